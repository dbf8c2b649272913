"""libcmol.so on the CPU: load, exports, host-only behaviour vs the reference.

No GPU is needed here: the library must load, export every function the
headers in include/ declare, and the host-side parts of the API (error
strings, ChatML formatting, version, the GGUF reader and the tokenizer) must
behave as the reference does on the same inputs (tests/golden/tokenizer.json
was produced by the reference's cmol_encode / cmol_decode_token /
cmol_strerror).
"""
import ctypes as C
import json
import os
import re
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden")


def _declared_functions():
    names = set()
    for h in ("cmol.h", "cmol_cuda.h", "cmolcu.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(cmol[a-z_0-9]*)\s*\(", src):
            names.add(m.group(1))
    return sorted(n for n in names if not n.endswith("_t"))


def test_library_exports_every_declared_function():
    from libcmol_b200 import lib
    L = lib()
    missing = [n for n in _declared_functions() if not hasattr(L, n)]
    assert not missing, missing
    assert len(_declared_functions()) > 30


def test_strerror_and_version_match_reference():
    from libcmol_b200.model import api
    gold = json.load(open(os.path.join(GOLD, "tokenizer.json")))
    for code, text in gold["strerror"].items():
        assert api().cmol_strerror(int(code)).decode() == text
    assert api().cmol_version().decode() == "0.1.0"


def test_chatml_helpers():
    from libcmol_b200.model import api
    L = api()
    buf = C.create_string_buffer(256)
    n = L.cmol_format_chatml(b"sys", b"hi", buf, 256)
    exp = b"<|im_start|>system\nsys<|im_end|>\n<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n"
    assert n == len(exp) and buf.value == exp
    n = L.cmol_format_chatml(None, b"hi", buf, 256)
    assert buf.value == b"<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n" and n == len(buf.value)
    assert L.cmol_format_chatml(b"", b"hi", None, 0) == n              # size probe
    assert L.cmol_format_chatml(b"", b"hi", buf, 5) == -8              # truncated
    assert L.cmol_format_chatml(b"", None, buf, 256) == -6
    n = L.cmol_format_chatml_turn(b"next", buf, 256)
    assert buf.value == b"<|im_end|>\n<|im_start|>user\nnext<|im_end|>\n<|im_start|>assistant\n"


def test_null_arguments_are_safe():
    from libcmol_b200.model import api
    L = api()
    L.cmol_free(None)
    assert L.cmol_session_acquire(None) is None
    L.cmol_session_release(None)
    L.cmol_session_reset(None)
    err = C.c_int(0)
    assert L.cmol_load(None, None, C.byref(err)) is None and err.value == -6
    assert L.cmol_load(b"/nonexistent.gguf", None, C.byref(err)) is None and err.value == -2


def _tok_path(tmp_path):
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg.gguf_path("q8_0", str(tmp_path))


def test_tokenizer_matches_reference(tmp_path):
    from libcmol_b200 import lib
    L = lib()
    L.cmolcu_tokenizer_open.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
    L.cmolcu_tokenizer_encode.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_int32), C.c_int]
    L.cmolcu_tokenizer_decode.restype = C.c_void_p
    L.cmolcu_tokenizer_decode.argtypes = [C.c_void_p, C.c_int32]
    L.cmolcu_tokenizer_free.argtypes = [C.c_void_p]
    gold = json.load(open(os.path.join(GOLD, "tokenizer.json")))
    t = C.c_void_p()
    assert L.cmolcu_tokenizer_open(_tok_path(tmp_path).encode(), C.byref(t)) == 0
    for text, exp in zip(gold["texts"], gold["encode"]):
        out = np.zeros(4096, np.int32)
        n = L.cmolcu_tokenizer_encode(t, text.encode(), out.ctypes.data_as(C.POINTER(C.c_int32)), 4096)
        assert n == exp["rc"], text
        assert out[:max(n, 0)].tolist() == exp["ids"], text
    for tid, hexv in gold["decode"].items():
        p = L.cmolcu_tokenizer_decode(t, int(tid))
        got = None if not p else C.string_at(p).hex()
        assert got == hexv, tid
    L.cmolcu_tokenizer_free(t)


def test_tokenizer_merge_order_matches_reference_live(tmp_path):
    """Random strings through both tokenizers (needs the reference build)."""
    from oracle.oracle import Reference, ReferenceModel
    if not Reference.available():
        pytest.skip("reference build (oracle/_ref) not present")
    from libcmol_b200 import lib
    L = lib()
    L.cmolcu_tokenizer_open.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
    L.cmolcu_tokenizer_encode.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_int32), C.c_int]
    path = _tok_path(tmp_path)
    t = C.c_void_p()
    assert L.cmolcu_tokenizer_open(path.encode(), C.byref(t)) == 0
    rm = ReferenceModel(path, 64)
    rng = np.random.default_rng(0)
    alphabet = list("abcdefghijklmnopqrstuvwxyz     ") + ["é", "☃", "<|im_end|>", "\n"]
    for _ in range(200):
        text = "".join(rng.choice(alphabet, size=int(rng.integers(0, 60))))
        n_ref, ids_ref = rm.encode(text)
        out = np.zeros(4096, np.int32)
        n = L.cmolcu_tokenizer_encode(t, text.encode(), out.ctypes.data_as(C.POINTER(C.c_int32)), 4096)
        assert n == n_ref and out[:max(n, 0)].tolist() == ids_ref.tolist(), text
    rm.close()


def test_tokenizer_parity_on_bench_texts(tmp_path, monkeypatch):
    """The tokenizer workload of bench.py (49152-token vocabulary, 4000-character
    texts near the 4096-symbol cap) encodes to the reference's ids, and a text
    past the cap gets the reference's answer too (needs the reference build)."""
    from oracle.oracle import Reference, ReferenceModel
    if not Reference.available():
        pytest.skip("reference build (oracle/_ref) not present")
    monkeypatch.setenv("CMOL_BENCH_CACHE", str(tmp_path))
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    from libcmol_b200 import lib
    path, texts = bench.tokenizer_setup()
    L = lib()
    L.cmolcu_tokenizer_open.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
    L.cmolcu_tokenizer_encode.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_int32), C.c_int]
    L.cmolcu_tokenizer_free.argtypes = [C.c_void_p]
    t = C.c_void_p()
    assert L.cmolcu_tokenizer_open(path.encode(), C.byref(t)) == 0
    rm = ReferenceModel(path, 64)
    try:
        for text in texts[:2] + [texts[2] + texts[3][:1000]]:
            n_ref, ids_ref = rm.encode(text.decode(), 8192)
            out = np.zeros(8192, np.int32)
            n = L.cmolcu_tokenizer_encode(t, text, out.ctypes.data_as(C.POINTER(C.c_int32)), 8192)
            assert n == n_ref and out[:max(n, 0)].tolist() == ids_ref.tolist(), (len(text), n, n_ref)
    finally:
        rm.close()
        L.cmolcu_tokenizer_free(t)
