"""Pins the CPU checker (oracle/cmol_oracle.c) to the reference.

1. The reference's own known-answer vectors (tests/test_quant.c:97-320,
   tests/test_model.c:128-166, tests/test_sampler.c:452-549 of the reference).
2. The golden fixtures under tests/golden/, produced by the unmodified
   reference (tests/golden/make_golden.py).  The restatement runs the
   reference's AVX-512 lane order, so model logits must be bit-identical.
3. Q4_0 (not implemented by the reference) against gguf-py 0.19.0.
"""
import hashlib
import json
import math
import os

import numpy as np
import pytest

from libcmol_b200 import synth
from oracle.oracle import GenParams, Oracle, OracleModel, fptr, iptr

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def f16(x):
    return np.frombuffer(np.float16(x).tobytes(), np.uint8)


def q8_block(d, entries):
    b = np.zeros(34, np.uint8)
    b[0:2] = f16(d)
    for i, v in entries.items():
        b[2 + i] = np.uint8(np.int8(v).view(np.uint8))
    return b


# ---- 1. reference known answers ---------------------------------------------

def test_known_answer_q8_0_dequant():
    out = Oracle.dequant(q8_block(2.0, {0: 3, 1: -1}), 32, synth.Q8_0)
    assert out[0] == 6.0 and out[1] == -2.0 and out[2] == 0.0 and out[31] == 0.0
    two = np.concatenate([q8_block(1.0, {0: 7}), q8_block(3.0, {0: 2})])
    out = Oracle.dequant(two, 64, synth.Q8_0)
    assert out[0] == 7.0 and out[32] == 6.0


def test_known_answer_q4_k_dequant():
    b = np.zeros(144, np.uint8)
    b[0:2], b[2:4] = f16(1.0), f16(0.0)
    b[4] = 1          # sub-block 0: sc=1
    b[5] = 1          # sub-block 1: sc=1
    b[16] = (10 << 4) | 3
    out = Oracle.dequant(b, 256, synth.Q4_K)
    assert out[0] == 3.0 and out[1] == 0.0 and out[2] == 0.0 and out[32] == 10.0 and out[255] == 0.0


def test_known_answer_q6_k_dequant():
    b = np.zeros(210, np.uint8)
    b[208:210] = f16(1.0)
    b[192] = 2        # scales[0]
    b[0] = 0x0A       # ql[0]
    b[128] = 0x02     # qh[0]
    out = Oracle.dequant(b, 256, synth.Q6_K)
    assert out[0] == 20.0 and out[1] == -64.0 and out[16] == 0.0


def test_known_answer_matmuls():
    A = np.array([1, 0, 0, 0, 0, 1, 0, 0, 1, 1, 0, 0], np.float32)
    out = Oracle.matmul(A.view(np.uint8), np.array([5, 7, 0, 0], np.float32), 3, 4, 1, synth.F32, lanes=1)
    assert out[:, 0].tolist() == [5.0, 7.0, 12.0]
    A2 = np.array([1, 0, 0, 0, 0, 1, 0, 0], np.float32)
    out = Oracle.matmul(A2.view(np.uint8), np.array([1, 2, 3, 4, 0, 0, 0, 0], np.float32), 2, 4, 2,
                        synth.F32, lanes=1)
    assert out.ravel().tolist() == [1.0, 2.0, 3.0, 4.0]
    A3 = np.concatenate([q8_block(1.0, {0: 1}), q8_block(3.0, {1: 1})])
    B = np.zeros(32, np.float32)
    B[0], B[1] = 1, 2
    assert Oracle.matmul(A3, B, 2, 32, 1, synth.Q8_0)[:, 0].tolist() == [1.0, 6.0]
    A4 = np.concatenate([q8_block(1.0, {0: 5}), q8_block(2.0, {0: 3})])
    B4 = np.zeros(64, np.float32)
    B4[0] = B4[32] = 1
    assert Oracle.matmul(A4, B4, 1, 64, 1, synth.Q8_0)[0, 0] == 11.0


def test_known_answer_dequant_noops():
    dst = np.full(32, 9.9, np.float32)
    Oracle.lib().orc_dequant_row(None, fptr(dst), 32, synth.Q8_0)
    Oracle.lib().orc_dequant_row(q8_block(1.0, {}).ctypes.data, fptr(dst), 0, synth.Q8_0)
    Oracle.lib().orc_dequant_row(q8_block(1.0, {}).ctypes.data, fptr(dst), 32, 99)
    assert np.all(dst == np.float32(9.9))


def test_known_answer_rope():
    L = Oracle.lib()
    q = np.array([1, 2, 3, 4, 5, 6, 7, 8], np.float32)
    k = np.array([1, 2, 3, 4], np.float32)
    q0, k0 = q.copy(), k.copy()
    L.orc_rope_apply(fptr(q), fptr(k), 0, 2, 1, 4, 10000.0)
    assert np.array_equal(q, q0) and np.array_equal(k, k0)
    q2 = np.array([1, 2, 3, 4], np.float32)
    k2 = q2.copy()
    L.orc_rope_apply(fptr(q2), fptr(k2), 1, 1, 1, 4, 10000.0)
    assert abs(q2[0] - (math.cos(1) - 2 * math.sin(1))) < 1e-3
    assert abs(q2[1] - (math.sin(1) + 2 * math.cos(1))) < 1e-3
    assert abs(math.hypot(q2[0], q2[1]) - math.hypot(1, 2)) < 1e-5


def test_known_answer_repeat_penalty():
    L = Oracle.lib()
    V = 8

    def pen(val, toks, p):
        l = np.full(V, val, np.float32)
        t = np.array(toks, np.int32)
        L.orc_apply_repeat_penalty(fptr(l), V, iptr(t), len(t), p)
        return l

    l = pen(2.0, [0, 3], 2.0)
    assert l[0] == 1.0 and l[3] == 1.0 and l[1] == 2.0
    l = pen(-2.0, [5], 3.0)
    assert l[5] == -6.0 and l[2] == -2.0
    assert pen(0.0, [4], 2.0)[4] == 0.0
    assert pen(5.0, [2], 1.0)[2] == 5.0 and pen(5.0, [2], 0.5)[2] == 5.0
    l = pen(3.0, [-1, V, 2], 2.0)
    assert l[2] == 1.5 and l[0] == 3.0
    l = np.arange(V, dtype=np.float32)
    t = np.array([7], np.int32)
    L.orc_apply_repeat_penalty(fptr(l), V, iptr(t), 1, 100.0)
    p = GenParams.make(temperature=0.0)
    assert L.orc_sample(fptr(l), V, p, None) == 6


def test_known_answer_rng_determinism():
    L = Oracle.lib()
    a = (np.ctypeslib.ctypes.c_uint64 * 4)()
    b = (np.ctypeslib.ctypes.c_uint64 * 4)()
    L.orc_rng_seed(a, 42)
    L.orc_rng_seed(b, 42)
    assert [L.orc_rng_next(a) for _ in range(8)] == [L.orc_rng_next(b) for _ in range(8)]


# ---- 2. golden fixtures from the reference ------------------------------------

def _gold(name):
    return np.load(os.path.join(GOLD, name), allow_pickle=False)


@pytest.mark.parametrize("dt", [synth.Q8_0, synth.Q5_0, synth.Q4_K, synth.Q6_K, synth.F16, synth.F32],
                         ids=lambda d: synth.DTYPE_NAMES[d])
def test_golden_gemv_bit_exact(dt):
    g = _gold("gemv.npz")
    name = synth.DTYPE_NAMES[dt]
    for n in (1, 3):
        blob, x = g[f"{name}_n{n}_blocks"], g[f"{name}_n{n}_x"]
        m, k = blob.shape[0], x.shape[0]
        assert np.array_equal(Oracle.matmul(blob, x, m, k, n, dt, lanes=16), g[f"{name}_n{n}_simd"])
        assert np.array_equal(Oracle.matmul(blob, x, m, k, n, dt, lanes=1), g[f"{name}_n{n}_scalar"])
    assert np.array_equal(Oracle.dequant(g[f"{name}_n1_blocks"][0], 512, dt), g[f"{name}_deq_row0"])


def test_q4_0_matches_gguf_py():
    g = _gold("gemv.npz")
    blob = g["Q4_0_blocks"]
    got = np.stack([Oracle.dequant(blob[r], 256, synth.Q4_0) for r in range(blob.shape[0])])
    assert np.array_equal(got, g["Q4_0_deq_ggufpy"])


def _golden_model(name, tmp_path):
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    path = mg.gguf_path(name, str(tmp_path))
    man = json.load(open(os.path.join(GOLD, "manifest.json")))
    h = hashlib.sha256(open(path, "rb").read()).hexdigest()
    assert h == man["models"][name]["sha256"], "synthetic GGUF writer output changed"
    return path


MODELS = ["q8_0", "q5_0", "q4_k", "q6_k", "smollm3", "mixed"]


@pytest.mark.parametrize("name", MODELS)
def test_golden_teacher_forced_logits_bit_exact(name, tmp_path):
    g = _gold("models.npz")
    om = OracleModel(_golden_model(name, tmp_path), lanes=16)
    s = om.session(64)
    toks = g[f"{name}_tokens"]
    got = np.stack([om.forward(s, int(t), i) for i, t in enumerate(toks)])
    om.free_session(s)
    assert np.array_equal(got, g[f"{name}_logits"])


@pytest.mark.parametrize("name", MODELS)
def test_golden_generate_loop(name, tmp_path):
    g = _gold("models.npz")
    om = OracleModel(_golden_model(name, tmp_path), lanes=16)
    eos = om.hp["eos"]
    toks = g[f"{name}_tokens"][:6]
    for tag, p in (("greedy", GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=20)),
                   ("greedy_pen", GenParams.make(0.0, repeat_penalty=1.3, repeat_last_n=8, max_new_tokens=20)),
                   ("topp", GenParams.make(0.9, top_p=0.9, top_k=40, seed=1234, repeat_penalty=1.1,
                                           max_new_tokens=20)),
                   ("topk", GenParams.make(1.2, top_p=1.0, top_k=5, seed=99, repeat_penalty=1.0,
                                           max_new_tokens=20))):
        s = om.session(64)
        ids, lg = om.generate_ids(s, toks, p, eos=eos, logits_cap=32)
        om.free_session(s)
        assert ids.tolist() == g[f"{name}_gen_{tag}"].tolist(), tag
        assert np.array_equal(lg, g[f"{name}_gen_{tag}_logits"]), tag


def test_golden_sampler():
    g = _gold("sampler.npz")
    L = Oracle.lib()
    for i in range(len(g["token"])):
        lg = g["logits"][i].copy()
        temp, top_p, top_k, pen, seed = g["params"][i]
        ring = g["ring"][i]
        ring = ring[ring >= 0].astype(np.int32)
        st = (np.ctypeslib.ctypes.c_uint64 * 4)()
        L.orc_rng_seed(st, int(seed))
        if pen > 1.0 and len(ring):
            L.orc_apply_repeat_penalty(fptr(lg), len(lg), iptr(ring), len(ring), float(pen))
        p = GenParams.make(float(temp), top_p=float(top_p), top_k=int(top_k), seed=int(seed),
                           repeat_penalty=float(pen))
        tok = L.orc_sample(fptr(lg), len(lg), p, st)
        assert tok == g["token"][i], i
        assert list(st) == [int(v) for v in g["rng_after"][i]], i


@pytest.mark.parametrize("kw", [dict(dt=synth.Q8_0), dict(dt=synth.Q4_K, arch="smollm3", no_rope_interval=2,
                                                          rope_base=5e6, qk_norm=True, tied=False, dt_head=8,
                                                          n_heads=4, n_kv_heads=1, d_model=512)],
                         ids=["q8_0", "smollm3-shape"])
def test_f16_kv_cache_stays_within_logit_tolerance(tmp_path, kw):
    """Groundwork for an f16 KV format (not in the reference, which stores
    f32): the oracle with K and V rounded to f16 on write, against the f32
    cache, over a 600-token context.  Every compared step must stay within
    the engine's logit tolerance (max-abs 2e-2, cosine 0.9999)."""
    kw = dict(kw)
    dt = kw.pop("dt")
    path = str(tmp_path / "kv.gguf")
    synth.write_gguf(path, synth.tiny_spec(dt, ctx=1024, **kw))
    om = OracleModel(path, lanes=16)
    rng = np.random.default_rng(5)
    toks = rng.integers(0, 512, size=600)
    worst_abs, worst_cos = 0.0, 1.0
    s32, s16 = om.session(1024), om.session(1024)
    try:
        for i, t in enumerate(toks):
            om.L.orc_set_kv_f16(0)
            a = om.forward(s32, int(t), i)
            om.L.orc_set_kv_f16(1)
            b = om.forward(s16, int(t), i)
            worst_abs = max(worst_abs, float(np.abs(a - b).max()))
            worst_cos = min(worst_cos, float(np.dot(a, b) / (np.linalg.norm(a) * np.linalg.norm(b))))
    finally:
        om.L.orc_set_kv_f16(0)
        om.free_session(s32)
        om.free_session(s16)
    print(f"f16 KV over 600 tokens: max-abs {worst_abs:.3g}, min cosine {worst_cos:.9f}")
    assert worst_abs <= 2e-2 and worst_cos >= 0.9999
