"""cmolcu_matmul_noalloc against cmolcu_matmul, through the C ABI.

The no-allocation variant keeps its working memory in a static device array
instead of cudaMalloc'd buffers; its results must equal those of the
allocating seam on the same GGUF blocks.  The file name sorts last so that,
in a full run, it also executes after every other test in the same process.
"""
import ctypes as C

import numpy as np
import pytest

from libcmol_b200 import synth

_fp = C.POINTER(C.c_float)
REL = 1e-6

CASES = [(synth.Q8_0, 96, 512, 1), (synth.Q4_K, 200, 2048, 3), (synth.Q5_0, 64, 768, 2),
         (synth.Q4_0, 130, 4352, 1), (synth.Q6_K, 40, 1024, 4)]


def _api():
    from libcmol_b200 import lib
    L = lib()
    for name in ("cmolcu_matmul", "cmolcu_matmul_noalloc"):
        f = getattr(L, name)
        f.restype = None
        f.argtypes = [_fp, C.c_void_p, _fp, C.c_int, C.c_int, C.c_int, C.c_int]
    L.cmolcu_last_error.restype = C.c_char_p
    L.cmolcu_last_error.argtypes = []
    return L


def _fp_of(a):
    return a.ctypes.data_as(_fp)


def _inputs(dtype, m, k, n, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((m, k), dtype=np.float32) * 0.02).astype(np.float32)
    blob = np.ascontiguousarray(synth.quantize(w, dtype))
    b = np.ascontiguousarray(rng.standard_normal((k, n), dtype=np.float32))
    return blob, b, np.abs(w) @ np.abs(b)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,m,k,n", CASES, ids=[f"{synth.DTYPE_NAMES[c[0]]}-{c[1]}x{c[2]}x{c[3]}" for c in CASES])
def test_noalloc_matches_matmul(gpu, dtype, m, k, n):
    import torch
    L = _api()
    for call in range(2):                       # two calls in a row, different inputs
        blob, b, mag = _inputs(dtype, m, k, n, seed=1000 * call + m + k + n)
        want = np.zeros((m, n), np.float32)
        L.cmolcu_matmul(_fp_of(want), blob.ctypes.data, _fp_of(b), m, k, n, dtype)
        assert np.isfinite(want).all() and np.any(want != 0), L.cmolcu_last_error()
        got = np.full((m, n), np.nan, np.float32)
        free0 = torch.cuda.mem_get_info()[0] if call else None
        L.cmolcu_matmul_noalloc(_fp_of(got), blob.ctypes.data, _fp_of(b), m, k, n, dtype)
        assert L.cmolcu_last_error() == b"", L.cmolcu_last_error()
        if call:                                # scratch already resolved: no memory taken
            assert torch.cuda.mem_get_info()[0] == free0
        bound = REL * mag + 1e-30
        err = np.abs(got - want)
        assert np.all(err <= bound), f"call {call}: max err {err.max()}"


@pytest.mark.gpu
def test_noalloc_rejects_oversize(gpu):
    """2048 x 16384 Q8_0 needs ~71 MB of scratch (> 64 MiB): rejected, out untouched."""
    L = _api()
    m, k, n = 2048, 16384, 1
    blob = np.zeros(m * (k // 32) * 34, np.uint8)
    b = np.zeros(k, np.float32)
    out = np.full(m, 7.25, np.float32)
    L.cmolcu_matmul_noalloc(_fp_of(out), blob.ctypes.data, _fp_of(b), m, k, n, synth.Q8_0)
    assert b"limit" in L.cmolcu_last_error()
    assert np.all(out == 7.25)
