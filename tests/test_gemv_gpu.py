"""Dequant-dot GEMV (cmolcu_gemv / cmolcu_matmul) against the CPU checker.

The checker is the oracle restatement of cmol_matmul_scalar / _avx512
(src/quant.c:334-566), run on the identical GGUF blocks.  Float results can
only differ by summation order, so the bound is relative to the sum of
absolute products:  |gpu - oracle| <= 2e-6 * sum_k |w_k x_k| + 1e-30.
"""
import numpy as np
import pytest

from libcmol_b200 import synth

DTYPES = [synth.Q8_0, synth.Q4_0, synth.Q5_0, synth.Q4_K, synth.Q6_K, synth.F16, synth.F32]
REL = 2e-6


def _blocks(dtype, m, k, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((m, k), dtype=np.float32) * 0.02).astype(np.float32)
    return synth.quantize(w, dtype)


def _abs_bound(blob, dtype, m, k, x):
    from oracle.oracle import Oracle
    W = np.stack([Oracle.dequant(blob[r], k, dtype) for r in range(m)])
    return np.abs(W) @ np.abs(x)          # [m, n]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES, ids=[synth.DTYPE_NAMES[d] for d in DTYPES])
@pytest.mark.parametrize("m,k,n", [(64, 256, 1), (200, 512, 2), (96, 2048, 3), (36, 768, 1),
                                   (130, 4352, 1), (40, 11008, 2)])
def test_gemv_matches_oracle(gpu, dtype, m, k, n):
    import torch
    from libcmol_b200 import Weight
    from oracle.oracle import Oracle
    if k % synth.BLOCK[dtype][0]:
        pytest.skip("k not a multiple of the block size")
    blob = _blocks(dtype, m, k, seed=m * 7 + k + n)
    x = np.random.default_rng(1).standard_normal((k, n), dtype=np.float32)
    ref = Oracle.matmul(blob, x, m, k, n, dtype, lanes=16)
    W = Weight(blob, dtype, m, k)
    xd = torch.from_numpy(x).to(gpu)                    # [k, n] row-major: x(c,i) = x[i*n + c]
    yd = torch.zeros((m, n), dtype=torch.float32, device=gpu)
    W.gemv(xd, yd, n, x_ld=1, x_inc=n, y_ld=1, y_inc=n)
    torch.cuda.synchronize()
    got = yd.cpu().numpy()
    bound = REL * _abs_bound(blob, dtype, m, k, x) + 1e-30
    err = np.abs(got - ref)
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert np.all(err <= bound), f"err {err[worst]} > bound {bound[worst]} at {worst}"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [synth.Q8_0, synth.Q4_K, synth.Q4_0])
def test_gemv_fused_rmsnorm(gpu, dtype):
    """norm_w != NULL: y = W . (w * x / rms(x)), as src/model.c:90-97 then matmul."""
    import torch
    from libcmol_b200 import Weight
    from oracle.oracle import Oracle, fptr
    m, k = 128, 1024
    blob = _blocks(dtype, m, k, seed=5)
    rng = np.random.default_rng(2)
    x = rng.standard_normal(k, dtype=np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    xn = np.zeros(k, np.float32)
    Oracle.lib().orc_rms_norm(fptr(x), fptr(nw), fptr(xn), k, 1e-5)
    ref = Oracle.matmul(blob, xn, m, k, 1, dtype)[:, 0]
    W = Weight(blob, dtype, m, k)
    y = torch.zeros(m, device=gpu)
    W.gemv(torch.from_numpy(x).to(gpu), y, 1, x_ld=k, x_inc=1, y_ld=m, y_inc=1,
           norm_w=torch.from_numpy(nw).to(gpu), eps=1e-5)
    got = y.cpu().numpy()
    bound = 1e-5 * _abs_bound(blob, dtype, m, k, xn[:, None])[:, 0] + 1e-30
    assert np.all(np.abs(got - ref) <= bound)


@pytest.mark.gpu
def test_matmul_host_seam_known_answers(gpu):
    """cmolcu_matmul with the reference's own known-answer blocks
    (tests/test_quant.c:272-320 of the reference): Q8_0 m=2,k=32 -> {1, 6};
    two blocks k=64 -> 11."""
    import ctypes as C
    from libcmol_b200 import lib
    from oracle.oracle import fptr

    def q8(d, entries):
        b = np.zeros(34, np.uint8)
        b[0:2] = np.frombuffer(np.float16(d).tobytes(), np.uint8)
        for i, v in entries.items():
            b[2 + i] = np.uint8(np.int8(v).view(np.uint8))
        return b

    A = np.concatenate([q8(1.0, {0: 1}), q8(3.0, {1: 1})])
    B = np.zeros(32, np.float32)
    B[0], B[1] = 1.0, 2.0
    out = np.zeros(2, np.float32)
    lib().cmolcu_matmul(fptr(out), A.ctypes.data, fptr(B), 2, 32, 1, synth.Q8_0)
    assert out.tolist() == [1.0, 6.0]
    A2 = np.concatenate([q8(1.0, {0: 5}), q8(2.0, {0: 3})])
    B2 = np.zeros(64, np.float32)
    B2[0] = B2[32] = 1.0
    out2 = np.zeros(1, np.float32)
    lib().cmolcu_matmul(fptr(out2), A2.ctypes.data, fptr(B2), 1, 64, 1, synth.Q8_0)
    assert out2[0] == 11.0
    # unknown dtype: out untouched (src/quant.c:337-338)
    out3 = np.full(2, 9.5, np.float32)
    lib().cmolcu_matmul(fptr(out3), A.ctypes.data, fptr(B), 2, 32, 1, 99)
    assert out3.tolist() == [9.5, 9.5]
