"""Batched dequant matmul on the tensor cores (cmolcu_matmul_batched).

The checker is the oracle's dequantisation of the identical GGUF blocks
(restating src/quant.c:152-194) times the activations in float64.  The
tensor-core path rounds the dequantised weights and the activations to f16
(11-bit significands) and accumulates in f32, so each product carries a
relative error of at most about 2 * 2^-11; the bound is

    |gpu - exact| <= 2.5e-3 * sum_k |w_k x_k| + 1e-6.
"""
import numpy as np
import pytest

from libcmol_b200 import synth

REL = 2.5e-3
CASES = [
    (synth.Q4_K, 256, 1024, 16),      # two row blocks, split K
    (synth.Q4_K, 384, 2048, 40),      # ragged column count
    (synth.Q8_0, 200, 960, 24),       # rows not a multiple of 128, a short last K-chunk
    (synth.Q4_0, 128, 576, 7),        # one K-chunk
    (synth.Q5_0, 512, 2048, 64),
    (synth.Q8_0, 19200, 512, 16),     # > 148 row blocks: no K split, epilogue from tensor memory
    (synth.Q4_K, 1024, 4096, 256),    # the widest column count
    # >= 64 blocks of 256 rows at 128 columns: two 128-row sub-tiles per CTA
    # (two tensor-memory accumulators share each activation tile); the last
    # block is ragged (a partial second sub-tile)
    (synth.Q4_K, 16512, 512, 256),
    (synth.Q4_0, 16448, 256, 128),
    # wider than 128 columns: every format, ragged widths, split K through a
    # cluster (also run with the dequantised tiles in tensor memory below)
    (synth.Q4_0, 16448, 256, 130),
    (synth.Q8_0, 300, 1024, 200),
    (synth.Q5_0, 2048, 1024, 256),
    (synth.Q4_K, 512, 8192, 256),
]


def _dequant(blob, rows, k, dtype):
    from oracle.oracle import Oracle
    return np.stack([Oracle.dequant(blob[r], k, dtype) for r in range(rows)]).astype(np.float64)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,rows,k,n", CASES,
                         ids=[f"{synth.DTYPE_NAMES[c[0]]}-{c[1]}x{c[2]}-n{c[3]}" for c in CASES])
@pytest.mark.parametrize("norm", [False, True], ids=["plain", "rmsnorm"])
def test_batched_matches_exact(gpu, dtype, rows, k, n, norm):
    import torch
    from libcmol_b200 import Weight
    rng = np.random.default_rng(rows + k + n)
    wq = (rng.standard_normal((rows, k), dtype=np.float32) * 0.02).astype(np.float32)
    blob = synth.quantize(wq, dtype)
    x = rng.standard_normal((n, k), dtype=np.float32)
    gains = (1.0 + 0.1 * rng.standard_normal(k)).astype(np.float32)
    W = Weight(blob, dtype, rows, k)
    xd = torch.from_numpy(x).to(gpu)
    yd = torch.full((n, rows), float("nan"), dtype=torch.float32, device=gpu)
    gd = torch.from_numpy(gains).to(gpu) if norm else None
    eps = 1e-5
    W.matmul_batched(xd, yd, n, norm_w=gd, eps=eps)
    torch.cuda.synchronize()
    got = yd.cpu().numpy().astype(np.float64)
    xn = x.astype(np.float64)
    if norm:
        inv = 1.0 / np.sqrt((xn * xn).mean(axis=1, keepdims=True) + eps)
        xn = xn * inv * gains.astype(np.float64)
    Wd = _dequant(blob, rows, k, dtype)
    want = xn @ Wd.T
    bound = REL * (np.abs(xn) @ np.abs(Wd).T) + 1e-6
    err = np.abs(got - want)
    assert np.isfinite(got).all()
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert np.all(err <= bound), f"err {err[worst]} > bound {bound[worst]} at {worst}"
    W.free()


@pytest.mark.gpu
def test_batched_rejects_unsupported(gpu):
    import torch
    from libcmol_b200 import CmolError, Weight
    blob = synth.quantize(np.zeros((64, 256), np.float32), synth.Q6_K)
    W = Weight(blob, synth.Q6_K, 64, 256)
    x = torch.zeros(16, 256, device=gpu)
    y = torch.zeros(16, 64, device=gpu)
    with pytest.raises(CmolError, match="tensor-core"):
        W.matmul_batched(x, y, 16)
    W.free()


@pytest.mark.gpu
def test_batched_global_partials(gpu):
    """With clusters off (CMOLCU_TC_CLUSTER=0, read once per process) the K
    splits add their partials through global scratch and the last CTA of the
    row block; same bound, in a fresh process."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    code = f"""
import sys
sys.path.insert(0, {os.path.dirname(here)!r})
sys.path.insert(0, {here!r})
import torch
import test_gemm_tc_gpu as t
dev = torch.device("cuda:0")
for case in [t.CASES[0], t.CASES[4], t.CASES[6]]:
    t.test_batched_matches_exact(dev, *case, norm=True)
print("ok")
"""
    env = dict(os.environ, CMOLCU_TC_CLUSTER="0")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.gpu
def test_batched_tensor_memory_tiles(gpu):
    """With CMOLCU_TC_TS=1 (read once per process) steps wider than 128
    columns keep the dequantised tiles in tensor memory and the tensor core
    reads A from there; the cases wider than 128 columns, same bound, in a
    fresh process."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    code = f"""
import sys
sys.path.insert(0, {os.path.dirname(here)!r})
sys.path.insert(0, {here!r})
import torch
import test_gemm_tc_gpu as t
dev = torch.device("cuda:0")
for case in [c for c in t.CASES if c[3] > 128]:
    t.test_batched_matches_exact(dev, *case, norm=True)
print("ok")
"""
    env = dict(os.environ, CMOLCU_TC_TS="1")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr
