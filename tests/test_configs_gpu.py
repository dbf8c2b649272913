"""Engine parity at the BASELINE configs' own layer shapes (GPU).

The models are reduced-depth versions of configs 1-4 (tests/golden/
make_golden.py: config_spec) that keep every per-layer shape the benchmarks
run: d_model 576 / 960 / 2048 / 2048, query / kv heads 9/3, 15/5, 32/32,
16/4 (group sizes 3, 3, 1, 4), d_head 64 or 128, the formats (Q8_0; Q4_0;
Q5_0 attention with Q4_K FFN; Q4_K with a Q8_0 head), vocabularies of 49152
and 128256, RoPE base 5e6 with NoPE on every 4th layer.  The expected values
come from the reference run on the same files (config 2 from the C
restatement, since the reference has no Q4_0), committed in
tests/golden/configs.npz.

Checked through the public API (cmol_forward_logits, cmol_forward_logits_batch,
cmol_generate_ids):
  * teacher-forced logits at every position: the reference's top 32 values,
    and the full vector at two positions: max-abs <= 2e-2 and cosine >=
    0.9999 (the specified tolerance; the f32 path stays below 1e-3);
  * greedy and seeded top-p streams identical to the reference's;
  * the tensor-core path forced on (CMOLCU_TC_MIN_COLS=1);
  * 16 sessions in one step at staggered positions (tensor cores at the
    default threshold), each column against the reference's logits at its
    own position.
"""
import hashlib
import importlib.util
import json
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ATOL, COS = 2e-2, 0.9999
CONFIGS = [1, 2, 3, 4]


def _mg():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLD, "configs.npz"))


@pytest.fixture(scope="module")
def cpaths(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("configs"))
    mg = _mg()
    man = json.load(open(os.path.join(GOLD, "manifest.json")))["configs"]
    out = {}
    for c in CONFIGS:
        p = mg.config_path(c, d)
        h = hashlib.sha256(open(p, "rb").read()).hexdigest()
        assert h == man[str(c)]["sha256"], f"config {c}: the synthetic writer changed; regenerate the goldens"
        out[c] = p
    return out


def _cos(a, b):
    return float(np.dot(a, b) / (np.linalg.norm(a) * np.linalg.norm(b)))


def _check_row(golden, c, i, got, tight=None):
    """Column logits `got` against the reference's at position i."""
    ids = golden[f"c{c}_top_ids"][i]
    d = float(np.abs(got[ids] - golden[f"c{c}_top_vals"][i]).max())
    assert d <= ATOL, (c, i, "top", d)
    nrm = float(golden[f"c{c}_norm"][i])
    assert abs(float(np.linalg.norm(got)) - nrm) <= 1e-3 * nrm, (c, i, "norm")
    if f"c{c}_full{i}" in golden:
        ref = golden[f"c{c}_full{i}"]
        d = max(d, float(np.abs(got - ref).max()))
        cs = _cos(got, ref)
        assert d <= ATOL and cs >= COS, (c, i, d, cs)
    if tight is not None:
        assert d < tight, (c, i, d)
    return d


@pytest.mark.gpu
@pytest.mark.parametrize("c", CONFIGS)
def test_config_teacher_forced_logits(gpu, golden, cpaths, c):
    from libcmol_b200.model import Model
    toks = golden[f"c{c}_tokens"]
    with Model(cpaths[c], max_ctx=64, max_sessions=2) as m:
        assert m.vocab == (128256 if c == 4 else 49152)
        s = m.acquire()
        worst = 0.0
        for i, t in enumerate(toks):
            worst = max(worst, _check_row(golden, c, i, s.forward_logits(int(t)), tight=1e-3))
        print(f"config {c}: f32 path worst max-abs {worst:.2e}")
        s.release()


@pytest.mark.gpu
@pytest.mark.parametrize("c", CONFIGS)
@pytest.mark.parametrize("tag", ["greedy", "topp"])
def test_config_streams(gpu, golden, cpaths, c, tag):
    from libcmol_b200.model import GenParams, Model
    p = {"greedy": GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=12),
         "topp": GenParams.make(0.9, top_p=0.9, top_k=40, seed=77, repeat_penalty=1.1, max_new_tokens=12)}[tag]
    with Model(cpaths[c], max_ctx=64, max_sessions=2) as m:
        s = m.acquire()
        rc, ids = s.generate_ids(golden[f"c{c}_tokens"][:6], p)
        assert rc == 0
        assert ids == golden[f"c{c}_gen_{tag}"].tolist()
        s.release()


@pytest.mark.gpu
@pytest.mark.parametrize("c", CONFIGS)
def test_config_tensor_cores(gpu, golden, cpaths, c, monkeypatch):
    """Every product on the tensor cores (f16 operands, f32 accumulation)."""
    from libcmol_b200.model import Model
    monkeypatch.setenv("CMOLCU_TC_MIN_COLS", "1")
    toks = golden[f"c{c}_tokens"]
    with Model(cpaths[c], max_ctx=64, max_sessions=2) as m:
        s = m.acquire()
        worst = 0.0
        for i, t in enumerate(toks):
            worst = max(worst, _check_row(golden, c, i, s.forward_logits(int(t))))
        print(f"config {c}: tensor-core worst max-abs {worst:.2e}")
        s.release()


@pytest.mark.gpu
@pytest.mark.parametrize("c", CONFIGS)
def test_config_wide_steps(gpu, golden, cpaths, c):
    """16 sessions fed the reference's token sequence with a stagger of one
    position each: step t holds session i at position t - i, so the columns
    of a step differ in token, position and context length.  The steps with
    all 16 columns take the tensor cores at the default threshold."""
    from libcmol_b200.model import Model
    toks = golden[f"c{c}_tokens"]
    T, NS = len(toks), 16
    with Model(cpaths[c], max_ctx=64, max_sessions=NS) as m:
        ss = [m.acquire() for _ in range(NS)]
        worst, wide = 0.0, 0
        for t in range(T + NS - 1):
            live = [i for i in range(NS) if 0 <= t - i < T]
            lg = m.forward_logits_batch([ss[i] for i in live], [int(toks[t - i]) for i in live])
            wide += len(live) == NS
            for row, i in enumerate(live):
                worst = max(worst, _check_row(golden, c, t - i, lg[row]))
        assert wide >= T - NS + 1
        print(f"config {c}: {wide} steps of {NS} columns, worst max-abs {worst:.2e}")
        for s in ss:
            assert s.n_tokens == T
            s.release()
