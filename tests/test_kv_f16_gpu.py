"""The f16 KV cache format (cmol_cuda_options_t.kv_dtype = 1) on a GPU.

Every K and V value is rounded to the nearest f16 when written and widened
exactly when read.  Two checks:
  * against the C restatement run with the same rounding (orc_set_kv_f16):
    logits within 1e-3 (only the summation order differs) and identical
    greedy streams, including long contexts (many pages and attention splits)
    and batched prefill (the group attention path);
  * against the reference's own f32-cache logits (tests/golden): within the
    engine's specified tolerance, max-abs <= 2e-2 and cosine >= 0.9999, at
    the benchmark configs' layer shapes too.
"""
import importlib.util
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ATOL, COS = 2e-2, 0.9999
MODELS = ["q8_0", "q4_k", "smollm3", "mixed"]


def _mg():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _cos(a, b):
    return float(np.dot(a, b) / (np.linalg.norm(a) * np.linalg.norm(b)))


@pytest.fixture
def oracle_f16():
    """The C restatement with its KV cache rounded to f16 (reset afterwards)."""
    from oracle.oracle import Oracle
    Oracle.lib().orc_set_kv_f16(1)
    yield
    Oracle.lib().orc_set_kv_f16(0)


@pytest.fixture(scope="module")
def cfg_path(tmp_path_factory):
    """Config-shape model files, written once per module on first use."""
    d = str(tmp_path_factory.mktemp("f16cfg"))
    mg = _mg()
    return lambda c: mg.config_path(c, d)


@pytest.fixture(scope="module")
def paths(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("f16kv"))
    mg = _mg()
    return {n: mg.gguf_path(n, d) for n in MODELS}


@pytest.mark.gpu
@pytest.mark.parametrize("name", MODELS)
def test_f16_kv_teacher_forced(gpu, paths, oracle_f16, name):
    from libcmol_b200.model import Model
    from oracle.oracle import OracleModel
    g = np.load(os.path.join(GOLD, "models.npz"))
    toks = g[f"{name}_tokens"]
    om = OracleModel(paths[name], lanes=16)
    os_ = om.session(64)
    with Model(paths[name], max_ctx=64, max_sessions=2, page_tokens=4, kv_dtype=1) as m:
        s = m.acquire()
        w_orc, w_ref = 0.0, 0.0
        for i, t in enumerate(toks):
            got = s.forward_logits(int(t))
            orc = om.forward(os_, int(t), i)
            ref = g[f"{name}_logits"][i]
            w_orc = max(w_orc, float(np.abs(got - orc).max()))
            d = float(np.abs(got - ref).max())
            w_ref = max(w_ref, d)
            assert d <= ATOL and _cos(got, ref) >= COS, (i, d)
        assert w_orc < 1e-3, w_orc
        print(f"{name}: f16 KV vs f16 checker {w_orc:.2e}, vs reference f32 cache {w_ref:.2e}")
        s.release()
    om.free_session(os_)


@pytest.mark.gpu
@pytest.mark.parametrize("name", MODELS)
def test_f16_kv_greedy_stream(gpu, paths, oracle_f16, name):
    from libcmol_b200.model import GenParams, Model
    from oracle.oracle import GenParams as OGen
    from oracle.oracle import OracleModel
    g = np.load(os.path.join(GOLD, "models.npz"))
    prompt = g[f"{name}_tokens"][:6]
    om = OracleModel(paths[name], lanes=16)
    os_ = om.session(64)
    want, _ = om.generate_ids(os_, prompt, OGen.make(0.0, repeat_penalty=1.0, max_new_tokens=20))
    om.free_session(os_)
    with Model(paths[name], max_ctx=64, max_sessions=2, kv_dtype=1) as m:
        s = m.acquire()
        rc, ids = s.generate_ids(prompt, GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=20))
        assert rc == 0 and ids == want.tolist()
        s.release()


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["q8_0", "smollm3"])
def test_f16_kv_long_context_and_prefill(gpu, tmp_path, oracle_f16, name):
    """300 + 170 token prompts in batched prefill (group attention over
    many pages and three 128-token splits), then greedy decode: streams as
    the f16-cache checker gives them for each prompt alone; then teacher
    forcing at long positions."""
    from libcmol_b200 import synth
    from libcmol_b200.model import GenParams, Model
    from oracle.oracle import GenParams as OGen
    from oracle.oracle import OracleModel
    kw = {"q8_0": dict(dtype=8),
          "smollm3": dict(dtype=12, n_layers=3, arch="smollm3", no_rope_interval=2, rope_base=5e6, qk_norm=True,
                          tied=False, dt_head=8, n_heads=4, n_kv_heads=1)}[name]
    dt = kw.pop("dtype")
    path = str(tmp_path / f"long_{name}.gguf")
    synth.write_gguf(path, synth.tiny_spec(dt, ctx=512, **kw))
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 512, size=300).astype(np.int32), rng.integers(0, 512, size=170).astype(np.int32)]
    om = OracleModel(path, lanes=16)
    want = []
    for pr in prompts:
        os_ = om.session(512)
        ids, _ = om.generate_ids(os_, pr, OGen.make(0.0, repeat_penalty=1.0, max_new_tokens=8))
        want.append(ids.tolist())
        om.free_session(os_)
    with Model(path, max_ctx=512, max_sessions=2, kv_dtype=1) as m:
        ss = [m.acquire() for _ in prompts]
        got = m.generate_batch(ss, prompts, [GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=8)] * 2)
        assert [x.tolist() for x in got] == want
        for s in ss:
            s.release()
        s = m.acquire()
        os_ = om.session(512)
        toks = rng.integers(0, 512, size=260)
        for i, t in enumerate(toks):
            got = s.forward_logits(int(t))
            ref = om.forward(os_, int(t), i)
            if i % 51 == 0 or i == len(toks) - 1:
                assert np.abs(got - ref).max() < 1e-3, i
        s.release()
        om.free_session(os_)


@pytest.mark.gpu
@pytest.mark.parametrize("c", [1, 3, 4])
def test_f16_kv_config_shapes(gpu, cfg_path, c):
    """The configs' layer shapes with the f16 cache, every position against
    the reference's f32-cache logits (spec tolerance), and 16-column steps
    (tensor cores) at staggered positions."""
    from libcmol_b200.model import Model
    path = cfg_path(c)
    gold = np.load(os.path.join(GOLD, "configs.npz"))
    toks = gold[f"c{c}_tokens"]

    def check(i, got):
        ids = gold[f"c{c}_top_ids"][i]
        d = float(np.abs(got[ids] - gold[f"c{c}_top_vals"][i]).max())
        if f"c{c}_full{i}" in gold:
            ref = gold[f"c{c}_full{i}"]
            d = max(d, float(np.abs(got - ref).max()))
            assert _cos(got, ref) >= COS, (i, "cos")
        assert d <= ATOL, (i, d)
        return d

    with Model(path, max_ctx=64, max_sessions=16, kv_dtype=1) as m:
        s = m.acquire()
        worst = max(check(i, s.forward_logits(int(t))) for i, t in enumerate(toks))
        s.release()
        ss = [m.acquire() for _ in range(16)]
        for t in range(len(toks) + 15):
            live = [i for i in range(16) if 0 <= t - i < len(toks)]
            lg = m.forward_logits_batch([ss[i] for i in live], [int(toks[t - i]) for i in live])
            for row, i in enumerate(live):
                worst = max(worst, check(t - i, lg[row]))
        print(f"config {c}: f16 KV worst max-abs vs reference {worst:.2e}")
        for x in ss:
            x.release()


@pytest.mark.gpu
@pytest.mark.parametrize("c", [1, 3, 4])
@pytest.mark.parametrize("tag", ["greedy", "topp"])
def test_f16_kv_config_streams_match_reference(gpu, cfg_path, c, tag):
    """With the f16 cache, the configs' greedy and seeded top-p streams are
    still the reference's own (f32 cache) streams."""
    from libcmol_b200.model import GenParams, Model
    path = cfg_path(c)
    gold = np.load(os.path.join(GOLD, "configs.npz"))
    p = {"greedy": GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=12),
         "topp": GenParams.make(0.9, top_p=0.9, top_k=40, seed=77, repeat_penalty=1.1, max_new_tokens=12)}[tag]
    with Model(path, max_ctx=64, max_sessions=2, kv_dtype=1) as m:
        s = m.acquire()
        rc, ids = s.generate_ids(gold[f"c{c}_tokens"][:6], p)
        assert rc == 0 and ids == gold[f"c{c}_gen_{tag}"].tolist()
        s.release()


@pytest.mark.gpu
@pytest.mark.parametrize("name", MODELS)
def test_f16_kv_tensor_core_attention(gpu, paths, monkeypatch, name):
    """Every step on the tensor cores (CMOLCU_TC_MIN_COLS=1): the weight
    products and, with the f16 cache, the persistent decode attention (f16
    queries and probabilities, f32 accumulation).  Logits against the
    reference's f32 cache at the specified tolerance."""
    from libcmol_b200.model import Model
    monkeypatch.setenv("CMOLCU_TC_MIN_COLS", "1")
    g = np.load(os.path.join(GOLD, "models.npz"))
    with Model(paths[name], max_ctx=64, max_sessions=2, page_tokens=4, kv_dtype=1) as m:
        s = m.acquire()
        worst = 0.0
        for i, t in enumerate(g[f"{name}_tokens"]):
            got = s.forward_logits(int(t))
            ref = g[f"{name}_logits"][i]
            d = float(np.abs(got - ref).max())
            worst = max(worst, d)
            assert d <= ATOL and _cos(got, ref) >= COS, (i, d)
        print(f"{name}: tensor-core attention, f16 cache: worst max-abs {worst:.2e}")
        s.release()


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["q8_0", "smollm3"])
def test_f16_kv_tensor_core_attention_long(gpu, tmp_path, monkeypatch, oracle_f16, name):
    """The persistent tensor-core attention over 400 positions (many 64-token
    sub-tiles, columns split into several chunks merged in order, partial
    last sub-tiles), and 16 staggered sessions at once: logits against the
    f16-cache checker within the specified tolerance."""
    from libcmol_b200 import synth
    from libcmol_b200.model import Model
    from oracle.oracle import OracleModel
    monkeypatch.setenv("CMOLCU_TC_MIN_COLS", "1")
    kw = {"q8_0": dict(dtype=8),
          "smollm3": dict(dtype=12, n_layers=3, arch="smollm3", no_rope_interval=2, rope_base=5e6, qk_norm=True,
                          tied=False, dt_head=8, n_heads=4, n_kv_heads=1)}[name]
    dt = kw.pop("dtype")
    path = str(tmp_path / f"tcattn_{name}.gguf")
    synth.write_gguf(path, synth.tiny_spec(dt, ctx=512, **kw))
    rng = np.random.default_rng(9)
    toks = rng.integers(0, 512, size=400)
    om = OracleModel(path, lanes=16)
    os_ = om.session(512)
    refs = {}
    for i, t in enumerate(toks):
        r = om.forward(os_, int(t), i)
        if i % 23 == 0 or i >= 390:
            refs[i] = r
    om.free_session(os_)
    with Model(path, max_ctx=512, max_sessions=16, kv_dtype=1) as m:
        s = m.acquire()
        worst = 0.0
        for i, t in enumerate(toks):
            got = s.forward_logits(int(t))
            if i in refs:
                d = float(np.abs(got - refs[i]).max())
                worst = max(worst, d)
                assert d <= ATOL and _cos(got, refs[i]) >= COS, (i, d)
        s.release()
        ss = [m.acquire() for _ in range(16)]
        for t in range(len(toks) + 15):
            live = [i for i in range(16) if 0 <= t - i < len(toks)]
            lg = m.forward_logits_batch([ss[i] for i in live], [int(toks[t - i]) for i in live])
            for row, i in enumerate(live):
                if t - i in refs:
                    d = float(np.abs(lg[row] - refs[t - i]).max())
                    worst = max(worst, d)
                    assert d <= ATOL and _cos(lg[row], refs[t - i]) >= COS, (t, i, d)
        print(f"{name}: tensor-core attention to position 400: worst max-abs {worst:.2e}")
        for x in ss:
            x.release()
