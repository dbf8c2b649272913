"""End-to-end parity of the decode engine (libcmol.so public API) on a GPU.

Checks, on the seeded synthetic GGUFs of tests/golden/:
  * teacher-forced logits (cmol_forward_logits) against the reference's
    cmol_model_forward logits: max-abs <= 2e-2 and cosine >= 0.9999 (the
    tolerance the engine is specified to), and in practice far tighter;
  * greedy token streams of cmol_generate_ids identical to the reference's
    generate loop; sampled streams (top-k / top-p, seeded) identical as long
    as no sampling decision falls within float rounding of a boundary;
  * continuous batching: sessions generated together equal each alone;
  * KV paging and split-context attention beyond one page / one split;
  * stop rules and session bookkeeping (max_new, EOS, abort, reset).
"""
import importlib.util
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MODELS = ["q8_0", "q5_0", "q4_k", "q6_k", "smollm3", "mixed"]
ATOL, COS = 2e-2, 0.9999
MODEL_KW = {
    "q8_0": dict(dtype=8),
    "smollm3": dict(dtype=12, n_layers=3, arch="smollm3", no_rope_interval=2, rope_base=5e6, qk_norm=True,
                    tied=False, dt_head=8, n_heads=4, n_kv_heads=1),
}


def _mg():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLD, "models.npz"))


@pytest.fixture(scope="module")
def paths(tmp_path_factory):
    d = tmp_path_factory.mktemp("gold")
    mg = _mg()
    return {n: mg.gguf_path(n, str(d)) for n in MODELS}


def _cos(a, b):
    return float(np.dot(a, b) / (np.linalg.norm(a) * np.linalg.norm(b)))


def _params(tag):
    from libcmol_b200.model import GenParams
    return {"greedy": GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=20),
            "greedy_pen": GenParams.make(0.0, repeat_penalty=1.3, repeat_last_n=8, max_new_tokens=20),
            "topp": GenParams.make(0.9, top_p=0.9, top_k=40, seed=1234, repeat_penalty=1.1, max_new_tokens=20),
            "topk": GenParams.make(1.2, top_p=1.0, top_k=5, seed=99, repeat_penalty=1.0, max_new_tokens=20)}[tag]


@pytest.mark.gpu
@pytest.mark.parametrize("name", MODELS)
def test_teacher_forced_logits(gpu, golden, paths, name):
    from libcmol_b200.model import Model
    with Model(paths[name], max_ctx=64, max_sessions=2, page_tokens=4) as m:
        s = m.acquire()
        toks = golden[f"{name}_tokens"]
        worst = 0.0
        for i, t in enumerate(toks):
            got = s.forward_logits(int(t))
            ref = golden[f"{name}_logits"][i]
            d = float(np.abs(got - ref).max())
            worst = max(worst, d)
            assert d <= ATOL and _cos(got, ref) >= COS, (i, d)
        assert s.n_tokens == len(toks)
        assert worst < 1e-3, worst          # f32 end to end: only summation order differs
        s.release()


@pytest.mark.gpu
@pytest.mark.parametrize("name", MODELS)
def test_teacher_forced_logits_tensor_cores(gpu, golden, paths, name, monkeypatch):
    """The tensor-core matmul forced on every step (CMOLCU_TC_MIN_COLS=1):
    f16 weights and activations, f32 accumulation.  Same tolerance as the
    engine's spec; formats without a tensor-core path (Q6_K) keep the GEMV."""
    from libcmol_b200.model import Model
    monkeypatch.setenv("CMOLCU_TC_MIN_COLS", "1")
    with Model(paths[name], max_ctx=64, max_sessions=2, page_tokens=4) as m:
        s = m.acquire()
        toks = golden[f"{name}_tokens"]
        worst, wcos = 0.0, 1.0
        for i, t in enumerate(toks):
            got = s.forward_logits(int(t))
            ref = golden[f"{name}_logits"][i]
            d = float(np.abs(got - ref).max())
            c = _cos(got, ref)
            worst, wcos = max(worst, d), min(wcos, c)
            assert d <= ATOL and c >= COS, (i, d, c)
        print(f"{name}: tensor-core logits max-abs {worst:.2e} cos {wcos:.7f}")
        s.release()


@pytest.mark.gpu
@pytest.mark.parametrize("env", [{"CMOLCU_ATTN_LIST": "1"}, {"CMOLCU_ATTN_DECODE": "0"}],
                         ids=["work_list", "split_items"])
@pytest.mark.parametrize("name", ["q4_k", "smollm3"])
def test_attention_work_list_launch(gpu, golden, paths, name, env):
    """The other decode attention launches, forced on every step in a fresh
    process: the work-list launch, and the per-split items (the path of
    head sizes and page sizes the streaming decode kernel does not take).
    Teacher-forced logits and greedy streams as the default gives them."""
    import subprocess
    import sys
    code = f"""
import numpy as np, sys
sys.path.insert(0, {os.path.dirname(GOLD)!r} + "/..")
from libcmol_b200.model import Model, GenParams
g = np.load({os.path.join(GOLD, "models.npz")!r})
with Model({paths[name]!r}, max_ctx=64, max_sessions=2, page_tokens=4) as m:
    s = m.acquire()
    for i, t in enumerate(g["{name}_tokens"]):
        got = s.forward_logits(int(t)); ref = g["{name}_logits"][i]
        assert float(np.abs(got - ref).max()) < 1e-3, i
    s.reset()
    rc, ids = s.generate_ids(g["{name}_tokens"][:6], GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=20))
    assert rc == 0 and ids == g["{name}_gen_greedy"].tolist(), ids
print("ok")
"""
    r = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, **env), capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["q4_k", "smollm3", "mixed", "q8_0"])
def test_wide_batch_uses_tensor_cores(gpu, paths, name):
    """32 sessions, each on its own random token sequence, advance together
    one token a step (32 columns: the tensor-core products at the default
    threshold).  Every column's logits are checked against the C
    restatement run on that session alone: max-abs <= 2e-2 and cosine >=
    0.9999, the engine's specified tolerance."""
    from libcmol_b200.model import Model
    from oracle.oracle import OracleModel
    NS, T = 32, 12
    rng = np.random.default_rng(21)
    seqs = rng.integers(0, 512, size=(NS, T)).astype(np.int32)
    om = OracleModel(paths[name], lanes=16)
    oss = [om.session(64) for _ in range(NS)]
    with Model(paths[name], max_ctx=64, max_sessions=NS) as m:
        ss = [m.acquire() for _ in range(NS)]
        worst, wcos = 0.0, 1.0
        for t in range(T):
            lg = m.forward_logits_batch(ss, seqs[:, t])
            for i in range(NS):
                ref = om.forward(oss[i], int(seqs[i, t]), t)
                d, c = float(np.abs(lg[i] - ref).max()), _cos(lg[i], ref)
                worst, wcos = max(worst, d), min(wcos, c)
                assert d <= ATOL and c >= COS, (t, i, d, c)
        print(f"{name}: 32-column steps, worst max-abs {worst:.2e} cos {wcos:.7f}")
        for s in ss:
            assert s.n_tokens == T
            s.release()
    for o in oss:
        om.free_session(o)


@pytest.mark.gpu
def test_wide_batch_generate(gpu, golden, paths):
    """Sixteen sessions generated together through cmol_generate_batch (their
    steps widen to the tensor-core threshold as the requests arrive): every
    stream has the requested length and starts with the reference's token;
    how many equal the reference's f32 stream throughout is reported, since
    a greedy decision within f16 rounding may differ.  The per-column
    numerics of wide steps are checked logit by logit in
    test_wide_batch_uses_tensor_cores."""
    from libcmol_b200.model import GenParams, Model
    name = "q4_k"
    with Model(paths[name], max_ctx=64, max_sessions=16) as m:
        ss = [m.acquire() for _ in range(16)]
        prompt = golden[f"{name}_tokens"][:6]
        p = GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=20)
        outs = m.generate_batch(ss, [prompt] * 16, [p] * 16)
        ref = golden[f"{name}_gen_greedy"].tolist()
        assert all(len(o) == len(ref) and o[0] == ref[0] for o in outs)
        same = sum(o.tolist() == ref for o in outs)
        print(f"wide batch: {same}/16 streams identical to the reference")
        st = m.stats(0)
        assert st.kernel_launches_per_step > 0
        for s in ss:
            s.release()


@pytest.mark.gpu
@pytest.mark.parametrize("name", MODELS)
@pytest.mark.parametrize("tag", ["greedy", "greedy_pen", "topp", "topk"])
def test_generate_matches_reference(gpu, golden, paths, name, tag):
    from libcmol_b200.model import Model
    with Model(paths[name], max_ctx=64, max_sessions=2) as m:
        s = m.acquire()
        rc, ids = s.generate_ids(golden[f"{name}_tokens"][:6], _params(tag))
        assert rc == 0
        assert ids == golden[f"{name}_gen_{tag}"].tolist()
        # the prompt and every sampled token but the last (EOS or max_new) are in the KV cache
        assert s.n_tokens == 6 + len(ids) - 1
        s.release()


@pytest.mark.gpu
def test_continuous_batching_equals_single(gpu, paths):
    from libcmol_b200.model import GenParams, Model
    prompts = [[5, 6, 7], [100, 200, 300, 400, 500, 7, 8], [42], [9, 8, 7, 6, 5, 4, 3, 2, 1, 0, 11]]
    params = [GenParams.make(0.0, max_new_tokens=12), GenParams.make(0.8, top_p=0.9, seed=5, max_new_tokens=9),
              GenParams.make(0.0, repeat_penalty=1.2, max_new_tokens=15), GenParams.make(1.0, top_k=3, seed=7,
                                                                                        max_new_tokens=10)]
    with Model(paths["q4_k"], max_ctx=64, max_sessions=4, page_tokens=4) as m:
        alone = []
        for p, pa in zip(prompts, params):
            s = m.acquire()
            rc, ids = s.generate_ids(p, pa)
            assert rc == 0
            alone.append(ids)
            s.release()
        sess = [m.acquire() for _ in prompts]
        together = m.generate_batch(sess, prompts, params)
        assert [t.tolist() for t in together] == alone
        for s in sess:
            s.release()


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["q8_0", "smollm3"])
def test_long_context_pages_and_splits(gpu, tmp_path, name):
    """300 tokens: many 16-token pages and three 128-token attention splits."""
    from libcmol_b200 import synth
    from libcmol_b200.model import Model
    from oracle.oracle import OracleModel
    kw = dict(MODEL_KW[name])
    dt = kw.pop("dtype")
    path = str(tmp_path / f"long_{name}.gguf")
    synth.write_gguf(path, synth.tiny_spec(dt, ctx=512, **kw))
    om = OracleModel(path, lanes=16)
    os_ = om.session(512)
    rng = np.random.default_rng(3)
    toks = rng.integers(0, 512, size=300)
    with Model(path, max_ctx=512, max_sessions=1) as m:
        s = m.acquire()
        for i, t in enumerate(toks):
            got = s.forward_logits(int(t))
            if i % 37 == 0 or i == len(toks) - 1:
                ref = om.forward(os_, int(t), i)
                assert np.abs(got - ref).max() <= ATOL and _cos(got, ref) >= COS, i
            else:
                om.forward(os_, int(t), i)
        s.release()
    om.free_session(os_)


@pytest.mark.gpu
@pytest.mark.parametrize("env", [{}, {"CMOLCU_ATTN_QB": "5"}, {"CMOLCU_ATTN_GROUP": "0"}],
                         ids=["leaders32", "leaders5", "per_column"])
@pytest.mark.parametrize("name", ["q8_0", "smollm3"])
def test_batched_prefill_long_prompts(gpu, tmp_path, monkeypatch, name, env):
    """Prompts of 300 and 170 tokens fed in chunks of up to 256 columns a step
    next to each other's columns: each chunk is one attention group whose
    block leaders (every 32 positions by default, 5 forced, or none) serve
    all its queries from one K / V load per split.  The greedy continuations
    equal the reference's for each prompt alone."""
    from libcmol_b200 import synth
    from libcmol_b200.model import GenParams, Model
    from oracle.oracle import GenParams as OGenParams
    from oracle.oracle import OracleModel
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    kw = dict(MODEL_KW[name])
    dt = kw.pop("dtype")
    path = str(tmp_path / f"prefill_{name}.gguf")
    synth.write_gguf(path, synth.tiny_spec(dt, ctx=512, **kw))
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, 512, size=300).astype(np.int32), rng.integers(0, 512, size=170).astype(np.int32)]
    om = OracleModel(path, lanes=16)
    want = []
    for pr in prompts:
        os_ = om.session(512)
        ids, _ = om.generate_ids(os_, pr, OGenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=8))
        want.append(ids.tolist())
        om.free_session(os_)
    with Model(path, max_ctx=512, max_sessions=2) as m:
        ss = [m.acquire() for _ in prompts]
        got = m.generate_batch(ss, prompts, [GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=8)] * 2)
        assert [g.tolist() for g in got] == want
        for s, pr, w in zip(ss, prompts, want):
            assert s.n_tokens == len(pr) + len(w) - 1
            s.release()


@pytest.mark.gpu
def test_stop_rules_and_session_state(gpu, paths):
    from libcmol_b200.model import GenParams, Model
    with Model(paths["q8_0"], max_ctx=32, max_sessions=2) as m:
        s = m.acquire()
        # max_new: generated tokens are forwarded except the last one
        rc, ids = s.generate_ids([5, 6, 7], GenParams.make(0.0, max_new_tokens=4))
        assert rc == 0 and len(ids) == 4 and s.n_tokens == 3 + 3
        # abort on the 2nd token: it is not forwarded, the call still returns OK
        s.reset()
        cnt = [0]

        def stop_second(t, e):
            cnt[0] += 1
            return 1 if cnt[0] >= 2 else 0

        rc, ids = s.generate_ids([5, 6, 7], GenParams.make(0.0, max_new_tokens=10), on_token=stop_second)
        assert rc == 0 and cnt[0] == 2
        assert s.n_tokens == 3 + 1
        # context full: the loop stops at max_ctx, the next call reports it
        s.reset()
        rc, ids = s.generate_ids(list(range(20)), GenParams.make(0.0, max_new_tokens=-1))
        assert rc == 0 and s.n_tokens == 32
        rc, ids = s.generate_ids([1], GenParams.make(0.0))
        assert rc == -7
        s.release()
        # pool: max_sessions slots, NULL when exhausted, fresh after release
        a, b = m.acquire(), m.acquire()
        assert a is not None and b is not None and m.acquire() is None
        a.release()
        c = m.acquire()
        assert c is not None and c.n_tokens == 0
        b.release()
        c.release()



@pytest.mark.gpu
def test_text_generate_and_tokenizer(gpu, paths):
    from libcmol_b200.model import GenParams, Model
    with Model(paths["q8_0"], max_ctx=64, max_sessions=1) as m:
        ids = m.encode("hello world")
        assert len(ids) > 0
        s = m.acquire()
        rc, pieces = s.generate("hello world", GenParams.make(0.0, max_new_tokens=5))
        assert rc == 0 and len(pieces) == 5
        s.release()
