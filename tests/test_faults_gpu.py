"""The device fault word, exercised without faulting the GPU.

cmol_cuda_debug_inject plants an error in the next decode step that the
kernels' own bounds checks catch: a token id past the vocabulary (the
embedding read is skipped, code 3), a page-table update naming a page
outside the pool (the table write is skipped, code 4), or a wait on a
barrier that nothing arrives on, which runs out after its bound (code 7):
the path every lost arrival takes.  The step must fail
with CMOL_ERR_INVALID carrying the code (the reference's generate loop
returns CMOL_ERR_INVALID when a forward fails, src/api.c:454,520), and the
next request on the same session pool must be served correctly.
"""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CMOL_ERR_INVALID = -3


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg.gguf_path("q8_0", str(tmp_path_factory.mktemp("faults")))


@pytest.mark.gpu
@pytest.mark.parametrize("kind,code", [(1, 3), (2, 4), (3, 7)], ids=["bad_token", "bad_page", "wait_runs_out"])
def test_planted_fault_fails_step_then_recovers(gpu, tiny, kind, code):
    from libcmol_b200.model import GenParams, Model
    g = np.load(os.path.join(GOLD, "models.npz"))
    prompt, want = g["q8_0_tokens"][:6], g["q8_0_gen_greedy"].tolist()
    p = GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=20)
    with Model(tiny, max_ctx=64, max_sessions=2) as m:
        s = m.acquire()
        assert m.stats(0).last_fault_code == 0
        m.debug_inject(kind)
        rc, ids = s.generate_ids(prompt, p)
        assert rc == CMOL_ERR_INVALID, rc
        assert m.stats(0).last_fault_code == code
        # the pool and the session stay usable: a fresh request is served exactly
        s.reset()
        rc, ids = s.generate_ids(prompt, p)
        assert rc == 0 and ids == want
        t = m.acquire()
        rc, ids = t.generate_ids(prompt, p)
        assert rc == 0 and ids == want
        t.release()
        s.release()


@pytest.mark.gpu
def test_planted_fault_in_a_shared_step(gpu, tiny):
    """A failed step fails every request in it; requests that come after it
    run normally."""
    from libcmol_b200.model import GenParams, Model
    g = np.load(os.path.join(GOLD, "models.npz"))
    want = g["q8_0_gen_greedy"].tolist()
    with Model(tiny, max_ctx=64, max_sessions=4) as m:
        ss = [m.acquire() for _ in range(2)]
        toks = g["q8_0_tokens"]
        m.debug_inject(1)
        with pytest.raises(Exception):
            m.forward_logits_batch(ss, [int(toks[0]), int(toks[1])])
        assert m.stats(0).last_fault_code == 3
        for s in ss:
            s.reset()
        outs = m.generate_batch(ss, [toks[:6]] * 2, [GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=20)] * 2)
        assert [o.tolist() for o in outs] == [want, want]
        for s in ss:
            s.release()
