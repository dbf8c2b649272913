"""The in-process multi-GPU path of the public API, on one GPU.

cmol_cuda_set_devices([0, 0]) gives the model two engines (two batchers,
streams, KV pools and slot tables) on the same device, which exercises what
a list of GPUs exercises: each GPU's share of max_sessions, placement at
acquire, per-GPU page pools and slots, release back to the right GPU.

Placement (the survey's multi-GPU row): a new session goes to the GPU with
the least outstanding work, tokens held in its sessions' KV caches plus tokens
its requests still have to run, among GPUs with a free slot.
"""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def model_path(tmp_path_factory):
    from libcmol_b200 import synth
    p = str(tmp_path_factory.mktemp("multi") / "m.gguf")
    synth.write_gguf(p, synth.tiny_spec(synth.Q4_K, ctx=512))
    return p


@pytest.fixture(autouse=True)
def default_devices_after():
    """The device list holds for every later cmol_load of the process:
    put the default (CMOL_CUDA_DEVICES, else device 0) back afterwards."""
    yield
    from libcmol_b200.model import api
    api().cmol_cuda_set_devices(None, 0)


def _greedy(n):
    from libcmol_b200.model import GenParams
    return GenParams.make(0.0, repeat_penalty=1.0, max_new_tokens=n)


@pytest.mark.gpu
def test_two_engines_share_sessions_and_match_one(gpu, model_path):
    from libcmol_b200.model import Model
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, 512, size=int(n)).astype(np.int32) for n in (5, 40, 17, 90)]
    with Model(model_path, max_ctx=256, max_sessions=4, devices=[0]) as m:
        want = []
        for p in prompts:
            s = m.acquire()
            rc, ids = s.generate_ids(p, _greedy(10))
            assert rc == 0
            want.append(ids)
            s.release()
    with Model(model_path, max_ctx=256, max_sessions=4, devices=[0, 0]) as m:
        assert m.n_gpus == 2
        ss = [m.acquire() for _ in range(4)]
        # each GPU holds its share (2) of max_sessions; ties go alternately
        assert [s.device for s in ss] == [0, 1, 0, 1]
        assert m.acquire() is None
        got = m.generate_batch(ss, prompts, [_greedy(10)] * 4)
        assert [g.tolist() for g in got] == want
        for s in ss:
            s.release()


@pytest.mark.gpu
def test_placement_follows_outstanding_work(gpu, model_path):
    from libcmol_b200.model import Model
    rng = np.random.default_rng(5)
    with Model(model_path, max_ctx=256, max_sessions=4, devices=[0, 0]) as m:
        a = m.acquire()
        assert a.device == 0
        rc, _ = a.generate_ids(rng.integers(0, 512, size=200).astype(np.int32), _greedy(1))
        assert rc == 0 and a.n_tokens == 200     # GPU 0 now holds 200 tokens of KV
        b = m.acquire()
        assert b.device == 1
        rc, _ = b.generate_ids(rng.integers(0, 512, size=10).astype(np.int32), _greedy(1))
        assert rc == 0
        # one session on each GPU: the next goes where less work is outstanding
        c = m.acquire()
        assert c.device == 1
        # GPU 1 has no free slot left (2 of 4): the next goes to GPU 0
        d = m.acquire()
        assert d.device == 0
        for s in (a, b, c, d):
            s.release()
        # released sessions give their slots and load back
        e = m.acquire()
        assert e.device == 0 and e.n_tokens == 0
        e.release()
