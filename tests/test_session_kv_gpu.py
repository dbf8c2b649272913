"""Session KV snapshots (cmol_cuda_session_save / _restore): multi-turn reuse.

A session runs the first half of a token sequence; its snapshot is restored
into another session (on the model's second engine, and back into the first
session after a reset): the logits of the second half are bit-identical to
the original session's, with f32 and with f16 KV.  Snapshots of another KV
format or page size are refused, and a short buffer is reported.
"""
import ctypes as C
import importlib.util
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CMOL_ERR_INVALID, CMOL_ERR_TRUNC = -3, -8


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLD, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg.gguf_path("q8_0", str(tmp_path_factory.mktemp("snap")))


@pytest.fixture(autouse=True)
def default_devices_after():
    yield
    from libcmol_b200.model import api
    api().cmol_cuda_set_devices(None, 0)


def _tokens():
    g = np.load(os.path.join(GOLD, "models.npz"))
    return [int(t) for t in g["q8_0_tokens"]]


@pytest.mark.gpu
@pytest.mark.parametrize("kv", [0, 1], ids=["f32", "f16"])
def test_snapshot_restores_context(gpu, tiny, kv):
    from libcmol_b200.model import Model
    toks = _tokens()
    k = len(toks) // 2
    with Model(tiny, max_ctx=64, max_sessions=4, devices=[0, 0], kv_dtype=kv) as m:
        a = m.acquire()
        for t in toks[:k]:
            a.forward_logits(t)
        snap = a.save()
        assert a.n_tokens == k
        want = [a.forward_logits(t) for t in toks[k:]]
        b = m.acquire()
        assert b.device != a.device            # the model's second engine
        b.restore(snap)
        assert b.n_tokens == k
        got = [b.forward_logits(t) for t in toks[k:]]
        assert all(np.array_equal(x, y) for x, y in zip(got, want))
        # back into a session that holds pages of its own
        a.reset()
        a.restore(snap)
        again = [a.forward_logits(t) for t in toks[k:]]
        assert all(np.array_equal(x, y) for x, y in zip(again, want))
        a.release()
        b.release()


@pytest.mark.gpu
def test_snapshot_refuses_other_shapes(gpu, tiny):
    from libcmol_b200.model import Model, api
    toks = _tokens()
    with Model(tiny, max_ctx=64, max_sessions=2) as m:
        a = m.acquire()
        for t in toks[:5]:
            a.forward_logits(t)
        snap = a.save()
        n = C.c_size_t(0)
        buf = C.create_string_buffer(len(snap) - 1)
        assert api().cmol_cuda_session_save(a.h, buf, len(snap) - 1, C.byref(n)) == CMOL_ERR_TRUNC
        assert n.value == len(snap)
        a.release()
    for kw in (dict(kv_dtype=1), dict(page_tokens=16)):
        with Model(tiny, max_ctx=64, max_sessions=2, **kw) as m:
            b = m.acquire()
            assert api().cmol_cuda_session_restore(b.h, snap, len(snap)) == CMOL_ERR_INVALID
            assert b.n_tokens == 0
            b.release()
