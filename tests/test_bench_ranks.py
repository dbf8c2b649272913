"""The multi-GPU bookkeeping of bench.py on CPU: two gloo ranks reduce their
numbers the way the GPU ranks do (tokens summed, device time = the slowest
rank), and config 4's sessions are partitioned over the ranks."""
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        sums, maxes = bench.reduce_ranks(dist, "cpu", sums=(100 * (rank + 1), 7), maxes=(10.0 + rank, 3.0 - rank))
        q.put((rank, sums, maxes, bench.sessions_per_rank(256, world, rank), bench.sessions_per_rank(5, world, rank)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_like_the_gpu_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, sums, maxes, s256, s5 in got:
        assert sums == [300.0, 14.0]            # tokens add up over the GPUs
        assert maxes == [11.0, 3.0]             # time: the slowest rank
        assert s256 == 128
        assert s5 == (3 if rank == 0 else 2)


def test_single_rank_is_identity():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.reduce_ranks(None, "cpu", sums=(1, 2), maxes=(3,)) == ([1.0, 2.0], [3.0])
    assert sum(bench.sessions_per_rank(256, 8, r) for r in range(8)) == 256
    assert sum(bench.sessions_per_rank(255, 8, r) for r in range(8)) == 255


@pytest.mark.parametrize("workload", ["c3", "c4"])
@pytest.mark.parametrize("scale", [1.0, 0.25])
def test_ranks_share_one_model_file(workload, scale):
    """Every rank of a config 3 / 4 run opens the model file rank 0 wrote:
    the synthetic spec (and so the file name) must not depend on the rank's
    own draw of prompt lengths, and its context covers every rank's."""
    import types
    sys.path.insert(0, ROOT)
    import bench
    args = types.SimpleNamespace(workload=workload, sessions=0, prompt_scale=scale)
    for world in (2, 8):
        plans = [bench.batched_plan(args, r, world) for r in range(world)]
        paths = {bench.model_path(p[4]) for p in plans}
        assert len(paths) == 1, paths
        assert all(p[4].ctx >= p[3] for p in plans)
