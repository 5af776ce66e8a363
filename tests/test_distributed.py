"""The N>1 host path on the CPU: two gloo ranks through bench.py's rank setup, barrier
and reductions (max of the per-rank device time, sum of tokens). The data path itself
has no collective: each rank is an independent replica."""
import os
import socket

import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(world),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist

    import bench

    w, r, local = bench.dist_setup(world)
    dev = torch.device("cpu")
    bench.barrier(w, dev)
    mx = bench.reduce(10.0 + r, "max", w, dev)
    sm = bench.reduce(100 * (r + 1), "sum", w, dev)
    q.put((r, w, mx, sm))
    dist.destroy_process_group()


def test_two_gloo_ranks_reduce_like_the_bench():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert [x[0] for x in res] == [0, 1] and all(x[1] == 2 for x in res)
    assert all(x[2] == 11.0 for x in res)  # max over ranks
    assert all(x[3] == 300 for x in res)  # sum over ranks


def _bcast_rank(rank, world, port, q):
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(world),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist

    from dan_b200.loader import broadcast_state

    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(7)
    want = {"a.weight": torch.randn(300, 70, generator=g).bfloat16(), "b.bias": torch.randn(17, generator=g),
            "c.A_log": torch.rand(5, generator=g), "d.ids": torch.arange(11, dtype=torch.int64)}
    got = broadcast_state(want if rank == 0 else None, "cpu", bucket_bytes=10_000)  # several buckets
    ok = set(got) == set(want) and all(got[k].dtype == want[k].dtype and torch.equal(got[k], want[k]) for k in want)
    q.put((rank, ok))
    dist.destroy_process_group()


def test_weight_broadcast_from_rank_zero():
    """Startup weight distribution for replicas: rank 0's state dict reaches every rank bit for bit
    (names, shapes, dtypes, several buckets), gloo on the CPU here, NCCL on GPUs."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_bcast_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert res == [(0, True), (1, True)]
