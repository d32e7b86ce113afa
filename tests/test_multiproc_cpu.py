"""Host-side multi-GPU plumbing of bench.py on CPU: two gloo ranks shard the frames without
overlap or gaps and agree on the max-over-ranks step time (the only exchange)."""
import importlib.util
import os
import socket

import torch.multiprocessing as mp

from conftest import ROOT


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", init_method="env://")
    b = _bench()
    lo, hi = b.shard(32 * world, world, rank)
    t = b.max_over_ranks(float(rank + 1) * 1.5, world)
    b.barrier(world)
    q.put((rank, lo, hi, t, b.dist_env()))
    dist.destroy_process_group()


def test_shards_and_max_over_two_gloo_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, lo0, hi0, t0, e0), (r1, lo1, hi1, t1, e1) = res
    assert (lo0, hi0, lo1, hi1) == (0, 32, 32, 64)
    assert t0 == t1 == 3.0
    assert e0 == (0, 2, 0) and e1 == (1, 2, 1)


def test_shard_uneven():
    b = _bench()
    got = [b.shard(10, 4, r) for r in range(4)]
    assert got == [(0, 3), (3, 6), (6, 8), (8, 10)]
