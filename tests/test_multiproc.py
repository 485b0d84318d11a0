"""The N > 1 host logic of bench.py on CPU: two `gloo` ranks exchange their
timings the way the GPU replicas do (the slowest rank's time is everyone's,
throughput counts every rank's tokens)."""
import os
import sys
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")
mp = pytest.importorskip("torch.multiprocessing")

ROOT = Path(__file__).resolve().parent.parent


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    import bench

    dist = bench.dist_init(world, rank, backend="gloo")
    try:
        ms = 100.0 + 50.0 * rank  # rank 1 is the slow one
        m = bench.max_over_ranks(dist, ms)
        v = bench.replica_tok_s(world, 256 * 3, m)
        dist.barrier()
        q.put((rank, m, v))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_take_the_slowest_time():
    world, port = 2, 29531
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, m, v in res:
        assert m == 150.0
        assert abs(v - 2 * 768 / 0.150) < 1e-6


def test_single_rank_needs_no_process_group():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.dist_init(1, 0) is None
    assert bench.max_over_ranks(None, 7.5) == 7.5
    assert bench.replica_tok_s(1, 256, 170.0) == pytest.approx(256 / 0.17)
