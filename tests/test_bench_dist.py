"""The multi-GPU bench logic on CPU: two gloo ranks split the one seeded request set by modelled
device work (request-level data parallelism, no data exchanged): every request runs on exactly
one rank, the ranks' modelled work is balanced, and the whole-job rate is all ranks' sequences
over the slowest rank's time."""
import os
import sys
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = Path(__file__).resolve().parents[1]


def _rank(rank, world, port, out):
    sys.path[:0] = [str(ROOT), str(ROOT / "laya-cuda_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        items, stats = bench.rank_workload(rank, world, 64, 50368)
        keys = [tuple(item[0][:12]) + (len(item[0]),) for item in items]
        everyone = [None] * world
        dist.all_gather_object(everyone, keys)
        local_ms = 100.0 * (rank + 1)              # rank 1 is the slow one
        rate, ms_max, total = bench.job_rate(local_ms, len(items), 3, world, "cpu")
        out[rank] = (everyone, stats, rate, ms_max, total)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_request_shards():
    world, port = 2, 29611
    with mp.Manager() as manager:
        out = manager.dict()
        mp.spawn(_rank, args=(world, port, out), nprocs=world, join=True)
        results = dict(out)
    everyone, stats, rate, ms_max, total = results[0]
    assert results[1][0] == everyone and results[1][1] == stats      # the same partition on both ranks
    import bench
    all_items, _ = bench.rank_workload(0, 1, 64, 50368)
    want = sorted(tuple(item[0][:12]) + (len(item[0]),) for item in all_items)
    got = sorted(everyone[0] + everyone[1])
    assert got == want                                               # every sequence exactly once
    assert not set(everyone[0]) & set(everyone[1])
    assert stats["requests_per_rank"] and sum(stats["requests_per_rank"]) == 64
    assert stats["cost_imbalance"] < 1.02
    assert ms_max == 200.0 and total == 64 * 3
    assert rate == pytest.approx(64 * 3 * 3 / 0.2)
