"""The multi-GPU bench logic on CPU: two gloo ranks, each with its own seeded workload
(request-level data parallelism, no data exchanged), and the whole-job rate as all ranks'
sequences over the slowest rank's time."""
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
        items = bench.rank_workload(rank, 8, 50368)
        local_ms = 100.0 * (rank + 1)              # rank 1 is the slow one
        rate, ms_max, total = bench.job_rate(local_ms, len(items), 3, world, "cpu")
        out[rank] = (len(items), sum(len(i[0]) for i in items), rate, ms_max, total, items[0][0][:8])
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_weak_scaling_rate():
    world, port = 2, 29611
    with mp.Manager() as manager:
        out = manager.dict()
        mp.spawn(_rank, args=(world, port, out), nprocs=world, join=True)
        results = dict(out)
    (n0, t0, r0, m0, tot0, head0), (n1, t1, r1, m1, tot1, head1) = results[0], results[1]
    assert n0 == n1 == 8 * 3                       # 8 requests x 3 questions per rank
    assert head0 != head1                          # independent per-rank request sets
    assert m0 == m1 == 200.0 and tot0 == tot1 == 48
    assert r0 == r1 == pytest.approx(48 * 3 / 0.2)
