"""Request sharding across GPUs (laya_cuda/sharding.py), on the host: the partition covers every
request once, balances the modelled work of the throughput configuration, and ShardedEngine
runs each device's share on its own thread and returns answers in request order."""
import threading

import numpy as np
import pytest

from laya_cuda import sharding
from laya_cuda import synthetic as S


def config5_costs(count=4096):
    reqs = S.throughput_requests(1000, count, 50368, (256, 1024), 3, 8)
    return [sharding.request_cost(r) for r in reqs], reqs


def test_sequence_flops_matches_the_bench_accounting():
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench
    arch = S.architecture("laya", max_len=1024)
    lengths = [1, 5, 64, 65, 129, 300, 1024]
    per_token = sum(bench.per_token_flops(arch).values())
    want = bench.attention_flops(lengths, arch) + per_token * sum(lengths)
    assert sum(sharding.sequence_flops(n) for n in lengths) == pytest.approx(want, rel=1e-12)


@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
def test_shard_covers_every_request_once_and_balances(n):
    costs, _ = config5_costs()
    parts = sharding.shard(costs, n)
    assert len(parts) == n
    flat = sorted(i for p in parts for i in p)
    assert flat == list(range(len(costs)))
    assert all(p == sorted(p) for p in parts)
    assert sharding.imbalance(costs, parts) < 1.001
    assert sharding.shard(costs, n) == parts                         # deterministic
    # Equal request counts would leave the longest shard late: the count split is worse.
    if n > 1:
        counts = [list(range(r, len(costs), n)) for r in range(n)]
        assert sharding.imbalance(costs, counts) > sharding.imbalance(costs, parts)


def test_shard_edge_cases():
    assert sharding.shard([], 3) == [[], [], []]
    assert sharding.shard([5.0], 3) == [[0], [], []]
    assert sharding.shard([1.0, 1.0, 1.0, 1.0], 2) == [[0, 2], [1, 3]]
    with pytest.raises(ValueError):
        sharding.shard([1.0], 0)


def test_micro_batches_keep_requests_whole():
    reqs = [(i, [None] * k) for i, k in enumerate([3, 3, 2, 70, 1, 3])]
    batches = sharding.micro_batches(reqs, 8)
    assert [[i for i, _ in b] for b in batches] == [[0, 1, 2], [3], [4, 5]]


class FakeRuntime:
    def __init__(self, device):
        self.device, self.calls = device, []

    def predict_many(self, batches):
        self.calls.append((threading.current_thread().name, [len(b) for b in batches]))
        out = []
        for items in batches:
            logits = np.array([[float(len(item[0])), self.device] for item in items], np.float32)
            out.append((logits, np.zeros((len(items), 2), np.float32), {"gpu_ms": 1.0}))
        return out


class FakeAdapter:
    width, layers, intermediate, global_every, window = 768, 12, 3072, 3, 64

    def prepare(self, state, questions):
        return [([0] * (len(state) + q), [1], 0) for q in range(questions)]

    def decode(self, logits, acts, questions, items):
        return {"tokens": [int(v) for v in logits[:, 0]], "device": int(logits[0, 1])}


class FakeEngine:
    def __init__(self, model, device, **options):
        self.device, self.closed = device, False
        self.runtime = FakeRuntime(int(device.split(":")[1]))
        self.adapter = FakeAdapter()

    def close(self):
        self.closed = True


def test_sharded_engine_routes_requests_and_keeps_order(monkeypatch):
    import laya_cuda.engine
    monkeypatch.setattr(laya_cuda.engine, "Engine", FakeEngine)
    rng = np.random.default_rng(0)
    requests = [("x" * int(rng.integers(200, 1000)), int(rng.integers(1, 4))) for _ in range(40)]
    with sharding.ShardedEngine("m", devices=["cuda:0", "cuda:1", "cuda:2"], micro_batch=8) as engine:
        answers = engine.predict_batch(requests)
        metrics = engine.last_metrics
        calls = [e.runtime.calls for e in engine.engines]
    for (state, q), answer in zip(requests, answers):
        assert answer["tokens"] == [len(state) + i for i in range(q)]
    assert sum(d["requests"] for d in metrics["devices"]) == 40
    assert {a["device"] for a in answers} == {0, 1, 2}
    assert metrics["imbalance"] < 1.1
    for rank, c in enumerate(calls):
        assert c and c[0][0] == f"laya-device-{rank}" and max(c[0][1]) <= 8
    assert all(e.closed for e in engine.engines)


def test_sharded_engine_prepares_through_prepare_many(monkeypatch):
    """With an adapter that has prepare_many, a batch of requests is prepared in one call (the
    tokenizer runs in parallel there); the first failing request's error is raised, as a loop
    over prepare() would raise it."""
    import laya_cuda.engine
    calls = []

    class ManyAdapter(FakeAdapter):
        def prepare_many(self, requests):
            calls.append(len(requests))
            return [ValueError(f"bad {i}") if state == "bad" else self.prepare(state, q)
                    for i, (state, q) in enumerate(requests)]

    class ManyEngine(FakeEngine):
        def __init__(self, model, device, **options):
            super().__init__(model, device, **options)
            self.adapter = ManyAdapter()

    monkeypatch.setattr(laya_cuda.engine, "Engine", ManyEngine)
    requests = [("x" * (100 + i), 1 + i % 3) for i in range(10)]
    with sharding.ShardedEngine("m", devices=["cuda:0", "cuda:1"]) as engine:
        answers = engine.predict_batch(requests)
        assert calls == [10]
        assert [a["tokens"] for a in answers] == [[len(s) + i for i in range(q)] for s, q in requests]
        with pytest.raises(ValueError, match="bad 3"):
            engine.predict_batch(requests[:3] + [("bad", 1), ("bad", 1)])
