"""Request-level data parallelism over the B200s of one host.

Requests are independent: no step of the forward pass combines two requests (the reference's
encoder schedule, runtime.py:90-113, and decision head, laya.py:214-245, work per packed row),
so N GPUs serve one request set with a full weight replica each and nothing exchanged between
them: no collective, no peer memory.  The only shared decision is which GPU runs which request,
and it decides the scaling: request lengths vary (256 to 1024 tokens in the throughput
configuration) and global-attention work grows with the square of the length, so equal request
counts per GPU leave the longest shard late.  `shard` balances the modelled device work instead.

`ShardedEngine` is the single-process form (one Engine per device, one host thread each; the
C ABI releases the GIL while a device call runs).  A multi-process launcher (one process per
GPU, as bench.py under torchrun) calls `shard` with the same inputs on every rank and takes its
own part; the partition is deterministic, so no rank has to tell another anything.
"""
import math
import threading
import time


def sequence_flops(tokens, width=768, layers=12, intermediate=3072, global_every=3, window=64):
    """Modelled device work of one packed sequence of `tokens` tokens: the encoder GEMMs
    (2 L d (4d + 3F) per token: QKV, attention output, GeGLU up and down) plus attention
    (4 d per visible query-key pair: all pairs on global layers, |i - j| <= window on the
    others).  The decision head and the per-row padding to 16 tokens are small next to these."""
    n = int(tokens)
    gemm = 2.0 * layers * width * (4 * width + 3 * intermediate) * n
    n_global = sum(1 for i in range(layers) if i % global_every == 0)
    w = min(window, max(n - 1, 0))
    # sum over q of (min(n, q + w + 1) - max(0, q - w)) = n (2w + 1) - w (w + 1)
    local_pairs = n * (2 * w + 1) - w * (w + 1)
    attention = 4.0 * width * (n_global * n * n + (layers - n_global) * local_pairs)
    return gemm + attention


def request_cost(items, **geometry):
    """Modelled work of one request: the sum over its question sequences (ids, markers, kind)."""
    return sum(sequence_flops(len(item[0]), **geometry) for item in items)


def shard(costs, n_shards):
    """Partition of request indices into `n_shards` lists with near-equal total cost.

    Longest-processing-time-first greedy: requests in decreasing cost (ties: lower index first)
    each go to the shard with the least cost so far (ties: lower shard).  Its makespan is within
    4/3 of the optimum, and with many requests far closer.  Deterministic; each shard lists its
    indices in increasing order."""
    if n_shards < 1:
        raise ValueError("n_shards must be positive")
    loads = [0.0] * n_shards
    parts = [[] for _ in range(n_shards)]
    for index in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        target = min(range(n_shards), key=lambda s: (loads[s], s))
        parts[target].append(index)
        loads[target] += costs[index]
    return [sorted(p) for p in parts]


def imbalance(costs, parts):
    """max / mean of the shards' total cost (1.0 is perfect balance)."""
    loads = [sum(costs[i] for i in p) for p in parts]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean > 0 else 1.0


def micro_batches(requests, limit):
    """Consecutive whole requests grouped into batches of at most `limit` sequences (a request
    with more questions than `limit` forms a batch of its own)."""
    batches, current, size = [], [], 0
    for index, items in requests:
        if current and size + len(items) > limit:
            batches.append(current)
            current, size = [], 0
        current.append((index, items))
        size += len(items)
    if current:
        batches.append(current)
    return batches


class ShardedEngine:
    """Engine replicas on several CUDA devices of this host, driven by one host thread each.

        with ShardedEngine("laya", devices=["cuda:0", "cuda:1"]) as engine:
            answers = engine.predict_batch([(state, questions), ...])

    `predict_batch` prepares every request (tokenised in parallel by the adapter's
    prepare_many, called on the calling thread), partitions them with `shard`
    by modelled work, and has each device's thread run its share as micro-batches of at most
    `micro_batch` packed sequences (two in flight per device), then decode.  Answers come back
    in request order; `last_metrics` reports each device's requests, sequences, tokens, GPU time
    and wall time, and the partition's cost imbalance.  Engine options (precision,
    max_cached_shapes, registry, revision) apply to every replica."""

    def __init__(self, model="laya", *, devices=("cuda:0",), micro_batch=64, **engine_options):
        from .engine import Engine
        if not devices:
            raise ValueError("at least one device")
        if type(micro_batch) is not int or micro_batch < 1:
            raise ValueError("micro_batch must be a positive integer")
        if engine_options.get("backend", "cuda") != "cuda":
            raise ValueError("ShardedEngine supports backend='cuda' only")
        self.micro_batch, self.devices, self.last_metrics = micro_batch, list(devices), {}
        self.engines = [None] * len(self.devices)
        errors = []

        def load(rank):
            try:
                self.engines[rank] = Engine(model, device=self.devices[rank], **engine_options)
            except BaseException as error:  # re-raised on the calling thread
                errors.append(error)
        self._each(load)
        if errors:
            self.close()
            raise errors[0]
        self.adapter = self.engines[0].adapter
        self.geometry = dict(width=self.adapter.width, layers=self.adapter.layers,
                             intermediate=self.adapter.intermediate, global_every=self.adapter.global_every,
                             window=self.adapter.window)

    def _each(self, work):
        threads = [threading.Thread(target=work, args=(rank,), name=f"laya-device-{rank}")
                   for rank in range(len(self.devices))]
        for thread in threads:
            thread.start()
        for thread in threads:
            thread.join()

    def predict_batch(self, requests):
        if any(engine is None or engine.closed for engine in self.engines):
            raise RuntimeError("Engine is closed")
        started = time.perf_counter()
        prepared = self._prepare(requests)
        costs = [request_cost(items, **self.geometry) for items in prepared]
        parts = shard(costs, len(self.engines))
        answers, per_device, errors = [None] * len(requests), [None] * len(self.engines), []

        def run(rank):
            try:
                engine, mine = self.engines[rank], parts[rank]
                t0 = time.perf_counter()
                batches = micro_batches([(i, prepared[i]) for i in mine], self.micro_batch)
                flat = [[item for _, items in batch for item in items] for batch in batches]
                results = engine.runtime.predict_many(flat) if flat else []
                gpu_ms = 0.0
                for batch, (logits, acts, metrics) in zip(batches, results):
                    gpu_ms += metrics["gpu_ms"]
                    offset = 0
                    for index, items in batch:
                        end = offset + len(items)
                        questions = requests[index][1]
                        answers[index] = engine.adapter.decode(logits[offset:end], acts[offset:end], questions, items)
                        offset = end
                per_device[rank] = {"device": self.devices[rank], "requests": len(mine),
                                    "sequences": sum(len(prepared[i]) for i in mine),
                                    "tokens": sum(len(item[0]) for i in mine for item in prepared[i]),
                                    "micro_batches": len(batches), "gpu_ms": gpu_ms,
                                    "wall_ms": (time.perf_counter() - t0) * 1000}
            except BaseException as error:
                errors.append(error)
        self._each(run)
        if errors:
            raise errors[0]
        self.last_metrics = {"devices": per_device, "imbalance": imbalance(costs, parts),
                             "api_ms": (time.perf_counter() - started) * 1000}
        return answers

    def _prepare(self, requests):
        """Every request's items (the first failing request's error is raised, as a loop over
        prepare() would); the adapter's prepare_many encodes them in parallel when it has one."""
        many = getattr(self.adapter, "prepare_many", None)
        if many is None or len(requests) < 2:
            return [self.adapter.prepare(state, questions) for state, questions in requests]
        prepared = many(list(requests))
        for items in prepared:
            if isinstance(items, Exception):
                raise items
        return prepared

    def close(self):
        for engine in self.engines:
            if engine is not None:
                engine.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def expected_speedup(costs, n_shards):
    """The speed-up over one device that the partition allows if device time is proportional to
    the modelled cost: total cost / the largest shard's cost."""
    parts = shard(costs, n_shards)
    loads = [sum(costs[i] for i in p) for p in parts]
    return sum(costs) / max(loads) if max(loads) > 0 else math.inf
