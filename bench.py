"""Benchmark of the Laya forward pass on B200 (one JSON line on rank 0).

Workload (one "step"): configuration 5 of the benchmark plan -- the `laya` encoder geometry
(12 layers, d 768, 12 heads, F 3072, vocab 50368) with positions extended to 1024, 4096
requests of uniform length in [256, 1024], 3 questions x 8 options each (12,288 packed
sequences), run as micro-batches of 64 sequences.  Under torchrun the one 4096-request set is
split across the ranks by modelled device work (laya_cuda.sharding.shard, the same partition on
every rank: strong scaling); each rank runs its share on its own weight replica and nothing is
exchanged between ranks (the NCCL group only carries the timing barrier and the max-reduction).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--latency none|basic]

metric: sequences/s over all ranks (device time, max over ranks).  Extra keys: batch-1 latency
(configs 1/2: 83 and 512 tokens through Engine.predict), per-kernel-family device times, the
roofline of the dominant kernel (FFN-up GEMM), the oracle on the host cores (cpu_baseline),
and the end-to-end number through the public Runtime.predict_many with host buffers (e2e).
"""
import argparse
import ctypes as ct
import json
import os
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "laya-cuda_b200"))

REQUESTS = 4096
QUESTIONS = 3
OPTIONS = 8
MICRO = 64
LENGTHS = (256, 1024)
FAMILIES = ["gemm_qkv_rope", "gemm_attn_out_residual", "gemm_ffn_up_geglu", "gemm_ffn_down_residual",
            "gemm_head", "attention", "row_kernels", "head_tail"]
CACHE = Path(os.environ.get("LAYA_BENCH_CACHE", Path(tempfile.gettempdir()) / "laya_b200_bench"))


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return data["hbm_gbs"], data["bf16_tflops"], data["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def per_token_flops(arch):
    """Encoder GEMM FLOPs per useful token: 2 * L * d * (3d + d + 2F + F)."""
    d, f, layers = arch["width"], arch["intermediate"], arch["layers"]
    return {"qkv": 2 * layers * d * 3 * d, "attn_out": 2 * layers * d * d, "ffn_up": 2 * layers * d * 2 * f,
            "ffn_down": 2 * layers * f * d}


def attention_flops(lengths, arch):
    """4 * d * sum over queries of visible keys, per layer (global: all keys; local: |i-j|<=w)."""
    d, w = arch["width"], arch["local_attention"] // 2
    n_global = sum(1 for layer in range(arch["layers"]) if layer % arch["global_every"] == 0)
    total = 0
    for n in lengths:
        q = np.arange(n)
        local = int((np.minimum(n, q + w + 1) - np.maximum(0, q - w)).sum())
        total += 4 * d * (n_global * n * n + (arch["layers"] - n_global) * local)
    return total


class Clocks:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    def __init__(self, index):
        self.index, self.samples, self.proc = index, [], None

    def __enter__(self):
        query = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={query}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([v.strip() for v in line.split(",")])

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        rows = [s for s in self.samples if len(s) >= 9 and s[1].isdigit()]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = sorted(int(r[1]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": int(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def rank_workload(rank, world, requests, vocab):
    """This rank's sequences: its share of the one seeded request set, partitioned across the
    `world` ranks by modelled device work (strong scaling: the job's work is fixed).  Every rank
    computes the same partition.  Returns (items, partition statistics)."""
    from laya_cuda import synthetic as S
    from laya_cuda.sharding import imbalance, request_cost, shard
    reqs = S.throughput_requests(1000, requests, vocab, LENGTHS, QUESTIONS, OPTIONS)
    costs = [request_cost(r) for r in reqs]
    parts = shard(costs, world)
    items = [item for i in parts[rank] for item in reqs[i]]
    stats = {"requests_per_rank": [len(p) for p in parts],
             "tokens_per_rank": [sum(len(it[0]) for i in p for it in reqs[i]) for p in parts],
             "cost_imbalance": round(imbalance(costs, parts), 5)}
    return items, stats


def job_rate(local_ms, local_sequences, steps, world, device):
    """Whole-job sequences/s: all ranks' sequences over the slowest rank's device time.
    Returns (sequences_per_second, max_ms, total_sequences_per_step)."""
    import torch
    t = torch.tensor([local_ms], dtype=torch.float64, device=device)
    n = torch.tensor([local_sequences], dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(n, op=dist.ReduceOp.SUM)
    ms_max, total = float(t.item()), float(n.item())
    return total * steps / (ms_max / 1000), ms_max, total


def build_micro_batches(items):
    batches = [items[i:i + MICRO] for i in range(0, len(items), MICRO)]
    return batches


def oracle_rate(arch, weights, items, budget_s):
    """Sequences/s of the FP32 oracle on the host cores over a bounded sample of the workload."""
    sys.path.insert(0, str(ROOT))
    from oracle.laya_oracle import Oracle
    oracle = Oracle(weights, arch)
    oracle.item(*items[0])  # warm caches
    done, t0 = 0, time.perf_counter()
    while done < len(items) and (time.perf_counter() - t0 < budget_s or done == 0):
        oracle.item(*items[done])
        done += 1
    return done / (time.perf_counter() - t0), done


def oracle_answer(adapter, oracle, state, questions):
    """The answer dict of one request with the FP32 oracle as the forward pass: the adapter's
    request contract and decoding around the CPU restatement."""
    items = adapter.prepare(state, questions)
    outs = [oracle.item(*item) for item in items]
    logits = np.zeros((len(items), max(len(item[1]) for item in items)), np.float32)
    for i, (option_logits, _) in enumerate(outs):
        logits[i, :len(option_logits)] = option_logits
    return adapter.decode(logits, np.stack([acts for _, acts in outs]).astype(np.float32), questions, items)


def cpu_checks(engine, arch, weights, repeats=30):
    """The cpu_baseline leg's other two parts, both with the FP32 oracle on the host cores:
    configuration 1 (batch 1, one 83-token question with 4 options: tokenise, forward, decode)
    as p50/p95 latency; and the reference's answer gates (laya_cuda.gates, benchmarks/run.py:23
    of the reference) between this engine and the oracle on the frozen request set."""
    from laya_cuda import gates
    from laya_cuda import synthetic as S
    sys.path.insert(0, str(ROOT))
    from oracle.laya_oracle import Oracle
    oracle = Oracle(weights, arch)
    state, questions, _ = S.request_texts(np.random.default_rng(0), 83, 4, arch["vocab"])
    times = []
    for i in range(repeats + 3):
        t0 = time.perf_counter()
        oracle_answer(engine.adapter, oracle, state, questions)
        if i >= 3:
            times.append((time.perf_counter() - t0) * 1000)
    config1 = {"p50_ms": round(float(np.percentile(times, 50)), 2), "p95_ms": round(float(np.percentile(times, 95)), 2),
               "repeats": repeats, "cores": os.cpu_count(), "kind": "port",
               "sample": "83-token request, 1 question x 4 options, FP32 numpy oracle (all host threads)"}
    requests = list(gates.frozen_requests(engine.adapter))
    candidate = gates.answers(engine, requests)
    reference = [{"id": rid, "answers": oracle_answer(engine.adapter, oracle, st, qs)["answers"]}
                 for rid, st, qs in requests]
    stats = gates.compare(candidate, reference)
    gate = {"requests": len(requests), "reference": "FP32 oracle", "thresholds": gates.GATES,
            **{k: (round(v, 8) if isinstance(v, float) else v) for k, v in stats.items()}, "passed": gates.passes(stats)}
    return config1, gate


def run_reference(args, rank, world):
    """--impl reference: the CPU implementation of this path (the oracle restatement; the
    reference's own path needs CuPy and a GPU), timed on this host's cores."""
    if rank != 0:
        return
    from laya_cuda import synthetic as S
    arch = S.architecture("laya", max_len=1024)
    weights = S.make_weights(arch, seed=0)
    requests = S.throughput_requests(1000, 64, arch["vocab"], LENGTHS, QUESTIONS, OPTIONS)
    items = [item for req in requests for item in req]
    cores = os.cpu_count()
    sys.path.insert(0, str(ROOT))
    from oracle.laya_oracle import Oracle
    oracle = Oracle(weights, arch)
    t0 = time.perf_counter()
    oracle.item(*items[0])
    per_seq = time.perf_counter() - t0
    per_step = max(1, min(len(items), int(2.0 / max(per_seq, 1e-3))))
    cursor = 0

    def step():
        nonlocal cursor
        for _ in range(per_step):
            oracle.item(*items[cursor % len(items)])
            cursor += 1
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    elapsed = time.perf_counter() - t0
    value = args.steps * per_step / elapsed
    sample = f"{per_step} sequences per step (lengths 256-1024, 8 options) of the config-5 workload"
    line = {"impl": "reference", "metric": "sequences/s", "value": round(value, 3), "unit": "sequences/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(elapsed / args.steps * 1000, 2), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config5-throughput laya 12L d768 F3072 V50368 ctx1024, 3q x 8 options",
                       "sample": sample},
            "cpu_baseline": {"value": round(value, 3), "unit": "sequences/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "sequences/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference GPU path requires CuPy (absent); CPU FP32 restatement of it timed with numpy BLAS"}
    print(json.dumps(line), flush=True)


def run_attention_only(args):
    """--attention-only: the attention kernel alone (laya_op_attention, the forward pass's
    key-split rule) on the first 64 sequences of the config-5 workload, 12 heads, f16, random
    q/k/v: 5 untimed + 30 timed launches of a global layer, then of a window-64 layer (CUDA
    events on the launching stream).  The command of the attention profile captures."""
    import torch
    from laya_cuda import _lib
    from laya_cuda import synthetic as S
    from laya_cuda.runtime import span
    lib = _lib.load()
    reqs = S.throughput_requests(1000, 22, 50368, LENGTHS, QUESTIONS, OPTIONS)
    lengths = [len(item[0]) for req in reqs for item in req][:MICRO]
    starts = np.cumsum([0] + [span(n) for n in lengths])[:-1].astype(np.int32)
    rows = int(span(sum(span(n) for n in lengths)) // 128 * 128 + 128)
    heads = 12
    lens = np.asarray(lengths, np.int32)
    cap = (rows + (128 - 16) * len(lengths) + 127) // 128 + 1
    tiles = np.zeros((cap, 4), np.int32)
    n_tiles = lib.laya_attention_tiles(starts.ctypes.data, lens.ctypes.data, len(lengths), rows, 128,
                                       tiles.ctypes.data, cap)
    gen = torch.Generator(device="cuda").manual_seed(0)
    qkv = torch.randn(3 * heads * rows * 64, dtype=torch.float16, device="cuda", generator=gen)
    out = torch.empty(rows * heads * 64, dtype=torch.float16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    dev = [torch.from_numpy(v).cuda() for v in (tiles, starts, lens)]
    stream = torch.cuda.current_stream()

    def run(window):
        _lib.check(lib.laya_op_attention(_lib.PRECISION_F16, 1, ct.c_void_p(qkv.data_ptr()), ct.c_void_p(out.data_ptr()),
                                         ct.c_void_p(dev[0].data_ptr()), cap, ct.c_void_p(dev[1].data_ptr()),
                                         ct.c_void_p(dev[2].data_ptr()), rows, heads, window,
                                         ct.c_void_p(err.data_ptr()), ct.c_void_p(stream.cuda_stream)))
    result = {"tokens": int(sum(lengths)), "rows": rows, "tiles": n_tiles}
    for window in (-1, 64):
        for _ in range(5):
            run(window)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(30):
            run(window)
        b.record(stream)
        torch.cuda.synchronize()
        us = a.elapsed_time(b) / 30 * 1000
        useful = 0
        for n in lengths:
            q = np.arange(n)
            keys = n * n if window < 0 else int((np.minimum(n, q + window + 1) - np.maximum(0, q - window)).sum())
            useful += 4 * 64 * heads * keys
        result["global" if window < 0 else "window64"] = {"us": round(us, 1), "useful_tflops": round(useful / us / 1e6, 1)}
    if int(err.item()) != 0:
        raise RuntimeError(f"attention reported device error {int(err.item())}")
    print(json.dumps({"attention_only": result}), flush=True)


def run_cold_load(args):
    """--cold-load NAME: in this fresh process, the wall time of Engine(checkpoint) (CUDA
    context, library, tokenizer, weight load and finalize) and of the first request after it (a
    512-token question with 4 options: cold shape class, graph capture included).  The checkpoint
    file is written beforehand, so it is read from the page cache, not from disk."""
    from laya_cuda import synthetic as S
    name = args.cold_load
    overrides = {"max_len": 1024} if name == "laya" else {}
    arch = S.architecture(name, **overrides)
    CACHE.mkdir(parents=True, exist_ok=True)
    path = S.cached_checkpoint(CACHE, name, seed=0, **overrides)
    state, questions, _ = S.request_texts(np.random.default_rng(7), 512, 4, arch["vocab"])
    size = (path / "model.safetensors").stat().st_size
    t0 = time.perf_counter()
    from laya_cuda import Engine
    engine = Engine(path, device="cuda:0")
    t1 = time.perf_counter()
    engine.predict(state, questions)
    t2 = time.perf_counter()
    engine.predict(state, questions)
    t3 = time.perf_counter()
    engine.close()
    print(json.dumps({"model": name, "load_s": round(t1 - t0, 3), "first_request_ms": round((t2 - t1) * 1000, 2),
                      "second_request_ms": round((t3 - t2) * 1000, 3), "checkpoint_bytes": size}), flush=True)


def cold_loads(names, runs=3):
    """Cold Engine construction and first request per model, each in `runs` fresh processes
    (the first process on a box also pays one-time driver work): the median run by load time,
    with every run's load time."""
    out = {}
    for name in names:
        results = []
        for _ in range(runs):
            run = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--cold-load", name], capture_output=True,
                                 text=True, timeout=600)
            lines = [l for l in run.stdout.splitlines() if l.startswith("{")]
            if run.returncode != 0 or not lines:
                results = None
                out[name] = {"error": run.stderr[-300:]}
                break
            results.append(json.loads(lines[-1]))
        if results:
            results.sort(key=lambda r: r["load_s"])
            out[name] = {**results[len(results) // 2], "load_s_runs": [r["load_s"] for r in results]}
    return out


def percentiles(values):
    return {"p50_ms": round(float(np.percentile(values, 50)), 4), "p95_ms": round(float(np.percentile(values, 95)), 4)}


def run_latency_only(args):
    """--latency-only: configurations 1/2 (+1024 tokens) on the `laya` geometry through
    Engine.predict, nothing else (a small command for profiler captures of the batch-1 path)."""
    from laya_cuda import Engine
    from laya_cuda import synthetic as S
    arch = S.architecture("laya", max_len=1024)
    CACHE.mkdir(parents=True, exist_ok=True)
    path = S.cached_checkpoint(CACHE, "laya", seed=0, max_len=1024)
    lengths = tuple(int(v) for v in args.lengths.split(","))
    with Engine(path, device="cuda:0") as engine:
        lat = latency(engine, arch, np.random.default_rng(0), lengths, repeats=args.repeats,
                      warmup=max(3, min(20, args.repeats)), tag="laya_")
    print(json.dumps({"latency_batch1": lat}), flush=True)


def latency(engine, arch, rng, lengths, repeats=200, warmup=20, zipf=None, tag=""):
    """Batch-1 latency of Engine.predict(text) at the given sequence lengths (one question with
    4 options): p50/p95 of the API time and of the device time."""
    from laya_cuda import synthetic as S
    out = {}
    for n in lengths:
        state, questions, _ = S.request_texts(rng, n, 4, arch["vocab"], zipf=zipf)
        for _ in range(warmup):
            engine.predict(state, questions)
        api, gpu = [], []
        for _ in range(repeats):
            engine.predict(state, questions)
            api.append(engine.last_metrics["api_ms"])
            gpu.append(engine.last_metrics["gpu_ms"])
        out[f"{tag}{n}tok"] = {"api_p50_ms": round(float(np.percentile(api, 50)), 4),
                          "api_p95_ms": round(float(np.percentile(api, 95)), 4),
                          "gpu_p50_ms": round(float(np.percentile(gpu, 50)), 4),
                          "gpu_p95_ms": round(float(np.percentile(gpu, 95)), 4),
                          "repeats": repeats, "graph_replay": engine.last_metrics["graph_replay"]}
    return out


def stream_latency(path, arch, count=200, seed=2):
    """Configuration 4: a mixed-shape request stream through BatchEngine, one request at a time
    (per-request API latency, cold shape classes included)."""
    from laya_cuda import BatchEngine
    from laya_cuda import synthetic as S
    rng = np.random.default_rng(seed)
    requests = [S.stream_request_texts(rng, arch["vocab"]) for _ in range(count)]
    api, gpu, cold, tokens = [], [], 0, []
    with BatchEngine(path, max_batch_size=8, max_batch_tokens=8192, max_wait_ms=0) as engine:
        for state, questions in requests:
            future = engine.submit(state, questions)
            future.result(120)
            m = future.metrics
            api.append(m["api_ms"])
            gpu.append(m["gpu_ms"])
            cold += bool(m.get("graph_capture"))
            tokens.append(sum(m["tokens_per_question"]))
    return {"requests": count, "api": percentiles(api), "gpu": percentiles(gpu), "cold_captures": cold,
            "tokens_per_request_mean": round(float(np.mean(tokens)), 1)}


def api_throughput(path, arch, count=1024, seed=5):
    """Configuration-5-shaped requests as text (states of U[256,1024] words, 3 choice questions x 8
    options) through the user-facing BatchEngine: tokenisation, batching under 64 questions and
    64 x 1024 packed tokens, packing, H2D, forward, D2H and decoding into answer dicts, all
    inside the timed region (first submit to last answer).  The graphs of the shape classes are
    captured by an untimed pass over the same requests first."""
    from laya_cuda import BatchEngine
    from laya_cuda import synthetic as S
    rng = np.random.default_rng(seed)
    requests = [S.stream_request_texts(rng, arch["vocab"], lengths=LENGTHS, questions=(QUESTIONS, QUESTIONS),
                                       options=(OPTIONS, OPTIONS)) for _ in range(count)]
    with BatchEngine(path, max_batch_size=MICRO, max_batch_tokens=MICRO * 1024, max_pending=count,
                     max_wait_ms=1, max_cached_shapes=64) as engine:
        for _ in range(2):
            t0 = time.perf_counter()
            futures = [engine.submit(state, questions) for state, questions in requests]
            answers = [f.result(300) for f in futures]
            seconds = time.perf_counter() - t0
    questions = sum(len(a["answers"]) for a in answers)
    return {"value": round(questions / seconds, 2), "unit": "sequences/s", "requests": count, "sequences": questions,
            "api": "BatchEngine.submit(text) -> answer dicts (tokenise, batch, pack, H2D, forward, D2H, decode)"}


def run_engine(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from laya_cuda import Engine
    from laya_cuda import _lib
    from laya_cuda import synthetic as S

    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta
        # rank 0's stdout carries exactly one JSON line: keep NCCL's version banner off it.
        os.environ["NCCL_DEBUG"] = "WARN"
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local_rank))
    arch = S.architecture("laya", max_len=1024)
    CACHE.mkdir(parents=True, exist_ok=True)
    if rank == 0:
        path = S.cached_checkpoint(CACHE, "laya", seed=0, max_len=1024)
    if world > 1:
        dist.barrier()
    path = S.cached_checkpoint(CACHE, "laya", seed=0, max_len=1024)
    engine = Engine(path, device=f"cuda:{local_rank}", max_cached_shapes=16)
    rt, lib = engine.runtime, engine.runtime._lib
    h = rt._handle

    items, sharding = rank_workload(rank, world, args.requests, arch["vocab"])
    batches = build_micro_batches(items)
    tokens = sum(len(i[0]) for i in items)
    packed, shapes, maxes = [], [], [0, 0, 0]
    from laya_cuda.runtime import classes, flatten
    for batch in batches:
        m, b, k = classes(batch)
        toks, lens, marks, counts, kinds = flatten(batch)
        buf = np.zeros(lib.laya_packed_ints(m, b, k), np.int32)
        _lib.check(lib.laya_pack(toks.ctypes.data, lens.ctypes.data, marks.ctypes.data, counts.ctypes.data,
                                 kinds.ctypes.data, len(batch), 0, m, b, k, buf.ctypes.data))
        packed.append(torch.from_numpy(buf).cuda())
        shapes.append((m, b, k))
        maxes = [max(a, v) for a, v in zip(maxes, (m, b, k))]
    _lib.check(lib.laya_reserve(h, *maxes), h)
    out_logits = torch.empty((maxes[1] * (maxes[2] + 1),), dtype=torch.float32, device="cuda")
    out_acts = torch.empty((maxes[1] * arch["n_act"],), dtype=torch.float32, device="cuda")
    stream = torch.cuda.ExternalStream(lib.laya_stream(h))

    def step():
        for buf, (m, b, k) in zip(packed, shapes):
            _lib.check(lib.laya_forward_device(h, ct.c_void_p(buf.data_ptr()), m, b, k, 2,
                                               ct.c_void_p(out_logits.data_ptr()), ct.c_void_p(out_acts.data_ptr())), h)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # Timed region: inputs resident in HBM; the working set of a step (12,288 sequences, ~7.9M
    # tokens, >40 GB of activations streamed) is far larger than L2, so no flush is needed.
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local_rank) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    # Per-kernel-family breakdown from one further, untimed step with an event pair around every
    # launch (the events keep consecutive kernels from overlapping, so it is not part of `value`).
    _lib.check(lib.laya_set_profiling(h, 1), h)
    step()
    torch.cuda.synchronize()
    _lib.check(lib.laya_set_profiling(h, 0), h)
    fam = {}
    launches = 0
    for i, name in enumerate(FAMILIES):
        t, n, fl = ct.c_double(), ct.c_int64(), ct.c_double()
        _lib.check(lib.laya_profile_read(h, i, ct.byref(t), ct.byref(n), ct.byref(fl)), h)
        fam[name] = {"ms": round(t.value, 3), "launches": n.value, "share": None}
        launches += n.value
    busy = sum(v["ms"] for v in fam.values())
    for v in fam.values():
        v["share"] = round(v["ms"] / busy, 4) if busy else None
    value, ms_max, _ = job_rate(ms, len(items), args.steps, world, "cuda")

    # Roofline of the dominant kernel: the FFN-up GEMM (+GeGLU epilogue), algorithmic FLOPs of
    # useful tokens, per launch, over its event-timed average launch duration.
    hbm, tf_burst, tf_sust, peak_kind = peaks()
    ptf = per_token_flops(arch)
    up = fam["gemm_ffn_up_geglu"]
    up_launch_ms = up["ms"] / max(up["launches"], 1)
    up_flops_per_launch = tokens * ptf["ffn_up"] / arch["layers"] / len(batches)
    achieved = up_flops_per_launch / (up_launch_ms / 1000) / 1e12
    enc_gemm_ms = sum(fam[k]["ms"] for k in FAMILIES[:4])
    enc_achieved = tokens * sum(ptf.values()) / (enc_gemm_ms / 1000) / 1e12
    roofline = {"kernel": "gemm_ffn_up_geglu (tcgen05, M=128 N=256 tiles)", "bound": "tensor",
                "achieved": round(achieved, 1), "peak": tf_sust, "unit": "TFLOP/s",
                "frac": round(achieved / tf_sust, 4), "peak_kind": f"{peak_kind} bf16 dense sustained (f16 same rate)",
                "traffic": round(TRAFFIC_FFN_UP_BYTES_PER_TOKEN * tokens / len(batches)),
                "all_encoder_gemms": {"achieved": round(enc_achieved, 1), "frac": round(enc_achieved / tf_sust, 4)}}

    # End to end through the public Runtime.predict_many on every rank: host items -> pinned
    # staging -> H2D -> forward -> D2H of logits/acts, every micro-batch (one step = the rank's
    # whole workload); whole-job rate = all ranks' sequences over the slowest rank's time.
    h2d, d2h = 0, 0
    for batch, (m, b, k) in zip(batches, shapes):
        h2d += lib.laya_packed_ints(m, b, k) * 4
        d2h += (b * (k + 1) + b * arch["n_act"] + 1) * 4
    rt.predict_many(batches[:4])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    rt.predict_many(batches)
    e2e_rate, _, _ = job_rate((time.perf_counter() - t0) * 1000, len(items), 1, world, "cuda")
    e2e = {"value": round(e2e_rate, 2), "unit": "sequences/s", "h2d_bytes_per_step": int(h2d) * world,
           "d2h_bytes_per_step": int(d2h) * world, "api": "Runtime.predict_many(64-sequence micro-batches), two in flight"}

    line = None
    if rank == 0:
        lat, stream = None, None
        if world == 1 and args.latency != "none":
            # Configurations 1/2 (83 and 512 tokens) and 1024 tokens on the `laya` geometry.
            lat = latency(engine, arch, np.random.default_rng(0), (83, 512, 1024), tag="laya_")
            if args.latency == "full":
                # Configuration 3: the multilingual geometry (250k vocabulary), Zipf(1.1) ids.
                from laya_cuda import Engine as _Engine
                ml = S.architecture("laya-multilingual")
                ml_path = S.cached_checkpoint(CACHE, "laya-multilingual", seed=0)
                with _Engine(ml_path, device=f"cuda:{local_rank}") as ml_engine:
                    lat.update(latency(ml_engine, ml, np.random.default_rng(3), (81, 1024), zipf=1.1,
                                       tag="multilingual_zipf_"))
                # Configuration 4: the typed-decisions geometry (1024 context) through BatchEngine.
                typed = S.architecture("laya-typed-decisions")
                stream = stream_latency(S.cached_checkpoint(CACHE, "laya-typed-decisions", seed=0), typed)
        loads = cold_loads(["laya", "laya-multilingual"]) if world == 1 and args.latency != "none" else None
        api_rate = api_throughput(path, arch) if world == 1 and args.latency == "full" else None
        cpu = None
        if world == 1 and args.cpu_budget > 0:
            weights = S.make_weights(arch, seed=0)
            rate, n = oracle_rate(arch, weights, items, args.cpu_budget)
            cpu = {"value": round(rate, 3), "unit": "sequences/s", "cores": os.cpu_count(), "kind": "port",
                   "sample": f"first {n} sequences of the rank-0 workload, FP32 numpy oracle, all host threads"}
            cpu["config1_batch1"], cpu["gates"] = cpu_checks(engine, arch, weights)
        line = {"metric": "sequences/s", "value": round(value, 2), "unit": "sequences/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
                "data": "synthetic (seeded random-init weights, uniform token ids)",
                "config": {"workload": "config5-throughput: laya 12L d768 h12 F3072 V50368, positions 1024; "
                                       f"{args.requests} requests x 3 questions x 8 options, lengths U[256,1024], "
                                       "64-sequence micro-batches, split across the GPUs by modelled work",
                           "sequences_rank0": len(items), "tokens_rank0": tokens, "micro_batches_rank0": len(batches),
                           "sharding": sharding, "parallelism": f"dp{world} (request shards, no collective)",
                           "l2": "inputs larger than L2 (no flush)"},
                "gpu_launches": launches * args.steps, "kernels": fam,
                "kernels_note": "per family over one profiled step (event pair around every launch), after the timed steps",
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "api_throughput": api_rate,
                "clocks": clocks.summary(), "latency_batch1": lat, "stream_config4": stream, "cold_load": loads,
                "attention_flops_per_step": attention_flops([len(i[0]) for i in items], arch)}
    engine.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


# dram__bytes_read.sum + dram__bytes_write.sum of one FFN-up GEMM launch per token (ncu capture
# of the first 64-sequence micro-batch, 39,518 tokens, of the current kernel: 71.1 + 190.7 MB);
# traffic grows in proportion to the rows, so a full launch is this times its tokens.
TRAFFIC_FFN_UP_BYTES_PER_TOKEN = 261.8e6 / 39518


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=3)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["laya_b200", "reference"], default="laya_b200")
    parser.add_argument("--latency", choices=["none", "basic", "full"], default="full",
                        help="basic: configurations 1/2 (+1024 tokens); full: also 3 (multilingual) and 4 (stream)")
    parser.add_argument("--cpu-budget", type=float, default=15.0, help="seconds of oracle time for cpu_baseline")
    parser.add_argument("--requests", type=int, default=REQUESTS,
                        help="requests per rank (4096 = configuration 5; smaller only for profiler captures)")
    parser.add_argument("--latency-only", action="store_true",
                        help="only the batch-1 latencies of the laya geometry (for profiler captures)")
    parser.add_argument("--lengths", default="83,512,1024", help="sequence lengths of --latency-only")
    parser.add_argument("--repeats", type=int, default=200, help="timed repeats per length of --latency-only")
    parser.add_argument("--cold-load", default=None, help="time Engine construction + first request of this model "
                                                          "in this fresh process (used by the main run)")
    parser.add_argument("--attention-only", action="store_true",
                        help="only the attention kernel on one config-5 micro-batch (for profiler captures)")
    args = parser.parse_args()
    if args.latency_only:
        return run_latency_only(args)
    if args.attention_only:
        return run_attention_only(args)
    if args.cold_load:
        return run_cold_load(args)
    if args.warmup < 3:
        parser.error("--warmup must be at least 3")
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", args.gpus if "RANK" in os.environ else 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_engine(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
