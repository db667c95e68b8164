"""Parity of the B200 engine with the FP32 oracle on every registered geometry the benchmark
times, on random-init weights of each architecture (N(0, 0.02), seed 0):

* `laya-multilingual`: 250,000-entry embedding table, 1024 positions, token ids Zipf(1.1)
  (scattered embedding reads), rows of 81 and 1024 tokens (configuration 3);
* `laya-typed-decisions`: 1024 context, packed batches of questions with up to 77 options, so
  the option class is k = 128 and each question's CLS + marker rows span two gathered-query
  attention tiles (configuration 4);
* `laya` with positions extended to 1024 and rows of 900-1024 tokens (configuration 5's rows);
* decision heads with 2 and 3 transformer layers (laya.py:82 allows any count >= 1; every layer
  but the last runs over all rows, laya.py:219-235), on classes that split K and ones that do not.

Gates (north star): per-option probabilities and action probabilities within 2e-3 of FP32; the
option logits themselves within 5e-3, so the probability gate is not met only because random-init
decisions are near uniform.  Usage counts are bit-exact by construction (the request contract is
pinned by tests/test_contract.py).
"""
import json

import numpy as np
import pytest

from laya_cuda import BatchEngine, Engine
from laya_cuda import synthetic as S
from laya_cuda.laya import softmax
from oracle.laya_oracle import Oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

PROB, ACT, LOGIT = 2e-3, 2e-3, 5e-3


@pytest.fixture(scope="module", autouse=True)
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")


def checkpoint(tmp_path_factory, name, **overrides):
    arch = S.architecture(name, **overrides)
    weights = S.make_weights(arch, seed=0)
    path = S.write_checkpoint(tmp_path_factory.mktemp(name), arch, weights=weights)
    return path, arch, weights


def errors(engine, oracle, items):
    logits, acts, metrics = engine.runtime.predict(items)
    rows = []
    for i, (ids, markers, kind) in enumerate(items):
        want_l, want_a = oracle.item(ids, markers, kind)
        k = len(markers)
        rows.append(dict(tokens=len(ids), options=k,
                         logit=float(np.max(np.abs(logits[i, :k] - want_l))),
                         prob=float(np.max(np.abs(softmax(logits[i, :k]) - softmax(want_l)))),
                         act=float(np.max(np.abs(softmax(acts[i]) - softmax(want_a))))))
    return rows, metrics


def check(rows, tag):
    summary = {key: max(r[key] for r in rows) for key in ("logit", "prob", "act")}
    print(json.dumps({"geometry": tag, "rows": len(rows), **summary}))
    assert summary["prob"] <= PROB and summary["act"] <= ACT and summary["logit"] <= LOGIT, (tag, rows)


def test_multilingual_zipf_ids_81_and_1024_tokens(tmp_path_factory):
    path, arch, weights = checkpoint(tmp_path_factory, "laya-multilingual")
    oracle = Oracle(weights, arch)
    rng = np.random.default_rng(3)
    single = [[S.build_item(rng, n, 4, arch["vocab"], zipf=1.1)] for n in (81, 1024)]
    packed = [S.build_item(rng, n, k, arch["vocab"], kind=j % 3, zipf=1.1)
              for j, (n, k) in enumerate([(1024, 8), (81, 4), (700, 6), (333, 3)])]
    rows = []
    with Engine(path) as engine:
        for items in single + [packed]:
            got, _ = errors(engine, oracle, items)
            rows += got
    # Zipf(1.1) ids are concentrated on low ranks but reach deep into the table.
    ids = np.concatenate([np.asarray(i[0]) for items in single + [packed] for i in items])
    assert ids.max() > 10_000
    check(rows, "laya-multilingual")


def test_typed_decisions_1024_context_77_options(tmp_path_factory):
    path, arch, weights = checkpoint(tmp_path_factory, "laya-typed-decisions")
    oracle = Oracle(weights, arch)
    rng = np.random.default_rng(2)
    batches = [
        # One request's questions packed together: 77 options force the k = 128 class.
        [S.build_item(rng, n, k, arch["vocab"], kind=j % 3) for j, (n, k) in
         enumerate([(1024, 77), (900, 40), (450, 77), (200, 4), (1000, 12)])],
        [S.build_item(rng, 1024, 77, arch["vocab"])],
        [S.build_item(rng, n, k, arch["vocab"], kind=1) for n, k in [(40, 4), (63, 9)]],
    ]
    rows = []
    with Engine(path) as engine:
        for items in batches:
            got, metrics = errors(engine, oracle, items)
            rows += got
            if max(len(i[1]) for i in items) > 64:
                assert metrics["shape"][2] == 128
    check(rows, "laya-typed-decisions")


def test_typed_decisions_stream_through_batch_engine(tmp_path_factory):
    """Configuration 4's request shapes through BatchEngine (1-5 questions of 4-77 options):
    every answer equals Engine.predict's within the probability gate."""
    path, arch, _ = checkpoint(tmp_path_factory, "laya-typed-decisions", layers=2)
    rng = np.random.default_rng(12)
    requests = [S.stream_request_texts(rng, arch["vocab"]) for _ in range(12)]
    with Engine(path) as engine:
        expected = [engine.predict(state, qs) for state, qs in requests]
    with BatchEngine(path, max_batch_size=8, max_batch_tokens=8192, max_wait_ms=2) as engine:
        futures = [engine.submit(state, qs) for state, qs in requests]
        for future, want in zip(futures, expected):
            got = future.result(120)
            assert got["usage"] == want["usage"]
            for key, answer in got["answers"].items():
                a = np.array(list(answer["probabilities"].values()))
                b = np.array(list(want["answers"][key]["probabilities"].values()))
                assert np.max(np.abs(a - b)) <= PROB


def test_laya_positions_1024_long_rows(tmp_path_factory):
    path, arch, weights = checkpoint(tmp_path_factory, "laya", max_len=1024)
    oracle = Oracle(weights, arch)
    rng = np.random.default_rng(5)
    batches = [[S.build_item(rng, 1024, 8, arch["vocab"])],
               [S.build_item(rng, n, 8, arch["vocab"], kind=j % 3) for j, n in enumerate([1024, 950, 900, 1000])]]
    rows = []
    with Engine(path) as engine:
        for items in batches:
            got, _ = errors(engine, oracle, items)
            rows += got
    check(rows, "laya-1024")


@pytest.mark.parametrize("head_layers", [2, 3])
def test_multi_layer_decision_head(tmp_path_factory, head_layers):
    """Every head layer but the last runs over all packed rows (out_proj + residual, norm2,
    linear1 + ReLU, linear2 + residual, next norm1): a small class (split-K residual GEMMs) and a
    class above 2048 rows (residual epilogues)."""
    path, arch, weights = checkpoint(tmp_path_factory, "small", max_len=256, head_layers=head_layers)
    oracle = Oracle(weights, arch)
    rng = np.random.default_rng(head_layers)
    small = [S.build_item(rng, n, k, arch["vocab"], kind=j % 3) for j, (n, k) in enumerate([(83, 4), (200, 7)])]
    large = [S.build_item(rng, int(rng.integers(150, 256)), int(rng.integers(2, 9)), arch["vocab"], kind=j % 3)
             for j in range(14)]
    rows = []
    with Engine(path) as engine:
        for items in (small, large):
            got, metrics = errors(engine, oracle, items)
            rows += got
        assert metrics["shape"][0] > 2048
    check(rows, f"small-head{head_layers}")
