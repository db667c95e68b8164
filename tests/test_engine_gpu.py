"""End-to-end parity and lifecycle of the B200 engine against the FP32 oracle.

Ports the reference's runtime contracts (tests/test_runtime.py, tests/test_custom_models.py,
tests/test_batching_gpu.py) onto seeded random-init checkpoints, and adds the north-star
parity gates: per-option probabilities within 2e-3 of FP32, argmax agreement, token/usage
counts bit-exact.  Logits are also compared directly, since random-init decisions are nearly
uniform and a probability gate alone is loose.
"""
import json

import numpy as np
import pytest

from laya_cuda import BatchEngine, Engine
from laya_cuda import synthetic as S
from laya_cuda.laya import Laya, softmax
from oracle.laya_oracle import Oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")


@pytest.fixture(scope="module")
def laya_ckpt(tmp_path_factory):
    """Full `laya` geometry (d 768, 12 layers, F 3072, vocab 50368), seed 0, max_len 512."""
    arch = S.architecture("laya")
    weights = S.make_weights(arch, seed=0)
    path = S.write_checkpoint(tmp_path_factory.mktemp("laya"), arch, weights=weights)
    return path, arch, weights


@pytest.fixture(scope="module")
def peaky_ckpt(tmp_path_factory):
    """Small geometry with 5x larger weights: decisive logits, so argmax parity means something."""
    arch = S.architecture("small", max_len=256)
    weights = S.make_weights(arch, seed=7, scale=0.1)
    path = S.write_checkpoint(tmp_path_factory.mktemp("peaky"), arch, weights=weights)
    return path, arch, weights


def compare(engine, oracle, items):
    logits, acts, _ = engine.runtime.predict(items)
    rows = []
    for i, (ids, markers, kind) in enumerate(items):
        want_l, want_a = oracle.item(ids, markers, kind)
        k = len(markers)
        got_p, want_p = softmax(logits[i, :k]), softmax(want_l)
        rows.append(dict(logit=float(np.max(np.abs(logits[i, :k] - want_l))),
                         prob=float(np.max(np.abs(got_p - want_p))),
                         act=float(np.max(np.abs(softmax(acts[i]) - softmax(want_a)))),
                         agree=bool(np.argmax(logits[i, :k]) == np.argmax(want_l)),
                         margin=float(np.sort(want_l)[-1] - np.sort(want_l)[-2]) if k > 1 else np.inf))
    return rows


@pytest.mark.parametrize("precision", ["bfloat16", "float16"])
def test_laya_geometry_matches_fp32_oracle(laya_ckpt, precision):
    path, arch, weights = laya_ckpt
    oracle = Oracle(weights, arch)
    rng = np.random.default_rng(1)
    # Config 1/2 shapes (83 and 512 tokens, 4 options), plus packed batches of mixed lengths/kinds.
    batches = [[S.build_item(rng, 83, 4, arch["vocab"])], [S.build_item(rng, 512, 4, arch["vocab"])],
               [S.build_item(rng, n, k, arch["vocab"], kind=j % 3) for j, (n, k) in
                enumerate([(40, 2), (300, 8), (129, 5), (512, 12), (64, 1)])]]
    with Engine(path, precision=precision) as engine:
        rows = [r for items in batches for r in compare(engine, oracle, items)]
    print(json.dumps(rows))
    assert max(r["prob"] for r in rows) <= 2e-3
    assert max(r["act"] for r in rows) <= 2e-3
    # Logit error must stay below the decision gaps it could flip.
    assert max(r["logit"] for r in rows) <= (0.02 if precision == "bfloat16" else 0.005)


@pytest.mark.parametrize("precision", ["bfloat16", "float16"])
def test_decisive_checkpoint_argmax_and_probabilities(peaky_ckpt, precision):
    path, arch, weights = peaky_ckpt
    oracle = Oracle(weights, arch)
    rng = np.random.default_rng(11)
    items_all = []
    for j in range(96):
        k = int(rng.integers(2, 12))
        items_all.append(S.build_item(rng, int(rng.integers(12 + 5 * k, 256)), k, arch["vocab"], kind=j % 3))
    rows = []
    with Engine(path, precision=precision) as engine:
        for start in range(0, len(items_all), 16):
            rows += compare(engine, oracle, items_all[start:start + 16])
    probs = [r["prob"] for r in rows]
    agree = np.mean([r["agree"] for r in rows if r["margin"] > 1e-3])
    print(json.dumps(dict(max_prob=max(probs), mean_prob=float(np.mean(probs)), agree=float(agree),
                          max_logit=max(r["logit"] for r in rows))))
    if precision == "float16":
        # The north-star gates: probabilities within 2e-3 of FP32, >= 99.5% identical argmax.
        assert max(probs) <= 2e-3
        assert agree >= 0.995
    else:
        # bfloat16 operands keep 8 mantissa bits: measured ~98% agreement on decisive logits,
        # short of the 99.5% gate, which is why float16 is the default precision.
        assert max(probs) <= 1e-2
        assert agree >= 0.95


def test_text_requests_usage_and_answers(laya_ckpt):
    """Engine.predict(text) end to end: token counts bit-exact, answers close to the oracle's."""
    path, arch, weights = laya_ckpt
    oracle = Oracle(weights, arch)
    rng = np.random.default_rng(5)
    with Engine(path) as engine:
        for length in (83, 200, 512):
            state, questions, ids = S.request_texts(rng, length, 4, arch["vocab"])
            answer = engine.predict(state, questions)
            items = engine.adapter.prepare(state, questions)
            assert items[0][0] == ids and answer["usage"]["input_tokens"] == length
            assert engine.last_metrics["tokens_per_question"] == [length]
            want_l, want_a = oracle.item(*items[0])
            want = engine.adapter.decode(want_l[None], want_a[None], questions, items)
            got_p = np.array(list(answer["answers"]["q"]["probabilities"].values()))
            want_p = np.array(list(want["answers"]["q"]["probabilities"].values()))
            assert np.max(np.abs(got_p - want_p)) <= 2e-3
            assert abs(answer["answers"]["q"]["action"]["act_probability"]
                       - want["answers"]["q"]["action"]["act_probability"]) <= 2e-3


def test_eager_graph_lifecycle(laya_ckpt):
    """tests/test_runtime.py:12-37: eager == graph bit-exact, repeats identical, one slot under
    max_cached_shapes=1, fresh contents on graph reuse, zero bytes after close, closed error."""
    path, arch, _ = laya_ckpt
    q = {"q": {"type": "choice", "instructions": "w7 w8", "criteria": ["w10 w11", "w12"]}}
    rng = np.random.default_rng(9)
    with Engine(path, max_cached_shapes=1) as e:
        for n in (5, 150, 400):
            state = " ".join(S.word(int(t)) for t in rng.integers(5, arch["vocab"], n))
            items = e.adapter.prepare(state, q)
            raw = e.runtime.predict(items, capture=False)
            captured = e.runtime.predict(items, capture=True)
            np.testing.assert_array_equal(raw[0], captured[0])
            np.testing.assert_array_equal(raw[1], captured[1])
            results = [e.predict(state, q) for _ in range(4)]
            assert all(r == results[0] for r in results)
            assert len(e.runtime.slots) == 1
        for state in ("w20 w21", "w30 " * 40, "w20 w21"):
            items = e.adapter.prepare(state, q)
            captured = e.runtime.predict(items, capture=True)
            eager = e.runtime.predict(items, capture=False)
            np.testing.assert_array_equal(captured[0], eager[0])
            np.testing.assert_array_equal(captured[1], eager[1])
    assert e.runtime.pool.used_bytes() == 0
    e.close()
    with pytest.raises(RuntimeError, match="closed"):
        e.predict("w5", q)


def test_cold_shape_captures_on_first_use_and_eviction(laya_ckpt):
    """tests/test_runtime.py:40-53."""
    path, _, _ = laya_ckpt
    q = {"q": {"type": "choice", "instructions": "w7", "criteria": ["w10", "w12"]}}
    with Engine(path, max_cached_shapes=1) as engine:
        first = engine.predict("w5 w6", q)
        m = engine.last_metrics
        assert m["cache_miss"] and m["graph_capture"] and m["graph_replay"]
        assert engine.predict("w5 w6", q) == first
        m = engine.last_metrics
        assert not m["cache_miss"] and not m["graph_capture"] and m["graph_replay"]
        engine.predict("w9 " * 300, q)
        assert engine.predict("w5 w6", q) == first
        assert engine.last_metrics["cache_miss"] and engine.last_metrics["graph_capture"]


def test_batched_rows_equal_single_rows(laya_ckpt):
    """Packing does not change a row's result: tile decomposition is per row, and every GEMM
    reduces K in the same order whatever the batch."""
    path, arch, _ = laya_ckpt
    rng = np.random.default_rng(21)
    items = [S.build_item(rng, n, k, arch["vocab"], kind=j % 3) for j, (n, k) in
             enumerate([(90, 3), (333, 9), (17, 1), (512, 4), (250, 6), (65, 1), (128, 16)])]
    with Engine(path) as engine:
        together = engine.runtime.predict(items)
        for i, item in enumerate(items):
            alone = engine.runtime.predict([item])
            k = len(item[1])
            np.testing.assert_allclose(together[0][i, :k], alone[0][0, :k], atol=2e-3)
            np.testing.assert_allclose(together[1][i], alone[1][0], atol=2e-3)


def test_custom_checkpoint_weights_registry_and_batching(tmp_path):
    """tests/test_custom_models.py:14-57 on a tiny synthetic checkpoint (d 64, 1 head, 1 layer)."""
    arch = S.architecture("tiny", layers=1, max_len=128, head_max_len=64)
    custom = tmp_path / "custom-weights"
    weights = {name: np.zeros(shape, np.float32) for name, shape in S.weight_shapes(arch).items()}
    registry = tmp_path / "models.json"
    registry.write_text(json.dumps({"my-finetune": {"path": "custom-weights"}}))
    queries = {"q": {"type": "choice", "instructions": "Choose", "criteria": ["yes", "no"]}}
    outputs = []
    for bias in ([-4, 4], [4, -4]):
        weights["act_head.2.bias"] = np.array(bias, np.float32)
        S.write_checkpoint(custom, arch, weights=weights)
        with Engine("my-finetune", registry=registry) as engine:
            output = engine.predict("custom input", queries)
            assert engine.path == custom
            np.testing.assert_array_equal(engine.runtime.weights["act_head.2.bias"].get(), bias)
            assert output == engine.predict("custom input", queries)
            outputs.append(output["answers"]["q"]["action"]["act_probability"])
        assert engine.runtime.pool.used_bytes() == 0
    assert outputs[0] < .001 and outputs[1] > .999
    with Engine(custom) as engine:
        expected = engine.predict("custom input", queries)
    with BatchEngine("my-finetune", registry=registry) as engine:
        assert engine.submit("custom input", queries).result(60) == expected
    weights["act_head.2.bias"] = np.zeros(3, np.float32)
    S.write_checkpoint(custom, arch, weights=weights)
    with pytest.raises(ValueError, match="Incompatible tensor shape"):
        Engine("my-finetune", registry=registry)


def test_batch_engine_matches_engine(laya_ckpt):
    """tests/test_batching_gpu.py:10-40 on synthetic requests."""
    path, arch, _ = laya_ckpt
    rng = np.random.default_rng(3)
    questions = {"same": {"type": "choice", "instructions": "w9 w10", "criteria": ["w11", "w12 w13"]},
                 "score": {"type": "score", "instructions": "w14", "criteria": ["w15", "w16", "w17"]},
                 "noul": {"type": "noul", "instructions": "w18 w19"}}
    states = [" ".join(S.word(int(t)) for t in rng.integers(5, arch["vocab"], n)) for n in (3, 40, 110, 500)]
    requests = [(s, questions) for s in states]
    requests.append((states[0], {"same": {"type": "choice", "instructions": "w9",
                                          "criteria": ["w20", "w21", "w22", "w23", "w24"]}}))
    requests.append((states[0], {"same": {"type": "choice", "instructions": "w9", "criteria": ["only"]}}))
    with Engine(path) as engine:
        expected = [engine.predict(s, q) for s, q in requests]
    with BatchEngine(path, max_batch_tokens=8192, max_wait_ms=5) as engine:
        futures = [engine.submit(s, q) for s, q in requests * 2]
        diffs = []
        for i, future in enumerate(futures):
            actual, reference = future.result(120), expected[i % len(requests)]
            assert actual["usage"] == reference["usage"]
            assert list(actual["answers"]) == list(reference["answers"])
            for key, a in actual["answers"].items():
                b = reference["answers"][key]
                pa = list(a["probabilities"].values()) if "probabilities" in a else [a["noul"]]
                pb = list(b["probabilities"].values()) if "probabilities" in b else [b["noul"]]
                diffs += list(np.abs(np.array(pa) - np.array(pb)))
                diffs.append(abs(a["action"]["act_probability"] - b["action"]["act_probability"]))
        assert futures[-1].result()["answers"]["same"]["probabilities"] == {"only": 1.0}
    assert max(diffs) <= 2e-3



def test_programmatic_launch_does_not_change_results(laya_ckpt):
    """Every kernel waits for its predecessor before reading its outputs, so results with
    programmatic dependent launch equal those of plain stream order bit for bit (a fresh
    engine per mode, so no graph captured under the other mode is reused)."""
    from laya_cuda import _lib
    path, arch, _ = laya_ckpt
    rng = np.random.default_rng(8)
    items = [S.build_item(rng, n, k, arch["vocab"], kind=j % 3) for j, (n, k) in enumerate([(83, 4), (512, 8), (300, 5)])]
    lib = _lib.load()
    results = []
    try:
        for pdl in (1, 0):
            assert lib.laya_set_launch_options(pdl, 0) == 0
            with Engine(path) as e:
                outs = [e.runtime.predict(items, capture=c) for c in (True, False)] + [e.runtime.predict(items[:1])]
            results.append([a for o in outs for a in o[:2]])
    finally:
        lib.laya_set_launch_options(1, 0)
    for a, b in zip(*results):
        np.testing.assert_array_equal(a, b)


def test_submit_collect_pipeline_matches_predict(laya_ckpt):
    """Runtime.submit/collect (two passes in flight, pinned staging per pass) returns exactly
    what predict returns for the same batches, in any collection order; a third submit while two
    are in flight is refused."""
    path, arch, _ = laya_ckpt
    rng = np.random.default_rng(11)
    batches = [[S.build_item(rng, n, k, arch["vocab"], kind=j % 3) for j, (n, k) in enumerate(shape)]
               for shape in ([(83, 4)], [(512, 8), (300, 5)], [(129, 2)] * 3, [(500, 4)], [(64, 1), (480, 6)])]
    with Engine(path) as engine:
        rt = engine.runtime
        expected = [rt.predict(b) for b in batches]
        got = rt.predict_many(batches)
        for (l0, a0, _), (l1, a1, _) in zip(expected, got):
            np.testing.assert_array_equal(l0, l1)
            np.testing.assert_array_equal(a0, a1)
        t0, t1 = rt.submit(batches[0]), rt.submit(batches[1])
        with pytest.raises(RuntimeError, match="in flight"):
            rt.submit(batches[2])
        l1, a1, _ = rt.collect(t1)
        l0, a0, _ = rt.collect(t0)
        np.testing.assert_array_equal(l0, expected[0][0])
        np.testing.assert_array_equal(l1, expected[1][0])
