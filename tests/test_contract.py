"""Request contract and decoding: golden fixtures from the reference adapter + its KATs.

tests/golden/contract.json was produced by tests/golden/make_golden.py from the reference's
own laya_cuda/laya.py; these tests require our adapter to reproduce it exactly (token ids,
markers, kinds, answer dicts, error types and messages).  The remaining tests port the
reference's tests/test_contract.py known-answer tests.
"""
import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from laya_cuda.laya import Laya, question, softmax

HERE = Path(__file__).resolve().parent
GOLDEN = json.loads((HERE / "golden/contract.json").read_text())
sys.path.insert(0, str(HERE / "golden"))
from make_golden import QUESTIONS, golden_checkpoint  # noqa: E402


@pytest.fixture(scope="module")
def adapter(tmp_path_factory):
    return Laya(golden_checkpoint(tmp_path_factory.mktemp("golden")))


def test_question_parsing_matches_reference():
    for qid, want in GOLDEN["questions"].items():
        kind, instruction, _, options = question(QUESTIONS[qid])
        assert (kind, instruction, options) == (want["kind"], want["instruction"], want["options"])


@pytest.mark.parametrize("case", range(len(GOLDEN["prepare"])))
def test_prepare_matches_reference(adapter, case):
    g = GOLDEN["prepare"][case]
    items = adapter.prepare(g["state"], {n: QUESTIONS[n] for n in g["questions"]})
    assert [[list(ids), list(markers), kind] for ids, markers, kind in items] == g["items"]


@pytest.mark.parametrize("case", range(len(GOLDEN["decode"])))
def test_decode_matches_reference(adapter, case):
    g = GOLDEN["decode"][case]
    qs = {n: QUESTIONS[n] for n in g["questions"]}
    items = [(ids, markers, kind) for ids, markers, kind in g["items"]]
    answer = adapter.decode(np.array(g["logits"], np.float32), np.array(g["acts"], np.float32), qs, items)
    assert json.loads(json.dumps(answer)) == g["answer"]


def test_errors_match_reference(adapter):
    cases = {"empty": ("x", {}), "badtype": ("x", {"q": {"type": "rank", "instructions": "i"}}),
             "nocriteria": ("x", {"q": {"type": "choice", "instructions": "i", "criteria": []}}),
             "scoredict": ("x", {"q": {"type": "score", "instructions": "i", "criteria": {"a": 1}}}),
             "noullist": ("x", {"q": {"type": "noul", "instructions": "i", "criteria": [1]}})}
    for g in GOLDEN["errors"]:
        if g["label"] == "nonfinite":
            with pytest.raises(RuntimeError) as info:
                adapter.decode(np.array([[np.nan, 1.0]], np.float32), np.zeros((1, 2), np.float32),
                               {"q": QUESTIONS["two"]}, [([1], [0], 0)])
        else:
            with pytest.raises(Exception) as info:
                adapter.prepare(*cases[g["label"]])
        assert type(info.value).__name__ == g["error"] and str(info.value) == g["message"]


def test_prepare_many_equals_prepare(adapter):
    """prepare_many (BatchEngine's path for several requests: each request's texts encoded on a
    helper thread) gives every request exactly prepare()'s items, and every failing request the
    error prepare() raises for it, whether parsing (before encoding) or the option budget (after)
    fails, without disturbing its neighbours."""
    requests = [(g["state"], {n: QUESTIONS[n] for n in g["questions"]}) for g in GOLDEN["prepare"]]
    many_options = {"type": "choice", "instructions": "i", "criteria": [f"option number {i}" for i in range(400)]}
    requests[1:1] = [("x", {}), ("x", {"q": {"type": "rank", "instructions": "i"}}), ("x", {"q": many_options})]
    results = adapter.prepare_many(requests)
    assert len(results) == len(requests)
    failed = 0
    for request, result in zip(requests, results):
        try:
            want = adapter.prepare(*request)
        except Exception as error:
            failed += 1
            assert type(result) is type(error) and str(result) == str(error)
        else:
            assert result == want
    assert failed == 3
    assert adapter.prepare_many([]) == []
    assert adapter.prepare_many(requests[:1]) == [adapter.prepare(*requests[0])]


def test_import_is_light():
    """tests/test_contract.py:11-17: importing the package pulls in no heavy libraries."""
    root = HERE.parent
    subprocess.run([sys.executable, "-c", f"""
import sys
sys.path.insert(0, {str(root / 'laya-cuda_b200')!r})
import laya_cuda
assert not {{'torch', 'transformers', 'cupy', 'psutil', 'pyarrow', 'safetensors'}} & sys.modules.keys()
assert set(laya_cuda.__all__) == {{'Engine', 'BatchEngine'}}
"""], check=True)


def test_kernel_sources_are_ascii():
    for path in (HERE.parent / "laya-cuda_b200/csrc").glob("*"):
        assert path.read_bytes().isascii(), path


def test_questions():
    """tests/test_contract.py:34-39."""
    q = question({"type": "choice", "instructions": {"ask": "team"}, "criteria": {"no": False, "zero": 0, "empty": None}})
    assert q[3] == ["no: false", "zero: 0", "empty"]
    assert question({"type": "noul", "instructions": "yes?"})[3] == ["false: no, the statement does not hold",
                                                                     "true: yes, the statement holds"]
    with pytest.raises(ValueError):
        question({"type": "choice", "instructions": "x", "criteria": []})


def test_softmax_stable():
    np.testing.assert_allclose(softmax([10000, 10000]), [.5, .5])


def test_decoding_single_option_calibration_and_nonfinite():
    """tests/test_contract.py:46-58."""
    adapter = object.__new__(Laya)
    adapter.cfg = {"temperature": [1, 1, 1], "temperature_by_options": {"choice:2": .1}}
    single = {"q": {"type": "choice", "instructions": "choose", "criteria": ["only"]}}
    items = [([1, 2], [1], 0)]
    answer = adapter.decode(np.array([[7.]]), np.array([[0., 0.]]), single, items)["answers"]["q"]
    assert answer["probabilities"] == {"only": 1.0} and answer["confidence"] == 1.0
    assert answer["action"] == {"act_probability": .5}
    double = {"q": {"type": "choice", "instructions": "choose", "criteria": ["a", "b"]}}
    output = adapter.decode(np.array([[0., 1.]]), np.array([[0., 0.]]), double, items)
    assert output["answers"]["q"]["probabilities"]["b"] == round(float(softmax([0, 2])[1]), 4)
    with pytest.raises(RuntimeError, match="Non-finite"):
        adapter.decode(np.array([[np.nan]]), np.array([[0., 0.]]), single, items)


def test_temperature_division_uses_fp32():
    """tests/test_contract.py:87-94."""
    adapter = object.__new__(Laya)
    adapter.cfg = {"temperature": [.7, 1, 1]}
    queries = {"q": {"type": "choice", "instructions": "choose", "criteria": ["a", "b"]}}
    logits = np.array([[32, 32.03125]], np.float16)
    result = adapter.decode(logits, np.array([[0, 0]], np.float16), queries, [([1, 2], [1, 2], 0)])
    expected = softmax(logits[0].astype(np.float32) / np.float32(.7))
    assert list(result["answers"]["q"]["probabilities"].values()) == [round(float(p), 4) for p in expected]


def test_missing_checkpoint_and_invalid_cache(tmp_path):
    from laya_cuda import Engine
    from laya_cuda.models import resolve
    with pytest.raises(FileNotFoundError, match="Incomplete checkpoint"):
        resolve(tmp_path)
    with pytest.raises(FileNotFoundError, match="Unknown alias"):
        resolve(tmp_path / "missing")
    for limit in (0, 65, True):
        with pytest.raises(ValueError, match="max_cached_shapes"):
            Engine(tmp_path, max_cached_shapes=limit)
    with pytest.raises(ValueError, match="CUDA device"):
        Engine(tmp_path, device="cpu")


def test_unsupported_encoder_config(monkeypatch, tmp_path):
    import laya_cuda.laya as implementation
    monkeypatch.setattr(implementation, "read_json", lambda _: {"model_type": "bert"})
    with pytest.raises(ValueError, match="ModernBERT"):
        Laya(tmp_path)


def test_state_requires_json_values():
    adapter = object.__new__(Laya)
    adapter.mask_text = "[MASK]"
    with pytest.raises(TypeError):
        adapter.prepare({"unsupported": object()}, {"q": {"type": "noul", "instructions": "yes?"}})


def test_synthetic_checkpoint_contract(tmp_path):
    """The synthetic checkpoints load through the adapter, and their token contract holds
    (tests/test_contract.py:97-108 on a generated checkpoint)."""
    from laya_cuda import synthetic as S
    a = Laya(S.write_checkpoint(tmp_path / "c", S.architecture("tiny"), weights={}))
    queries = {"q": {"type": "choice", "instructions": "Choose [MASK] a team", "criteria": {"billing": "payment", "other": None}}}
    seq, markers, kind = a.prepare("w9 " * 5000, queries)[0]
    assert len(seq) == a.max_len and seq[0] == a.cls and seq[-1] == a.sep
    assert len(markers) == 2 and all(seq[i] == a.mask for i in markers) and kind == 0
    with pytest.raises(ValueError):
        a.prepare("", {})


def test_fingerprint_equals_compact_json_digest(adapter):
    """The fingerprint is sha256 of json.dumps(items, separators=(",", ":")) (laya.py:192-193)."""
    import hashlib
    rng = np.random.default_rng(5)
    for n in (1, 2, 7):
        items = []
        for _ in range(n):
            ids = [int(v) for v in rng.integers(0, 250000, rng.integers(1, 600))]
            markers = [int(v) for v in rng.integers(0, 500, rng.integers(1, 80))]
            item = (ids, markers, int(rng.integers(0, 3)))
            items.append(item if rng.random() < 0.5 else list(item))
        want = hashlib.sha256(json.dumps(items, separators=(",", ":")).encode()).hexdigest()
        assert adapter.fingerprint(items) == want


@pytest.mark.skipif(not hasattr(__import__("os"), "fork"), reason="needs fork")
@pytest.mark.filterwarnings("ignore:This process .* is multi-threaded:DeprecationWarning")
def test_prepare_many_in_a_forked_child(adapter):
    """A child forked after prepare_many has run gets its own helper threads (the parent's do not
    exist in the child), so its prepare_many completes with the same items."""
    import multiprocessing
    requests = [(g["state"], {n: QUESTIONS[n] for n in g["questions"]}) for g in GOLDEN["prepare"][:4]]
    want = adapter.prepare_many(requests)
    ctx = multiprocessing.get_context("fork")
    queue = ctx.Queue()
    child = ctx.Process(target=lambda: queue.put(adapter.prepare_many(requests)))
    child.start()
    try:
        got = queue.get(timeout=60)
    finally:
        child.join(60)
        if child.is_alive():
            child.kill()
    assert child.exitcode == 0 and got == want
