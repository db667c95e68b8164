"""Parity gates between two backends' answers on one frozen request set.

The gates and their thresholds are the reference's (benchmarks/run.py:23 GATES; compare and
passes at benchmarks/run.py:180-219): over every question of every request, the mean and the
largest absolute difference of the option probabilities and of the action probability, and
the share of questions whose decision label agrees.  They must be alike for a comparison with
the reference's published gate results to mean the same thing.

    python -m laya_cuda.gates --model laya [--registry R] [--device cuda:0]

runs this library (backend="cuda") and the official SDK in FP32 (backend="official", when it is
installed) on `frozen_requests` and prints the statistics and the verdict.  bench.py applies the
same gates with the FP32 restatement of the reference forward pass as the reference answers.
"""
import argparse
import json

import numpy as np

# benchmarks/run.py:23 of the reference (the gates that concern answers).
GATES = {"probability_mae": 1e-3, "probability_max": 1e-2, "agreement": 0.995}


def label(answer):
    """The decision of one answer: the choice, the noul side, or the most probable score level."""
    if answer["type"] == "choice":
        return answer["choice"]
    if answer["type"] == "noul":
        return "true" if answer["noul"] >= 0.5 else "false"
    return max(answer["probabilities"], key=answer["probabilities"].get)


def probabilities(answer):
    p = answer.get("probabilities")
    return list(p.values()) if p is not None else [1 - answer["noul"], answer["noul"]]


def compare(candidate, reference):
    """Statistics over aligned answer records [{"id", "answers"}]: probability and action MAE and
    maximum, label agreement, decision count, all finite."""
    diffs, actions, agree, total = [], [], 0, 0
    for x, y in zip(candidate, reference, strict=True):
        if x["id"] != y["id"]:
            raise ValueError("answer records do not align")
        for q, a in x["answers"].items():
            b = y["answers"][q]
            diffs.extend(np.abs(np.array(probabilities(a)) - np.array(probabilities(b))).tolist())
            actions.append(abs(a["action"]["act_probability"] - b["action"]["act_probability"]))
            agree += label(a) == label(b)
            total += 1
    return {"decisions": total, "mae": float(np.mean(diffs)) if diffs else None,
            "max": float(max(diffs)) if diffs else None, "agreement": agree / total if total else None,
            "finite": bool(np.isfinite(diffs).all()) if diffs else False,
            "action_mae": float(np.mean(actions)) if actions else None,
            "action_max": float(max(actions)) if actions else None}


def passes(stats):
    """The reference's verdict: every gate met, on at least one decision, all values finite."""
    return bool(stats["decisions"] and stats["finite"]
                and stats["mae"] <= GATES["probability_mae"] and stats["max"] <= GATES["probability_max"]
                and stats["action_mae"] <= GATES["probability_mae"] and stats["action_max"] <= GATES["probability_max"]
                and stats["agreement"] >= GATES["agreement"])


def _state_of_length(adapter, questions, target, word):
    """A state whose longest question sequence is exactly `target` tokens, or None if the
    tokenizer cannot hit it with whole words."""
    def length(n):
        return max(len(v[0]) for v in adapter.prepare(" ".join(word(i) for i in range(n)), questions))
    lo, hi = 0, target
    while lo < hi:
        mid = (lo + hi) // 2
        if length(mid) < target:
            lo = mid + 1
        else:
            hi = mid
    state = " ".join(word(i) for i in range(lo))
    return state if length(lo) == target else None


def frozen_requests(adapter, seed=0, lengths=(32, 128, 512, 1024), counts=(1, 5), word=None):
    """A deterministic request set in the shape of the reference's timing cases
    (benchmarks/run.py:51-71): every (length, question count) pair up to the context budget,
    the tile boundaries 127 / 129 and max_len - 1, and a request whose questions differ in
    length.  Choice questions with 2-4 labels; states of seeded words (`word(i)` -> text,
    default the synthetic checkpoints' "w<id>" vocabulary).  Yields (id, state, questions)."""
    rng = np.random.default_rng(seed)
    vocab = adapter.config.get("vocab_size", 1000)
    ids = rng.integers(5, max(vocab, 6), 4096)
    word = word or (lambda i: f"w{ids[i % len(ids)]}")

    def question(i):
        labels = [f"{word(100 + 7 * i + j)} {word(200 + 5 * i + j)}" for j in range(2 + i % 3)]
        return {"type": "choice", "instructions": " ".join(word(300 + 3 * i + j) for j in range(4)), "criteria": labels}

    for length in lengths:
        if length > adapter.max_len:
            continue
        for count in counts:
            questions = {str(i): question(i) for i in range(count)}
            state = _state_of_length(adapter, questions, length, word)
            if state is not None:
                yield f"l{length}-q{count}", state, questions
    for length in (127, 129, adapter.max_len - 1):
        questions = {"0": question(0)}
        state = _state_of_length(adapter, questions, length, word)
        if state is not None:
            yield f"boundary-l{length}", state, questions
    mixed = {str(i): dict(question(i), instructions=question(i)["instructions"] + " " + " ".join(
        word(400 + k) for k in range(9 * i))) for i in range(5)}
    yield "mixed-lengths", " ".join(word(500 + k) for k in range(40)), mixed


def answers(engine, requests):
    return [{"id": rid, "answers": engine.predict(state, questions)["answers"]} for rid, state, questions in requests]


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--model", default="laya")
    parser.add_argument("--registry")
    parser.add_argument("--device", default="cuda:0")
    args = parser.parse_args()
    from .engine import Engine
    with Engine(args.model, registry=args.registry, device=args.device) as engine:
        requests = list(frozen_requests(engine.adapter))
        candidate = answers(engine, requests)
    with Engine(args.model, registry=args.registry, device=args.device, backend="official") as reference:
        reference.runtime.agent.dtype = reference.runtime.torch.float32
        expected = answers(reference, requests)
    stats = compare(candidate, expected)
    print(json.dumps({"gates": GATES, "stats": stats, "passed": passes(stats), "requests": len(requests)}))


if __name__ == "__main__":
    main()
