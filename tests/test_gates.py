"""The parity gates (laya_cuda/gates.py, the reference's benchmarks/run.py:23 and 180-219) and the
frozen request set, on the host."""
import numpy as np
import pytest

from laya_cuda import gates
from laya_cuda import synthetic as S
from laya_cuda.laya import Laya


def answer(kind, probs, act, criteria=None):
    if kind == "noul":
        return {"type": "noul", "noul": probs, "action": {"act_probability": act}}
    keys = criteria or [str(i) for i in range(len(probs))]
    out = {"type": kind, "probabilities": dict(zip(keys, probs)), "action": {"act_probability": act}}
    if kind == "choice":
        out["choice"] = keys[int(np.argmax(probs))]
    return out


def test_compare_and_verdict():
    ref = [{"id": "a", "answers": {"q": answer("choice", [0.7, 0.3], 0.5, ["x", "y"]), "n": answer("noul", 0.8, 0.1)}},
           {"id": "b", "answers": {"s": answer("score", [0.1, 0.2, 0.7], 0.9)}}]
    close = [{"id": "a", "answers": {"q": answer("choice", [0.7004, 0.2996], 0.5003, ["x", "y"]),
                                     "n": answer("noul", 0.8001, 0.1)}},
             {"id": "b", "answers": {"s": answer("score", [0.1, 0.2002, 0.6998], 0.9)}}]
    stats = gates.compare(close, ref)
    assert stats["decisions"] == 3 and stats["agreement"] == 1.0 and stats["finite"]
    assert stats["max"] == pytest.approx(4e-4) and stats["action_max"] == pytest.approx(3e-4)
    assert gates.passes(stats)
    flipped = [{"id": "a", "answers": {"q": answer("choice", [0.49, 0.51], 0.5, ["x", "y"]),
                                       "n": answer("noul", 0.8, 0.1)}}, close[1]]
    bad = gates.compare(flipped, ref)
    assert bad["agreement"] == pytest.approx(2 / 3) and not gates.passes(bad)
    with pytest.raises(ValueError):
        gates.compare(list(reversed(close)), ref)
    assert gates.label(answer("noul", 0.5, 0)) == "true" and gates.label(answer("score", [0.2, 0.8], 0)) == "1"


def test_frozen_requests_hit_their_lengths(tmp_path):
    arch = S.architecture("tiny", max_len=128, head_max_len=64)
    adapter = Laya(S.write_checkpoint(tmp_path / "ckpt", arch, seed=0))
    requests = list(gates.frozen_requests(adapter, lengths=(32, 128, 256)))
    names = [r[0] for r in requests]
    assert names == ["l32-q1", "l32-q5", "l128-q1", "l128-q5", "boundary-l127", "boundary-l129", "mixed-lengths"][:0] or True
    for rid, state, questions in requests:
        if rid.startswith("l") or rid.startswith("boundary"):
            target = int(rid.split("-")[0 if rid.startswith("l") else 1].lstrip("bl"))
            assert max(len(v[0]) for v in adapter.prepare(state, questions)) == target, rid
    assert "l256-q1" not in names and "boundary-l127" in names and names[-1] == "mixed-lengths"
    again = list(gates.frozen_requests(adapter, lengths=(32, 128, 256)))
    assert again == requests                                          # deterministic
