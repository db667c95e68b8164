"""Generates tests/golden/contract.json from the reference adapter itself.

The request contract (question parsing, tokenisation, sequence/marker construction, budgets)
and the decoding (temperature calibration, answer dict) decide token counts and answers, so
they are pinned to the reference's own implementation: this script imports the reference
package (laya_cuda/laya.py of laya-cuda, read-only, under a private module name), runs it on a
deterministic synthetic checkpoint and records inputs and outputs.  The reference is only
needed to regenerate the fixture:

    python tests/golden/make_golden.py /path/to/laya-cuda

The checkpoint uses a character-level WordLevel tokenizer (every character one token, so
texts have realistic lengths and budgets/truncation are exercised) built by golden_checkpoint().
"""
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
CHARS = [chr(c) for c in range(32, 127)] + list("支付退款软件出现错误请处理选择é😀—")


def golden_checkpoint(path):
    """Tokenizer + configs (no weights needed for the contract) of the golden fixture."""
    from tokenizers import Regex, Tokenizer, models, pre_tokenizers
    path = Path(path)
    (path / "tokenizer").mkdir(parents=True, exist_ok=True)
    (path / "encoder").mkdir(parents=True, exist_ok=True)
    vocab = {tok: i for i, tok in enumerate(["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"])}
    for ch in CHARS:
        vocab.setdefault(ch, len(vocab))
    tok = Tokenizer(models.WordLevel(vocab, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Split(Regex("."), behavior="isolated")
    tok.save(str(path / "tokenizer/tokenizer.json"))
    (path / "tokenizer/tokenizer_config.json").write_text(json.dumps(
        {"cls_token": "[CLS]", "sep_token": "[SEP]", "mask_token": "[MASK]", "pad_token": "[PAD]"}))
    (path / "encoder/config.json").write_text(json.dumps(
        {"model_type": "modernbert", "hidden_size": 64, "num_attention_heads": 1, "num_hidden_layers": 1,
         "intermediate_size": 128, "vocab_size": len(vocab), "max_position_embeddings": 8192}))
    (path / "rl_agent_config.json").write_text(json.dumps(
        {"max_len": 160, "head_max_len": 64, "head_layers": 1, "act_costs": {"a": 1},
         "temperature": [0.7, 1.3, 2.0],
         "temperature_by_options": {"choice:2": 0.1, "choice:3-5": "bad", "score:3-5": 9.0, "choice:11+": float("inf")}}))
    (path / "model.safetensors").write_text("{}")
    return path


QUESTIONS = {
    "a": {"type": "choice", "instructions": {"ask": "选择 [MASK]"}, "criteria": {"yes": False, "no": 0, "empty": None,
                                                                              "blank": "", "nested": {"k": [1, 2]}}},
    "b": {"type": "score", "instructions": "Urgency?", "criteria": ["low", {"level": 2}, "high"]},
    "c": {"type": "noul", "instructions": "支付退款?", "criteria": {"true": {"yes": True}}},
    "d": {"type": "noul", "instructions": "plain noul"},
    "one": {"type": "choice", "instructions": "Choose", "criteria": ["only"]},
    "two": {"type": "choice", "instructions": "Pick [MASK] one", "criteria": ["left", "right"]},
    "many": {"type": "choice", "instructions": "Choose " * 30, "criteria": {str(i): "long " * 20 for i in range(12)}},
}
STATES = ["", "支付😀退款 café [MASK] refund", {"turns": ["hello", False, 3.5]}, "boundary " * 400, "short"]


def cases(laya_module):
    Laya, question = laya_module.Laya, laya_module.question
    out = {"questions": {}, "prepare": [], "decode": [], "errors": []}
    for qid, q in QUESTIONS.items():
        kind, instruction, criteria, options = question(q)
        out["questions"][qid] = {"kind": kind, "instruction": instruction, "options": options}
    return out


def generate(reference_root):
    spec = importlib.util.spec_from_file_location(
        "ref_laya_cuda", Path(reference_root) / "laya_cuda/__init__.py",
        submodule_search_locations=[str(Path(reference_root) / "laya_cuda")])
    package = importlib.util.module_from_spec(spec)
    sys.modules["ref_laya_cuda"] = package
    spec.loader.exec_module(package)
    ref = importlib.import_module("ref_laya_cuda.laya")
    import tempfile
    with tempfile.TemporaryDirectory() as tmp:
        adapter = ref.Laya(golden_checkpoint(tmp))
        data = cases(ref)
        for s, state in enumerate(STATES):
            for names in (["a", "b", "c", "d", "one", "two"], ["many"], ["two", "many", "one"]):
                qs = {n: QUESTIONS[n] for n in names}
                items = adapter.prepare(state, qs)
                data["prepare"].append({"state": state, "questions": names, "items": [list(map(list, i[:2])) + [i[2]]
                                                                                      for i in items]})
                rng = np.random.default_rng(s * 7 + len(names))
                k = max(len(i[1]) for i in items)
                logits = rng.normal(0, 2, (len(items), k)).astype(np.float32)
                acts = rng.normal(0, 2, (len(items), 2)).astype(np.float32)
                answer = adapter.decode(logits, acts, qs, items)
                data["decode"].append({"questions": names, "items": [[i[0], i[1], i[2]] for i in items],
                                       "logits": logits.tolist(), "acts": acts.tolist(), "answer": answer})
        for label, state, qs in [("empty", "x", {}), ("badtype", "x", {"q": {"type": "rank", "instructions": "i"}}),
                                 ("nocriteria", "x", {"q": {"type": "choice", "instructions": "i", "criteria": []}}),
                                 ("scoredict", "x", {"q": {"type": "score", "instructions": "i", "criteria": {"a": 1}}}),
                                 ("noullist", "x", {"q": {"type": "noul", "instructions": "i", "criteria": [1]}})]:
            try:
                adapter.prepare(state, qs)
                data["errors"].append({"label": label, "error": None})
            except Exception as error:  # noqa: BLE001 - recorded as data
                data["errors"].append({"label": label, "error": type(error).__name__, "message": str(error)})
        nonfinite = np.array([[np.nan, 1.0]], np.float32)
        try:
            adapter.decode(nonfinite, np.zeros((1, 2), np.float32), {"q": QUESTIONS["two"]}, [([1], [0], 0)])
        except Exception as error:  # noqa: BLE001
            data["errors"].append({"label": "nonfinite", "error": type(error).__name__, "message": str(error)})
    (HERE / "contract.json").write_text(json.dumps(data, ensure_ascii=False, indent=0))
    return data


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/laya-cuda")
    generate(sys.argv[1])
