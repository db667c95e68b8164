"""Laya decision-model adapter: checkpoint validation, the request contract and decoding.

The request contract (question parsing, tokenisation, sequence and marker construction,
budgets) and the decoding (temperature-calibrated softmax, confidence, answer dict) define
token counts and answers, so they follow the reference adapter exactly
(laya_cuda/laya.py:17-165); golden fixtures generated from it pin them
(tests/golden/contract.json).  The device forward pass lives in liblaya_b200.so.
"""
from concurrent.futures import ThreadPoolExecutor
import hashlib
import json
import math
import os
from threading import Lock

import numpy as np

from .models import read_json

# A request holds a few short texts and one state text; handing them to the tokenizer's thread
# pool costs more than encoding them on the calling thread (a 6-text, 83-word request: ~310 us
# through the pool, ~55 us without it).  A process that sets the variable keeps its own choice.
os.environ.setdefault("TOKENIZERS_PARALLELISM", "false")

# Several requests at once (a burst taken by BatchEngine) are encoded on helper threads, one
# task per request: the tokenizer releases the GIL while it encodes, so they run in parallel (a
# config-5-shaped request of ~640 words: ~710 us on one thread, ~230 us each with four).  Only
# the tokenizer runs there; the calling thread parses the questions and builds the items.
TOKENIZE_THREADS = max(2, min(4, (os.cpu_count() or 2) // 2))
_helpers, _helpers_pid, _helpers_lock = None, None, Lock()


def _tokenize_helpers():
    """The process's helper threads (a forked child makes its own: it inherits none)."""
    global _helpers, _helpers_pid
    with _helpers_lock:
        if _helpers is None or _helpers_pid != os.getpid():
            _helpers = ThreadPoolExecutor(TOKENIZE_THREADS, thread_name_prefix="laya-tokenize")
            _helpers_pid = os.getpid()
        return _helpers

TYPES = ("choice", "score", "noul")
NOUL_DEFAULTS = (("false", "no, the statement does not hold"), ("true", "yes, the statement holds"))


def text(value):
    """Strings pass through; anything else is JSON (non-ASCII kept, str() for the rest)."""
    return value if isinstance(value, str) else json.dumps(value, ensure_ascii=False, default=str)


def _choice_options(criteria):
    if isinstance(criteria, list):
        criteria = dict.fromkeys(criteria)
    if not isinstance(criteria, dict) or not all(isinstance(k, str) for k in criteria):
        raise ValueError("Choice criteria must be a mapping or list of string labels")
    options = []
    for label, detail in criteria.items():
        options.append(label if detail is None or detail == "" else f"{label}: {text(detail)}")
    return criteria, options


def _score_options(criteria):
    if not isinstance(criteria, list):
        raise ValueError("Score criteria must be a list")
    return criteria, [f"level {i}: {text(v)}" for i, v in enumerate(criteria)]


def _noul_options(criteria):
    criteria = criteria or {}
    if not isinstance(criteria, dict):
        raise ValueError("Noul criteria must be a mapping")
    options = []
    for key, default in NOUL_DEFAULTS:
        given = criteria.get(key)
        options.append(f"{key}: {default if given in (None, '') else text(criteria[key])}")
    return criteria, options


def question(value):
    """(kind, instruction, criteria, options) of one question definition (laya.py:21-45)."""
    kind, instruction, criteria = value["type"], value["instructions"], value.get("criteria")
    if kind not in TYPES:
        raise ValueError(f"Unsupported question type: {kind}")
    build = {"choice": _choice_options, "score": _score_options, "noul": _noul_options}[kind]
    criteria, options = build(criteria)
    if not options:
        raise ValueError("Each question must have at least one option")
    if not isinstance(instruction, str):
        instruction = json.dumps(instruction)
    return kind, instruction, criteria, options


def softmax(values):
    """Numerically stable fp32 softmax over the last axis."""
    values = np.asarray(values, np.float32)
    shifted = np.exp(values - values.max(axis=-1, keepdims=True))
    return shifted / shifted.sum(axis=-1, keepdims=True)


def _bucket(count):
    if count <= 2:
        return "2"
    if count <= 5:
        return "3-5"
    return "6-10" if count <= 10 else "11+"


class Laya:
    """ModernBERT/mmBERT encoder + decision head checkpoint (laya.py:54-99)."""

    def __init__(self, path):
        from tokenizers import Tokenizer
        self.path = path
        self.cfg = read_json(path / "rl_agent_config.json")
        self.config = c = read_json(path / "encoder/config.json")
        if c.get("model_type") != "modernbert" or c.get("hidden_activation", "gelu") != "gelu":
            raise ValueError("Only ModernBERT/mmBERT with exact GELU is supported")
        self.width, self.heads = c["hidden_size"], c["num_attention_heads"]
        if self.width % self.heads or self.width // self.heads != 64:
            raise ValueError("v1 requires 64-wide attention heads")
        if any(c.get(flag, False) for flag in ("attention_bias", "mlp_bias", "norm_bias", "rope_scaling")):
            raise ValueError("Biased or scaled-RoPE encoder variants are unsupported")
        self.layers, self.intermediate = c["num_hidden_layers"], c["intermediate_size"]
        self.ff_width = max(2 * self.intermediate, 4 * self.width)
        self.global_every = c.get("global_attn_every_n_layers", 3)
        self.window = c.get("local_attention", 128) // 2
        topology = ["full_attention" if i % self.global_every == 0 else "sliding_attention" for i in range(self.layers)]
        if c.get("layer_types", topology) != topology:
            raise ValueError("Unsupported attention topology")
        self.theta = self._rope_thetas(c)
        self.eps = float(c.get("norm_eps", 1e-5))
        self.max_len, self.head_max_len = self.cfg["max_len"], self.cfg["head_max_len"]
        self.head_layers = self.cfg["head_layers"]
        self.n_act = len(self.cfg.get("act_costs", {})) + 1
        if not 0 < self.max_len <= min(1024, c["max_position_embeddings"]) or self.head_layers < 1:
            raise ValueError("Invalid context budget or decision head")
        self.tokenizer = Tokenizer.from_file(str(path / "tokenizer/tokenizer.json"))
        self.tokenizer.no_padding()
        self.tokenizer.no_truncation()
        self._load_specials()

    @staticmethod
    def _rope_thetas(c):
        thetas = []
        for kind, default, legacy in (("full_attention", 160000, "global_rope_theta"),
                                      ("sliding_attention", 10000, "local_rope_theta")):
            rope = c.get("rope_parameters", {}).get(kind, {})
            if rope.get("rope_type", "default") != "default":
                raise ValueError("Only default RoPE is supported")
            thetas.append(float(rope.get("rope_theta", c.get(legacy, default)) or thetas[0]))
        return thetas

    def _load_specials(self):
        specials = {}
        for name in ("tokenizer_config.json", "special_tokens_map.json"):
            file = self.path / "tokenizer" / name
            if file.is_file():
                specials.update(read_json(file))
        for key in ("cls", "sep", "mask", "pad"):
            token = specials.get(key + "_token")
            if isinstance(token, dict):
                token = token.get("content")
            value = self.tokenizer.token_to_id(token) if isinstance(token, str) else None
            if value is None:
                raise ValueError(f"Missing tokenizer special token: {key}")
            setattr(self, key, value)
            if key == "mask":
                self.mask_text = token

    def encode(self, value):
        return self.tokenizer.encode(value.replace(self.mask_text, " "), add_special_tokens=False).ids

    def _encode_all(self, texts):
        texts = [v.replace(self.mask_text, " ") for v in texts]
        # Each text is encoded independently, so one batch call gives the same ids as per-text
        # calls; the "fast" batch path skips offset tracking, which the contract never reads.
        fast = getattr(self.tokenizer, "encode_batch_fast", None)
        if fast is not None:
            return [e.ids for e in fast(texts, add_special_tokens=False)]
        return [e.ids for e in self.tokenizer.encode_batch(texts, add_special_tokens=False)]

    def prepare(self, state, questions):
        """One (ids, markers, kind) item per question (laya.py:104-135):
        [CLS] question [SEP] ([MASK] option)... [SEP] state [SEP], truncated to max_len."""
        parsed, texts = self._texts(state, questions)
        return self._items(questions, parsed, self._encode_all(texts))

    def prepare_many(self, requests):
        """prepare() of several (state, questions) requests: per request its items, or the
        exception prepare() raises for it.  Each request's texts are encoded on a helper thread
        while this thread builds the items of the requests already encoded (same ids: the
        tokenizer encodes every text independently)."""
        results, work = [None] * len(requests), []
        for i, (state, questions) in enumerate(requests):
            try:
                parsed, texts = self._texts(state, questions)
            except Exception as error:
                results[i] = error
                continue
            work.append((i, questions, parsed, _tokenize_helpers().submit(self._encode_all, texts)))
        for i, questions, parsed, encoded in work:
            try:
                results[i] = self._items(questions, parsed, encoded.result())
            except Exception as error:
                results[i] = error
        return results

    def _texts(self, state, questions):
        """The parsed questions and the texts to encode: the state, then per question its
        heading and its options."""
        if not isinstance(questions, dict) or not questions:
            raise ValueError("Provide a nonempty mapping of questions")
        parsed = [question(definition) for definition in questions.values()]
        texts = [state if isinstance(state, str) else json.dumps(state, ensure_ascii=False)]
        for kind, instruction, _, options in parsed:
            texts.append(f"{kind} question: {instruction}")
            texts.extend(" " + option for option in options)
        return parsed, texts

    def _items(self, questions, parsed, encoded):
        """The items of one request from its encoded texts (in _texts' order)."""
        encoded = iter(encoded)
        state_ids = next(encoded)
        items = []
        for qid, (kind, _, _, options) in zip(questions, parsed):
            head = next(encoded)
            opts = [[self.mask] + next(encoded)[:48] for _ in options]
            budget = self.head_max_len - sum(len(o) for o in opts)
            if budget < 16:
                cap = max(4, (self.head_max_len - 16) // len(opts))
                opts = [o[:cap] for o in opts]
                budget = self.head_max_len - sum(len(o) for o in opts)
            ids = [self.cls] + head[:max(8, budget)] + [self.sep]
            markers = []
            for option in opts:
                markers.append(len(ids))
                ids += option
            ids.append(self.sep)
            room = max(0, self.max_len - len(ids) - 1)
            ids.extend(state_ids[:room])  # in place: ids is this item's own list
            ids.append(self.sep)
            del ids[self.max_len:]
            if markers[-1] >= len(ids):
                raise ValueError(f"Question {qid!r} exceeds the option token budget")
            items.append((ids, markers, TYPES.index(kind)))
        return items

    def _temperature(self, kind, count):
        qt = TYPES.index(kind)
        fallback = self.cfg.get("temperature", [1] * 3)[qt]
        value = self.cfg.get("temperature_by_options", {}).get(f"{kind}:{_bucket(count)}", fallback)
        try:
            value = float(value)
        except (TypeError, ValueError):
            return 1.0
        # Scalar clamp: the value np.clip gives a finite float, without its per-call setup.
        return min(max(value, .5), 5.0) if math.isfinite(value) else 1.0

    def decode_plan(self, questions):
        """The parts of decode() that need no model output: per question (id, kind, criteria,
        option count, calibration temperature)."""
        plan = []
        for qid, definition in questions.items():
            kind, _, criteria, options = question(definition)
            plan.append((qid, kind, criteria, len(options), self._temperature(kind, len(options))))
        return plan

    def decode(self, logits, acts, questions, items, plan=None):
        """Answer dict of the SDK (laya.py:137-165) from option logits [b, >=k] and action logits.
        `plan` is decode_plan(questions), when the caller computed it already."""
        if not np.isfinite(logits).all() or not np.isfinite(acts).all():
            raise RuntimeError("Non-finite model output; no decision returned")
        actions, answers = softmax(acts), {}
        for row, (qid, kind, criteria, count, temp) in enumerate(plan if plan is not None else self.decode_plan(questions)):
            prob = softmax(logits[row, :count].astype(np.float32) / np.float32(temp))
            if count > 1:
                entropy = (prob * np.log(np.maximum(prob, 1e-12))).sum()
                conf = float(min(max(1 + entropy / math.log(count), 0), 1))  # finite: as np.clip
            else:
                conf = 1.0
            answer = {"type": kind, "confidence": round(conf, 4),
                      "action": {"act_probability": round(float(actions[row, 0]), 4)}}
            if kind == "noul":
                yes = float(prob[1])
                answer.update(noul=round(yes, 4), confidence=round(float(max(prob[1], 1 - prob[1])), 4))
            else:
                keys = list(criteria) if kind == "choice" else [str(i) for i in range(count)]
                answer["probabilities"] = {key: round(p, 4) for key, p in zip(keys, prob.tolist())}
                if kind == "choice":
                    answer["choice"] = keys[int(prob.argmax())]
                else:
                    answer.update(score=round(float(np.arange(count) @ prob), 4), legend=dict(zip(keys, criteria)))
            answers[qid] = answer
        usage = {"input_tokens": sum(len(item[0]) for item in items), "output_tokens": 0}
        return {"model": "laya-rl-agent", "answers": answers, "usage": usage}

    def weight_shapes(self):
        """Checkpoint tensor names and shapes (laya.py:167-190)."""
        w, f = self.width, self.intermediate
        shapes = {"encoder.embeddings.tok_embeddings.weight": (self.config["vocab_size"], w),
                  "encoder.embeddings.norm.weight": (w,), "encoder.final_norm.weight": (w,),
                  "type_emb.weight": (3, w), "temperature": (3,),
                  "scorer.0.weight": (w,), "scorer.0.bias": (w,), "scorer.1.weight": (w, w),
                  "scorer.1.bias": (w,), "scorer.3.weight": (1, w), "scorer.3.bias": (1,),
                  "act_head.0.weight": (256, w + 4), "act_head.0.bias": (256,),
                  "act_head.2.weight": (self.n_act, 256), "act_head.2.bias": (self.n_act,)}
        for i in range(self.layers):
            p = f"encoder.layers.{i}."
            shapes[p + "attn.Wqkv.weight"] = (3 * w, w)
            shapes[p + "attn.Wo.weight"] = (w, w)
            shapes[p + "mlp.Wi.weight"] = (2 * f, w)
            shapes[p + "mlp.Wo.weight"] = (w, f)
            shapes[p + "mlp_norm.weight"] = (w,)
            if i:
                shapes[p + "attn_norm.weight"] = (w,)
        for i in range(self.head_layers):
            p = f"head.layers.{i}."
            for name, shape in (("self_attn.in_proj_weight", (3 * w, w)), ("self_attn.in_proj_bias", (3 * w,)),
                                ("self_attn.out_proj.weight", (w, w)), ("self_attn.out_proj.bias", (w,)),
                                ("linear1.weight", (4 * w, w)), ("linear1.bias", (4 * w,)),
                                ("linear2.weight", (w, 4 * w)), ("linear2.bias", (w,)),
                                ("norm1.weight", (w,)), ("norm1.bias", (w,)),
                                ("norm2.weight", (w,)), ("norm2.bias", (w,))):
                shapes[p + name] = shape
        return shapes

    def fingerprint(self, items):
        """sha256 of the items' compact JSON (laya.py:192-193), built directly: for lists of
        ints the text equals json.dumps(items, separators=(",", ":")) at a third of the cost."""
        text = ",".join(f"[[{','.join(map(str, ids))}],[{','.join(map(str, markers))}],{int(kind)}]"
                        for ids, markers, kind in items)
        return hashlib.sha256(f"[{text}]".encode()).hexdigest()

    def official(self, device):
        from .official import Official
        return Official(self.path, device)
