"""Seeded synthetic checkpoints and workloads for benchmarks and tests.

No trained checkpoint or dataset is available offline, so the benchmark configurations run on
random-init checkpoints with each registered architecture's geometry: matrices, embeddings and
biases ~ N(0, 0.02), LayerNorm weights ~ 1 + N(0, 0.02).  A checkpoint directory is complete
(model.safetensors, encoder/config.json, rl_agent_config.json, tokenizer/), so the registry,
adapter and Engine load it unchanged.  The tokenizer is a whitespace WordLevel vocabulary in
which token id i (i >= 5) is the word "w<i>", so a request text maps to known ids exactly.
"""
import json
from pathlib import Path

import numpy as np

SPECIALS = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"]
PAD, UNK, CLS, SEP, MASK = range(5)
FIRST_WORD = len(SPECIALS)

ARCHITECTURES = {
    # The three registered aliases (models.json); dims per the benchmark configurations.
    "laya": dict(vocab=50368, width=768, heads=12, layers=12, intermediate=3072, max_len=512),
    "laya-multilingual": dict(vocab=250000, width=768, heads=12, layers=12, intermediate=3072, max_len=1024),
    "laya-typed-decisions": dict(vocab=50368, width=768, heads=12, layers=12, intermediate=3072, max_len=1024),
    # Small geometries for CPU tests.
    "tiny": dict(vocab=512, width=64, heads=1, layers=3, intermediate=128, max_len=128),
    "small": dict(vocab=2048, width=128, heads=2, layers=4, intermediate=256, max_len=256),
}


def word(i):
    return f"w{i}"


def architecture(name, **overrides):
    arch = dict(ARCHITECTURES[name])
    arch.update(head_layers=1, head_max_len=256, global_every=3, local_attention=128,
                theta_global=160000.0, theta_local=10000.0, eps=1e-5, n_act=2)
    arch.update(overrides)
    return arch


def encoder_config(arch):
    return {"model_type": "modernbert", "hidden_size": arch["width"], "num_attention_heads": arch["heads"],
            "num_hidden_layers": arch["layers"], "intermediate_size": arch["intermediate"],
            "vocab_size": arch["vocab"], "max_position_embeddings": 8192, "hidden_activation": "gelu",
            "global_attn_every_n_layers": arch["global_every"], "local_attention": arch["local_attention"],
            "global_rope_theta": arch["theta_global"], "local_rope_theta": arch["theta_local"],
            "norm_eps": arch["eps"], "attention_bias": False, "mlp_bias": False, "norm_bias": False,
            "pad_token_id": PAD, "cls_token_id": CLS, "sep_token_id": SEP}


def agent_config(arch):
    costs = {f"act{i}": 0.1 for i in range(arch["n_act"] - 1)}
    return {"max_len": arch["max_len"], "head_max_len": arch["head_max_len"], "head_layers": arch["head_layers"],
            "act_costs": costs, "temperature": [1.0, 1.0, 1.0]}


def weight_shapes(arch):
    w, f = arch["width"], arch["intermediate"]
    shapes = {"encoder.embeddings.tok_embeddings.weight": (arch["vocab"], w),
              "encoder.embeddings.norm.weight": (w,), "encoder.final_norm.weight": (w,),
              "type_emb.weight": (3, w), "temperature": (3,),
              "scorer.0.weight": (w,), "scorer.0.bias": (w,), "scorer.1.weight": (w, w), "scorer.1.bias": (w,),
              "scorer.3.weight": (1, w), "scorer.3.bias": (1,), "act_head.0.weight": (256, w + 4),
              "act_head.0.bias": (256,), "act_head.2.weight": (arch["n_act"], 256), "act_head.2.bias": (arch["n_act"],)}
    for i in range(arch["layers"]):
        p = f"encoder.layers.{i}."
        shapes.update({p + "attn.Wqkv.weight": (3 * w, w), p + "attn.Wo.weight": (w, w),
                       p + "mlp.Wi.weight": (2 * f, w), p + "mlp.Wo.weight": (w, f), p + "mlp_norm.weight": (w,)})
        if i:
            shapes[p + "attn_norm.weight"] = (w,)
    for i in range(arch["head_layers"]):
        p = f"head.layers.{i}."
        shapes.update({p + "self_attn.in_proj_weight": (3 * w, w), p + "self_attn.in_proj_bias": (3 * w,),
                       p + "self_attn.out_proj.weight": (w, w), p + "self_attn.out_proj.bias": (w,),
                       p + "linear1.weight": (4 * w, w), p + "linear1.bias": (4 * w,),
                       p + "linear2.weight": (w, 4 * w), p + "linear2.bias": (w,),
                       p + "norm1.weight": (w,), p + "norm1.bias": (w,), p + "norm2.weight": (w,),
                       p + "norm2.bias": (w,)})
    return shapes


def make_weights(arch, seed=0, scale=0.02):
    """Random-init weights in a fixed (sorted-name) order, so a seed names one checkpoint."""
    rng = np.random.default_rng(seed)
    weights = {}
    for name, shape in sorted(weight_shapes(arch).items()):
        if name == "temperature":
            weights[name] = np.ones(shape, np.float32)
            continue
        values = rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)
        if "norm" in name and name.endswith("weight") or name == "scorer.0.weight":
            values += np.float32(1.0)
        weights[name] = values
    return weights


def write_tokenizer(directory, vocab):
    from tokenizers import Tokenizer, models, pre_tokenizers
    directory.mkdir(parents=True, exist_ok=True)
    table = {tok: i for i, tok in enumerate(SPECIALS)}
    table.update({word(i): i for i in range(FIRST_WORD, vocab)})
    tokenizer = Tokenizer(models.WordLevel(table, unk_token="[UNK]"))
    tokenizer.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tokenizer.save(str(directory / "tokenizer.json"))
    (directory / "tokenizer_config.json").write_text(json.dumps(
        {"cls_token": "[CLS]", "sep_token": "[SEP]", "mask_token": "[MASK]", "pad_token": "[PAD]",
         "unk_token": "[UNK]"}))


def write_checkpoint(path, arch, seed=0, scale=0.02, weights=None):
    """Writes a complete checkpoint directory; returns its Path."""
    from safetensors.numpy import save_file
    path = Path(path)
    (path / "encoder").mkdir(parents=True, exist_ok=True)
    (path / "encoder/config.json").write_text(json.dumps(encoder_config(arch)))
    (path / "rl_agent_config.json").write_text(json.dumps(agent_config(arch)))
    write_tokenizer(path / "tokenizer", arch["vocab"])
    save_file(weights if weights is not None else make_weights(arch, seed, scale), str(path / "model.safetensors"))
    return path


def cached_checkpoint(root, name, seed=0, **overrides):
    """A checkpoint for architecture `name` under `root`, written once per (name, seed, overrides)."""
    arch = architecture(name, **overrides)
    tag = "-".join([name, f"s{seed}"] + [f"{k}{v}" for k, v in sorted(overrides.items())])
    path = Path(root) / tag
    if not (path / "model.safetensors").is_file():
        tmp = Path(root) / (tag + ".tmp")
        write_checkpoint(tmp, arch, seed)
        tmp.rename(path)
    return path


# ---------------------------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------------------------
def draw_ids(rng, n, vocab, zipf=None):
    """n token ids in [5, vocab): uniform, or Zipf(a) ranks (scattered embedding reads)."""
    if zipf is None:
        return rng.integers(FIRST_WORD, vocab, n).tolist()
    ranks = rng.zipf(zipf, n)
    return np.clip(ranks + FIRST_WORD - 1, FIRST_WORD, vocab - 1).tolist()


def build_item(rng, length, options, vocab, kind=0, question_len=8, zipf=None, option_len=(2, 4)):
    """(ids, markers, kind) of exactly `length` tokens:
    [CLS] question [SEP] ([MASK] option)... [SEP] state [SEP] (the adapter's sequence layout)."""
    ids = [CLS] + draw_ids(rng, question_len, vocab, zipf) + [SEP]
    markers = []
    for _ in range(options):
        markers.append(len(ids))
        ids += [MASK] + draw_ids(rng, int(rng.integers(option_len[0], option_len[1] + 1)), vocab, zipf)
    ids.append(SEP)
    state = length - len(ids) - 1
    if state < 0:
        raise ValueError(f"{options} options do not fit in {length} tokens")
    return ids + draw_ids(rng, state, vocab, zipf) + [SEP], markers, kind


def item_text(ids, markers):
    """(state, questions) texts that the adapter turns back into `ids` exactly (one question)."""
    close = len(ids) - 1
    first_marker = markers[0]
    instruction = " ".join(word(t) for t in ids[1:first_marker - 1])
    bounds = markers + [ids.index(SEP, markers[-1])]
    labels = [" ".join(word(t) for t in ids[a + 1:b]) for a, b in zip(bounds[:-1], bounds[1:])]
    state = " ".join(word(t) for t in ids[bounds[-1] + 1:close])
    return state, instruction, labels


def request_texts(rng, length, options, vocab, zipf=None):
    """An Engine.predict request (state, questions) whose single question tokenises to `length`
    ids.  The question header encodes as [UNK] [UNK] + instruction ("choice", "question:")."""
    ids, markers, _ = build_item(rng, length, options, vocab, question_len=6, zipf=zipf)
    # The adapter encodes its "choice question:" prefix as two unknown words.
    ids[1] = ids[2] = UNK
    state, instruction, labels = item_text(ids, markers)
    questions = {"q": {"type": "choice", "instructions": " ".join(instruction.split(" ")[2:]), "criteria": labels}}
    return state, questions, ids


def stream_requests(rng, count, vocab, max_len, lengths=(40, 900), questions=(1, 5), options=(4, 77)):
    """Mixed-shape request stream: per request a length, 1-5 questions of 4-77 options each."""
    out = []
    for _ in range(count):
        n_q = int(rng.integers(questions[0], questions[1] + 1))
        req = []
        length = int(rng.integers(lengths[0], lengths[1] + 1))
        for q in range(n_q):
            k = int(rng.integers(options[0], options[1] + 1))
            need = 3 + 8 + k * 5 + 2
            req.append(build_item(rng, min(max(length, need), max_len), k, vocab, kind=q % 3))
        out.append(req)
    return out


def throughput_requests(seed, count, vocab, lengths=(256, 1024), questions=3, options=8):
    """Throughput sweep: `count` requests, each `questions` sequences of one request length."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(count):
        length = int(rng.integers(lengths[0], lengths[1] + 1))
        out.append([build_item(rng, length, options, vocab, kind=q % 3) for q in range(questions)])
    return out


def stream_request_texts(rng, vocab, lengths=(40, 900), questions=(1, 5), options=(4, 77)):
    """One request of the mixed-shape stream as texts for Engine/BatchEngine: a state of
    U[lengths] words and U[questions] choice questions with U[options] labels of 1-3 words.
    The adapter's budgets and max_len truncation apply exactly as for real text."""
    state = " ".join(word(int(t)) for t in rng.integers(FIRST_WORD, vocab, int(rng.integers(lengths[0], lengths[1] + 1))))
    qs = {}
    for q in range(int(rng.integers(questions[0], questions[1] + 1))):
        k = int(rng.integers(options[0], options[1] + 1))
        labels = []
        while len(labels) < k:
            label = " ".join(word(int(t)) for t in rng.integers(FIRST_WORD, vocab, int(rng.integers(1, 4))))
            if label not in labels:
                labels.append(label)
        instruction = " ".join(word(int(t)) for t in rng.integers(FIRST_WORD, vocab, 6))
        qs[f"q{q}"] = {"type": "choice", "instructions": instruction, "criteria": labels}
    return state, qs

