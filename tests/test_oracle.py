"""Pins the FP32 oracle before it is trusted as the parity reference.

The reference's own GPU path cannot run in this image (it needs CuPy), so the oracle is pinned
against independent implementations of the same architecture (transformers ModernBERT for the
encoder, torch's pre-norm TransformerEncoderLayer for the head layer) and against the in-test
formulas the reference's kernel tests use (tests/test_gpu.py, tests/test_attention.py).
"""
import math

import numpy as np
import pytest

from laya_cuda import synthetic as S
from oracle import laya_oracle as O

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def small():
    arch = S.architecture("small")
    return arch, S.make_weights(arch, seed=3, scale=0.05)


def test_encoder_matches_transformers_modernbert(small):
    transformers = pytest.importorskip("transformers")
    arch, w = small
    types = ["full_attention" if i % arch["global_every"] == 0 else "sliding_attention" for i in range(arch["layers"])]
    cfg = transformers.ModernBertConfig(
        vocab_size=arch["vocab"], hidden_size=arch["width"], intermediate_size=arch["intermediate"],
        num_hidden_layers=arch["layers"], num_attention_heads=arch["heads"], layer_types=types,
        local_attention=arch["local_attention"], norm_eps=arch["eps"], pad_token_id=0, hidden_activation="gelu",
        rope_parameters={"full_attention": {"rope_type": "default", "rope_theta": arch["theta_global"]},
                         "sliding_attention": {"rope_type": "default", "rope_theta": arch["theta_local"]}},
        max_position_embeddings=8192, attention_dropout=0.0, embedding_dropout=0.0, mlp_dropout=0.0)
    cfg._attn_implementation = "eager"
    model = transformers.ModernBertModel(cfg).eval()
    state = {k[len("encoder."):]: torch.from_numpy(v) for k, v in w.items() if k.startswith("encoder.")}
    missing, unexpected = model.load_state_dict(state, strict=False)
    assert not unexpected and not [m for m in missing if "rotary" not in m and "inv_freq" not in m]
    ids = np.random.default_rng(0).integers(5, arch["vocab"], 200)
    with torch.no_grad():
        ours = model(input_ids=torch.from_numpy(ids)[None]).last_hidden_state[0].double().numpy()
    oracle = O.Oracle(w, arch, np.float64).encoder(ids.tolist())
    # 200 tokens > the 129-key local window, so the sliding-window layers are exercised.
    assert np.max(np.abs(ours - oracle)) < 2e-4


def test_head_layer_matches_torch_transformer_layer(small):
    arch, w = small
    d, h = arch["width"], arch["heads"]
    layer = torch.nn.TransformerEncoderLayer(d, h, 4 * d, dropout=0.0, activation="relu", batch_first=True,
                                             norm_first=True, layer_norm_eps=1e-5).double().eval()
    p = "head.layers.0."
    sd = {"self_attn.in_proj_weight": p + "self_attn.in_proj_weight", "self_attn.in_proj_bias": p + "self_attn.in_proj_bias",
          "self_attn.out_proj.weight": p + "self_attn.out_proj.weight", "self_attn.out_proj.bias": p + "self_attn.out_proj.bias",
          "linear1.weight": p + "linear1.weight", "linear1.bias": p + "linear1.bias", "linear2.weight": p + "linear2.weight",
          "linear2.bias": p + "linear2.bias", "norm1.weight": p + "norm1.weight", "norm1.bias": p + "norm1.bias",
          "norm2.weight": p + "norm2.weight", "norm2.bias": p + "norm2.bias"}
    layer.load_state_dict({k: torch.from_numpy(w[v]).double() for k, v in sd.items()})
    x = np.random.default_rng(1).normal(0, 1, (77, d))
    with torch.no_grad():
        expected = layer(torch.from_numpy(x)[None])[0].numpy()
    oracle = O.Oracle(w, arch, np.float64)
    np.testing.assert_allclose(oracle.head_layer(x, 0), expected, atol=1e-10)
    picks = [0, 5, 9, 13]
    np.testing.assert_allclose(oracle.head_layer(x, 0, picks), expected[picks], atol=1e-10)


def test_rope_matches_reference_test_formula():
    """tests/test_gpu.py:36-53: x*cat(cos,cos) + cat(-x[32:], x[:32])*cat(sin,sin), with the
    tables built as the runtime builds them (runtime.py:163-164: angle = pos * (1 / theta^e);
    the reference test divides instead, which differs by an ulp in some angles)."""
    rng = np.random.default_rng(17)
    x = rng.normal(size=(768, 2, 64)).astype(np.float32)
    freq = 1 / (np.float32(10000) ** (np.arange(0, 64, 2, dtype=np.float32) / 64))
    angle = np.arange(768, dtype=np.float32)[:, None] * freq
    cos, sin = np.cos(angle), np.sin(angle)
    ours = O.rotate(x, *O.rope_tables(10000, 768))
    rotated = np.concatenate((-x[..., 32:], x[..., :32]), axis=-1)
    expected = x * np.concatenate((cos, cos), -1)[:, None] + rotated * np.concatenate((sin, sin), -1)[:, None]
    np.testing.assert_array_equal(ours, expected)


@pytest.mark.parametrize("n,window", [(32, -1), (96, 64), (250, 64), (500, 64), (333, -1)])
def test_attention_matches_reference_test_oracle(n, window):
    """tests/test_attention.py:47-53 (float64, mask |i-j| > window)."""
    x = np.random.default_rng(n).normal(0, 1, (n, 3, 2, 64))
    q, k, v = x.transpose(1, 0, 2, 3)
    ours = O.attention(q, k, v, window)
    qq, kk, vv = x.transpose(1, 2, 0, 3)
    s = qq @ kk.transpose(0, 2, 1) / 8
    if window >= 0:
        s[:, np.abs(np.arange(n)[:, None] - np.arange(n)) > window] = -np.inf
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    np.testing.assert_allclose(ours, (p @ vv).transpose(1, 0, 2).reshape(n, 128), atol=1e-12)


def test_layernorm_matches_reference_test_formula():
    """tests/test_gpu.py:68-75 / 96-103: (x-mean)/sqrt(var+eps)*gamma+beta."""
    rng = np.random.default_rng(11)
    x = rng.normal(2, .3, (3, 768))
    g, b = rng.normal(1, .1, 768), rng.normal(0, .1, 768)
    expected = (x - x.mean(-1, keepdims=True)) / np.sqrt(x.var(-1, keepdims=True) + 1e-5) * g + b
    np.testing.assert_allclose(O.layer_norm(x, g, b), expected, atol=1e-12)


def test_features_match_reference_scan():
    """kernels.cu:167-183: serial top-2 scan, entropy with p clamped at 1e-9."""
    oracle = O.Oracle({}, dict(max_len=16, theta_global=1e4, theta_local=1e4), np.float64)
    for logits in ([1.0, 2.0, 2.0, -1.0], [3.0], [0.5, -0.5], [0.0] * 9, []):
        logits = np.array(logits)
        top, total, p1, p2, entropy = -math.inf, 0.0, 0.0, 0.0, 0.0
        for v in logits:
            top = max(top, v)
        for v in logits:
            total += math.exp(v - top)
        for v in logits:
            pv = math.exp(v - top) / total
            entropy -= pv * math.log(max(pv, 1e-9))
            if pv > p1:
                p2, p1 = p1, pv
            else:
                p2 = max(p2, pv)
        c2 = max(len(logits), 2)
        np.testing.assert_allclose(oracle.features(logits), [p1, p1 - p2, entropy / math.log(c2), c2 / 255], atol=1e-12)


def test_full_forward_is_finite_and_deterministic(small):
    arch, w = small
    oracle = O.Oracle(w, arch)
    rng = np.random.default_rng(4)
    items = [S.build_item(rng, 150, 5, arch["vocab"], kind=1), S.build_item(rng, 40, 3, arch["vocab"])]
    a, b = oracle.predict(items), oracle.predict(items)
    for (la, aa), (lb, ab), item in zip(a, b, items):
        assert la.shape == (len(item[1]),) and aa.shape == (arch["n_act"],)
        assert np.isfinite(la).all() and np.isfinite(aa).all()
        np.testing.assert_array_equal(la, lb)
        np.testing.assert_array_equal(aa, ab)
