"""Kernel-level parity of the sm_100a library against float64 / fp32 references.

Mirrors the reference's kernel tests (tests/test_gpu.py, tests/test_attention.py): GEMM with
every fused epilogue, RoPE layout, LayerNorm, embedding gather, packed varlen attention with
sliding windows and padding rows.  Device memory comes from torch (plumbing only); every kernel
runs through the C ABI.
"""
import ctypes as ct
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from laya_cuda import _lib  # noqa: E402
from laya_cuda.runtime import span  # noqa: E402

PRECISIONS = {"bf16": (_lib.PRECISION_BF16, torch.bfloat16), "f16": (_lib.PRECISION_F16, torch.float16)}
# Output rounding of one 16-bit value (relative); bf16 keeps 8 mantissa bits, f16 11.
ROUND = {"bf16": 2.0 ** -8, "f16": 2.0 ** -11}


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return _lib.load()


def ptr(t):
    return ct.c_void_p(t.data_ptr()) if t is not None else None


def stream():
    return ct.c_void_p(torch.cuda.current_stream().cuda_stream)


def gemm(lib, prec, epi, x, w, out=None, ldo=0, residual=None, ldr=0, bias=None, heads=0, rope_tab=None,
         positions=None, splits=1, block_n=0):
    """rope_tab: RoPE table [16][rope_rows][4] = (cos f_2k, cos f_2k+1, sin f_2k, sin f_2k+1), or None."""
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    M, K = x.shape
    N = w.shape[0]
    rope_rows = rope_tab.shape[1] if rope_tab is not None else 0
    _lib.check(lib.laya_op_gemm(PRECISIONS[prec][0], epi, ptr(x), ptr(w), M, N, K, ptr(out), ldo, ptr(residual), ldr,
                                ptr(bias), heads, ptr(rope_tab), rope_rows, ptr(positions), splits, block_n,
                                ptr(err), stream()))
    torch.cuda.synchronize()
    assert int(err.item()) == 0


def rand16(shape, prec, rng, scale=1.0):
    a = rng.normal(0, scale, shape).astype(np.float32)
    t = torch.from_numpy(a).to(PRECISIONS[prec][1])
    return t.cuda(), t.float().double().numpy()


@pytest.mark.parametrize("prec", ["bf16", "f16"])
@pytest.mark.parametrize("M,N,K,block_n", [(7, 64, 64, 0), (96, 768, 768, 0), (200, 2304, 768, 256),
                                           (513, 768, 3072, 128), (1000, 256, 768, 64), (128, 512, 256, 0)])
def test_gemm_store_matches_fp64(lib, prec, M, N, K, block_n):
    rng = np.random.default_rng(M + N + K)
    x, xd = rand16((M, K), prec, rng)
    w, wd = rand16((N, K), prec, rng, 0.05)
    bias = torch.from_numpy(rng.normal(0, 0.1, N).astype(np.float32)).cuda()
    out = torch.full((M, N), float("nan"), dtype=PRECISIONS[prec][1], device="cuda")
    gemm(lib, prec, 0, x, w, out, N, bias=bias, block_n=block_n)
    expected = xd @ wd.T + bias.double().cpu().numpy()
    got = out.double().cpu().numpy()
    tol = ROUND[prec] * np.abs(expected) + 1e-4 * math.sqrt(K)
    assert np.all(np.abs(got - expected) <= tol), float(np.max(np.abs(got - expected) - tol))


@pytest.mark.parametrize("prec", ["bf16", "f16"])
@pytest.mark.parametrize("epi", [1, 2])
def test_gemm_relu_gelu_epilogues(lib, prec, epi):
    rng = np.random.default_rng(3 + epi)
    M, N, K = 150, 3072, 768
    x, xd = rand16((M, K), prec, rng)
    w, wd = rand16((N, K), prec, rng, 0.05)
    bias = torch.from_numpy(rng.normal(0, 0.1, N).astype(np.float32)).cuda()
    out = torch.empty((M, N), dtype=PRECISIONS[prec][1], device="cuda")
    gemm(lib, prec, epi, x, w, out, N, bias=bias)
    pre = xd @ wd.T + bias.double().cpu().numpy()
    expected = np.maximum(pre, 0) if epi == 1 else 0.5 * pre * (1 + np.vectorize(math.erf)(pre / math.sqrt(2)))
    got = out.double().cpu().numpy()
    assert np.max(np.abs(got - expected) - ROUND[prec] * np.abs(expected)) < 3e-3


@pytest.mark.parametrize("prec", ["bf16", "f16"])
@pytest.mark.parametrize("M,F", [(96, 3072), (333, 512)])
def test_gemm_geglu_epilogue(lib, prec, M, F):
    rng = np.random.default_rng(M)
    K = 768
    x, xd = rand16((M, K), prec, rng)
    w, wd = rand16((2 * F, K), prec, rng, 0.05)
    host = w.cpu().view(torch.int16).numpy().astype(np.uint16)
    inter = np.empty_like(host)
    _lib.check(lib.laya_interleave_geglu(host.ctypes.data, inter.ctypes.data, F, K))
    wi = torch.from_numpy(inter.view(np.int16)).view(PRECISIONS[prec][1]).cuda()
    out = torch.empty((M, F), dtype=PRECISIONS[prec][1], device="cuda")
    gemm(lib, prec, 3, x, wi, out, F)
    h = xd @ wd.T
    g, u = h[:, :F], h[:, F:]
    expected = 0.5 * g * (1 + np.vectorize(math.erf)(g / math.sqrt(2))) * u
    got = out.double().cpu().numpy()
    assert np.max(np.abs(got - expected) - ROUND[prec] * np.abs(expected)) < 3e-3


def rope_tables(theta, rows):
    freq = 1 / (np.float32(theta) ** (np.arange(0, 64, 2, dtype=np.float32) / 64))
    angle = np.arange(rows, dtype=np.float32)[:, None] * freq
    return np.cos(angle).astype(np.float32), np.sin(angle).astype(np.float32)


def rope_table_device(cos, sin):
    """[rows][32] cos/sin -> the kernel's table [16][rows][4] = (cos 2k, cos 2k+1, sin 2k, sin 2k+1)."""
    rows = cos.shape[0]
    tab = np.stack([cos[:, 0::2], cos[:, 1::2], sin[:, 0::2], sin[:, 1::2]], -1)  # [rows][16][4]
    return torch.from_numpy(np.ascontiguousarray(tab.transpose(1, 0, 2))).cuda()


@pytest.mark.parametrize("prec", ["bf16", "f16"])
@pytest.mark.parametrize("rope,M,block_n", [(True, 208, 0), (False, 208, 0), (True, 2320, -256), (False, 2320, -128),
                                            (True, 203, 0)])
def test_gemm_qkv_rope_layout(lib, prec, rope, M, block_n):
    """Encoder QKV (RoPE, no bias) and head in_proj (bias, no RoPE) epilogues, 1-CTA and CTA-pair
    kernels; cf. tests/test_gpu.py:36-53."""
    rng = np.random.default_rng(17)
    heads, K = 4, 128
    N = 3 * heads * 64
    x, xd = rand16((M, K), prec, rng)
    w, wd = rand16((N, K), prec, rng, 0.1)
    positions = (np.arange(M) % 112).astype(np.int32)
    cos, sin = rope_tables(10000, 128)
    bias = None if rope else torch.from_numpy(rng.normal(0, 0.1, N).astype(np.float32)).cuda()
    out = torch.full((3, heads, M, 64), float("nan"), dtype=PRECISIONS[prec][1], device="cuda")
    gemm(lib, prec, 4, x, w, out, heads=heads, rope_tab=rope_table_device(cos, sin) if rope else None,
         positions=torch.from_numpy(positions).cuda(), bias=bias, block_n=block_n)
    h = xd @ wd.T
    if bias is not None:
        h = h + bias.double().cpu().numpy()
    h = h.reshape(M, 3, heads, 64).transpose(1, 2, 0, 3).copy()       # [3][heads][M][64]
    if rope:
        c = np.concatenate([cos, cos], -1)[positions].astype(np.float64)
        s = np.concatenate([sin, sin], -1)[positions].astype(np.float64)
        for part in (0, 1):
            o = h[part]
            rot = np.concatenate([-o[..., 32:], o[..., :32]], -1)
            h[part] = o * c + rot * s
    got = out.double().cpu().numpy()
    # v is stored transposed: the buffer's third plane is [heads][64][M].
    got[2] = got[2].reshape(heads, 64, M).transpose(0, 2, 1)
    assert np.max(np.abs(got - h) - ROUND[prec] * np.abs(h)) < 2e-3


@pytest.mark.parametrize("prec", ["f16", "bf16"])
@pytest.mark.parametrize("epi,bn", [(0, -256), (0, -128), (2, -256), (3, -256), (3, -128), (5, -256), (5, -128)])
def test_gemm_cta_pair_kernel(lib, prec, epi, bn):
    """The cta_group::2 kernel (256-row tiles over a CTA pair), with a row count that leaves the
    second CTA of the last pair partly and wholly out of range."""
    rng = np.random.default_rng(abs(bn) + epi)
    M, K = 2500, 768
    N = 2048 if epi == 3 else 768
    x, xd = rand16((M, K), prec, rng)
    w, wd = rand16((N, K), prec, rng, 0.05)
    bias = torch.from_numpy(rng.normal(0, 0.1, N).astype(np.float32)).cuda() if epi in (0, 2, 5) else None
    h = xd @ wd.T + (bias.double().cpu().numpy() if bias is not None else 0)
    if epi == 3:
        host = w.cpu().view(torch.int16).numpy().astype(np.uint16)
        inter = np.empty_like(host)
        _lib.check(lib.laya_interleave_geglu(host.ctypes.data, inter.ctypes.data, N // 2, K))
        w = torch.from_numpy(inter.view(np.int16)).view(PRECISIONS[prec][1]).cuda()
        out = torch.empty((M, N // 2), dtype=PRECISIONS[prec][1], device="cuda")
        gemm(lib, prec, 3, x, w, out, N // 2, block_n=bn)
        g, u = h[:, :N // 2], h[:, N // 2:]
        expected = 0.5 * g * (1 + np.vectorize(math.erf)(g / math.sqrt(2))) * u
    elif epi == 5:
        base = rng.normal(0, 1, (M, N)).astype(np.float32)
        out = torch.from_numpy(base.copy()).cuda()
        gemm(lib, prec, 5, x, w, residual=out, ldr=N, bias=bias, block_n=bn)
        expected = base + h
        assert np.max(np.abs(out.cpu().double().numpy() - expected)) < 2e-4 * math.sqrt(K)
        return
    else:
        out = torch.full((M, N), float("nan"), dtype=PRECISIONS[prec][1], device="cuda")
        gemm(lib, prec, epi, x, w, out, N, bias=bias, block_n=bn)
        expected = h if epi == 0 else 0.5 * h * (1 + np.vectorize(math.erf)(h / math.sqrt(2)))
    got = out.double().cpu().numpy()
    assert np.max(np.abs(got - expected) - ROUND[prec] * np.abs(expected)) < 3e-3


@pytest.mark.parametrize("prec", ["bf16"])
@pytest.mark.parametrize("splits", [1, 3])
def test_gemm_residual_and_partials(lib, prec, splits):
    rng = np.random.default_rng(5)
    M, N, K = 300, 768, 3072
    x, xd = rand16((M, K), prec, rng)
    w, wd = rand16((N, K), prec, rng, 0.02)
    base = rng.normal(0, 1, (M, N)).astype(np.float32)
    bias = rng.normal(0, 0.1, N).astype(np.float32)
    residual = torch.from_numpy(base.copy()).cuda()
    gemm(lib, prec, 5, x, w, residual=residual, ldr=N, bias=torch.from_numpy(bias).cuda())
    expected = base + xd @ wd.T + bias
    assert np.max(np.abs(residual.cpu().numpy() - expected)) < 2e-4 * math.sqrt(K)
    partial = torch.zeros((splits, M, N), dtype=torch.float32, device="cuda")
    gemm(lib, prec, 6, x, w, residual=partial, ldr=N, splits=splits, block_n=64)
    assert np.max(np.abs(partial.sum(0).double().cpu().numpy() - xd @ wd.T)) < 2e-4 * math.sqrt(K)


@pytest.mark.parametrize("prec", ["bf16", "f16"])
@pytest.mark.parametrize("M,N,K,block_n,splits", [(128, 64, 320, 64, 1), (200, 128, 192, 128, 1), (96, 256, 448, 64, 1),
                                                  (300, 384, 1536, 128, 3), (64, 768, 768, 64, 3)])
def test_gemm_issuer_shares(lib, prec, M, N, K, block_n, splits):
    """Grids with one tile per CTA spread a tile's k-blocks over several MMA-issuing threads
    (4 for 64-column tiles, 2 for 128), each into its own accumulator: shares that do not divide
    evenly (5 k-blocks over 4 issuers, 3 over 2, 7 over 4), and split-K partials whose split
    ranges are shared out again, all against float64."""
    rng = np.random.default_rng(M + N + K + splits)
    x, xd = rand16((M, K), prec, rng)
    w, wd = rand16((N, K), prec, rng, 0.05)
    if splits == 1:
        bias = torch.from_numpy(rng.normal(0, 0.1, N).astype(np.float32)).cuda()
        out = torch.full((M, N), float("nan"), dtype=PRECISIONS[prec][1], device="cuda")
        gemm(lib, prec, 0, x, w, out, N, bias=bias, block_n=block_n)
        expected = xd @ wd.T + bias.double().cpu().numpy()
        got = out.double().cpu().numpy()
        tol = ROUND[prec] * np.abs(expected) + 1e-4 * math.sqrt(K)
        assert np.all(np.abs(got - expected) <= tol), float(np.max(np.abs(got - expected) - tol))
    else:
        partial = torch.zeros((splits, M, N), dtype=torch.float32, device="cuda")
        gemm(lib, prec, 6, x, w, residual=partial, ldr=N, splits=splits, block_n=block_n)
        assert np.max(np.abs(partial.sum(0).double().cpu().numpy() - xd @ wd.T)) < 2e-4 * math.sqrt(K)


def packed_case(lengths):
    starts = np.cumsum([0] + [span(n) for n in lengths])[:-1].astype(np.int32)
    M = span(sum(span(n) for n in lengths) + 16)  # include tokens past the last row
    return starts, np.asarray(lengths, np.int32), M


@pytest.mark.parametrize("prec,impl", [("f16", 1), ("bf16", 1), ("f16", 2), ("bf16", 2), ("f16", 3), ("bf16", 3),
                                       ("f16", 4), ("bf16", 4), ("f16", 5), ("bf16", 5), ("f16", 6), ("bf16", 6)])
@pytest.mark.parametrize("lengths,window", [([32], -1), ([7, 96], 64), ([128, 1], -1), ([250, 131], 64),
                                            ([256, 219, 145], -1), ([500], 64), ([1024, 333], -1), ([300, 77], 40)])
def test_packed_attention_matches_oracle(lib, prec, impl, lengths, window):
    """Cases and float64 oracle of tests/test_attention.py:12-56 (h=2, seeded by M), for the
    tcgen05 kernel over 128-query tiles (impl 1: key split chosen as the forward pass does;
    2: never; 3: over 2 CTAs; 4: over 4 CTAs, ranks without a key block included; 5: one tile
    per CTA; 6: the persistent kernel on one CTA, which then runs every (tile, head) item,
    zero-fill and unused table entries included, through one pipeline)."""
    check_packed_attention(lib, prec, impl, lengths, window, ramp=False)


@pytest.mark.parametrize("prec,impl", [("f16", 1), ("bf16", 1), ("f16", 2), ("bf16", 3), ("f16", 4), ("f16", 6),
                                       ("bf16", 6)])
@pytest.mark.parametrize("lengths,window", [([1024, 333], -1), ([700], 64), ([513, 200], -1)])
def test_packed_attention_growing_scores(lib, prec, impl, lengths, window):
    """Scores that grow along the row (keys scaled up with position), so the running maximum
    rises by far more than 2^8 between key blocks: exercises the rescaling of O."""
    check_packed_attention(lib, prec, impl, lengths, window, ramp=True)


@pytest.mark.parametrize("prec,impl", [("f16", 1), ("bf16", 1), ("f16", 6), ("bf16", 6)])
@pytest.mark.parametrize("window", [-1, 64])
def test_packed_attention_large_grid(lib, prec, impl, window):
    """12 heads over 48 rows of 40-900 tokens: impl 1 runs the persistent kernel on the SMs'
    resident slots (several items per CTA, longest rows first), impl 6 on its fewest CTAs
    (up to 128 items each).  Ten rows, the longest and shortest among them, are checked
    against the float64 oracle; every other real row must be finite and the rest zero."""
    lengths = [int(v) for v in np.random.default_rng(48).integers(40, 901, 48)]
    check_packed_attention(lib, prec, impl, lengths, window, ramp=False, h=12,
                           check_rows=sorted({int(np.argmax(lengths)), int(np.argmin(lengths)), 0, 5, 11, 17, 23,
                                              31, 40, 47}))


# Worst |error| - 16-bit output rounding, by precision: the 16-bit rounding of the
# probabilities.  Scores that grow along the row concentrate the softmax on a few keys, so one
# rounded bf16 probability weighs more.
ATTN_LIMIT = {"bf16": 6e-3, "f16": 1.5e-3}
ATTN_LIMIT_RAMP = {"bf16": 1e-2, "f16": 1.5e-3}


def check_packed_attention(lib, prec, impl, lengths, window, ramp, h=2, check_rows=None):
    tile_q = 128
    starts, lens, M = packed_case(lengths)
    cap = (M + (tile_q - 16) * len(lengths) + tile_q - 1) // tile_q + 1
    tiles = np.zeros((cap, 4), np.int32)
    n_tiles = lib.laya_attention_tiles(starts.ctypes.data, lens.ctypes.data, len(lengths), M, tile_q,
                                       tiles.ctypes.data, cap)
    assert n_tiles > 0
    x = np.random.default_rng(M).normal(0, 1, (M, 3, h, 64)).astype(np.float32)
    if ramp:
        for start, n in zip(starts, lengths):
            x[start:start + n, 0] *= 2.0
            x[start:start + n, 1] *= (1.0 + np.arange(n, dtype=np.float32) / 64.0)[:, None, None]
    xt = torch.from_numpy(x).to(PRECISIONS[prec][1])
    xd = xt.double().numpy()
    layout = xt.permute(1, 2, 0, 3).contiguous()                  # [3][h][M][64]
    layout[2] = layout[2].transpose(1, 2).reshape(h, M, 64)       # v stored transposed: [h][64][M]
    layout = layout.cuda()
    out = torch.full((M, h * 64), float("nan"), dtype=PRECISIONS[prec][1], device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    dev = [torch.from_numpy(v).cuda() for v in (tiles, starts, lens)]
    _lib.check(lib.laya_op_attention(PRECISIONS[prec][0], impl, ptr(layout), ptr(out), ptr(dev[0]), cap, ptr(dev[1]),
                                     ptr(dev[2]), M, h, window, ptr(err), stream()))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = out.double().cpu().numpy()
    real = np.zeros(M, bool)
    worst = 0.0
    for row, (start, n) in enumerate(zip(starts, lens)):
        real[start:start + n] = True
        if check_rows is not None and row not in check_rows:
            assert np.isfinite(got[start:start + n]).all()
            continue
        q, k, v = xd[start:start + n].transpose(1, 2, 0, 3)
        s = q @ k.transpose(0, 2, 1) / 8
        if window >= 0:
            s[:, np.abs(np.arange(n)[:, None] - np.arange(n)) > window] = -np.inf
        p = np.exp(s - s.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        expected = (p @ v).transpose(1, 0, 2).reshape(n, h * 64)
        err_ = np.abs(got[start:start + n] - expected) - ROUND[prec] * np.abs(expected)
        worst = max(worst, float(err_.max()))
    limit = (ATTN_LIMIT_RAMP if ramp else ATTN_LIMIT)[prec]
    assert worst < limit, worst
    np.testing.assert_array_equal(got[~real], 0)


@pytest.mark.parametrize("prec", ["bf16", "f16"])
@pytest.mark.parametrize("width", [64, 768, 1024])
def test_embed_norm(lib, prec, width):
    rng = np.random.default_rng(width)
    vocab, rows = 1000, 77
    table = rng.normal(0, 0.5, (vocab, width)).astype(np.float32)
    gamma = rng.normal(1, 0.1, width).astype(np.float32)
    ids = rng.integers(0, vocab, rows).astype(np.int32)
    residual = torch.empty((rows, width), dtype=torch.float32, device="cuda")
    x = torch.empty((rows, width), dtype=PRECISIONS[prec][1], device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    t = [torch.from_numpy(v).cuda() for v in (ids, table, gamma)]
    _lib.check(lib.laya_op_embed_norm(PRECISIONS[prec][0], ptr(t[0]), ptr(t[1]), ptr(t[2]), 1e-5, rows, width, vocab,
                                      ptr(residual), ptr(x), ptr(err), stream()))
    torch.cuda.synchronize()
    e = table[ids].astype(np.float64)
    expected = (e - e.mean(-1, keepdims=True)) / np.sqrt(e.var(-1, keepdims=True) + 1e-5) * gamma
    np.testing.assert_allclose(residual.cpu().numpy(), expected, atol=2e-5, rtol=1e-5)
    np.testing.assert_array_equal(x.cpu().float().numpy(), residual.to(PRECISIONS[prec][1]).cpu().float().numpy())
    assert int(err.item()) == 0


@pytest.mark.parametrize("prec", ["bf16", "f16"])
@pytest.mark.parametrize("width", [64, 768, 1024])
@pytest.mark.parametrize("splits,beta", [(0, False), (0, True), (2, False), (2, True)])
@pytest.mark.parametrize("rows", [29, 2371])
def test_norm_residual_partials(lib, prec, width, splits, beta, rows):
    """cf. tests/test_gpu.py:68-103: residual accumulation then LayerNorm with/without beta.
    2,371 rows launch 8-warp blocks with a partly filled last block; 29 rows one-warp blocks."""
    rng = np.random.default_rng(31)
    source = rng.normal(2, .3, (rows, width)).astype(np.float32)
    parts = rng.normal(0, .1, (max(splits, 1), rows, width)).astype(np.float32)
    gamma = rng.normal(1, .1, width).astype(np.float32)
    b = rng.normal(0, .1, width).astype(np.float32)
    residual = torch.from_numpy(source.copy()).cuda()
    x = torch.empty((rows, width), dtype=PRECISIONS[prec][1], device="cuda")
    t = [torch.from_numpy(v).cuda() for v in (parts, gamma, b)]
    _lib.check(lib.laya_op_norm(PRECISIONS[prec][0], ptr(residual), ptr(t[0]) if splits else None, splits, ptr(t[1]),
                                ptr(t[2]) if beta else None, 1e-5, ptr(x), rows, width, stream()))
    torch.cuda.synchronize()
    added = source.astype(np.float64) + (parts[:splits].sum(0) if splits else 0)
    np.testing.assert_allclose(residual.cpu().numpy(), added, atol=1e-6, rtol=1e-6)
    expected = (added - added.mean(-1, keepdims=True)) / np.sqrt(added.var(-1, keepdims=True) + 1e-5) * gamma
    if beta:
        expected = expected + b
    got = x.cpu().double().numpy()
    assert np.max(np.abs(got - expected) - ROUND[prec] * np.abs(expected)) < 1e-4


@pytest.mark.parametrize("prec", ["f16", "bf16"])
@pytest.mark.parametrize("lengths,q_per_row", [([300, 77, 1024], 9), ([129], 1), ([700, 40], 130)])
def test_gathered_query_attention_matches_oracle(lib, prec, lengths, q_per_row):
    """Global attention from gathered query rows only (CLS + markers of the decision head, with
    duplicate indices as packing pads them): those rows match the float64 oracle, every other
    row of the output is left untouched, and an unused (length-0) row is skipped."""
    h = 2
    starts, lens, M = packed_case(lengths)
    starts = np.append(starts, 0).astype(np.int32)
    lens = np.append(lens, 0).astype(np.int32)                       # unused row of the class
    rng = np.random.default_rng(M + q_per_row)
    index = np.zeros((len(lens), q_per_row), np.int32)
    for r, (s0, n) in enumerate(zip(starts, lens)):
        if n:
            picks = rng.integers(0, n, q_per_row)
            picks[0] = 0
            picks[-1] = 0 if q_per_row > 1 else picks[-1]             # duplicate of the CLS row
            index[r] = s0 + picks
    x = rng.normal(0, 1, (M, 3, h, 64)).astype(np.float32)
    xt = torch.from_numpy(x).to(PRECISIONS[prec][1])
    xd = xt.double().numpy()
    layout = xt.permute(1, 2, 0, 3).contiguous()
    layout[2] = layout[2].transpose(1, 2).reshape(h, M, 64)
    layout = layout.cuda()
    out = torch.full((M, h * 64), 7.0, dtype=PRECISIONS[prec][1], device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    dev = [torch.from_numpy(np.ascontiguousarray(v)).cuda() for v in (index, starts, lens)]
    _lib.check(lib.laya_op_attention_gathered(PRECISIONS[prec][0], ptr(layout), ptr(out), ptr(dev[0]), q_per_row,
                                              ptr(dev[1]), ptr(dev[2]), len(lens), M, h, ptr(err), stream()))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = out.double().cpu().numpy()
    written = np.zeros(M, bool)
    worst = 0.0
    for r, (s0, n) in enumerate(zip(starts, lens)):
        if not n:
            continue
        q, k, v = xd[s0:s0 + n].transpose(1, 2, 0, 3)
        s = q @ k.transpose(0, 2, 1) / 8
        p = np.exp(s - s.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        expected = (p @ v).transpose(1, 0, 2).reshape(n, h * 64)
        for t in index[r]:
            written[t] = True
            e = expected[t - s0]
            worst = max(worst, float(np.max(np.abs(got[t] - e) - ROUND[prec] * np.abs(e))))
    assert worst < ATTN_LIMIT[prec], worst
    np.testing.assert_array_equal(got[~written], 7.0)


@pytest.mark.parametrize("prec", ["f16", "bf16"])
@pytest.mark.parametrize("M,N,K,with_bias", [(300, 768, 768, False), (4099, 768, 3072, False), (200, 256, 128, True),
                                             (513, 512, 768, True), (130, 1024, 256, False), (257, 384, 256, True),
                                             (300, 576, 512, False)])
def test_gemm_residual_layernorm_matches_fp64(lib, prec, M, N, K, with_bias):
    """Fused residual GEMM + LayerNorm (clusters of CTAs exchanging row statistics):
    residual += x W^T + bias and out = LN(residual) * gamma (+ beta) against float64."""
    rng = np.random.default_rng(M + N + K)
    x, xd = rand16((M, K), prec, rng)
    w, wd = rand16((N, K), prec, rng, 0.02)
    base = rng.normal(0, 1, (M, N)).astype(np.float32) + rng.normal(0, 0.5, (M, 1)).astype(np.float32)
    bias = rng.normal(0, 0.1, N).astype(np.float32) if with_bias else None
    gamma = (1 + rng.normal(0, 0.1, N)).astype(np.float32)
    beta = rng.normal(0, 0.1, N).astype(np.float32) if with_bias else None
    residual = torch.from_numpy(base.copy()).cuda()
    out = torch.full((M, N), float("nan"), dtype=PRECISIONS[prec][1], device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    dev = lambda a: torch.from_numpy(a).cuda() if a is not None else None  # noqa: E731
    b_t, g_t, be_t = dev(bias), dev(gamma), dev(beta)
    _lib.check(lib.laya_op_gemm_ln(PRECISIONS[prec][0], ptr(x), ptr(w), M, N, K, ptr(residual), N, ptr(b_t), ptr(g_t),
                                   ptr(be_t), 1e-5, ptr(out), N, ptr(err), stream()))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want_r = base.astype(np.float64) + xd @ wd.T + (bias if with_bias else 0)
    assert np.max(np.abs(residual.cpu().numpy() - want_r)) < 2e-4 * math.sqrt(K)
    mean = want_r.mean(1, keepdims=True)
    var = ((want_r - mean) ** 2).mean(1, keepdims=True)
    want = (want_r - mean) / np.sqrt(var + 1e-5) * gamma + (beta if with_bias else 0)
    got = out.double().cpu().numpy()
    assert np.max(np.abs(got - want) - ROUND[prec] * np.abs(want)) < 2e-3


@pytest.mark.parametrize("prec", ["f16", "bf16"])
@pytest.mark.parametrize("width", [128, 768])
def test_head_tail_features_logits_and_actions(lib, prec, width):
    """The decision-head tail against the oracle's features (kernels.cu:167-183, laya.py:241-245):
    option counts 0, 1, 2, a tied top-2, 77 options and a random question in a k = 128 class.
    scorer.3 is the unit vector e0 so the option logits are chosen values (16-bit exact), and p1,
    p1 - p2, entropy / log(max(c, 2)) and max(c, 2) / 255 are compared directly."""
    import types
    from oracle.laya_oracle import Oracle, gelu
    rng = np.random.default_rng(width)
    counts = np.array([0, 1, 2, 2, 77, 5], np.int32)
    b, k, d, n_act = len(counts), 128, width, 3
    option_logits = np.zeros((b, k + 1), np.float32)
    for q, c in enumerate(counts):
        option_logits[q, 1:c + 1] = rng.normal(0, 2, c)
    option_logits[3, 1:3] = 1.5                                     # tied top-2
    t16 = PRECISIONS[prec][1]
    option_logits = torch.from_numpy(option_logits).to(t16).float().numpy()
    scored = np.zeros((b, k + 1, d), np.float32)
    scored[:, :, 0] = option_logits
    scored[:, :, 1:] = rng.normal(0, 1, (b, k + 1, d - 1))          # ignored by w3 = e0
    selected = rng.normal(0, 1, (b, k + 1, d)).astype(np.float32)
    w3 = np.zeros(d, np.float32); w3[0] = 1.0
    b3 = np.array([0.25], np.float32)
    wa0 = rng.normal(0, 0.05, (256, d + 4)).astype(np.float32)
    ba0 = rng.normal(0, 0.1, 256).astype(np.float32)
    wa2 = rng.normal(0, 0.05, (n_act, 256)).astype(np.float32)
    ba2 = rng.normal(0, 0.1, n_act).astype(np.float32)
    dev = {name: torch.from_numpy(v).cuda() for name, v in dict(selected=selected, w3=w3, b3=b3, wa0=wa0, ba0=ba0,
                                                                 wa2=wa2, ba2=ba2, counts=counts).items()}
    dev["scored"] = torch.from_numpy(scored).to(t16).cuda()
    logits = torch.full((b, k + 1), float("nan"), device="cuda")
    acts = torch.full((b, n_act), float("nan"), device="cuda")
    feats = torch.full((b, 4), float("nan"), device="cuda")
    hidden = torch.zeros((b, 256), device="cuda")
    arrivals = torch.zeros(b, dtype=torch.int32, device="cuda")
    _lib.check(lib.laya_op_head_tail(PRECISIONS[prec][0], ptr(dev["selected"]), ptr(dev["scored"]), ptr(dev["counts"]),
                                     b, k, d, ptr(dev["w3"]), ptr(dev["b3"]), ptr(dev["wa0"]), ptr(dev["ba0"]),
                                     ptr(dev["wa2"]), ptr(dev["ba2"]), n_act, ptr(logits), ptr(acts), ptr(feats),
                                     ptr(hidden), ptr(arrivals), stream()))
    torch.cuda.synchronize()
    want_logits = option_logits.astype(np.float64) + 0.25
    np.testing.assert_allclose(logits.cpu().numpy(), want_logits, atol=1e-6, rtol=0)
    shim = types.SimpleNamespace(dtype=np.float64)
    for q, c in enumerate(counts):
        want_f = Oracle.features(shim, want_logits[q, 1:c + 1])
        got_f = feats[q].cpu().numpy()
        np.testing.assert_allclose(got_f, want_f, atol=2e-6, rtol=1e-5, err_msg=f"question {q}, {c} options")
        feat = np.concatenate([selected[q, 0].astype(np.float64), want_f])
        want_a = gelu(wa0.astype(np.float64) @ feat + ba0) @ wa2.astype(np.float64).T + ba2
        np.testing.assert_allclose(acts[q].cpu().numpy(), want_a, atol=1e-4, rtol=0)
    assert feats[3, 1].item() == 0.0                                 # tie: p1 - p2 exactly 0
    np.testing.assert_array_equal(arrivals.cpu().numpy(), 0)         # left zero for the next launch


def test_gathered_attention_reports_out_of_range_indices(lib):
    """Gathered query indices outside the packed rows set the error word (kErrBadIndex = 4),
    are not stored, and leave the valid rows exact: the kernel clamps instead of reading or
    writing out of bounds."""
    prec, h, q_per_row = "f16", 2, 4
    starts, lens, M = packed_case([300, 77])
    s1 = int(starts[1])
    index = np.array([[0, 5, M + 7, 299], [s1, -3, s1 + 10, s1 + 76]], np.int32)
    rng = np.random.default_rng(17)
    x = rng.normal(0, 1, (M, 3, h, 64)).astype(np.float32)
    xt = torch.from_numpy(x).to(torch.float16)
    xd = xt.double().numpy()
    layout = xt.permute(1, 2, 0, 3).contiguous()
    layout[2] = layout[2].transpose(1, 2).reshape(h, M, 64)
    out = torch.full((M, h * 64), 7.0, dtype=torch.float16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    dev = [torch.from_numpy(np.ascontiguousarray(v)).cuda() for v in (index, starts, lens)]
    _lib.check(lib.laya_op_attention_gathered(PRECISIONS[prec][0], ptr(layout.cuda()), ptr(out), ptr(dev[0]), q_per_row,
                                              ptr(dev[1]), ptr(dev[2]), 2, M, h, ptr(err), stream()))
    torch.cuda.synchronize()
    assert int(err.item()) == 4
    got = out.double().cpu().numpy()
    written = np.zeros(M, bool)
    for r, (s0, n) in enumerate(zip(starts, lens)):
        q, k, v = xd[s0:s0 + n].transpose(1, 2, 0, 3)
        s = q @ k.transpose(0, 2, 1) / 8
        p = np.exp(s - s.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        expected = (p @ v).transpose(1, 0, 2).reshape(n, h * 64)
        for t in index[r]:
            if 0 <= t < M:
                written[t] = True
                e = expected[t - s0]
                assert np.max(np.abs(got[t] - e) - ROUND[prec] * np.abs(e)) < ATTN_LIMIT[prec]
    np.testing.assert_array_equal(got[~written], 7.0)
