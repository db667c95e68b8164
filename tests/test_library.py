"""The C ABI library on the host (no GPU needed): it loads, exports every symbol the header
declares, and its host-side packing, shape classes and attention tile tables match a Python
restatement of the reference's Slot.fill (laya_cuda/runtime.py:52-68) and classes (20-25)."""
import ctypes as ct
import math
import re
from pathlib import Path

import numpy as np
import pytest

from laya_cuda import _lib
from laya_cuda.runtime import classes, flatten, span

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    header = (ROOT / "include/laya_b200.h").read_text()
    declared = set(re.findall(r"^\s*(?:int|int64_t|void\*|const char\*)\s+(laya_\w+)\s*\(", header, re.M))
    assert declared == set(_lib.EXPORTS)
    for name in declared:
        assert hasattr(lib, name), name


def test_create_without_device_fails_cleanly(lib):
    """No GPU here: laya_create must return an error status with a message, not crash."""
    cfg = _lib.Config(vocab=100, width=64, heads=1, layers=1, intermediate=128, global_every=3, window=64,
                      theta_global=160000., theta_local=10000., eps=1e-5, max_len=128, head_layers=1, n_act=2,
                      precision=0)
    handle = ct.c_void_p()
    code = lib.laya_create(ct.byref(cfg), 0, 4, ct.byref(handle))
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except ImportError:
        has_gpu = False
    if has_gpu:
        lib.laya_destroy(handle)
        pytest.skip("a GPU is present")
    assert code == _lib.ERR_NO_DEVICE and not handle.value
    assert lib.laya_last_error(None)


def fill_reference(items, pad, m, b, k):
    """Python restatement of Slot.fill: ids/positions/rows/kinds per token, starts/lengths/
    counts per question, (k+1) gather indices per question (CLS, then marker tokens)."""
    ids = np.full(m, pad, np.int32)
    positions = np.zeros(m, np.int32)
    rows = np.full(m, -1, np.int32)
    kinds = np.zeros(m, np.int32)
    starts, lengths, counts = (np.zeros(b, np.int32) for _ in range(3))
    indices = np.zeros(b * (k + 1), np.int32)
    offset = 0
    for r, (tok, markers, kind) in enumerate(items):
        n = len(tok)
        end = offset + span(n)
        ids[offset:offset + n] = tok
        positions[offset:end] = np.arange(end - offset)
        rows[offset:end], kinds[offset:end] = r, kind
        starts[r], lengths[r], counts[r] = offset, n, len(markers)
        block = indices[r * (k + 1):(r + 1) * (k + 1)]
        block[:] = offset
        block[1:len(markers) + 1] += markers
        offset = end
    return ids, positions, rows, kinds, starts, lengths, counts, indices


def pack(lib, items, pad=0):
    m, b, k = classes(items)
    tokens, lengths, markers, counts, kinds = flatten(items)
    out = np.zeros(lib.laya_packed_ints(m, b, k), np.int32)
    code = lib.laya_pack(tokens.ctypes.data, lengths.ctypes.data, markers.ctypes.data, counts.ctypes.data,
                         kinds.ctypes.data, len(items), pad, m, b, k, out.ctypes.data)
    return code, out, (m, b, k)


@pytest.mark.parametrize("seed", range(6))
def test_pack_matches_reference_fill(lib, seed):
    rng = np.random.default_rng(seed)
    items = []
    for j in range(int(rng.integers(1, 9))):
        n = int(rng.integers(1, 700))
        markers = sorted(rng.choice(n, size=int(rng.integers(1, min(n, 40) + 1)), replace=False).tolist())
        items.append((rng.integers(0, 1000, n).tolist(), markers, j % 3))
    code, out, (m, b, k) = pack(lib, items, pad=7)
    assert code == 0
    want = fill_reference(items, 7, m, b, k)
    o = 0
    for field, size in zip(want, (m, m, m, m, b, b, b, b * (k + 1))):
        np.testing.assert_array_equal(out[o:o + size], field)
        o += size
    # Attention tile table (128 queries): every token of every row span is covered exactly once
    # by a tile of its row; tokens past the last row by zero-fill tiles; no tile straddles rows.
    o = (o + 3) // 4 * 4
    for tile_q in (128,):
        cap = (m + (tile_q - 16) * b + tile_q - 1) // tile_q + 1
        tiles = out[o:o + 4 * cap].reshape(-1, 4)
        o += 4 * cap
        cover = np.zeros(m, np.int32)
        # Order: row tiles with rows longest first, then zero-fill tiles, then unused slots.
        kinds = [0 if row >= 0 else 1 if row == -1 else 2 for row in tiles[:, 2]]
        assert kinds == sorted(kinds)
        row_lengths = [want[5][row] for row in tiles[:, 2] if row >= 0]
        assert row_lengths == sorted(row_lengths, reverse=True)
        for t0, t1, row, _ in tiles:
            if row == -2:
                continue
            assert 0 <= t0 < t1 <= m and t1 - t0 <= tile_q
            cover[t0:t1] += 1
            if row >= 0:
                s, n = want[4][row], want[5][row]
                assert s <= t0 and t1 <= s + span(n) and (t0 - s) % tile_q == 0
            else:
                assert np.all(want[2][t0:t1] == -1)
        np.testing.assert_array_equal(cover, 1)
    assert o == len(out)


def test_shape_class_matches_reference(lib):
    cases = [[([1] * 17, [1, 2], 0), ([1] * 250, [1] * 9, 1)], [([1] * 83, [1, 2, 3, 4], 0)],
             [([1] * 600, [3], 0)] * 5, [([1] * 1, [0], 2)], [([1] * 300, list(range(77)), 0)] * 3]
    for items in cases:
        _, lengths, _, counts, _ = flatten(items)
        got = [ct.c_int32() for _ in range(3)]
        assert lib.laya_shape_class(lengths.ctypes.data, counts.ctypes.data, len(items), *map(ct.byref, got)) == 0
        assert tuple(v.value for v in got) == classes(items)
    assert classes(cases[0]) == (320, 2, 16) and classes(cases[1]) == (96, 1, 8)


@pytest.mark.parametrize("bad", ["marker", "kind", "empty"])
def test_pack_rejects_invalid_items(lib, bad):
    items = [([5] * 20, [3, 9], 0)]
    if bad == "marker":
        items = [([5] * 20, [3, 20], 0)]
    elif bad == "kind":
        items = [([5] * 20, [3], 3)]
    elif bad == "empty":
        items = [([], [], 0)]
    if bad == "empty":
        lengths = np.zeros(1, np.int32)
        counts = np.zeros(1, np.int32)
        got = [ct.c_int32() for _ in range(3)]
        assert lib.laya_shape_class(lengths.ctypes.data, counts.ctypes.data, 1, *map(ct.byref, got)) == _lib.ERR_INVALID
        return
    code, _, _ = pack(lib, items)
    assert code == _lib.ERR_INVALID
    assert lib.laya_last_error(None)


def test_geglu_interleave(lib):
    F, K = 128, 8
    src = np.arange(2 * F * K, dtype=np.uint16).reshape(2 * F, K)
    dst = np.zeros_like(src)
    assert lib.laya_interleave_geglu(src.ctypes.data, dst.ctypes.data, F, K) == 0
    for blk in range(F // 64):
        np.testing.assert_array_equal(dst[blk * 128:blk * 128 + 64], src[blk * 64:blk * 64 + 64])
        np.testing.assert_array_equal(dst[blk * 128 + 64:blk * 128 + 128], src[F + blk * 64:F + blk * 64 + 64])


def test_gelu_erf_approximation_restated():
    """The GEMM epilogues' GELU uses erf from Abramowitz & Stegun 7.1.26 (common.cuh,
    gelu_erf).  Restated here in float32 with the same constants and operation order: its
    absolute error against the exact erf GELU stays below 6e-7 on [-12, 12]."""
    x = np.linspace(-12, 12, 24001).astype(np.float32)
    z = np.abs(x) * np.float32(0.70710678118654752)
    t = np.float32(1) / (np.float32(0.3275911) * z + np.float32(1))
    poly = np.float32(1.061405429) * t + np.float32(-1.453152027)
    for a in (1.421413741, -0.284496736, 0.254829592):
        poly = poly * t + np.float32(a)
    poly = poly * t
    e = np.exp2(-z * z * np.float32(1.4426950408889634)).astype(np.float32)
    erf_v = np.copysign(np.float32(1) - poly * e, x)
    got = (np.float32(0.5) * x * (np.float32(1) + erf_v)).astype(np.float64)
    xd = x.astype(np.float64)
    want = 0.5 * xd * (1 + np.array([math.erf(v / math.sqrt(2)) for v in xd]))
    assert np.max(np.abs(got - want)) < 6e-7


def _scan(lib, path):
    n, elems = ct.c_int64(), ct.c_int64()
    code = lib.laya_scan_checkpoint(str(path).encode(), ct.byref(n), ct.byref(elems))
    return code, n.value, elems.value


def test_checkpoint_header_parser_matches_safetensors(lib, tmp_path):
    """laya_scan_checkpoint parses the safetensors header the native loader uses: tensor count
    and elements agree with the safetensors library on a synthetic checkpoint with metadata,
    F32/F16/BF16 tensors and escaped names."""
    from safetensors.numpy import save_file
    from laya_cuda import synthetic as S
    arch = S.architecture("tiny", layers=2)
    weights = S.make_weights(arch, seed=1)
    weights["encoder.final_norm.weight"] = weights["encoder.final_norm.weight"].astype(np.float16)
    weights['odd "name"\\é'] = np.zeros((2, 3), np.float32)
    path = tmp_path / "model.safetensors"
    save_file(weights, str(path), metadata={"format": "pt", "note": 'a "quoted" {value}'})
    code, n, elems = _scan(lib, path)
    assert code == 0, lib.laya_last_error(None)
    assert n == len(weights) and elems == sum(v.size for v in weights.values())
    # bfloat16 through the torch writer, when present.
    torch = pytest.importorskip("torch")
    from safetensors.torch import save_file as save_torch
    save_torch({"a": torch.zeros(4, 5, dtype=torch.bfloat16), "b": torch.ones(7)}, str(tmp_path / "bf.safetensors"))
    assert _scan(lib, tmp_path / "bf.safetensors") == (0, 2, 27)


@pytest.mark.parametrize("damage", ["truncated", "header", "offsets", "json", "dtype", "empty"])
def test_checkpoint_header_parser_rejects_malformed_files(lib, tmp_path, damage):
    import json as _json
    import struct
    header = {"w": {"dtype": "F32", "shape": [2, 2], "data_offsets": [0, 16]}}
    body = b"\0" * 16
    if damage == "offsets":
        header["w"]["data_offsets"] = [0, 20]
    if damage == "dtype":
        header["w"]["dtype"] = "I64"
    text = _json.dumps(header).encode()
    if damage == "json":
        text = text[:-3]
    blob = struct.pack("<Q", len(text)) + text + body
    if damage == "truncated":
        blob = blob[:-4]
    if damage == "header":
        blob = struct.pack("<Q", 1 << 40) + blob[8:]
    if damage == "empty":
        blob = b"\0\0"
    path = tmp_path / "bad.safetensors"
    path.write_bytes(blob)
    code, _, _ = _scan(lib, path)
    assert code == _lib.ERR_INVALID
    assert lib.laya_last_error(None)


def test_exp2_polynomial_restated():
    """The attention's FMA-pipe 2^x (common.cuh, exp2_poly2): range reduction by adding
    1.5 * 2^23 and a degree-3 minimax polynomial on [-0.5, 0.5], restated in float32 with the same
    constants and operation order.  Its relative error against exact 2^x stays below 8e-5 over
    the softmax's input range, below the 2^-11 rounding of the 16-bit probabilities."""
    x = np.concatenate([np.linspace(-64, 8, 400001), np.array([-64.0, -0.5, 0.5, 0.0, 8.0])]).astype(np.float32)
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    n = (t - magic).astype(np.float32)
    f = (x - n).astype(np.float32)
    p = np.float32(0.0551716685) * f + np.float32(0.2426111251)
    p = (p * f + np.float32(0.6932609677)).astype(np.float32)
    p = (p * f + np.float32(0.9999280572)).astype(np.float32)
    bits = p.view(np.int32) + (t.view(np.int32) << 23)
    got = bits.view(np.float32).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    assert np.max(np.abs(got - want) / want) < 8e-5
