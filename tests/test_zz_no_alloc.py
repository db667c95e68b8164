"""The allocation-free split-K residual GEMM (laya_op_gemm_residual_static).

Some callers cannot allocate device memory on this path: a serving host whose own allocator
owns all of the GPU's memory, or a latency-critical loop where cudaMalloc/cudaFree would
implicitly synchronise the device.  This entry point keeps its split-K partial sums in a static
device array of the library instead.  The test drives it through the C ABI and checks two calls
in a row against the allocating entry point (laya_op_gemm, residual epilogue) within the GEMM
tolerance of the kernel tests.  The file name makes pytest collect it last.
"""
import ctypes as ct
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from laya_cuda import _lib  # noqa: E402


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return _lib.load()


def ptr(t):
    return ct.c_void_p(t.data_ptr()) if t is not None else None


def case(seed, M, N, K):
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(rng.normal(0, 1, (M, K)).astype(np.float32)).half().cuda()
    w = torch.from_numpy(rng.normal(0, 0.02, (N, K)).astype(np.float32)).half().cuda()
    base = torch.from_numpy(rng.normal(0, 1, (M, N)).astype(np.float32)).cuda()
    bias = torch.from_numpy(rng.normal(0, 0.1, N).astype(np.float32)).cuda()
    return x, w, base, bias


def allocating(lib, x, w, base, bias):
    out = base.clone()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    M, K = x.shape
    N = w.shape[0]
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.laya_op_gemm(_lib.PRECISION_F16, 5, ptr(x), ptr(w), M, N, K, None, 0, ptr(out), N, ptr(bias), 0,
                                None, 0, None, 1, 0, ptr(err), stream))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


def static(lib, x, w, base, bias, splits):
    out = base.clone()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    M, K = x.shape
    N = w.shape[0]
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.laya_op_gemm_residual_static(_lib.PRECISION_F16, ptr(x), ptr(w), M, N, K, splits, ptr(out),
                                                ptr(bias), ptr(err), stream))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


def test_static_scratch_matches_allocating_entry_point_twice(lib):
    # Two calls in a row: a larger problem first, then a smaller one with other data, so a
    # stale partial from the first call would show up in the second.
    for seed, (M, N, K, splits) in ((1, (600, 768, 3072, 4)), (2, (96, 768, 768, 3))):
        x, w, base, bias = case(seed, M, N, K)
        expected = allocating(lib, x, w, base, bias).cpu().numpy()
        got = static(lib, x, w, base, bias, splits).cpu().numpy()
        assert np.max(np.abs(got - expected)) < 2e-4 * math.sqrt(K)


def test_static_scratch_rejects_oversized_problems(lib):
    x, w, base, bias = case(3, 2048, 768, 768)
    limit = _lib.STATIC_SCRATCH_FLOATS
    splits = 3  # 2048 * 768 * 3 > 4 Mi floats
    assert 2048 * 768 * splits > limit
    out = base.clone()
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    code = lib.laya_op_gemm_residual_static(_lib.PRECISION_F16, ptr(x), ptr(w), 2048, 768, 768, splits, ptr(out),
                                            ptr(bias), None, stream)
    assert code == _lib.ERR_INVALID
    assert b"static scratch" in lib.laya_last_error(None)
    torch.cuda.synchronize()
    assert torch.equal(out, base)


def test_static_scratch_rejects_a_misaligned_residual(lib):
    """The partial sums are added to the residual four floats at a time, so a residual that is
    not 16-byte aligned is refused on the host (LAYA_ERR_INVALID) before anything is launched,
    and the residual is left as it was."""
    x, w, base, bias = case(4, 96, 768, 768)
    out = torch.zeros(96 * 768 + 4, dtype=torch.float32, device="cuda")
    out[1:1 + 96 * 768] = base.flatten()
    shifted = out[1:1 + 96 * 768]                         # 4-byte offset from an aligned buffer
    assert shifted.data_ptr() % 16 != 0
    before = out.clone()
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    code = lib.laya_op_gemm_residual_static(_lib.PRECISION_F16, ptr(x), ptr(w), 96, 768, 768, 3, ptr(shifted),
                                            ptr(bias), None, stream)
    assert code == _lib.ERR_INVALID
    assert b"16-byte aligned" in lib.laya_last_error(None)
    torch.cuda.synchronize()
    assert torch.equal(out, before)
