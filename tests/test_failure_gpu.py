"""Failure paths on the GPU, in the forms that fault and hang nothing (no trap, no bad address,
no endless wait):

* an out-of-range token id reaches the embedding kernel, which clamps the read, sets the
  launch's error word and lets the pass finish: the call reports LAYA_ERR_DEVICE (RuntimeError)
  and the engine's next pass is exact;
* a bounded pipeline wait runs out on a valid, correctly addressed GEMM because the test sets
  the wait limit to 1 ns (laya_set_launch_options): the kernel unwinds, drains the copies and
  MMAs it issued, frees its TMEM and sets its error word; the next launch with the default limit
  is exact.  The 1-CTA GEMM kernel is used: its producer, MMA issuer and epilogue share one CTA,
  so the drain covers every copy the kernel issued.
"""
import ctypes as ct
import math

import numpy as np
import pytest

from laya_cuda import Engine, _lib
from laya_cuda import synthetic as S

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return _lib.load()


def ptr(t):
    return ct.c_void_p(t.data_ptr()) if t is not None else None


def test_out_of_range_token_id_reports_device_error_then_recovers(lib, tmp_path):
    arch = S.architecture("small", max_len=256)
    path = S.write_checkpoint(tmp_path / "ckpt", arch, seed=3)
    rng = np.random.default_rng(4)
    items = [S.build_item(rng, 120, 4, arch["vocab"]), S.build_item(rng, 60, 2, arch["vocab"], kind=1)]
    bad_ids = list(items[0][0])
    bad_ids[20] = arch["vocab"] + 1000
    bad = [(bad_ids, items[0][1], 0), items[1]]
    with Engine(path) as engine:
        expected = engine.runtime.predict(items, capture=False)
        for capture in (False, True):
            with pytest.raises(RuntimeError, match="device error 4"):
                engine.runtime.predict(bad, capture=capture)
            again = engine.runtime.predict(items, capture=capture)
            np.testing.assert_array_equal(again[0], expected[0])
            np.testing.assert_array_equal(again[1], expected[1])


def gemm_store(lib, x, w, out):
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    M, K = x.shape
    N = w.shape[0]
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    # 1-CTA kernel with 64-column tiles (block_n 64), plain store epilogue.
    _lib.check(lib.laya_op_gemm(_lib.PRECISION_F16, 0, ptr(x), ptr(w), M, N, K, ptr(out), N, None, 0, None, 0, None,
                                0, None, 1, 64, ptr(err), stream))
    torch.cuda.synchronize()
    return int(err.item())


def test_gemm_wait_limit_runs_out_then_recovers(lib):
    """One 128 x 64 tile over K = 65536 (1024 k-blocks): its epilogue waits for the accumulator
    for well over 100 us, far past a 1 ns limit however long one try_wait suspends."""
    rng = np.random.default_rng(6)
    M, N, K = 128, 64, 65536
    x = torch.from_numpy(rng.normal(0, 1, (M, K)).astype(np.float32)).half().cuda()
    w = torch.from_numpy(rng.normal(0, 0.02, (N, K)).astype(np.float32)).half().cuda()
    expected = x.double().cpu().numpy() @ w.double().cpu().numpy().T
    out = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    try:
        assert lib.laya_set_launch_options(1, 1) == 0
        code = gemm_store(lib, x, w, out)
    finally:
        assert lib.laya_set_launch_options(1, 0) == 0
    # 1: producer, 2: MMA issuer, 3: epilogue wait ran out (whichever role gave up first).
    assert code in (1, 2, 3), code
    out.fill_(0)
    assert gemm_store(lib, x, w, out) == 0
    got = out.double().cpu().numpy()
    assert np.max(np.abs(got - expected) - 2.0 ** -11 * np.abs(expected)) < 1e-4 * math.sqrt(K)
