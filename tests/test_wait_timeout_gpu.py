"""Failure detection on the GPU without a fault: a bounded device wait that
nothing completes gives up after its limit, records its code in the device
error word and returns, and the context stays usable (a GEMM right after is
correct and the error word is clean again)."""

import ctypes as C

import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]


@pytest.mark.parametrize("limit_ms", [5, 50])
def test_expired_wait_reports_and_context_survives(limit_ms):
    import ridge_b200 as rb
    code, waited = C.c_int32(-1), C.c_int64(0)
    st = rb.lib.ridge_selftest_wait_timeout(limit_ms * 1000000, C.byref(code), C.byref(waited))
    assert st == 0, rb.lib.ridge_status_string(st).decode()
    assert code.value == 6
    assert limit_ms * 1e6 <= waited.value < limit_ms * 1e6 + 5e8
    assert rb.device_error() == 0
    a, b = rb.synthetic_inputs(512, 512, 256)
    c = rb.gemm(a, b, config=rb.TileConfig(128, 128, 64, 4, 4, 8))
    ref = (a.float() @ b.float().t()).half()
    torch.cuda.synchronize()
    assert rb.device_error() == 0
    assert ((c.float() - ref.float()).norm() / ref.float().norm()).item() < 1e-3


def test_selftest_rejects_out_of_range_limits():
    import ridge_b200 as rb
    code, waited = C.c_int32(), C.c_int64()
    for bad in (0, 999999, 2000000001):
        assert rb.lib.ridge_selftest_wait_timeout(bad, C.byref(code), C.byref(waited)) == -1


def test_cleared_error_resets_cached_workspace_counters():
    """Stale split-K counters in the library's cached workspace (the state a
    GEMM that gave up can leave) are reset by ridge_device_error(clear): the
    next split launch through ridge_gemm_launch matches the FP64 oracle."""
    import numpy as np

    import oracle
    import ridge_b200 as rb
    M, N, K = 512, 512, 4096
    cfg = rb.TileConfig(128, 128, 64, 4, 4, 8)
    a, b = oracle.unit_inputs(M, N, K, seed=9)
    ad = torch.from_numpy(a.view(np.float16)).cuda()
    bd = torch.from_numpy(b.view(np.float16)).cuda()
    ref = oracle.gemm_f64(a, b)
    rb.gemm(ad, bd, config=cfg)                  # the stream's workspace exists
    torch.cuda.synchronize()
    assert rb.lib.ridge_selftest_stale_counters(3) == 0
    assert rb.device_error(clear=True) == 7
    for _ in range(2):
        c = rb.gemm(ad, bd, config=cfg)
        torch.cuda.synchronize()
        assert rb.device_error() == 0
        rel, _m, excess = oracle.fp16_stats(c.cpu().numpy().view(np.uint16), ref)
        assert rel <= oracle.REL_FROB_TOL and excess <= oracle.MAX_ABS_EXCESS_TOL, (rel, excess)
