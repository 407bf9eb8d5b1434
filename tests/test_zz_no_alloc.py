"""ridge_gemm_launch_noalloc: the GEMM entry point for callers that may not
allocate device memory (code living inside a host framework's memory pool, or
on a path where cudaMalloc is off limits because it synchronises the device).
It uses the library's fixed per-device scratch array instead of an allocated
split-K workspace. These tests call it through the C ABI, on shapes whose
launch does split K, and check it against ridge_gemm_launch twice in a row
(the second call proves the shared scratch was left ready for reuse).

This file is collected last on purpose, and works both alone in a fresh
process and after the rest of the suite."""

import ctypes

import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

CASES = [
    ((512, 512, 4096), (128, 128, 64, 4, 4, 8)),
    ((2048, 2560, 512), (256, 256, 64, 4, 8, 8, 2)),
    ((1000, 1000, 296), (128, 128, 32, 3, 4, 8)),     # ragged, 2-way split: ~8 MB of scratch
]


def _launch_noalloc(rb, cfg, a, b, c, M, N, K):
    cc = cfg.to_c()
    return rb.lib.ridge_gemm_launch_noalloc(ctypes.byref(cc), a.data_ptr(), b.data_ptr(),
                                            c.data_ptr(), M, N, K, K, K, N,
                                            torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("shape,c", CASES, ids=lambda x: "x".join(map(str, x)))
def test_noalloc_matches_allocating_entry_point(shape, c):
    import ridge_b200 as rb
    M, N, K = shape
    cfg = rb.TileConfig(*c)
    need = ctypes.c_int64(0)
    cc = cfg.to_c()
    assert rb.lib.ridge_gemm_workspace_size(ctypes.byref(cc), M, N, K, ctypes.byref(need)) == 0
    assert 0 < need.value <= rb.lib.ridge_gemm_noalloc_scratch_bytes()
    a, b = oracle.unit_inputs(M, N, K, seed=21)
    ad = torch.from_numpy(a.view(np.float16)).cuda()
    bd = torch.from_numpy(b.view(np.float16)).cuda()
    ref = rb.gemm(ad, bd, config=cfg)            # the allocating entry point
    torch.cuda.synchronize()
    ref64 = ref.float().cpu().numpy().astype(np.float64)
    for _ in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        assert _launch_noalloc(rb, cfg, ad, bd, out, M, N, K) == 0
        torch.cuda.synchronize()
        assert rb.device_error() == 0
        rel, _max_abs, excess = oracle.fp16_stats(out.cpu().numpy().view(np.uint16), ref64)
        assert rel <= oracle.REL_FROB_TOL and excess <= oracle.MAX_ABS_EXCESS_TOL, (rel, excess)


def test_noalloc_rejects_launch_that_needs_more_scratch():
    import ridge_b200 as rb
    from ridge_b200._native import RIDGE_ENOSCRATCH
    M, N, K = 16, 8192, 8192          # 32 single-CTA 256x256 tiles split 4 ways: ~25 MB
    cfg = rb.TileConfig(256, 256, 32, 3, 4, 8, 1)
    need = ctypes.c_int64(0)
    cc = cfg.to_c()
    assert rb.lib.ridge_gemm_workspace_size(ctypes.byref(cc), M, N, K, ctypes.byref(need)) == 0
    assert need.value > rb.lib.ridge_gemm_noalloc_scratch_bytes()
    a = torch.zeros((M, K), dtype=torch.float16, device="cuda")
    b = torch.zeros((N, K), dtype=torch.float16, device="cuda")
    c = torch.zeros((M, N), dtype=torch.float16, device="cuda")
    assert _launch_noalloc(rb, cfg, a, b, c, M, N, K) == RIDGE_ENOSCRATCH


def test_noalloc_scratch_recovers_after_an_aborted_launch():
    """A GEMM that gives up mid-launch can leave split-K counters non-zero in
    the shared scratch, which lives as long as the process. Plant that state on
    the host (ridge_selftest_stale_counters: no kernel, no fault), show that a
    split launch then misses its reduction, and that ridge_device_error(clear)
    restores the scratch so the next launch matches the FP64 oracle."""
    import ridge_b200 as rb
    (M, N, K), c = CASES[0]
    cfg = rb.TileConfig(*c)
    a, b = oracle.unit_inputs(M, N, K, seed=5)
    ad = torch.from_numpy(a.view(np.float16)).cuda()
    bd = torch.from_numpy(b.view(np.float16)).cuda()
    ref = oracle.gemm_f64(a, b)
    out = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    assert _launch_noalloc(rb, cfg, ad, bd, out, M, N, K) == 0   # scratch set up
    torch.cuda.synchronize()
    assert rb.device_error() == 0

    assert rb.lib.ridge_selftest_stale_counters(1) == 0
    out.fill_(float("nan"))
    assert _launch_noalloc(rb, cfg, ad, bd, out, M, N, K) == 0
    torch.cuda.synchronize()
    assert torch.isnan(out.float()).any(), "stale counters should have hidden the split tiles"
    assert rb.device_error(clear=True) == 7        # the planted code; clearing resets the scratch

    for _ in range(2):
        out.fill_(float("nan"))
        assert _launch_noalloc(rb, cfg, ad, bd, out, M, N, K) == 0
        torch.cuda.synchronize()
        assert rb.device_error() == 0
        rel, _max_abs, excess = oracle.fp16_stats(out.cpu().numpy().view(np.uint16), ref)
        assert rel <= oracle.REL_FROB_TOL and excess <= oracle.MAX_ABS_EXCESS_TOL, (rel, excess)
