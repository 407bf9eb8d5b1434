"""GPU smoke tests of the calibration microbenchmarks (include/ridge_b200_calibrate.h):
each runs on a small case and its constant must land in the datasheet band the
calibration driver checks before it writes a hardware file (BANDS in
ridge_b200/calibrate.py), as the reference's run-calibration.py:113-137 checks
its bands; repeated runs must agree (the reference's spread check,
bench/calibrate/cal-common.cuh:107-115)."""

import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]


def _band(key, v):
    from ridge_b200.calibrate import BANDS
    lo, hi = BANDS[key]
    assert lo <= v <= hi, "%s = %g outside its band [%g, %g]" % (key, v, lo, hi)


def test_umma_cycles_clock_and_smem_feed():
    from ridge_b200 import calibrate as cal
    cyc = {}
    for n in (64, 128, 256):
        cyc[n], hz = cal.umma(128, n, iters=4000)
    _band("ummaCycles128x256", cyc[256])
    _band("clockHz", hz)
    c256, smem_bpc, overlap = cal.fit_smem(cyc)
    _band("smemBytesPerCycle", smem_bpc)
    assert overlap in (0.0, 1.0)
    # the tensor issue rate scales with N: 128x128 costs about half of 128x256
    assert 0.4 <= cyc[128] / cyc[256] <= 0.75
    again, _ = cal.umma(128, 256, iters=4000)
    assert abs(again - cyc[256]) / cyc[256] < 0.05, (again, cyc[256])


def test_umma_m64_costs_like_m128():
    from ridge_b200 import calibrate as cal
    c128, _ = cal.umma(128, 256, iters=2000)
    c64, _ = cal.umma(64, 256, iters=2000)
    assert 0.4 <= c64 / c128 <= 1.1


def test_tma_fill_rates_in_band():
    from ridge_b200 import calibrate as cal
    per_sm, total = cal.tma(32 << 20, 128, 8)          # L2-resident tensor
    _band("l2BytesPerSec", total)
    assert 8.0 <= per_sm <= 256.0
    _per_sm_h, total_h = cal.tma(1 << 30, 128, 8)      # 8x L2: streams from DRAM
    _band("hbmBytesPerSec", total_h)


def test_tma_fill_scales_with_issuers_and_box_bytes():
    """What the benchmark measures on B200: the rate of one issuing thread is
    set by boxes, not by bytes in flight -- a second issuer or a box of twice
    the bytes (two 128-byte K atoms) nearly doubles it, a deeper ring does not
    lower it."""
    from ridge_b200 import calibrate as cal
    d1, _ = cal.tma(96 << 20, 128, 1, 1, 1)
    d4, _ = cal.tma(96 << 20, 128, 4, 1, 1)
    two_issuers, _ = cal.tma(96 << 20, 128, 4, 1, 1, 2)
    two_atoms, _ = cal.tma(96 << 20, 128, 3, 1, 1, 1, 128)
    assert d4 >= 0.95 * d1
    assert two_issuers >= 1.5 * d4, (two_issuers, d4)
    assert two_atoms >= 1.5 * d4, (two_atoms, d4)
    latency = 128 * 128 / d1
    assert 200 <= latency <= 5000, latency


def test_epilogue_drain_and_write_bandwidth():
    from ridge_b200 import calibrate as cal
    w4, _ = cal.epi(4)
    w8, _ = cal.epi(8)
    assert 2.0 <= w4 <= 256.0 and 2.0 <= w8 <= 256.0
    wr = cal.write_bw(256 << 20)
    cp = cal.copy_bw(512 << 20)
    assert 2e12 <= wr <= 9e12, wr
    assert 2e12 <= cp <= 9e12, cp


def test_launch_overhead():
    from ridge_b200 import calibrate as cal
    s = cal.launch_overhead()
    assert 5e-7 <= s <= 5e-5, s
