"""GPU parity of the tcgen05 GEMM family against the FP64 CPU oracle.

Inputs are the benchmark fill (LCG, U(-1,1), seed 0, A then B) unless noted.
Acceptance: relative Frobenius error <= 1e-3 and max |dC| <= 2e-2 beyond the
half-ulp rounding of the FP16 output (oracle.REL_FROB_TOL / MAX_ABS_EXCESS_TOL).
"""

import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

if torch.cuda.is_available():
    import ridge_b200 as rb
    from _gpu import assert_close, run_gemm, to_dev, to_host_bits
    TileConfig = rb.TileConfig
else:  # collected on CPU only to be skipped
    TileConfig = None


def _cfg(*a):
    from ridge_b200 import TileConfig as T
    return T(*a)


# A spread of tile configs over BM, BN, BK, warps, stages (one per shape kind).
CONFIGS = [
    (128, 128, 32, 3, 4, 8),
    (128, 256, 64, 4, 4, 8),
    (128, 64, 64, 4, 8, 8),
    (64, 128, 32, 2, 4, 1),
    (64, 64, 64, 5, 8, 4),
    (256, 128, 64, 3, 4, 8),
    (256, 256, 32, 3, 8, 16),
    (64, 256, 64, 4, 4, 2),
    (256, 128, 64, 4, 4, 8, 2),   # 2-CTA pair tiles
    (256, 256, 64, 4, 8, 8, 2),
    (256, 64, 32, 3, 4, 3, 2),
    (256, 128, 32, 2, 8, 8, 1),   # single-CTA 256-row tile
    (128, 128, 128, 3, 4, 8),     # BK=128: two K atoms per TMA box (3-D map)
    (256, 128, 128, 4, 4, 8, 2),
    (256, 256, 128, 3, 8, 8, 2),
    (64, 256, 128, 2, 4, 4),
]


@pytest.fixture(scope="module")
def shape_1024():
    a, b = oracle.unit_inputs(1024, 1024, 1024, seed=0)
    ref = oracle.gemm_f64(a, b)
    return a, b, ref


@pytest.mark.parametrize("c", CONFIGS, ids=lambda c: "x".join(map(str, c)))
def test_config1_shape_all_kinds(c, shape_1024):
    a, b, ref = shape_1024
    cfg = _cfg(*c)
    out = run_gemm(cfg, to_dev(a), to_dev(b), 1024, 1024, 1024)
    assert_close(to_host_bits(out), ref, cfg.tag())


# Ragged shapes: M/N/K tails in every dimension, K below one BK, single tiles.
RAGGED = [(200, 136, 72), (1, 8, 8), (129, 257, 33), (64, 64, 16), (300, 520, 1000),
          (17, 1000, 264)]


@pytest.mark.parametrize("shape", RAGGED, ids=lambda s: "%dx%dx%d" % s)
@pytest.mark.parametrize("c", [CONFIGS[0], CONFIGS[1], CONFIGS[3], CONFIGS[5], CONFIGS[8],
                               CONFIGS[10]],
                         ids=lambda c: "x".join(map(str, c)))
def test_ragged_shapes(shape, c):
    M, N, K = shape
    a, b = oracle.unit_inputs(M, N, K, seed=7)
    ref = oracle.gemm_f64(a, b)
    cfg = _cfg(*c)
    # TMA needs 16-byte row pitches: a K that is not a multiple of 8 runs with
    # padded leading dimensions (the pad columns hold garbage the GEMM must ignore).
    ld = (K + 7) // 8 * 8
    ad = torch.full((M, ld), 7.0, dtype=torch.float16, device="cuda")
    bd = torch.full((N, ld), -3.0, dtype=torch.float16, device="cuda")
    ad[:, :K] = to_dev(a)
    bd[:, :K] = to_dev(b)
    out = run_gemm(cfg, ad, bd, M, N, K)
    assert_close(to_host_bits(out), ref, "%s %dx%dx%d" % (cfg.tag(), M, N, K))


def test_every_registered_variant():
    """The whole variant table on one shape with tails in M and N."""
    M, N, K = 520, 392, 256
    a, b = oracle.unit_inputs(M, N, K, seed=3)
    ref = oracle.gemm_f64(a, b)
    ad, bd = to_dev(a), to_dev(b)
    for v in rb.variants():
        out = run_gemm(v.config, ad, bd, M, N, K)
        assert_close(to_host_bits(out), ref, v.config.tag())


@pytest.mark.parametrize("c", [CONFIGS[0], CONFIGS[3], CONFIGS[8]], ids=lambda c: "x".join(map(str, c)))
def test_padded_ldc_leaves_padding_untouched(c):
    """C with a padded row pitch: the epilogue's clipped TMA stores must not
    write the padding columns (sentinel NaN survives)."""
    M, N, K = 300, 200, 128
    a, b = oracle.unit_inputs(M, N, K, seed=11)
    ref = oracle.gemm_f64(a, b)
    cfg = _cfg(*c)
    out = run_gemm(cfg, to_dev(a), to_dev(b), M, N, K, ldc=N + 24)
    bits = to_host_bits(out)
    assert np.isnan(bits[:, N:].view(np.float16).astype(np.float32)).all()
    assert_close(np.ascontiguousarray(bits[:, :N]), ref, cfg.tag())


@pytest.mark.parametrize("c", [CONFIGS[0], CONFIGS[4], CONFIGS[8]], ids=lambda c: "x".join(map(str, c)))
def test_unaligned_c_uses_direct_stores(c):
    """A C pointer that is not 16-byte aligned, or a pitch that is not a
    multiple of 8, takes the register-to-global epilogue; results must match."""
    M, N, K = 130, 77, 64
    a, b = oracle.unit_inputs(M, N, K, seed=5)
    ref = oracle.gemm_f64(a, b)
    cfg = _cfg(*c)
    ldc = N + 2
    buf = torch.full((M * ldc + 8,), float("nan"), dtype=torch.float16, device="cuda")
    cview = buf[1:1 + M * ldc]           # 2-byte offset: not 16-byte aligned
    ad, bd = to_dev(a), to_dev(b)
    st = rb.launch_raw(cfg, ad.data_ptr(), bd.data_ptr(), cview.data_ptr(), M, N, K, K, K, ldc,
                       torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    assert rb.device_error() == 0
    got = to_host_bits(cview).reshape(M, ldc)
    assert np.isnan(got[:, N:].view(np.float16).astype(np.float32)).all()
    assert_close(np.ascontiguousarray(got[:, :N]), ref, cfg.tag())


def test_k_zero_writes_zeros():
    M, N = 64, 48
    cfg = _cfg(*CONFIGS[0])
    a = torch.empty((M, 8), dtype=torch.float16, device="cuda")
    b = torch.empty((N, 8), dtype=torch.float16, device="cuda")
    c = torch.full((M, N), 3.0, dtype=torch.float16, device="cuda")
    assert rb.launch_raw(cfg, a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, 0, 8, 8, N, 0) == 0
    torch.cuda.synchronize()
    assert bool((c == 0).all())


# Split-K tail: (shape, config) pairs whose tile count leaves the last round of
# the persistent grid partly idle, so the launcher splits tiles along K.
SPLITK_CASES = [
    ((512, 512, 4096), (128, 128, 64, 4, 4, 8)),          # 16 tiles -> 8-way split
    ((16, 2048, 4096), (128, 256, 64, 4, 8, 8)),          # skinny M
    ((512, 768, 2048), (256, 256, 64, 4, 4, 8, 2)),       # 2-CTA pairs, 8-way
    ((1000, 1000, 1000), (128, 128, 32, 3, 4, 8)),        # ragged + 2-way
    ((1280, 2048, 1024), (128, 128, 64, 4, 4, 8)),        # whole rounds + split tail
    ((2048, 2560, 512), (256, 256, 64, 4, 8, 8, 2)),      # pairs: whole rounds + split tail
    ((640, 384, 1024), (64, 128, 64, 4, 4, 1)),           # M=64 UMMA rows
]


@pytest.mark.parametrize("shape,c", SPLITK_CASES, ids=lambda x: "x".join(map(str, x)))
def test_split_k_tail(shape, c):
    import ctypes
    M, N, K = shape
    cfg = _cfg(*c)
    ws = ctypes.c_int64(0)
    cc = cfg.to_c()
    assert rb.lib.ridge_gemm_workspace_size(ctypes.byref(cc), M, N, K, ctypes.byref(ws)) == 0
    assert ws.value > 0, "expected this case to split"
    a, b = oracle.unit_inputs(M, N, K, seed=13)
    ref = oracle.gemm_f64(a, b)
    ad, bd = to_dev(a), to_dev(b)
    for _ in range(2):  # twice: counters must come back to zero
        out = run_gemm(cfg, ad, bd, M, N, K)
        assert_close(to_host_bits(out), ref, "split " + cfg.tag())
    import dataclasses
    whole = run_gemm(dataclasses.replace(cfg, split_k=1), ad, bd, M, N, K)
    assert_close(to_host_bits(whole), ref, "no split " + cfg.tag())


def test_caller_workspace_launch():
    """ridge_gemm_launch_ws on a caller-owned, zeroed workspace; a too-small
    workspace is refused."""
    import ctypes
    M, N, K = 512, 512, 4096
    cfg = _cfg(128, 128, 64, 4, 4, 8)
    cc = cfg.to_c()
    need = ctypes.c_int64(0)
    assert rb.lib.ridge_gemm_workspace_size(ctypes.byref(cc), M, N, K, ctypes.byref(need)) == 0
    ws = torch.zeros(need.value // 4 + 64, dtype=torch.int32, device="cuda")
    a, b = oracle.unit_inputs(M, N, K, seed=17)
    ref = oracle.gemm_f64(a, b)
    ad, bd = to_dev(a), to_dev(b)
    c = torch.empty((M, N), dtype=torch.float16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert rb.lib.ridge_gemm_launch_ws(ctypes.byref(cc), ad.data_ptr(), bd.data_ptr(),
                                       c.data_ptr(), M, N, K, K, K, N, ws.data_ptr(),
                                       need.value - 4, s) == -1
    for _ in range(2):
        assert rb.lib.ridge_gemm_launch_ws(ctypes.byref(cc), ad.data_ptr(), bd.data_ptr(),
                                           c.data_ptr(), M, N, K, K, K, N, ws.data_ptr(),
                                           need.value, s) == 0
        torch.cuda.synchronize()
        assert rb.device_error() == 0
        assert_close(to_host_bits(c), ref, "caller workspace")


@pytest.mark.parametrize("shape", [(200, 136, 192), (129, 257, 64), (300, 520, 1088)],
                         ids=lambda s: "%dx%dx%d" % s)
@pytest.mark.parametrize("c", [CONFIGS[11], CONFIGS[12], CONFIGS[13], CONFIGS[14]],
                         ids=lambda c: "x".join(map(str, c)))
def test_bk128_tails(shape, c):
    """BK=128 stages with M/N tails and a K that ends mid-stage (K = 64 mod 128)."""
    M, N, K = shape
    a, b = oracle.unit_inputs(M, N, K, seed=9)
    ref = oracle.gemm_f64(a, b)
    cfg = _cfg(*c)
    out = run_gemm(cfg, to_dev(a), to_dev(b), M, N, K)
    assert_close(to_host_bits(out), ref, "%s %dx%dx%d" % (cfg.tag(), M, N, K))


def test_split_k_launches_overlap_on_two_streams():
    """Two split-K launches running at once on two streams, each with the
    library's workspace for its stream. A split tile is reduced by whichever
    split arrives last, so neither grid waits on CTAs the other grid may be
    keeping off the SMs; both results match the FP64 oracle."""
    M, N, K = 1280, 2048, 1024
    cfg = _cfg(128, 128, 64, 4, 4, 8)
    a1, b1 = oracle.unit_inputs(M, N, K, seed=31)
    a2, b2 = oracle.unit_inputs(M, N, K, seed=32)
    ref1, ref2 = oracle.gemm_f64(a1, b1), oracle.gemm_f64(a2, b2)
    d = [(to_dev(a1), to_dev(b1)), (to_dev(a2), to_dev(b2))]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [torch.empty((M, N), dtype=torch.float16, device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    for _ in range(4):
        for o in outs:
            o.fill_(float("nan"))
        torch.cuda.synchronize()
        for (ad, bd), o, s in zip(d, outs, streams):
            assert rb.launch_raw(cfg, ad.data_ptr(), bd.data_ptr(), o.data_ptr(), M, N, K, K, K,
                                 N, s.cuda_stream) == 0
        torch.cuda.synchronize()
        assert rb.device_error() == 0
        assert_close(to_host_bits(outs[0]), ref1, "stream 1")
        assert_close(to_host_bits(outs[1]), ref2, "stream 2")


# Split tails after many whole-tile rounds: the launcher puts split ranges
# after the whole tiles there (with few rounds it puts them first).
MANY_ROUND_CASES = [
    ((3072, 11648, 1024), (128, 128, 32, 3, 4, 8)),        # 7 rounds of 296 units + 112 split
    ((6400, 6400, 1024), (256, 256, 128, 3, 8, 8, 2)),     # 8 rounds of 74 pairs + 33 split
]


@pytest.mark.parametrize("shape,c", MANY_ROUND_CASES, ids=lambda x: "x".join(map(str, x)))
def test_split_k_after_many_rounds(shape, c):
    import ctypes
    M, N, K = shape
    cfg = _cfg(*c)
    ws = ctypes.c_int64(0)
    cc = cfg.to_c()
    assert rb.lib.ridge_gemm_workspace_size(ctypes.byref(cc), M, N, K, ctypes.byref(ws)) == 0
    assert ws.value > 0, "expected this case to split"
    a, b = oracle.unit_inputs(M, N, K, seed=41)
    rows = np.unique(np.concatenate([np.arange(8), np.arange(M - 8, M),
                                     np.random.default_rng(3).choice(M, 48, replace=False)]))
    ref = oracle.gemm_f64(a, b, rows=rows)
    ad, bd = to_dev(a), to_dev(b)
    for _ in range(2):
        out = run_gemm(cfg, ad, bd, M, N, K)
        assert_close(to_host_bits(out)[rows], ref, "split after rounds " + cfg.tag())
