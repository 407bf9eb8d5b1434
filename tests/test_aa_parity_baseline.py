"""GPU parity at the workloads that are timed, and on the reference's own
correctness cases. Collected first, so a `-x` run cannot stop before them.

1. The reference's six correctness shapes with its own fill and seeds
   (bench/check-gemm.cu:87-94, :266-267; fillDeterministic :139-145), checked
   with the reference's tolerances (errorStats, relative Frobenius <= 1e-2 and
   max |d| / max |ref| <= 5e-2, check-gemm.cu:32-37) and with this build's
   FP16 tolerances (oracle.REL_FROB_TOL / MAX_ABS_EXCESS_TOL).
2. The reference's own kernel (gemmMmaKernel, compiled unchanged for sm_100a
   into oracle/_ref) on identical inputs, B in its row-major K x N layout and C
   in FP32: both it and this build's kernel agree with the FP64 oracle.
3. BASELINE shapes, compared with the FP64 oracle on a row sample (first,
   last and seeded random rows): 4096^3 with the bench tile and the best
   single-CTA tile; 8192 x 8192 x 128 on BK=32, 64 and 128 tiles; one
   16384^3 N-slab (as one rank of an 8-way split) launched on one GPU.

Inputs for 3 are the benchmark fill (LCG U(-1,1), seed 0, A then B), generated
on the host by the oracle, independent of the device fill.
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

# Reference tolerances (bench/check-gemm.cu:32, :37).
REF_REL_TOL = 1e-2
REF_MAX_ELEM_TOL = 5e-2

# bench/check-gemm.cu:87-94
REF_SHAPES = [(256, 256, 64), (256, 512, 128), (512, 256, 192), (1024, 1024, 64),
              (1024, 512, 1024), (2048, 2048, 2048)]

BENCH_TILE = (256, 256, 64, 6, 4, 8, 2)        # bench.py's headline tile
BEST_1CTA_4096 = (128, 256, 64, 4, 4, 8, 1)    # best single-CTA tile of the 4096^3 sweep

TILES_REF_SHAPES = [
    (128, 128, 32, 3, 4, 8),
    (128, 256, 64, 4, 4, 8),
    (64, 64, 64, 4, 8, 8),
    (256, 256, 64, 6, 4, 8, 2),    # bench tile
    (256, 128, 128, 4, 4, 8, 2),
]


def _cfg(t):
    return rb.TileConfig(*t)


def _sample_rows(M, n_rand=32, edge=16, seed=1):
    rng = np.random.default_rng(seed)
    rows = set(range(min(edge, M))) | set(range(max(0, M - edge), M))
    rows |= set(rng.choice(M, size=min(n_rand, M), replace=False).tolist())
    return np.array(sorted(rows), np.int64)


def _ref_inputs(M, N, K):
    a = oracle.fill_reference(M * K, 0x1234 + M).reshape(M, K)
    b_kn = oracle.fill_reference(K * N, 0x9ABC + N).reshape(K, N)
    return a, b_kn


@pytest.fixture(scope="module")
def ref_cases():
    out = {}
    for (M, N, K) in REF_SHAPES:
        a, b_kn = _ref_inputs(M, N, K)
        b_nk = np.ascontiguousarray(b_kn.T)
        out[(M, N, K)] = (a, b_kn, b_nk, oracle.gemm_f64(a, b_nk))
    return out


@pytest.mark.parametrize("shape", REF_SHAPES, ids=lambda s: "%dx%dx%d" % s)
@pytest.mark.parametrize("tile", TILES_REF_SHAPES, ids=lambda t: "x".join(map(str, t)))
def test_reference_correctness_shapes(shape, tile, ref_cases):
    M, N, K = shape
    a, _, b_nk, ref = ref_cases[shape]
    cfg = _cfg(tile)
    if not rb.valid_for_shape(cfg, M, N, K):
        pytest.skip("tile not valid for this shape")
    c = to_host_bits(run_gemm(cfg, to_dev(a), to_dev(b_nk), M, N, K))
    # the reference's own criteria on the output as the reference reads it (FP32)
    frob, max_rel = oracle.error_stats(oracle.f16_to_f32(c), ref)
    assert frob <= REF_REL_TOL and max_rel <= REF_MAX_ELEM_TOL, (frob, max_rel)
    # and this build's stricter FP16 criteria
    assert_close(c, ref, "%s %dx%dx%d (reference fill)" % (cfg.tag(), M, N, K))


def test_reference_kernel_on_b200_agrees(ref_cases):
    """The reference's own gemmMmaKernel, built for sm_100a from its sources,
    and this build's kernel, run on identical inputs: both pass the reference's
    checker against the FP64 oracle, and they agree with each other to the
    FP16 output rounding."""
    if not oracle.reference_available():
        pytest.skip("oracle/_ref/libridge_ref.so not built (needs the reference sources)")
    ref_lib = oracle.Reference()
    variants = ref_lib.variants()
    assert variants, "reference variant table is empty"
    ran = 0
    for (M, N, K) in [(256, 512, 128), (1024, 512, 1024), (2048, 2048, 2048)]:
        a, b_kn, b_nk, ref = ref_cases[(M, N, K)]
        a_d, bkn_d, bnk_d = to_dev(a), to_dev(b_kn), to_dev(b_nk)
        ours = to_host_bits(run_gemm(_cfg(BENCH_TILE), a_d, bnk_d, M, N, K))
        ours_f = oracle.f16_to_f32(ours)
        for i, v in enumerate(variants):
            if M % v["BM"] or N % v["BN"] or K % v["BK"]:
                continue
            c32 = torch.zeros((M, N), dtype=torch.float32, device="cuda")
            st = ref_lib.launch(i, a_d.data_ptr(), bkn_d.data_ptr(), c32.data_ptr(), M, N, K,
                                torch.cuda.current_stream().cuda_stream)
            assert st == 0, "reference launch %d returned %d" % (i, st)
            torch.cuda.synchronize()
            got = c32.cpu().numpy()
            frob, max_rel = oracle.error_stats(got, ref)
            assert frob <= REF_REL_TOL and max_rel <= REF_MAX_ELEM_TOL, (v, frob, max_rel)
            # FP32-output reference kernel vs FP16-output B200 kernel: they
            # differ by the FP16 rounding of C plus accumulation order.
            d = np.abs(got.astype(np.float64) - ours_f)
            assert d.max() <= 2.0 ** -10 * max(1.0, float(np.abs(got).max())) + 1e-3, (v, d.max())
            ran += 1
    assert ran >= 3, "no reference variant divided the shapes"


@pytest.fixture(scope="module")
def inputs_4096():
    M = N = K = 4096
    a, b = oracle.unit_inputs(M, N, K, seed=0)
    rows = _sample_rows(M)
    return a, b, rows, oracle.gemm_f64(a, b, rows=rows)


@pytest.mark.parametrize("tile", [BENCH_TILE, BEST_1CTA_4096, (256, 256, 128, 3, 8, 8, 2)],
                         ids=lambda t: "x".join(map(str, t)))
def test_baseline_4096_cube(tile, inputs_4096):
    a, b, rows, ref = inputs_4096
    cfg = _cfg(tile)
    c = run_gemm(cfg, to_dev(a), to_dev(b), 4096, 4096, 4096)
    got = to_host_bits(c)[rows]
    assert_close(got, ref, "%s 4096^3 (%d sampled rows)" % (cfg.tag(), rows.size))


@pytest.fixture(scope="module")
def inputs_short_k():
    M, N, K = 8192, 8192, 128
    a, b = oracle.unit_inputs(M, N, K, seed=0)
    rows = _sample_rows(M, n_rand=64)
    return a, b, rows, oracle.gemm_f64(a, b, rows=rows)


@pytest.mark.parametrize("tile", [(128, 256, 64, 4, 8, 8), (128, 256, 128, 2, 8, 8),
                                  (128, 128, 32, 3, 4, 8), (256, 256, 32, 4, 8, 8, 1),
                                  (256, 128, 128, 3, 4, 8, 2), (64, 128, 32, 4, 4, 8)],
                         ids=lambda t: "x".join(map(str, t)))
def test_baseline_short_k(tile, inputs_short_k):
    a, b, rows, ref = inputs_short_k
    cfg = _cfg(tile)
    c = run_gemm(cfg, to_dev(a), to_dev(b), 8192, 8192, 128)
    assert_close(to_host_bits(c)[rows], ref, "%s 8192x8192x128" % cfg.tag())


def test_baseline_16384_slab():
    """One rank's slab of the 16384^3 GEMM split 8 ways: M=16384, N=2048 (B rows
    [0, 2048) of the N x K storage), K=16384, with the bench tile."""
    M, NS, K = 16384, 2048, 16384
    a, b = oracle.unit_inputs(M, NS, K, seed=0)
    rows = _sample_rows(M, n_rand=24, edge=4)
    ref = oracle.gemm_f64(a, b, rows=rows)
    a_d = to_dev(a)
    b_d = to_dev(b)
    del a, b
    c = run_gemm(_cfg(BENCH_TILE), a_d, b_d, M, NS, K)
    assert_close(to_host_bits(c)[rows], ref, "16384x2048x16384 slab")
