"""Pins the CPU oracle (oracle/ridge_oracle.c) to the reference's own code:
golden vectors in tests/golden/reference_gemm.json were produced by the
reference's fillDeterministic, referenceGemm and errorStats
(bench/check-gemm.cu:98-145, :201-259) compiled from its sources. Runs on CPU."""

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = json.loads((Path(__file__).parent / "golden" / "reference_gemm.json").read_text())


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("case", GOLDEN["shapes"], ids=lambda c: "%dx%dx%d" % (c["M"], c["N"], c["K"]))
def test_fill_matches_reference(case):
    M, N, K = case["M"], case["N"], case["K"]
    a = oracle.fill_reference(M * K, case["seed_a"])
    b = oracle.fill_reference(K * N, case["seed_b"])
    assert a[:16].tolist() == case["a_head"]
    assert sha(a) == case["a_sha256"]
    assert sha(b) == case["b_sha256"]


@pytest.mark.parametrize("case", GOLDEN["shapes"], ids=lambda c: "%dx%dx%d" % (c["M"], c["N"], c["K"]))
def test_fp64_gemm_matches_reference(case):
    """Same products, same k order: the oracle's FP64 result is bit-identical to
    referenceGemm's at every sampled element, and the full-matrix sums agree."""
    M, N, K = case["M"], case["N"], case["K"]
    a = oracle.fill_reference(M * K, case["seed_a"]).reshape(M, K)
    b_kn = oracle.fill_reference(K * N, case["seed_b"]).reshape(K, N)
    c = oracle.gemm_f64(a, np.ascontiguousarray(b_kn.T))   # column-major B = (N, K) storage
    for i, j, v in case["samples"]:
        assert c[i, j] == v, (i, j, c[i, j], v)
    assert c.sum() == pytest.approx(case["c_sum"], rel=1e-12, abs=1e-9)
    assert np.abs(c).sum() == pytest.approx(case["c_abs_sum"], rel=1e-12)
    assert (c * c).sum() == pytest.approx(case["c_sq_sum"], rel=1e-12)


def test_reference_loop_order_variant_agrees():
    """The literal reference loop (row-major K x N B) and the column-major fast
    path give identical doubles."""
    case = GOLDEN["shapes"][0]
    M, N, K = case["M"], case["N"], case["K"]
    a = oracle.fill_reference(M * K, case["seed_a"]).reshape(M, K)
    b_kn = oracle.fill_reference(K * N, case["seed_b"]).reshape(K, N)
    c1 = oracle.gemm_f64_reference_loop(a, b_kn)
    c2 = oracle.gemm_f64(a, np.ascontiguousarray(b_kn.T))
    assert np.array_equal(c1, c2)
    rows = np.array([3, 0, M - 1])
    assert np.array_equal(oracle.gemm_f64(a, np.ascontiguousarray(b_kn.T), rows=rows), c1[rows])


def test_checker_self_test_matches_reference():
    """check-gemm.cu:201-259: the statistics of the four self-test vectors equal
    the reference errorStats', and the tolerances accept the clean copy and
    reject the three corruptions."""
    n = 4096
    s = 0xC0FFEE
    ref = np.empty(n, np.float64)
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        ref[i] = ((s >> 16) & 0x7FFF) / 32767.0 - 0.5
    cases = {"exact copy": ref.astype(np.float32),
             "systematic 5% scale": (ref * 1.05).astype(np.float32)}
    bad = ref.astype(np.float32).copy()
    bad[int(n * 0.97):] = (ref[int(n * 0.97):] * 0.5).astype(np.float32)
    cases["last 3% of outputs halved"] = bad
    bad = ref.astype(np.float32).copy()
    bad[n // 3] = np.float32(ref[n // 3] + 1.0)
    cases["one element off by a full unit"] = bad
    for name, got in cases.items():
        frob, max_rel = oracle.error_stats(got, ref)
        gf, gm = GOLDEN["self_test"][name]
        assert frob == pytest.approx(gf, rel=1e-12, abs=1e-15)
        assert max_rel == pytest.approx(gm, rel=1e-12, abs=1e-15)
        rejected = frob > 1e-2 or max_rel > 5e-2   # the reference tolerances
        assert rejected == (name != "exact copy"), name


def test_f16_conversion_round_trip_and_rounding():
    """Binary16 conversion: every finite half round-trips, and ties round to even."""
    bits = np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)
    f = oracle.f16_to_f32(bits)
    finite = np.isfinite(f)
    back = oracle.f32_to_f16(f[finite])
    # -0 and +0 both round-trip to themselves
    assert np.array_equal(back, bits[finite])
    # numpy's float16 cast is IEEE round-to-nearest-even: compare on a sweep
    x = np.linspace(-70000, 70000, 200001, dtype=np.float32)
    x = np.concatenate([x, np.float32(2.0) ** np.arange(-30, 16, dtype=np.float32) * 1.0009765625])
    assert np.array_equal(oracle.f32_to_f16(x), x.astype(np.float16).view(np.uint16))


def test_fp16_stats_accepts_rounded_reference_and_rejects_corruption():
    M, N, K = 64, 48, 4096
    a, b = oracle.unit_inputs(M, N, K, seed=0)
    ref = oracle.gemm_f64(a, b)
    rounded = oracle.f32_to_f16(ref.astype(np.float32))
    rel, max_abs, excess = oracle.fp16_stats(rounded, ref)
    assert rel <= oracle.REL_FROB_TOL and excess <= oracle.MAX_ABS_EXCESS_TOL
    assert max_abs > 0.02 or np.abs(ref).max() < 32   # half-ulp rounding alone can exceed 2e-2
    bad = rounded.copy()
    bad[5, 7] = oracle.f32_to_f16(np.array([ref[5, 7] + 0.25], np.float32))[0]
    assert oracle.fp16_stats(bad, ref)[2] > oracle.MAX_ABS_EXCESS_TOL


def test_unit_inputs_range_and_stream():
    a, b = oracle.unit_inputs(16, 8, 32, seed=0)
    fa, fb = oracle.f16_to_f32(a), oracle.f16_to_f32(b)
    assert fa.min() >= -1 and fa.max() <= 1 and fb.min() >= -1 and fb.max() <= 1
    # B continues A's stream: drawing A and B as one run gives the same bits
    both, _ = oracle.unit_inputs(16 * 32 + 8 * 32, 0, 1, seed=0)
    assert np.array_equal(both.ravel(), np.concatenate([a.ravel(), b.ravel()]))


@pytest.mark.skipif(not oracle.reference_available(), reason="reference library not built here")
def test_reference_a100_model_matches_its_hand_derived_example():
    """The reference's own model (src/model.cpp, linked into oracle/_ref) on its
    worked example, checked against the hand-derived values of
    test/test-model.cpp:47-101 -- pins the parity shim."""
    p = oracle.Reference().predict_a100(4096, 4096, 4096, 128, 128, 32, 64, 64, 3, 128)
    assert p["tComputeCycles"] == pytest.approx(512.0)
    assert p["tSmemCycles"] == pytest.approx(256.0)
    assert p["ctasPerSM"] == 3
    assert p["waveEfficiency"] == pytest.approx(1024.0 / 1296.0)
    assert p["envelopeEfficiency"] == pytest.approx(0.975248, abs=1e-6)
    assert p["predictedTFLOPS"] == pytest.approx(120.158068, abs=1e-4)
    assert p["bottleneck"] == 1  # Smem
