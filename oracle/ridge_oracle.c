/*
 * ridge_oracle.c -- CPU oracle for the ridge GEMM hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker, never the product: only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
 * load it. The product path (ridge_b200/, libridge_b200.so) never calls into it.
 *
 * A plain-C restatement of the reference's host-side algorithms for the path,
 * each function citing the reference file:line it follows (paths relative to
 * the reference project root, i-nahc/ridge):
 *   - the deterministic LCG fill              bench/check-gemm.cu:139-145
 *   - the FP64 host GEMM                       bench/check-gemm.cu:98-108
 *   - the two-criterion error statistics       bench/check-gemm.cu:121-135
 *   - IEEE binary16 conversion (what __float2half / __half2float compute on the host)
 *
 * Parity is pinned in tests/test_oracle.py against golden vectors produced by
 * the reference's own code (oracle/_ref, built from the reference sources by
 * oracle/Makefile) and committed under tests/golden/.
 *
 * Build: cc -O2 -fPIC -shared -fopenmp ridge_oracle.c -o libridge_oracle.so -lm
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

/* ------------------------------------------------------------ binary16 */

/* IEEE 754 binary32 -> binary16, round to nearest even, with subnormals,
 * infinities and NaN (quiet, payload truncated). Written from the format
 * definition. */
uint16_t oracle_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) { /* inf or nan */
        if (absx > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((absx >> 13) & 0x3ffu));
        return (uint16_t)(sign | 0x7c00u);
    }
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520 -> inf */
    if (absx < 0x38800000u) {                                     /* result subnormal or zero */
        if (absx < 0x33000000u) return (uint16_t)sign;            /* < 2^-25: rounds to 0 */
        const uint32_t e = absx >> 23;                            /* 102..112 */
        const uint32_t mant = (absx & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126u - e;                          /* 14..24 */
        uint32_t r = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (r & 1u))) r += 1u;
        return (uint16_t)(sign | r);
    }
    /* normal: rebias exponent 127 -> 15, keep 10 mantissa bits, RNE */
    uint32_t r = ((absx - 0x38000000u) >> 13);
    const uint32_t rem = absx & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r += 1u;
    return (uint16_t)(sign | r);
}

float oracle_f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t e = ((uint32_t)h >> 10) & 0x1fu;
    const uint32_t m = (uint32_t)h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else { /* subnormal: value = m * 2^-24 */
            float v = (float)m * 5.9604644775390625e-08f;
            memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

void oracle_f32_to_f16_array(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = oracle_f32_to_f16(in[i]);
}

void oracle_f64_to_f16_array(const double* in, uint16_t* out, size_t n) {
    /* double -> float -> half matches fp16(C) only up to double rounding, which
     * is irrelevant at the tolerances used; callers that need exact fp16(x)
     * of a double use this for the comparison target. */
    for (size_t i = 0; i < n; ++i) out[i] = oracle_f32_to_f16((float)in[i]);
}

void oracle_f16_to_f32_array(const uint16_t* in, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = oracle_f16_to_f32(in[i]);
}

/* ------------------------------------------------------------ inputs */

/* The reference fill (check-gemm.cu:139-145, measure.cu:96-102): 32-bit LCG
 * s = s*1664525 + 1013904223, value = ((s>>16)&0x7fff)/32767 - 0.5 in FP32,
 * rounded to FP16. */
void oracle_fill_reference(uint16_t* out, size_t n, uint32_t seed) {
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) {
        s = s * 1664525u + 1013904223u;
        const float v = ((float)((s >> 16) & 0x7fffu) / 32767.0f) - 0.5f;
        out[i] = oracle_f32_to_f16(v);
    }
}

/* The benchmark fill: the same LCG recurrence mapped to U(-1,1),
 * value = 2*((s>>16)&0x7fff)/32767 - 1, continuing from *state so that A and
 * then B can be drawn from one stream seeded with 0. */
void oracle_fill_unit(uint16_t* out, size_t n, uint32_t* state) {
    uint32_t s = *state;
    for (size_t i = 0; i < n; ++i) {
        s = s * 1664525u + 1013904223u;
        const float v = 2.0f * ((float)((s >> 16) & 0x7fffu) / 32767.0f) - 1.0f;
        out[i] = oracle_f32_to_f16(v);
    }
    *state = s;
}

/* ------------------------------------------------------------ FP64 GEMM */

/* FP64 host GEMM (check-gemm.cu:98-108): for each (i, j) a sequential k loop
 * accumulating double(a) * double(b) in double. A is M x K row-major (lda). B
 * is addressed as B(k, j) = B[k * sbk + j * sbj]: the reference's row-major
 * K x N B is (sbk, sbj) = (N, 1); this build's column-major B (N x K storage,
 * ldb) is (1, ldb). C is M x N row-major (ldc). Rows [row0, row1) only, so a
 * caller can sample rows or split the work across threads. */
void oracle_gemm_f64_rows(const uint16_t* A, int64_t lda, const uint16_t* B, int64_t sbk,
                          int64_t sbj, double* C, int64_t ldc, int64_t N, int64_t K, int64_t row0,
                          int64_t row1) {
    for (int64_t i = row0; i < row1; ++i) {
        for (int64_t j = 0; j < N; ++j) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; ++k) {
                acc += (double)oracle_f16_to_f32(A[i * lda + k]) *
                       (double)oracle_f16_to_f32(B[k * sbk + j * sbj]);
            }
            C[i * ldc + j] = acc;
        }
    }
}

/* Same product with B converted to double once up front (numerically
 * identical: every product and the summation order are unchanged) and the
 * requested rows spread over OpenMP threads. Bnk is the N x K storage of a
 * column-major B (ldb). rows == NULL means all M rows; otherwise C row r holds
 * output row rows[r]. scratch_b must hold N*K doubles. */
void oracle_gemm_f64_fast(const uint16_t* A, int64_t lda, const uint16_t* Bnk, int64_t ldb,
                          double* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                          const int64_t* rows, int64_t nrows, double* scratch_b) {
    for (int64_t j = 0; j < N; ++j)
        for (int64_t k = 0; k < K; ++k) scratch_b[j * K + k] = oracle_f16_to_f32(Bnk[j * ldb + k]);
    const int64_t count = rows ? nrows : M;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t r = 0; r < count; ++r) {
        const int64_t i = rows ? rows[r] : r;
        const uint16_t* a = A + i * lda;
        for (int64_t j = 0; j < N; ++j) {
            const double* b = scratch_b + j * K;
            double acc = 0.0;
            for (int64_t k = 0; k < K; ++k) acc += (double)oracle_f16_to_f32(a[k]) * b[k];
            C[r * ldc + j] = acc;
        }
    }
}

/* ------------------------------------------------------------ checking */

/* errorStats (check-gemm.cu:121-135): relative Frobenius norm of (got - ref)
 * and the largest single-element error scaled by max|ref|, with the same
 * zero-denominator conventions. */
void oracle_error_stats(const float* got, const double* ref, size_t n, double* frob,
                        double* max_rel) {
    double num = 0.0, den = 0.0, max_diff = 0.0, max_ref = 0.0;
    for (size_t i = 0; i < n; ++i) {
        const double r = ref[i];
        const double d = (double)got[i] - r;
        num += d * d;
        den += r * r;
        if (fabs(d) > max_diff) max_diff = fabs(d);
        if (fabs(r) > max_ref) max_ref = fabs(r);
    }
    *frob = den > 0.0 ? sqrt(num) / sqrt(den) : (num == 0.0 ? 0.0 : 1.0);
    *max_rel = max_ref > 0.0 ? max_diff / max_ref : (max_diff == 0.0 ? 0.0 : 1.0);
}

/* The B200 acceptance statistics for FP16 output. rel_frob as above; the
 * elementwise bound is stated on |C_fp16 - C_fp64| minus half an FP16 ulp of
 * the reference value (the unavoidable output rounding), so "max_abs_excess
 * <= 2e-2" is the absolute 2e-2 criterion applied to the arithmetic, not to
 * the final rounding step. Also returns the plain max |dC|. */
void oracle_fp16_stats(const uint16_t* got, int64_t ldg, const double* ref, int64_t ldr,
                       int64_t M, int64_t N, double* rel_frob, double* max_abs,
                       double* max_abs_excess) {
    double num = 0.0, den = 0.0, ma = 0.0, mx = -1e300;
    for (int64_t i = 0; i < M; ++i) {
        for (int64_t j = 0; j < N; ++j) {
            const double r = ref[i * ldr + j];
            const double g = (double)oracle_f16_to_f32(got[i * ldg + j]);
            const double d = fabs(g - r);
            num += d * d;
            den += r * r;
            if (d > ma) ma = d;
            /* half ulp of |r| in binary16: 2^(floor(log2|r|) - 11), min 2^-25 */
            double half_ulp = ldexp(1.0, -25);
            if (fabs(r) >= ldexp(1.0, -14)) {
                int e;
                frexp(fabs(r), &e); /* |r| = f * 2^e, f in [0.5, 1) */
                half_ulp = ldexp(1.0, e - 1 - 11);
            }
            const double excess = d - half_ulp;
            if (excess > mx) mx = excess;
        }
    }
    *rel_frob = den > 0.0 ? sqrt(num) / sqrt(den) : (num == 0.0 ? 0.0 : 1.0);
    *max_abs = ma;
    *max_abs_excess = (M * N > 0) ? mx : 0.0;
}
