/*
 * ridge_b200_calibrate.h -- sm_100a calibration microbenchmarks for the B200
 * cost model (C ABI; same status convention as ridge_b200.h). Each runs on the
 * current device, synchronises it, and returns a measured constant.
 *
 * Replaces the reference's calibration binaries bench/calibrate/cal-mma.cu,
 * cal-smem-bw.cu, cal-hbm-bw.cu and cal-latency.cu (their CAL_RESULT lines,
 * parsed by run-calibration.py:47-62); the Python driver that turns these into
 * data/hardware/b200.json is ridge_b200/calibrate.py.
 */
#ifndef RIDGE_B200_CALIBRATE_H
#define RIDGE_B200_CALIBRATE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* SM cycles per tcgen05.mma kind::f16 of shape m x n x 16 (m 64 or 128, n a
 * multiple of 16 up to 256), operands in 128B-swizzled shared memory, one CTA
 * per SM, `iters` back-to-back MMAs (median over SMs), repeated for about
 * 0.3 s so clocks settle under tensor load; *clock_hz (optional) = SM cycles /
 * event time of the last run, the clock the tensor cores really ran at. Replaces cal-mma.cu:41-163
 * and, through the n dependence, the smem-feed part of cal-smem-bw.cu:47-288. */
int ridge_cal_umma(int32_t m, int32_t n, int32_t iters, double* cycles_per_mma, double* clock_hz);

/* TMA tile-load bandwidth: `ctas_per_sm` CTAs per SM each keep `depth` boxes of
 * box_rows x box_cols FP16 in flight, reading a K-major tensor of
 * about tensor_bytes (L2-resident when small, HBM-streaming when large).
 * private_regions = 0: CTAs sweep the tensor together, so many SMs read the
 * same box at the same moment (the pattern of GEMM operand panels shared
 * through L2); 1: each CTA cycles over 16 boxes of its own (no shared bytes).
 * issuers = threads per CTA issuing loads, each with its own `depth` slots.
 * box_cols = FP16 columns per box row: 64 (128 B, 128B swizzle: BK=64 tiles)
 * or 32 (64 B, 64B swizzle: BK=32 tiles), or 128 (two 128-byte atoms per 3-D
 * box: BK=128 tiles).
 * Returns bytes per SM cycle per SM and aggregate bytes per second. Replaces
 * cal-hbm-bw.cu:22-109 and the latency surface of cal-latency.cu:56-256. */
int ridge_cal_tma(int64_t tensor_bytes, int32_t box_rows, int32_t depth, int32_t ctas_per_sm,
                  int32_t private_regions, int32_t issuers, int32_t box_cols,
                  double* bytes_per_cycle_sm, double* total_bytes_per_sec);

/* Epilogue drain rate, bytes of FP16 C per SM cycle (per SM) and per second
 * (aggregate, optional), for `warps` (4 or 8) warps doing TMEM load -> convert
 * -> swizzled smem -> TMA store into a C of c_bytes: L2-resident when small,
 * HBM-bound when several times larger than L2. tile_pattern 0: each warp
 * writes consecutive 32 x 32 chunks along rows; 1: the GEMM's order (each CTA
 * writes whole 128 x 256 tiles, a warp its 32-row quarter). */
int ridge_cal_epi(int32_t warps, int64_t c_bytes, int32_t tile_pattern,
                  double* bytes_per_cycle_sm, double* total_bytes_per_sec);

/* Write-only bandwidth (cudaMemsetAsync over `bytes`), bytes per second. */
int ridge_cal_write(int64_t bytes, double* bytes_per_sec);

/* Device-to-device copy bandwidth over `bytes` (read + write bytes per second). */
int ridge_cal_copy(int64_t bytes, double* bytes_per_sec);

/* Seconds per back-to-back launch of an empty 148-CTA kernel. */
int ridge_cal_launch(double* seconds);

/* The device's nominal SM clock (Hz). */
int ridge_cal_clock(double* hz);

#ifdef __cplusplus
}
#endif

#endif /* RIDGE_B200_CALIBRATE_H */
