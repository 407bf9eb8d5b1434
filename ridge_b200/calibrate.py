"""Runs the sm_100a calibration microbenchmarks and writes the B200 hardware
model (data/hardware/b200.json by default).

Reference: bench/calibrate/run-calibration.py runs four CUDA binaries, parses
their CAL_RESULT lines, checks each constant against a datasheet band and
writes a flat JSON that HardwareModel::loadFromJson reads. Same contract here,
with the microbenchmarks built into libridge_b200.so
(include/ridge_b200_calibrate.h) and constants for the tcgen05/TMA kernel:

  ummaCycles128x256  cycles per 128x256x16 tcgen05.mma (tensor issue rate)
  ummaM64Ratio       cycles(64x256x16) / cycles(128x256x16)
  smemBytesPerCycle  operand bytes/cycle/SM the tensor core reads from shared
                     memory, from the MMA cycle count at small N
  smemMmaOverlap     1 when those reads overlap the MMA (cycles = max), 0 when
                     they add (cycles = sum); whichever fits the N sweep better
  l2BytesPerSec      TMA fill cap from an L2-resident tensor (best bytes per SM
                     cycle of several issuer / box / residency mixes, at clockHz)
  hbmBytesPerSec     aggregate TMA fill rate from a tensor 8x larger than L2
  epiBytesPerCycleW4/W8  epilogue drain rate per SM with 4 / 8 warps (C in L2)
  cWriteBytesPerSec  aggregate rate the epilogue writes a C far larger than L2
  tmaBoxCycles       cycles (at the loaded clock) one issuing thread needs per box;
                     tmaBoxCycles32Ratio / tmaBoxCycles128Ratio: BK=32 / BK=128 boxes
  tmaLatencyCycles   load latency: bytes in flight / per-SM rate at depth 1
  tmaLatencyHbmCycles  the same with the tensor in DRAM (8 GB, L2 misses)
  launchOverheadSec  back-to-back launch cost of an empty kernel
  clockHz            SM clock measured under full tensor load

Usage: python -m ridge_b200.calibrate [--out data/hardware/b200.json]
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import sys
import time
from pathlib import Path

from ._native import check, lib

ROOT = Path(__file__).resolve().parent.parent

# Datasheet-derived sanity bands (run-calibration.py:113-126 in the reference):
# a constant outside its band means the benchmark, not the chip, is wrong.
BANDS = {
    "ummaCycles128x256": (100.0, 200.0),   # 128 nominal (8192 FLOP/cycle/SM)
    "smemBytesPerCycle": (64.0, 512.0),
    "l2BytesPerSec": (4e12, 40e12),
    "hbmBytesPerSec": (3e12, 8.5e12),
    "clockHz": (0.8e9, 2.1e9),
}


def umma(m, n, iters=20000):
    cyc, hz = C.c_double(), C.c_double()
    check(lib.ridge_cal_umma(m, n, iters, C.byref(cyc), C.byref(hz)), "ridge_cal_umma")
    return cyc.value, hz.value


def tma(tensor_bytes, box_rows, depth, ctas=1, private=0, issuers=1, box_cols=64):
    per_sm, total = C.c_double(), C.c_double()
    check(lib.ridge_cal_tma(tensor_bytes, box_rows, depth, ctas, private, issuers, box_cols,
                            C.byref(per_sm),
                            C.byref(total)),
          "ridge_cal_tma")
    return per_sm.value, total.value


def epi(warps, c_bytes=32 << 20, tile_pattern=0):
    v, t = C.c_double(), C.c_double()
    check(lib.ridge_cal_epi(warps, c_bytes, tile_pattern, C.byref(v), C.byref(t)),
          "ridge_cal_epi")
    return v.value, t.value


def write_bw(nbytes=1 << 30):
    v = C.c_double()
    check(lib.ridge_cal_write(nbytes, C.byref(v)), "ridge_cal_write")
    return v.value


def copy_bw(nbytes=1 << 31):
    v = C.c_double()
    check(lib.ridge_cal_copy(nbytes, C.byref(v)), "ridge_cal_copy")
    return v.value


def launch_overhead():
    v = C.c_double()
    check(lib.ridge_cal_launch(C.byref(v)), "ridge_cal_launch")
    return v.value


# The one constant taken from the GEMM itself: a long, tensor-bound launch on a
# shape outside the validation sweep, with every other constant already
# measured; efficiency = measured / modelled-at-efficiency-1.
def _cal_gemm():
    from .gemm import TileConfig
    return (6144, 6144, 6144, TileConfig(256, 256, 128, 3, 8, 8, 2))


CAL_GEMM = None


def pipeline_efficiency(res):
    global CAL_GEMM
    import torch

    from ._native import HwC
    from .gemm import synthetic_inputs
    from .model import HW_KEYS, predict
    CAL_GEMM = _cal_gemm()
    M, N, K, cfg = CAL_GEMM
    meas = 2.0 * M * N * K / (_time_tflops(M, N, K, cfg) * 1e-3) / 1e12
    hw = HwC()
    lib.ridge_hw_b200(C.byref(hw))
    for k, f in HW_KEYS.items():
        if k in res:
            setattr(hw, f, type(getattr(hw, f))(res[k]))
    ideal = predict(M, N, K, cfg, hw)["predicted_tflops"]
    return min(1.0, meas / ideal), meas, ideal


TURN_SHAPE = (6144, 6144, 64)


def _hw_from(res):
    from ._native import HwC
    from .model import HW_KEYS
    hw = HwC()
    lib.ridge_hw_b200(C.byref(hw))
    for k, f in HW_KEYS.items():
        if k in res:
            setattr(hw, f, type(getattr(hw, f))(res[k]))
    return hw


def _time_tflops(M, N, K, cfg):
    """Milliseconds per launch, timed the way the autotuner and the headline
    benchmark time a GEMM (L2 flushed before every launch)."""
    import torch

    from .gemm import synthetic_inputs
    a, b = synthetic_inputs(M, N, K)
    c = torch.empty((M, N), dtype=torch.float16, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    ms = C.c_double()
    cc = cfg.to_c()
    check(lib.ridge_time_gemm_cold(C.byref(cc), a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N,
                                   K, K, K, N, flush.data_ptr(), flush.numel(), 5, 30,
                                   torch.cuda.current_stream().cuda_stream, C.byref(ms)),
          "ridge_time_gemm_cold")
    return ms.value


def tile_overhead(res, cfg_tuple):
    """Per-tile turnover cost: a K=64 GEMM (one K-block per tile, outside the
    validation sweep) is nothing but tile turnovers; whatever its measured time
    per tile exceeds the model's drain-and-mainloop time is the hand-off cost."""
    from .gemm import TileConfig
    from .model import predict
    M, N, K = TURN_SHAPE
    cfg = TileConfig(*cfg_tuple)
    ms = _time_tflops(M, N, K, cfg)
    hw = _hw_from(res)
    p = predict(M, N, K, cfg, hw)
    tiles_per_unit = p["total_tiles"] / min(p["total_tiles"], p["tile_slots"])
    meas_cycles = (ms * 1e-3 - hw.launch_overhead_sec) * hw.clock_hz / tiles_per_unit
    model_cycles = (p["predicted_seconds"] - hw.launch_overhead_sec) * hw.clock_hz / tiles_per_unit
    return max(0.0, meas_cycles - model_cycles), meas_cycles, model_cycles


def fit_smem(cycles_by_n, m=128):
    """From cycles(n) of m x n x 16 MMAs: tensor cycles per 128x256 MMA, smem
    bytes/cycle, and whether operand reads overlap (max) or add (sum).
    Operand bytes per MMA: (m + n) * 16 * 2."""
    c256 = cycles_by_n[256]
    best = None
    for overlap in (1, 0):
        # the tensor part scales with n; solve the smem rate from the smallest n
        n0 = min(cycles_by_n)
        bytes0 = (m + n0) * 32
        t0 = c256 * n0 / 256.0
        if overlap:
            bw = bytes0 / cycles_by_n[n0] if cycles_by_n[n0] > t0 * 1.02 else 1e9
        else:
            extra = cycles_by_n[n0] - t0
            bw = bytes0 / extra if extra > 1e-6 else 1e9
        err = 0.0
        for n, c in cycles_by_n.items():
            t = c256 * n / 256.0
            s = (m + n) * 32 / bw
            pred = max(t, s) if overlap else t + s
            err += abs(pred - c) / c
        if best is None or err < best[0]:
            best = (err, overlap, bw)
    _, overlap, bw = best
    return c256, min(bw, 1024.0), float(overlap)


def calibrate(verbose=True):
    log = (lambda *a: print(*a, flush=True)) if verbose else (lambda *a: None)
    res, raw = {}, {}
    cyc = {}
    for n in (64, 128, 256):
        cyc[n], hz = umma(128, n)
        raw["umma_128x%d" % n] = cyc[n]
        log("umma 128x%dx16: %.2f cycles (clock %.0f MHz)" % (n, cyc[n], hz / 1e6))
    c64, _ = umma(64, 256)
    raw["umma_64x256"] = c64
    c256, hz = umma(128, 256, 40000)
    cyc[256] = c256
    res["clockHz"] = hz
    res["ummaCycles128x256"], res["smemBytesPerCycle"], res["smemMmaOverlap"] = fit_smem(cyc)
    res["ummaM64Ratio"] = c64 / c256
    log("m64 ratio %.3f, smem %.1f B/cycle, overlap %d" % (
        res["ummaM64Ratio"], res["smemBytesPerCycle"], res["smemMmaOverlap"]))
    # TMA fill: L2-resident (32 MB tensor) vs HBM-streaming (8 GB) at deep rings.
    l2_best, hbm_best = 0.0, 0.0
    for box, depth in ((256, 6), (128, 12), (256, 3)):
        per_sm, tot = tma(32 << 20, box, depth)
        raw["tma_l2_box%d_d%d" % (box, depth)] = [per_sm, tot]
        l2_best = max(l2_best, tot)
        log("tma L2  box %3d depth %2d: %.1f B/cycle/SM  %.2f TB/s" % (box, depth, per_sm, tot / 1e12))
    for box, depth in ((256, 6), (128, 12)):
        per_sm, tot = tma(8 << 30, box, depth)
        raw["tma_hbm_box%d_d%d" % (box, depth)] = [per_sm, tot]
        hbm_best = max(hbm_best, tot)
        log("tma HBM box %3d depth %2d: %.1f B/cycle/SM  %.2f TB/s" % (box, depth, per_sm, tot / 1e12))
    res["l2BytesPerSec"] = l2_best
    res["hbmBytesPerSec"] = hbm_best
    # the same loads, but no two SMs ever read the same bytes (76-96 MB, in L2)
    for box, depth, tb in ((256, 6, 80 << 20), (128, 8, 96 << 20), (64, 12, 96 << 20)):
        per_sm, tot = tma(tb, box, depth, 1, 1)
        raw["tma_l2_private_box%d_d%d" % (box, depth)] = [per_sm, tot]
        log("tma L2 private box %3d depth %2d: %.1f B/cycle/SM  %.2f TB/s" % (box, depth, per_sm,
                                                                             tot / 1e12))
    # several issuing threads in one CTA
    for iss in (2, 4):
        per_sm, tot = tma(32 << 20, 128, 8 // iss, 1, 0, iss)
        raw["tma_l2_box128_issuers%d" % iss] = [per_sm, tot]
        log("tma L2  box 128 depth %d, %d issuers: %.1f B/cycle/SM  %.2f TB/s" % (8 // iss, iss, per_sm,
                                                                                tot / 1e12))
    per_sm, tot = tma(8 << 30, 128, 2, 1, 0, 4)
    raw["tma_hbm_box128_d2_issuers4"] = [per_sm, tot]
    log("tma HBM box 128 depth  2, 4 issuers: %.1f B/cycle/SM  %.2f TB/s" % (per_sm, tot / 1e12))
    # two CTAs per SM, shared boxes
    per_sm, tot = tma(32 << 20, 128, 6, 2)
    raw["tma_l2_box128_d6_2cta"] = [per_sm, tot]
    log("tma L2  box 128 depth  6, 2 CTAs/SM: %.1f B/cycle/SM  %.2f TB/s" % (per_sm, tot / 1e12))
    # latency: fill rate against bytes in flight (one box per ring slot)
    curve = {}
    for depth in (1, 2, 4, 8):
        per_sm, tot = tma(32 << 20, 128, depth)
        curve[depth] = per_sm
        log("tma L2  box 128 depth %2d: %.1f B/cycle/SM  %.2f TB/s" % (depth, per_sm, tot / 1e12))
    raw["tma_l2_box128_depth_curve"] = curve
    res["tmaLatencyCycles"] = 128 * 128 / curve[1]
    log("tma latency (depth 1): %.0f cycles" % res["tmaLatencyCycles"])
    # the same from a tensor far larger than L2: every box waits for DRAM
    ps_hbm, _ = tma(8 << 30, 128, 1)
    raw["tma_hbm_box128_d1"] = ps_hbm
    res["tmaLatencyHbmCycles"] = 128 * 128 / ps_hbm
    log("tma latency from DRAM (depth 1): %.0f cycles" % res["tmaLatencyHbmCycles"])
    res["epiBytesPerCycleW4"], _ = epi(4)
    res["epiBytesPerCycleW8"], _ = epi(8)
    log("epilogue (C in L2): %.1f / %.1f B/cycle/SM (4 / 8 warps)" % (
        res["epiBytesPerCycleW4"], res["epiBytesPerCycleW8"]))
    big4, tot4 = epi(4, 1 << 30)
    big8, tot8 = epi(8, 1 << 30)
    raw["epi_hbm_w4"] = [big4, tot4]
    raw["epi_hbm_w8"] = [big8, tot8]
    log("epilogue (C 1 GiB, row stripes): %.1f / %.1f B/cycle/SM, %.2f / %.2f TB/s" % (
        big4, big8, tot4 / 1e12, tot8 / 1e12))
    t4, tt4 = epi(4, 1 << 30, 1)
    t8, tt8 = epi(8, 1 << 30, 1)
    raw["epi_hbm_tiles_w4"] = [t4, tt4]
    raw["epi_hbm_tiles_w8"] = [t8, tt8]
    res["cWriteBytesPerSec"] = max(tt4, tt8)
    log("epilogue (C 1 GiB, GEMM tile order): %.1f / %.1f B/cycle/SM, %.2f / %.2f TB/s" % (
        t4, t8, tt4 / 1e12, tt8 / 1e12))
    raw["memset_bytes_per_sec"] = write_bw()
    log("memset %.2f TB/s" % (raw["memset_bytes_per_sec"] / 1e12))
    # Per-box cost with ONE issuing thread (below the L2 cap): cycles per
    # box at the GEMM's loaded clock (the microbenchmark runs faster; its own
    # clock is total / (SMs x per-SM rate)), and the cost of 64-byte (BK=32)
    # and two-atom (BK=128) boxes relative to one-atom 128-byte boxes.
    box1 = {}
    for cols in (32, 64, 128):
        ps, tot = tma(32 << 20, 128, 2, 1, 0, 1, cols)
        box1[cols] = (ps, tot)
        raw["tma_l2_box128x%d_d2_issuers1" % cols] = [ps, tot]
    ps64, tot64 = box1[64]
    micro_hz = tot64 / (148 * ps64)
    res["tmaBoxCycles"] = 128 * 128 / ps64 * res["clockHz"] / micro_hz
    res["tmaBoxCycles32Ratio"] = ps64 / (2.0 * box1[32][0])
    res["tmaBoxCycles128Ratio"] = 2.0 * ps64 / box1[128][0]
    log("tma box, 1 issuer: %.0f cycles at the loaded clock; 64-byte box x%.2f, two-atom box x%.2f"
        % (res["tmaBoxCycles"], res["tmaBoxCycles32Ratio"], res["tmaBoxCycles128Ratio"]))
    # The L2 -> shared memory cap: the best of several issuer / box / residency
    # mixes, in bytes per SM cycle at whatever clock the run holds, stated at
    # the loaded clock.
    cap_per_cycle = 0.0
    for rows, depth, ctas, iss, cols in ((128, 2, 1, 4, 64), (256, 2, 1, 2, 64),
                                         (256, 1, 1, 4, 64), (128, 1, 2, 4, 64),
                                         (128, 2, 1, 2, 128), (128, 1, 1, 8, 64)):
        ps, tot = tma(32 << 20, rows, depth, ctas, 0, iss, cols)
        raw["tma_l2_box%dx%d_d%d_c%d_issuers%d" % (rows, cols, depth, ctas, iss)] = [ps, tot]
        cap_per_cycle = max(cap_per_cycle, ps)
        log("tma L2 box %dx%d depth %d, %d CTA(s), %d issuers: %.1f B/cycle/SM  %.2f TB/s" % (
            rows, cols, depth, ctas, iss, ps, tot / 1e12))
    res["l2BytesPerSec"] = cap_per_cycle * 148 * res["clockHz"]
    log("tma L2 fill cap %.1f B/cycle/SM = %.2f TB/s at the loaded clock" % (
        cap_per_cycle, res["l2BytesPerSec"] / 1e12))
    raw["copy_bytes_per_sec"] = copy_bw()
    res["launchOverheadSec"] = launch_overhead()
    log("copy %.2f TB/s, launch %.2f us" % (raw["copy_bytes_per_sec"] / 1e12,
                                           res["launchOverheadSec"] * 1e6))
    res.update({"numSMs": 148, "l2Bytes": 126.0 * 1024 * 1024, "smemBytesPerSM": 233472,
                "tmemColsPerSM": 512, "maxCtasPerSM": 32})
    res["pipelineEfficiency"] = 1.0
    res["tileOverheadCycles"] = 0.0
    res["pairTileOverheadCycles"] = 0.0
    for key, cfg in (("tileOverheadCycles", (128, 256, 64, 4, 8, 8, 1)),
                     ("pairTileOverheadCycles", (256, 256, 64, 4, 8, 8, 2))):
        res[key], meas_t, model_t = tile_overhead(res, cfg)
        raw[key] = {"shape": list(TURN_SHAPE), "config": list(cfg), "measured_tile_cycles": meas_t,
                    "modelled_tile_cycles_without_overhead": model_t}
        log("tile turnover %s: %.0f cycles measured vs %.0f modelled -> %s %.0f" % (
            cfg, meas_t, model_t, key, res[key]))
    eff, meas, ideal = pipeline_efficiency(res)
    res["pipelineEfficiency"] = eff
    raw["calibration_gemm"] = {"shape": list(CAL_GEMM[:3]), "config": CAL_GEMM[3].tag(),
                               "measured_tflops": meas, "model_tflops_at_efficiency_1": ideal}
    log("calibration GEMM %s %s: %.1f TF measured, %.1f ideal -> pipeline efficiency %.3f" % (
        "x".join(map(str, CAL_GEMM[:3])), CAL_GEMM[3].tag(), meas, ideal, eff))
    bad = {k: v for k, v in res.items() if k in BANDS and not BANDS[k][0] <= v <= BANDS[k][1]}
    return res, raw, bad


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(ROOT / "data" / "hardware" / "b200.json"))
    a = ap.parse_args(argv)
    res, raw, bad = calibrate()
    if bad:
        print("constants outside their datasheet bands, not written: %s" % bad, file=sys.stderr)
        return 1
    import torch
    name = torch.cuda.get_device_name()
    doc = {"name": name, "note": "measured by ridge_b200.calibrate (sm_100a microbenchmarks) on %s"
           % time.strftime("%Y-%m-%d"), **res}
    Path(a.out).parent.mkdir(parents=True, exist_ok=True)
    Path(a.out).write_text(json.dumps(doc, indent=1) + "\n")
    Path(a.out).with_suffix(".raw.json").write_text(json.dumps(raw, indent=1) + "\n")
    print("wrote", a.out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
