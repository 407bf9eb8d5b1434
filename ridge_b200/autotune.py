"""Model-pruned empirical autotuning and the regret report.

The model ranks, the hardware decides (reference: tools/ridge-autotune.py). For
each shape every valid registered variant is ranked by ridge_predict, the top k
are benchmarked on the GPUs (libridge_b200's C++ farm: one worker thread per
device, jobs pulled from a shared queue), and the fastest measured one wins.

`sweep()` with k=0 benchmarks every candidate -- the exhaustive B200 sweep --
and writes it as CSV (the reference's measured schema, bench/measure.cu:233-234,
extended with warps, groupM, cta_group and device). `regret()` replays top-k
selection against such a sweep exactly as the reference does against its CSV:
for each k, pick the best measured config among the model's top k and report
(best - picked) / best against the exhaustive best.

    python -m ridge_b200.autotune --k 10 --devices 0,1          # tune the registered sweep
    python -m ridge_b200.autotune --exhaustive out.csv           # measure every candidate
    python -m ridge_b200.autotune --regret data/measured/b200.csv
"""

from __future__ import annotations

import argparse
import collections
import csv
import ctypes as C
import statistics
import sys
import time
from pathlib import Path

from ._native import BOTTLENECKS, TuneEntryC, TuneResultC, check, lib
from .gemm import TileConfig
from .model import HwC, default_hw, hw_to_dict, load_hw, predict

ROOT = Path(__file__).resolve().parent.parent
REGISTERED = ROOT / "data" / "sweep" / "b200-registered.csv"
CSV_FIELDS = ["M", "N", "K", "tag", "BM", "BN", "BK", "stages", "warps", "groupM", "cta_group",
              "smemBytes", "threads", "tmemCols", "tflops", "pred_tflops", "pred_bottleneck",
              "device"]


def load_sweep(path=REGISTERED):
    shapes = []
    for line in Path(path).read_text().splitlines():
        if not line.strip() or line.startswith("#"):
            continue
        f = line.split(",")
        if len(f) < 4:
            raise ValueError("%s: malformed row %r" % (path, line))
        shapes.append((int(f[0]), int(f[1]), int(f[2]), f[3]))
    if not shapes:
        raise ValueError("%s has no shapes" % path)
    return shapes


def autotune(shapes, k=10, devices=(0,), hw: HwC | None = None, warmup=3, iters=10):
    """Runs the farm. Returns (results, entries): per shape the best measured
    config, and every ranked candidate (benchmarked or not) in model order.
    Each benchmarked candidate is timed over L2-flushed launches (at least
    `iters`; ridge_time_gemm_cold)."""
    hw = hw if hw is not None else default_hw()
    n = len(shapes)
    mnk = (C.c_int64 * (3 * n))(*[v for s in shapes for v in s[:3]])
    devs = (C.c_int32 * len(devices))(*devices)
    res = (TuneResultC * n)()
    cap = lib.ridge_num_variants()
    ent = (TuneEntryC * (n * cap))()
    st = lib.ridge_autotune(mnk, n, k, devs, len(devices), C.byref(hw), warmup, iters, res, ent,
                            cap)
    check(st, "ridge_autotune")
    results, entries = [], []
    for s in range(n):
        r = res[s]
        results.append({"M": r.M, "N": r.N, "K": r.K, "best": TileConfig.from_c(r.best),
                        "best_tflops": r.best_tflops, "benchmarked": r.benchmarked,
                        "candidates": r.candidates})
        rows = []
        for i in range(r.candidates):
            e = ent[s * cap + i]
            rows.append({"config": TileConfig.from_c(e.tile), "pred_tflops": e.predicted_tflops,
                         "tflops": e.measured_tflops, "device": e.device, "status": e.status})
        entries.append(rows)
    return results, entries


def write_header(path, hw: HwC, note=""):
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, "w", newline="") as f:
        f.write("# ridge B200 measured sweep (libridge_b200 ridge_autotune, exhaustive)\n")
        f.write("# hw_model,%s\n" % hw.name.decode())
        if note:
            f.write("# %s\n" % note)
        csv.writer(f).writerow(CSV_FIELDS)


def append_rows(path, shape, rows, hw: HwC):
    from .gemm import config_info
    M, N, K, tag = shape
    with open(path, "a", newline="") as f:
        w = csv.writer(f)
        for r in rows:
            c = r["config"]
            info = config_info(c)
            p = predict(M, N, K, c, hw)
            w.writerow([M, N, K, tag, c.BM, c.BN, c.BK, c.stages, c.warps, c.groupM,
                        info.config.cta_group, info.smem_bytes, info.threads, info.tmem_cols,
                        "%.3f" % r["tflops"], "%.3f" % p["predicted_tflops"], p.label,
                        r["device"]])


def append_meta(path, key, value):
    with open(path, "a") as f:
        f.write("# %s,%s\n" % (key, value))


def write_csv(path, shapes, entries, hw: HwC, note=""):
    write_header(path, hw, note)
    for shape, rows in zip(shapes, entries):
        append_rows(path, shape, rows, hw)


def completed_shapes(path):
    """Shapes whose rows are all in an existing sweep file (resume)."""
    from .gemm import num_variants
    if not Path(path).exists():
        return set()
    counts = collections.Counter()
    with open(path, newline="") as f:
        for r in csv.DictReader(l for l in f if not l.startswith("#")):
            counts[(int(r["M"]), int(r["N"]), int(r["K"]))] += 1
    n = num_variants()
    return {k for k, v in counts.items() if v >= n}


def merge_best(out_path, in_paths):
    """Per configuration the best throughput over several complete sweeps of the
    same registered cross product (e.g. on separate boxes): single
    configurations can move by tens of percent between sweeps while the median
    barely moves, and those outliers decide top-k regret."""
    key = ("M", "N", "K", "BM", "BN", "BK", "stages", "warps", "cta_group")
    merged, order, meta = {}, [], []
    fields = None
    for i, path in enumerate(in_paths):
        lines = Path(path).read_text().splitlines()
        meta += ["# sweep %d %s" % (i + 1, l[2:]) for l in lines if l.startswith("# ")][1:]
        rows = list(csv.DictReader(l for l in lines if not l.startswith("#")))
        fields = fields or list(rows[0].keys())
        for r in rows:
            k = tuple(r[x] for x in key)
            if k not in merged:
                merged[k] = r
                order.append(k)
            elif float(r["tflops"]) > float(merged[k]["tflops"]):
                merged[k] = r
    with open(out_path, "w", newline="") as f:
        f.write("# ridge B200 measured sweep (libridge_b200 ridge_autotune, exhaustive)\n")
        f.write("# per configuration the best of %d complete sweeps (each best of 3 timed runs)\n"
                % len(in_paths))
        for m in meta:
            f.write(m + "\n")
        w = csv.DictWriter(f, fieldnames=fields)
        w.writeheader()
        w.writerows(merged[k] for k in order)
    return len(order)


CANARY = (4096, 4096, 4096)


def canary_tflops(device=0):
    """A fixed 4096^3 launch (the bench tile) timed cold on `device` -- the
    drift check of the reference's measure.cu, between shapes of a long sweep."""
    import torch

    from .gemm import synthetic_inputs
    M, N, K = CANARY
    cfg = TileConfig(256, 256, 128, 3, 8, 8, 2)
    with torch.cuda.device(device):
        dev = torch.device("cuda", device)
        a, b = synthetic_inputs(M, N, K, device=dev)
        c = torch.empty((M, N), dtype=torch.float16, device=dev)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        ms = C.c_double()
        cc = cfg.to_c()
        check(lib.ridge_time_gemm_cold(C.byref(cc), a.data_ptr(), b.data_ptr(), c.data_ptr(), M,
                                       N, K, K, K, N, flush.data_ptr(), flush.numel(), 3, 20,
                                       torch.cuda.current_stream().cuda_stream, C.byref(ms)),
              "canary")
    return 2.0 * M * N * K / (ms.value * 1e-3) / 1e12


def exhaustive(path, shapes, devices, hw: HwC, warmup=3, iters=10, resume=False, log=print):
    """Every candidate of every shape, appended shape by shape (a killed sweep
    resumes with resume=True), with a canary before the first and after every
    shape; returns the canary drift fraction (max - min) / median."""
    done = completed_shapes(path) if resume else set()
    if not resume or not Path(path).exists():
        write_header(path, hw, "devices %s" % list(devices))
    canaries = [canary_tflops(devices[0])]
    append_meta(path, "canary_tflops", "%.1f" % canaries[-1])
    for shape in shapes:
        if shape[:3] in done:
            log("%6d x %6d x %6d  already measured, skipped" % shape[:3])
            continue
        t0 = time.time()
        results, entries = autotune([shape], 0, devices, hw, warmup, iters)
        append_rows(path, shape, entries[0], hw)
        canaries.append(canary_tflops(devices[0]))
        append_meta(path, "canary_tflops", "%.1f" % canaries[-1])
        r = results[0]
        log("%6d x %6d x %6d  best %8.1f TFLOP/s  %s  (%d candidates, %.1f s, canary %.0f)" % (
            r["M"], r["N"], r["K"], r["best_tflops"], r["best"].tag(), r["candidates"],
            time.time() - t0, canaries[-1]))
    drift = (max(canaries) - min(canaries)) / statistics.median(canaries)
    append_meta(path, "canary_drift_fraction", "%.4f" % drift)
    return drift


def load_measured(path):
    with open(path, newline="") as f:
        rows = list(csv.DictReader(l for l in f if not l.startswith("#")))
    for r in rows:
        for k in ("M", "N", "K", "BM", "BN", "BK", "stages", "warps", "groupM", "cta_group"):
            r[k] = int(r[k])
        r["tflops"] = float(r["tflops"])
        r["config"] = TileConfig(r["BM"], r["BN"], r["BK"], r["stages"], r["warps"], r["groupM"],
                                 r["cta_group"])
    return rows


def regret(rows, ks=(1, 3, 5, 10, 20), hw: HwC | None = None):
    """Top-k regret of the model against an exhaustive measured sweep.
    Predictions are recomputed with `hw` (the current model), never read
    from the CSV. Returns {k: (mean%, worst%, exact_hits, shapes, per-shape)}."""
    hw = hw if hw is not None else default_hw()
    by_shape = {}
    for r in rows:
        p = predict(r["M"], r["N"], r["K"], r["config"], hw)["predicted_tflops"]
        by_shape.setdefault((r["M"], r["N"], r["K"], r["tag"]), []).append((p, r["tflops"]))
    out = {}
    for k in ks:
        regrets, hits, detail = [], 0, {}
        for key, rs in by_shape.items():
            best = max(m for _, m in rs)
            # stable: equal predictions keep sweep (table) order, as the farm does
            short = sorted(rs, key=lambda x: -x[0])[:k]
            picked = max(m for _, m in short)
            rg = (best - picked) / best * 100.0 if best > 0 else 0.0
            regrets.append(rg)
            hits += picked == best
            detail[key] = rg
        out[k] = (statistics.mean(regrets), max(regrets), hits, len(by_shape), detail)
    return out


def model_error(rows, hw: HwC | None = None):
    """Mean / median / p90 / max absolute percentage error of predicted vs
    measured TFLOP/s over a sweep (reference: bench/validate.py:252-259)."""
    hw = hw if hw is not None else default_hw()
    errs = []
    for r in rows:
        if r["tflops"] <= 0:
            continue
        p = predict(r["M"], r["N"], r["K"], r["config"], hw)["predicted_tflops"]
        errs.append(abs(p - r["tflops"]) / r["tflops"] * 100.0)
    errs.sort()
    return {"mape": statistics.mean(errs), "median": statistics.median(errs),
            "p90": errs[int(0.9 * (len(errs) - 1))], "max": errs[-1], "n": len(errs)}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--sweep", default=str(REGISTERED))
    ap.add_argument("--hw", default=None, help="calibration JSON (default data/hardware/b200.json)")
    ap.add_argument("--devices", default="0")
    ap.add_argument("--k", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--exhaustive", default=None, help="benchmark every candidate, write CSV")
    ap.add_argument("--regret", default=None, help="report regret against this measured CSV")
    ap.add_argument("--ks", default="1,3,5,10,20")
    ap.add_argument("--resume", action="store_true",
                    help="with --exhaustive: keep the shapes already complete in the file")
    ap.add_argument("--merge", nargs="+", default=None, metavar="CSV",
                    help="OUT IN1 IN2 ...: per configuration the best of several sweeps")
    a = ap.parse_args(argv)
    if a.merge:
        n = merge_best(a.merge[0], a.merge[1:])
        print("merged %d configurations from %d sweeps into %s" % (n, len(a.merge) - 1,
                                                                  a.merge[0]))
        return 0
    hw = load_hw(a.hw) if a.hw else default_hw()
    ks = [int(x) for x in a.ks.split(",")]
    if a.regret:
        rows = load_measured(a.regret)
        rg = regret(rows, ks, hw)
        err = model_error(rows, hw)
        print("model: %s" % hw.name.decode())
        print("MAPE %.2f%%  median %.2f%%  p90 %.2f%%  max %.2f%%  (%d configs)" % (
            err["mape"], err["median"], err["p90"], err["max"], err["n"]))
        print("%5s %12s %12s %10s" % ("top_k", "mean regret", "worst regret", "exact"))
        for k in ks:
            m, w, h, n, _ = rg[k]
            print("%5d %11.2f%% %11.2f%% %6d/%-3d" % (k, m, w, h, n))
        return 0
    shapes = load_sweep(a.sweep)
    devices = [int(x) for x in a.devices.split(",")]
    if a.exhaustive:
        drift = exhaustive(a.exhaustive, shapes, devices, hw, a.warmup, a.iters, a.resume)
        print("canary drift %.1f%%%s" % (100 * drift, "  (above 5%: clocks moved during the "
                                         "sweep, treat it with care)" if drift > 0.05 else ""))
        print("wrote", a.exhaustive)
        return 0
    t0 = time.time()
    results, entries = autotune(shapes, a.k, devices, hw, a.warmup, a.iters)
    dt = time.time() - t0
    for r in results:
        print("%6d x %6d x %6d  best %8.1f TFLOP/s  %s  (%d of %d benchmarked)" % (
            r["M"], r["N"], r["K"], r["best_tflops"], r["best"].tag(), r["benchmarked"],
            r["candidates"]))
    print("farm: %d devices, %.1f s" % (len(devices), dt))
    return 0


if __name__ == "__main__":
    sys.exit(main())
