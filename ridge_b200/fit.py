"""Fits the cost model's pipeline constants to a calibration sweep.

The microbenchmarks (ridge_b200.calibrate) measure each mechanism alone: a TMA
box, a drain, a hand-off. Inside the GEMM they overlap and contend, so a few of
them carry an effective value that no isolated benchmark shows. This step
measures every registered variant on a CALIBRATION shape set that is disjoint
from the registered validation sweep (data/sweep/b200-calibration.csv), then
adjusts those constants, each within a bounded band around its microbenchmark
value, to minimise the mean |log(predicted / measured)| over that set without
raising the top-10 autotune regret on it. Each
configuration can be weighted by (its throughput / its shape's best) ** p
(--weight-power; default 0, unweighted) so that the top of the ranking, where
the autotuner picks, counts more. The
validation sweep is never read here, so its model error and autotune regret stay
out-of-sample.

The reference has no such step: its constants come straight from datasheet
bands and four microbenchmarks (bench/calibrate/run-calibration.py:113-126).

    python -m ridge_b200.fit --measure            # on a B200: sweep + fit
    python -m ridge_b200.fit --from data/measured/b200-calibration.csv   # refit offline
"""

from __future__ import annotations

import argparse
import json
import math
import sys
import time
from pathlib import Path

from .model import DEFAULT_HW_JSON, HW_KEYS, load_hw

ROOT = Path(__file__).resolve().parent.parent
CAL_SWEEP = ROOT / "data" / "sweep" / "b200-calibration.csv"
CAL_MEASURED = ROOT / "data" / "measured" / "b200-calibration.csv"

# JSON key -> (low, high) as multiples of the microbenchmark value, or, for the
# hand-off costs that the microbenchmarks can measure as 0, absolute cycles.
FIT_BANDS = {
    "tmaBoxCycles": (0.5, 2.0),
    "tmaBoxCycles128Ratio": (0.5, 2.0),
    "tmaBoxCycles32Ratio": (0.5, 2.0),
    "tmaLatencyCycles": (0.5, 3.0),
    "tmaLatencyHbmCycles": (0.5, 3.0),
    "pipelineEfficiency": (0.7, 1.0),
    "epiBytesPerCycleW4": (0.5, 2.0),
    "epiBytesPerCycleW8": (0.5, 2.0),
    "cWriteBytesPerSec": (0.7, 1.3),
    "hbmBytesPerSec": (0.8, 1.1),
    "launchOverheadSec": (0.5, 3.0),
}
# the microbenchmark value of a fitted constant is kept under this key prefix
MICRO = "microbenchmark_"
WEIGHT_POWER = 0.0
GUARD_K = 10
# Constants with a direct measurement of their own are not fitted: the tile
# turnover costs are measured on a K=64 GEMM where every tile is one K-block
# (ridge_b200.calibrate.tile_overhead); the calibration shapes, which turn
# tiles over rarely, barely constrain them.
ABS_BANDS = {}


def _hw_with(base: dict, values: dict, tmp: Path):
    doc = dict(base)
    doc.update(values)
    tmp.write_text(json.dumps(doc))
    return load_hw(tmp)


def _weights(rows, power):
    """Per row (measured / best measured of its shape) ** power: the autotuner
    only ever benchmarks the top of the ranking, so the fit cares most about
    the configurations near each shape's best."""
    best = {}
    for r in rows:
        key = (r["M"], r["N"], r["K"])
        best[key] = max(best.get(key, 0.0), r["tflops"])
    return [(r["tflops"] / best[(r["M"], r["N"], r["K"])]) ** power if r["tflops"] > 0 else 0.0
            for r in rows]


def _objective(rows, hw, weights):
    from .model import predict
    tot, wsum = 0.0, 0.0
    for r, w in zip(rows, weights):
        if w <= 0:
            continue
        p = predict(r["M"], r["N"], r["K"], r["config"], hw)["predicted_tflops"]
        if p <= 0:
            return float("inf")
        tot += w * abs(math.log(p / r["tflops"]))
        wsum += w
    return tot / max(wsum, 1e-30)


def _topk_regret(rows, hw, k=GUARD_K):
    """Mean top-k autotune regret (fraction) over the shapes in `rows`."""
    from .model import predict
    by = {}
    for r in rows:
        p = predict(r["M"], r["N"], r["K"], r["config"], hw)["predicted_tflops"]
        by.setdefault((r["M"], r["N"], r["K"]), []).append((p, r["tflops"]))
    tot = 0.0
    for rs in by.values():
        best = max(m for _, m in rs)
        picked = max(m for _, m in sorted(rs, key=lambda x: -x[0])[:k])
        tot += (best - picked) / best if best > 0 else 0.0
    return tot / max(len(by), 1)


def fit(rows, base: dict, passes=4, steps=9, weight_power=WEIGHT_POWER, log=print):
    """Coordinate descent over FIT_BANDS / ABS_BANDS, each constant on a
    geometric (or linear, for ABS_BANDS) grid that narrows every pass. A move
    is taken only if it lowers the error without raising the top-GUARD_K
    autotune regret on the same calibration shapes: the constants exist to
    rank configurations, so a better average error bought with a worse ranking
    is refused."""
    weights = _weights(rows, weight_power)
    tmp = Path("/tmp") / ("ridge_fit_%d.json" % id(rows))
    start = {k: float(base[k]) for k in list(FIT_BANDS) + list(ABS_BANDS)}
    lo = {k: start[k] * FIT_BANDS[k][0] for k in FIT_BANDS}
    hi = {k: start[k] * FIT_BANDS[k][1] for k in FIT_BANDS}
    lo.update({k: ABS_BANDS[k][0] for k in ABS_BANDS})
    hi.update({k: ABS_BANDS[k][1] for k in ABS_BANDS})
    cur = dict(start)
    hw0 = _hw_with(base, cur, tmp)
    best = _objective(rows, hw0, weights)
    guard = _topk_regret(rows, hw0)
    log("fit: start mean |log error| %.4f, top-%d regret %.2f%%" % (best, GUARD_K, 100 * guard))
    width = {k: 1.0 for k in cur}  # fraction of the band searched around the current value
    for ps in range(passes):
        for k in cur:
            if k in ABS_BANDS:
                span = (hi[k] - lo[k]) * width[k] / 2
                cands = [min(hi[k], max(lo[k], cur[k] + span * (2 * i / (steps - 1) - 1)))
                         for i in range(steps)]
            else:
                lspan = math.log(hi[k] / lo[k]) * width[k] / 2
                cands = [min(hi[k], max(lo[k], cur[k] * math.exp(lspan * (2 * i / (steps - 1) - 1))))
                         for i in range(steps)]
            for v in cands:
                trial = dict(cur)
                trial[k] = v
                hw = _hw_with(base, trial, tmp)
                obj = _objective(rows, hw, weights)
                if obj < best - 1e-6:
                    rg = _topk_regret(rows, hw)
                    if rg <= guard + 1e-12:
                        best, cur, guard = obj, trial, rg
            width[k] *= 0.5
        log("fit: pass %d mean |log error| %.4f, top-%d regret %.2f%%" % (
            ps + 1, best, GUARD_K, 100 * guard))
    tmp.unlink(missing_ok=True)
    return cur, best


def measure(devices=(0,), hw=None):
    from .autotune import autotune, load_sweep, write_csv
    shapes = load_sweep(CAL_SWEEP)
    hw = hw if hw is not None else load_hw(DEFAULT_HW_JSON)
    t0 = time.time()
    _, entries = autotune(shapes, 0, devices, hw)
    write_csv(CAL_MEASURED, shapes, entries, hw,
              note="calibration shapes, devices %s, %.1f s" % (list(devices), time.time() - t0))
    return CAL_MEASURED


def main(argv=None):
    from .autotune import load_measured
    ap = argparse.ArgumentParser()
    ap.add_argument("--measure", action="store_true", help="sweep the calibration shapes first")
    ap.add_argument("--from", dest="src", default=str(CAL_MEASURED))
    ap.add_argument("--hw", default=str(DEFAULT_HW_JSON), help="microbenchmark JSON to start from")
    ap.add_argument("--out", default=str(DEFAULT_HW_JSON))
    ap.add_argument("--devices", default="0")
    ap.add_argument("--weight-power", type=float, default=WEIGHT_POWER)
    a = ap.parse_args(argv)
    src = Path(a.src)
    if a.measure:
        src = measure([int(x) for x in a.devices.split(",")], load_hw(a.hw))
    base = json.loads(Path(a.hw).read_text())
    # start from the microbenchmark values when a previous fit is present
    base_raw = dict(base)
    base_raw.update({k[len(MICRO):]: v for k, v in base.items() if k.startswith(MICRO)})
    rows = load_measured(src)
    fitted, obj = fit(rows, {k: v for k, v in base_raw.items() if k in HW_KEYS or k == "name"},
                      weight_power=a.weight_power)
    doc = dict(base)
    doc.update({MICRO + k: base_raw[k] for k in fitted})
    doc.update(fitted)
    doc["fitSource"] = str(src.relative_to(ROOT)) if src.is_relative_to(ROOT) else str(src)
    doc["fitRows"] = len(rows)
    doc["fitWeightPower"] = a.weight_power
    doc["fitWeightedMeanAbsLogError"] = obj
    Path(a.out).write_text(json.dumps(doc, indent=1) + "\n")
    for k in fitted:
        print("%-24s microbenchmark %12.5g  fitted %12.5g" % (k, base_raw[k], fitted[k]))
    print("wrote", a.out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
