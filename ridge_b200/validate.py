"""Model validation report for the B200 sweep.

Reference: bench/validate.py. Same gates, same questions, for the B200 model:

- the measured sweep must be exactly the registered cross product (every
  registered shape x every registered variant of libridge_b200.so), so a sweep
  that lost its inconvenient rows cannot produce a better number;
- absolute accuracy: MAPE (gate <= 20%), median, p90, max, mean signed error,
  the worst configurations;
- ranking, per shape (an autotuner ranks one shape at a time): Spearman's rho
  with tied predictions given their average rank, where the measured best sits
  in the predicted order (a range when it is inside a tie group), regret@1 (a
  range under ties) and the top-k regret the autotuner actually pays;
- the label distribution the model emits on the sweep.

Predictions are recomputed from the current model (ridge_predict with the
committed calibration), never read from the CSV.

    python -m ridge_b200.validate [--measured data/measured/b200-exhaustive.csv]
"""

from __future__ import annotations

import argparse
import collections
import statistics
import sys
from pathlib import Path

from .autotune import REGISTERED, load_measured, load_sweep
from .gemm import config_info, variants
from .model import DEFAULT_HW_JSON, load_hw, predict

ROOT = Path(__file__).resolve().parent.parent
MEASURED = ROOT / "data" / "measured" / "b200-exhaustive.csv"
MAPE_GATE = 20.0
TOPK = 10


def _key(M, N, K, cfg):
    return (M, N, K, cfg.BM, cfg.BN, cfg.BK, cfg.stages, cfg.warps, cfg.cta_group)


def registration_gap(rows, shapes, table):
    """(missing, extra) against the registered shapes x variant table."""
    expected = set()
    for (M, N, K, _tag) in shapes:
        for v in table:
            expected.add(_key(M, N, K, v.config))
    got = set()
    for r in rows:
        info = config_info(r["config"])
        got.add(_key(r["M"], r["N"], r["K"], info.config))
    return expected - got, got - expected


def average_ranks(values):
    """1-based ranks, highest value first; ties share their average rank."""
    order = sorted(range(len(values)), key=lambda i: -values[i])
    ranks = [0.0] * len(values)
    i = 0
    while i < len(order):
        j = i
        while j + 1 < len(order) and values[order[j + 1]] == values[order[i]]:
            j += 1
        avg = (i + j) / 2.0 + 1.0
        for k in range(i, j + 1):
            ranks[order[k]] = avg
        i = j + 1
    return ranks


def spearman(x, y):
    """Pearson correlation of the average ranks; nan without variance."""
    rx, ry = average_ranks(x), average_ranks(y)
    mx, my = statistics.mean(rx), statistics.mean(ry)
    sxy = sum((a - mx) * (b - my) for a, b in zip(rx, ry))
    sxx = sum((a - mx) ** 2 for a in rx)
    syy = sum((b - my) ** 2 for b in ry)
    if sxx == 0 or syy == 0:
        return float("nan")
    return sxy / (sxx * syy) ** 0.5


def best_rank_range(pred, meas):
    """Where the measured-best config sits in the predicted order: (first,
    last) position it could take when its prediction is tied with others."""
    b = max(range(len(meas)), key=lambda i: meas[i])
    above = sum(1 for p in pred if p > pred[b])
    tied = sum(1 for p in pred if p == pred[b])
    return above + 1, above + tied


def regret1_range(pred, meas):
    """regret@1 as (worst, best) over the configs tied for the top prediction."""
    best = max(meas)
    top = max(pred)
    tied = [m for p, m in zip(pred, meas) if p == top]
    return (best - min(tied)) / best, (best - max(tied)) / best, len(tied)


def topk_regret(pred, meas, k):
    best = max(meas)
    order = sorted(range(len(pred)), key=lambda i: -pred[i])[:k]
    return (best - max(meas[i] for i in order)) / best


def report(measured=MEASURED, registered=REGISTERED, hw_path=DEFAULT_HW_JSON, out=print):
    rows = load_measured(measured)
    shapes = load_sweep(registered)
    table = variants()
    hw = load_hw(hw_path)
    failures = []
    out("=" * 78)
    out("ridge B200 model validation")
    out("=" * 78)
    out("  measured  %s" % measured)
    out("  model     %s (%s)" % (hw_path, hw.name.decode()))
    missing, extra = registration_gap(rows, shapes, table)
    out("registered cross product: %d shapes x %d variants = %d; measured rows: %d" % (
        len(shapes), len(table), len(shapes) * len(table), len(rows)))
    if missing or extra:
        out("  MISSING %d, EXTRA %d" % (len(missing), len(extra)))
        for m in sorted(missing)[:5]:
            out("    missing %s" % (m,))
        failures.append("measured set does not match the registered sweep")
    else:
        out("  matches the registered sweep exactly")
    out("")

    labels = collections.Counter()
    for r in rows:
        p = predict(r["M"], r["N"], r["K"], r["config"], hw)
        r["pred"] = p["predicted_tflops"]
        r["label"] = p.label
        labels[p.label] += 1
        r["err"] = (r["pred"] - r["tflops"]) / r["tflops"] * 100.0
    errs = sorted(abs(r["err"]) for r in rows)
    mape = statistics.mean(errs)
    pct = lambda q: errs[min(len(errs) - 1, int(q * (len(errs) - 1) + 0.5))]
    out("absolute accuracy")
    out("  MAPE               %7.2f %%   (gate <= %.0f%%)" % (mape, MAPE_GATE))
    out("  median abs error   %7.2f %%" % pct(0.5))
    out("  p90 abs error      %7.2f %%" % pct(0.9))
    out("  max abs error      %7.2f %%" % errs[-1])
    out("  mean signed error  %+7.2f %%   (negative = model under-predicts)" %
        statistics.mean(r["err"] for r in rows))
    out("  worst 8 configurations:")
    for r in sorted(rows, key=lambda r: -abs(r["err"]))[:8]:
        out("    %-18s %-24s meas %8.1f pred %8.1f %+7.1f%%" % (
            "%dx%dx%d" % (r["M"], r["N"], r["K"]), r["config"].tag(), r["tflops"], r["pred"],
            r["err"]))
    if mape > MAPE_GATE:
        failures.append("MAPE %.1f%% above the %.0f%% gate" % (mape, MAPE_GATE))
    out("")

    out("ranking, per shape")
    out("  %-26s %8s %6s %12s %9s %14s %10s" % ("shape", "spearman", "ties", "rank of best",
                                                 "recall@3", "regret@1 %", "top-%d %%" % TOPK))
    by = collections.OrderedDict()
    for r in rows:
        by.setdefault((r["M"], r["N"], r["K"], r["tag"]), []).append(r)
    rhos, worst1, regk = [], [], []
    for (M, N, K, tag), rs in by.items():
        pred = [r["pred"] for r in rs]
        meas = [r["tflops"] for r in rs]
        rho = spearman(pred, meas)
        lo, hi = best_rank_range(pred, meas)
        w, b, nt = regret1_range(pred, meas)
        rk = topk_regret(pred, meas, TOPK)
        rhos.append(rho)
        worst1.append(w)
        regk.append(rk)
        ties = max(collections.Counter(round(p, 6) for p in pred).values())
        out("  %-26s %8s %6d %12s %9s %14s %10.2f" % (
            ("%s %dx%dx%d" % (tag, M, N, K))[:26],
            "n/a" if rho != rho else "%.3f" % rho, ties,
            "%d" % lo if lo == hi else "%d-%d" % (lo, hi),
            "yes" if hi <= 3 else ("maybe" if lo <= 3 else "no"),
            "%.1f" % (100 * w) if nt == 1 else "%.1f-%.1f" % (100 * w, 100 * b), 100 * rk))
    valid = [x for x in rhos if x == x]
    out("")
    out("  mean Spearman       %7.3f" % (statistics.mean(valid) if valid else float("nan")))
    out("  worst regret@1      %7.2f %%" % (100 * max(worst1)))
    out("  mean top-%d regret  %7.2f %%   worst %.2f %%" % (
        TOPK, 100 * statistics.mean(regk), 100 * max(regk)))
    out("")
    out("labels the model emits on the sweep: %s" % ", ".join(
        "%s %d" % kv for kv in labels.most_common()))
    out("")
    if failures:
        out("FAIL: " + "; ".join(failures))
    else:
        out("PASS: registered sweep complete, MAPE within the gate")
    return {"mape": mape, "spearman": statistics.mean(valid) if valid else float("nan"),
            "topk_regret_mean": statistics.mean(regk), "topk_regret_worst": max(regk),
            "failures": failures, "labels": dict(labels)}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--measured", default=str(MEASURED))
    ap.add_argument("--registered", default=str(REGISTERED))
    ap.add_argument("--hw", default=str(DEFAULT_HW_JSON))
    a = ap.parse_args(argv)
    res = report(a.measured, a.registered, a.hw)
    return 1 if res["failures"] else 0


if __name__ == "__main__":
    sys.exit(main())
