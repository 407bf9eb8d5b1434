"""The B200 bottleneck-label check: collect hardware counters for the
registered configurations and score the model's labels against them.

Reference: bench/run-ncu-validation.sh collects counters for twelve registered
configs under `ncu`; the counters-to-label table and the pass criterion were
fixed in a separate file before any run. Same split here: the configurations
live in data/sweep/b200-ncu-configs.csv and the table below (RULES) was
committed with them before the first run; `collect` only gathers counters and
`score` only applies RULES. Neither may be edited to improve a result.

    python -m ridge_b200.ncu_validate collect --out ncu-labels.csv   # on a B200
    python -m ridge_b200.ncu_validate score data/measured/b200-ncu-labels.csv
    python -m ridge_b200.ncu_validate table --out ncu-table.csv       # on a B200
    python -m ridge_b200.ncu_validate render data/measured/b200-ncu-table.csv

`table` gathers a per-configuration counter table (tensor pipe, DRAM bytes
and GB/s, L2 -> SM bytes, shared-memory wavefronts of the tensor-core data
path) for the configurations in data/sweep/b200-ncu-table.csv, the same way
(plain run first, then one captured launch); `render` prints it as Markdown.

`collect` runs every configuration once without the profiler (the same command
line), and only if that exits 0 runs it under
`ncu --clock-control none -k regex:ridge_gemm_sm100 -s 1 -c 1` (one warm-up
launch skipped, one launch captured, a handful of counters): small captures
that end by themselves.
"""

from __future__ import annotations

import argparse
import csv
import io
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
CONFIGS = ROOT / "data" / "sweep" / "b200-ncu-configs.csv"
TABLE_CONFIGS = ROOT / "data" / "sweep" / "b200-ncu-table.csv"

METRICS = [
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
    "sm__cycles_active.avg.pct_of_peak_sustained_elapsed",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
    "l1tex__m_xbar2l1tex_read_bytes.sum",
    "l1tex__m_l1tex2xbar_write_bytes.sum",
    "sm__cycles_active.sum",
]

# Counters of the per-configuration table.
TABLE_METRICS = [
    "gpu__time_duration.sum",
    "sm__cycles_elapsed.avg.per_second",
    "sm__cycles_active.avg.pct_of_peak_sustained_elapsed",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
    "l1tex__m_xbar2l1tex_read_bytes.sum",
    "l1tex__data_pipe_tc_wavefronts_mem_shared.sum",
]

# The registered thresholds.
FILL_CAP = 72.0          # B/cycle/SM, the calibrated TMA fill cap
PASS_AGREE = 12          # of 16


def label_from_counters(c: dict) -> str:
    """The registered decision table, first match wins."""
    dram = c["gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed"]
    active = c["sm__cycles_active.avg.pct_of_peak_sustained_elapsed"]
    tensor = c["sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active"]
    cycles = max(c["sm__cycles_active.sum"], 1.0)
    fill = c["l1tex__m_xbar2l1tex_read_bytes.sum"] / cycles
    write = c["l1tex__m_l1tex2xbar_write_bytes.sum"] / cycles
    if dram >= 70:
        return "HBM"
    if active < 80:
        return "WAVES"
    if tensor >= 85:
        return "TENSOR_CORE"
    if fill >= 0.75 * FILL_CAP:
        return "L2"
    if write >= 12 and tensor < 50:
        return "EPILOGUE"
    if tensor < 60:
        return "OCC"
    return "ENVELOPE"


def load_configs(path=CONFIGS):
    with open(path, newline="") as f:
        rows = list(csv.DictReader(l for l in f if not l.startswith("#")))
    for r in rows:
        for k in ("M", "N", "K", "BM", "BN", "BK", "stages", "warps", "groupM", "cta_group"):
            r[k] = int(r[k])
    return rows


def run_one(M, N, K, cfg_tuple, launches=2):
    """`launches` launches of one configuration (the first is the warm-up the
    profiler skips)."""
    import torch

    import ridge_b200 as rb
    cfg = rb.TileConfig(*cfg_tuple)
    a, b = rb.synthetic_inputs(M, N, K)
    c = torch.empty((M, N), dtype=torch.float16, device="cuda")
    for _ in range(launches):
        rb.gemm(a, b, c, config=cfg)
    torch.cuda.synchronize()
    if rb.device_error() != 0:
        raise RuntimeError("device error word set")


def _cmd(r):
    cfg = "%d,%d,%d,%d,%d,%d,%d" % (r["BM"], r["BN"], r["BK"], r["stages"], r["warps"],
                                    r["groupM"], r["cta_group"])
    return [sys.executable, "-m", "ridge_b200.ncu_validate", "one", str(r["M"]), str(r["N"]),
            str(r["K"]), cfg]


def _parse_ncu_csv(text: str) -> dict:
    lines = [l for l in text.splitlines() if l.startswith('"')]
    out = {}
    for row in csv.DictReader(io.StringIO("\n".join(lines))):
        name, val = row.get("Metric Name"), row.get("Metric Value")
        if name in METRICS and val not in (None, ""):
            out[name] = float(val.replace(",", ""))
    return out


def collect(out_path, configs=CONFIGS, log=print):
    ncu = shutil.which("ncu") or "/usr/local/cuda/bin/ncu"
    rows = load_configs(configs)
    out_path = Path(out_path)
    out_path.parent.mkdir(parents=True, exist_ok=True)
    with open(out_path, "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(["predicted_label", "tag", "M", "N", "K", "BM", "BN", "BK", "stages", "warps",
                    "groupM", "cta_group", *METRICS])
        for i, r in enumerate(rows):
            cmd = _cmd(r)
            plain = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
            if plain.returncode != 0:
                log("[%2d] %s plain run failed (%d), not profiled:\n%s" % (
                    i + 1, r["tag"], plain.returncode, plain.stderr[-2000:]))
                continue
            prof = subprocess.run([ncu, "--csv", "--clock-control", "none", "--metrics",
                                   ",".join(METRICS), "-k", "regex:ridge_gemm_sm100", "-s", "1",
                                   "-c", "1", *cmd], capture_output=True, text=True,
                                  timeout=600)
            vals = _parse_ncu_csv(prof.stdout)
            if len(vals) != len(METRICS):
                log("[%2d] %s: %d of %d counters (rc %d):\n%s" % (
                    i + 1, r["tag"], len(vals), len(METRICS), prof.returncode,
                    (prof.stdout + prof.stderr)[-2000:]))
                continue
            w.writerow([r["predicted_label"], r["tag"], r["M"], r["N"], r["K"], r["BM"], r["BN"],
                        r["BK"], r["stages"], r["warps"], r["groupM"], r["cta_group"],
                        *[vals[m] for m in METRICS]])
            f.flush()
            log("[%2d] %-5s %-14s done" % (i + 1, r["predicted_label"], r["tag"]))
    return out_path


def _ncu_metrics(cmd, metrics, ncu):
    """Plain run of `cmd` first; only if it exits 0, one captured launch of the
    GEMM (the second; the first is a warm-up) with `metrics`. Returns the
    counters (name -> float, in ncu's base units), or an error string."""
    plain = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    if plain.returncode != 0:
        return "plain run failed (%d): %s" % (plain.returncode, plain.stderr[-500:])
    prof = subprocess.run([ncu, "--csv", "--print-units", "base", "--clock-control", "none",
                           "--metrics", ",".join(metrics), "-k", "regex:ridge_gemm_sm100", "-s",
                           "1", "-c", "1", *cmd], capture_output=True, text=True, timeout=600)
    lines = [l for l in prof.stdout.splitlines() if l.startswith('"')]
    vals = {}
    for row in csv.DictReader(io.StringIO("\n".join(lines))):
        name, val = row.get("Metric Name"), row.get("Metric Value")
        if name in metrics and val not in (None, ""):
            vals[name] = float(val.replace(",", ""))
    if len(vals) != len(metrics):
        return "%d of %d counters (rc %d): %s" % (len(vals), len(metrics), prof.returncode,
                                                 (prof.stdout + prof.stderr)[-500:])
    return vals


def table(out_path, configs=TABLE_CONFIGS, log=print):
    ncu = shutil.which("ncu") or "/usr/local/cuda/bin/ncu"
    rows = load_configs(configs)
    out_path = Path(out_path)
    out_path.parent.mkdir(parents=True, exist_ok=True)
    with open(out_path, "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(["tag", "M", "N", "K", "BM", "BN", "BK", "stages", "warps", "groupM",
                    "cta_group", *TABLE_METRICS])
        for i, r in enumerate(rows):
            vals = _ncu_metrics(_cmd(r), TABLE_METRICS, ncu)
            if isinstance(vals, str):
                log("[%2d] %s: %s" % (i + 1, r["tag"], vals))
                continue
            w.writerow([r["tag"], r["M"], r["N"], r["K"], r["BM"], r["BN"], r["BK"], r["stages"],
                        r["warps"], r["groupM"], r["cta_group"], *[vals[m] for m in TABLE_METRICS]])
            f.flush()
            log("[%2d] %s %sx%sx%s done" % (i + 1, r["tag"], r["BM"], r["BN"], r["BK"]))
    return out_path


def render(path, hbm_peak_gbs=None, log=print):
    """The counter table as Markdown: per configuration the captured launch's
    time, TFLOP/s, tensor-pipe share of active and elapsed cycles, DRAM bytes
    and GB/s (and % of the measured copy peak when given), algorithmic bytes,
    L2 -> SM bytes per SM cycle, and shared-memory wavefronts per SM cycle of
    the tensor-core data path (128 B each)."""
    with open(path, newline="") as f:
        rows = list(csv.DictReader(l for l in f if not l.startswith("#")))
    log("| cfg | shape | tile | us | TFLOP/s | tensor %% active | tensor %% elapsed | SM active %% "
        "| DRAM MB (alg.) | DRAM GB/s%s | L2->SM B/clk/SM | smem wavefronts/clk/SM |"
        % (" (%% of peak)" if hbm_peak_gbs else ""))
    log("|---|---|---|---|---|---|---|---|---|---|---|---|")
    for r in rows:
        g = {k: float(r[k]) for k in TABLE_METRICS}
        M, N, K = int(r["M"]), int(r["N"]), int(r["K"])
        sec = g["gpu__time_duration.sum"] * 1e-9
        cycles = sec * g["sm__cycles_elapsed.avg.per_second"] * 148
        dram = g["dram__bytes_read.sum"] + g["dram__bytes_write.sum"]
        alg = 2.0 * (M * K + N * K + M * N)
        gbs = dram / sec / 1e9
        log("| %s | %dx%dx%d | %sx%sx%s s%s w%s c%s | %.1f | %.0f | %.1f | %.1f | %.1f | %.1f (%.1f) "
            "| %.0f%s | %.1f | %.2f |" % (
                r["tag"], M, N, K, r["BM"], r["BN"], r["BK"], r["stages"], r["warps"],
                r["cta_group"], sec * 1e6, 2.0 * M * N * K / sec / 1e12,
                g["sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active"],
                g["sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed"],
                g["sm__cycles_active.avg.pct_of_peak_sustained_elapsed"], dram / 1e6, alg / 1e6,
                gbs, (" (%.0f%%)" % (100.0 * gbs / hbm_peak_gbs)) if hbm_peak_gbs else "",
                g["l1tex__m_xbar2l1tex_read_bytes.sum"] / cycles,
                g["l1tex__data_pipe_tc_wavefronts_mem_shared.sum"] / cycles))
    return len(rows)


def score(path, log=print):
    with open(path, newline="") as f:
        rows = list(csv.DictReader(l for l in f if not l.startswith("#")))
    agree = 0
    log("%-6s %-14s %-22s %6s %6s %6s %6s %6s  %s" % (
        "model", "shape", "config", "DRAM%", "SMact%", "tens%", "fillB", "writeB", "counters"))
    for r in rows:
        c = {m: float(r[m]) for m in METRICS}
        got = label_from_counters(c)
        agree += got == r["predicted_label"]
        cyc = max(c["sm__cycles_active.sum"], 1.0)
        log("%-6s %-14s %-22s %6.1f %6.1f %6.1f %6.1f %6.1f  %s%s" % (
            r["predicted_label"], r["tag"],
            "%sx%sx%s_s%s_w%s_c%s" % (r["BM"], r["BN"], r["BK"], r["stages"], r["warps"],
                                      r["cta_group"]),
            c[METRICS[0]], c[METRICS[1]], c[METRICS[2]],
            c["l1tex__m_xbar2l1tex_read_bytes.sum"] / cyc,
            c["l1tex__m_l1tex2xbar_write_bytes.sum"] / cyc, got,
            "" if got == r["predicted_label"] else "  (disagrees)"))
    n = len(rows)
    verdict = "PASS" if agree >= PASS_AGREE and n == 16 else "FAIL"
    log("agreement %d of %d (registered pass: >= %d of 16): %s" % (agree, n, PASS_AGREE, verdict))
    return agree, n, verdict


def main(argv=None):
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    o = sub.add_parser("one")
    o.add_argument("M", type=int)
    o.add_argument("N", type=int)
    o.add_argument("K", type=int)
    o.add_argument("config")
    c = sub.add_parser("collect")
    c.add_argument("--out", default="ncu-labels.csv",
                   help="CSV of counters per configuration (default: ./ncu-labels.csv)")
    s = sub.add_parser("score")
    s.add_argument("path")
    t = sub.add_parser("table")
    t.add_argument("--out", default="ncu-table.csv")
    r = sub.add_parser("render")
    r.add_argument("path")
    r.add_argument("--hbm-peak-gbs", type=float, default=None)
    a = ap.parse_args(argv)
    if a.cmd == "table":
        print("wrote", table(a.out))
        return 0
    if a.cmd == "render":
        render(a.path, a.hbm_peak_gbs)
        return 0
    if a.cmd == "one":
        run_one(a.M, a.N, a.K, tuple(int(x) for x in a.config.split(",")))
        return 0
    if a.cmd == "collect":
        print("wrote", collect(a.out))
        return 0
    _, _, verdict = score(a.path)
    return 0 if verdict == "PASS" else 1


if __name__ == "__main__":
    sys.exit(main())
