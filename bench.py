"""Headline benchmark: FP16 GEMM TFLOP/s at 4096^3 on B200 (ridge hot path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ridge|reference]

One step = one launch of the GEMM (C = A * B, FP16 in, FP32 accumulate, FP16
out) over one batch of synthetic input: A 4096 x 4096 row-major and this rank's
4096 x 4096 N-column slab of B (column-major), drawn U(-1,1) from the
reference's LCG seeded 0 (A first, then B). At N GPUs the GEMM is
4096 x (4096*N) x 4096, split by N-column slabs of B with A replicated: every
rank computes one 4096^3 slab, no collective on the data path (weak scaling).

value   = whole-job TFLOP/s with inputs resident in HBM: sum over ranks of
          2*M*N_slab*K per step / (max over ranks of the summed per-step GEMM
          time). L2 is flushed (256 MiB write) before every timed launch and
          only the GEMM sits between the CUDA events.
e2e     = the same metric through the public C ABI with host buffers: each step
          copies A and the B slab from pinned host memory, launches, and copies
          C back, all inside the timed region.
--impl reference  times the reference's own CPU GEMM (referenceGemm, FP64,
          bench/check-gemm.cu:98-108, built from the reference sources into
          oracle/_ref) on all host cores over a row sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

M = K = 4096
N_SLAB = 4096
METRIC = "FP16 GEMM TFLOP/s (4096^3) vs B200 peak"
UNIT = "TFLOP/s"
# Best 4096^3 config from the autotuner on B200 (model-pruned, top-k measured).
BEST_CONFIG = dict(BM=256, BN=256, BK=64, stages=6, warps=4, groupM=8, cta_group=2)
L2_FLUSH_BYTES = 256 << 20


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def _traffic(workload: str):
    """Per-launch DRAM bytes of the GEMM from the committed ncu summary, or None."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(workload)
    except ValueError:
        return None


class ClockSampler:
    """SM clock and throttle reasons sampled DURING the timed region: an NVML
    thread polling every millisecond between __enter__ and __exit__ (the timed
    region is milliseconds long, too short for nvidia-smi's 100 ms loop), with
    nvidia-smi as the fallback when NVML cannot be opened."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event-reason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40}

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.nvml = None
        self.samples = []      # (sm_mhz, reason bits)
        self.max_mhz = None
        self.lines = []

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        prop = torch.cuda.get_device_properties(self.index)
        # the CUDA device as NVML sees it (CUDA_VISIBLE_DEVICES may renumber)
        uuid = getattr(prop, "uuid", None)
        if uuid is not None:
            u = str(uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(u if u.startswith("GPU-")
                                                             else "GPU-" + u)
        if "CUDA_VISIBLE_DEVICES" in os.environ:
            raise RuntimeError("cannot map the CUDA device to NVML")
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _poll(self):
        nv, h = self.nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((float(mhz), int(bits)))
            except Exception:
                break
            time.sleep(0.001)

    def __enter__(self):
        import threading
        try:
            self.nvml = self._nvml_handle()
            nv, h = self.nvml
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._poll, daemon=True)
            self._thread.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.nvml is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            return
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], self.max_mhz, set()
        if self.nvml is not None:
            for mhz, bits in self.samples:
                sm.append(mhz)
                for name, bit in self.REASONS.items():
                    if bits & bit:
                        reasons.add(name)
            source = "nvml 1 ms"
        else:
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for line in self.lines:
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    mx = float(f[2])
                except ValueError:
                    continue
                for name, val in zip(names, f[5:9]):
                    if val.lower() == "active":
                        reasons.add(name)
            source = "nvidia-smi 100 ms"
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": ["unsampled"], "samples": 0}
        busy = [x for x in sm if mx and x > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": source}


def _dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


class CpuReference:
    """The reference's own CPU GEMM (referenceGemm, FP64, bench/check-gemm.cu:98-108,
    compiled from the reference sources into oracle/_ref) over a row sample of the
    4096^3 workload: output rows [0, rows), split across `threads` host threads.
    Falls back to this repo's C restatement (kind "port", 1 thread) when the
    reference library was not built."""

    def __init__(self, threads: int):
        import numpy as np
        import oracle
        a, b = oracle.unit_inputs(M, N_SLAB, K, seed=0)
        self.a = a
        self.b_kn = np.ascontiguousarray(b.T)  # the reference takes row-major K x N
        if oracle.reference_available():
            self.ref = oracle.Reference()
            self.kind = "reference"
            self.threads = max(1, threads)
        else:
            self.ref = None
            self.kind = "port"
            self.threads = 1

    def run(self, rows: int) -> float:
        import oracle
        t0 = time.perf_counter()
        if self.ref is not None:
            self.ref.gemm_f64(self.a[:rows], self.b_kn, threads=self.threads)
        else:
            oracle.gemm_f64_reference_loop(self.a[:rows], self.b_kn)
        return time.perf_counter() - t0

    def rows_for(self, seconds: float) -> int:
        """Row count whose sample takes about `seconds` (a short probe first)."""
        rows = self.threads
        dt = self.run(rows)
        while dt < 0.2 and rows < M:
            rows = min(M, rows * 4)
            dt = self.run(rows)
        rows = int(rows * seconds / max(dt, 1e-6))
        rows = max(self.threads, (rows // self.threads) * self.threads)
        return min(M, rows)

    def tflops(self, rows: int, dt: float) -> float:
        return 2.0 * rows * N_SLAB * K / dt / 1e12

    def sample_text(self, rows: int, dt: float) -> str:
        return ("output rows [0, %d) of the 4096x4096x4096 GEMM (%.2f%% of it), FP64 %s loop, "
                "%d thread(s), %.1f s" % (rows, 100.0 * rows / M,
                                          "referenceGemm" if self.ref else "restated", self.threads,
                                          dt))


def run_reference(args):
    rank, world, _ = _dist_env()
    if rank != 0:
        return 0
    ref = CpuReference(os.cpu_count() or 1)
    per_step = min(10.0, max(0.5, 150.0 / (args.steps + args.warmup)))
    rows = ref.rows_for(per_step)
    for _ in range(args.warmup):
        ref.run(rows)
    times = [ref.run(rows) for _ in range(args.steps)]
    dt = statistics.median(times)
    value = ref.tflops(rows, dt)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic: reference LCG mapped to U(-1,1), seed 0, A then B",
        "config": {"workload": "%dx%dx%d FP16 GEMM (host FP64 reference loop, row sample)"
                               % (M, N_SLAB, K), "threads": ref.threads},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": ref.threads, "kind": ref.kind,
                         "sample": ref.sample_text(rows, dt)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ridge(args):
    import ctypes as C

    import torch
    import torch.distributed as dist

    import ridge_b200 as rb

    rank, world, local = _dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    cfg = rb.TileConfig(**BEST_CONFIG)
    if args.config:
        cfg = rb.TileConfig(*[int(x) for x in args.config.split(",")])
    # Inputs: one LCG stream from seed 0: A, then the full B (N x K storage);
    # each rank keeps its N-slab (rows [rank*N_SLAB, (rank+1)*N_SLAB) of B).
    a = torch.empty((M, K), dtype=torch.float16, device=dev)
    st = rb.fill_lcg(a, 0)
    b = torch.empty((N_SLAB, K), dtype=torch.float16, device=dev)
    if rank > 0:
        # advance the stream past the earlier ranks' slabs
        skip = torch.empty((N_SLAB, K), dtype=torch.float16, device=dev)
        for _ in range(rank):
            st = rb.fill_lcg(skip, st)
        del skip
    rb.fill_lcg(b, st)
    c = torch.empty((M, N_SLAB), dtype=torch.float16, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream

    def launch(a_t, b_t, c_t):
        s = rb.launch_raw(cfg, a_t.data_ptr(), b_t.data_ptr(), c_t.data_ptr(), M, N_SLAB, K, K,
                          K, N_SLAB, sh)
        if s != 0:
            raise rb.RidgeError(s, "ridge_gemm_launch")

    for _ in range(args.warmup):
        flush.zero_()
        launch(a, b, c)
    torch.cuda.synchronize()
    if rb.device_error() != 0:
        raise RuntimeError("device error during warm-up")

    # ------------------------------------------------ device-resident timing
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            launch(a, b, c)
            ends[i].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    per_step = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(per_step)
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    flops_step = 2.0 * M * N_SLAB * K
    value = world * flops_step * args.steps / (total_ms * 1e-3) / 1e12
    kernel_ms = total_ms / args.steps
    if rb.device_error() != 0:
        raise RuntimeError("device error during the timed region")

    # ------------------------------------------------ end to end (host buffers)
    # The user-facing host-buffer call, ridge_gemm_host: page-locked A and B in,
    # C out, the copies pipelined against the kernel by M-panels inside the call.
    a_h = torch.empty((M, K), dtype=torch.float16).pin_memory()
    b_h = torch.empty((N_SLAB, K), dtype=torch.float16).pin_memory()
    c_h = torch.empty((M, N_SLAB), dtype=torch.float16).pin_memory()
    a_h.copy_(a)
    b_h.copy_(b)
    cc = cfg.to_c()

    def host_call():
        s = rb.lib.ridge_gemm_host(C.byref(cc), a_h.data_ptr(), b_h.data_ptr(), c_h.data_ptr(),
                                   M, N_SLAB, K, K, K, N_SLAB, args.panels, sh)
        if s != 0:
            raise rb.RidgeError(s, "ridge_gemm_host")

    for _ in range(max(1, args.warmup)):
        host_call()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        host_call()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * flops_step * args.steps / (e2e_ms * 1e-3) / 1e12
    # Same kernel, but panels change the split-K tail plan (summation order):
    # agreement to FP16 rounding, not bit for bit.
    cr = c.float().cpu()
    ok = bool(((c_h.float() - cr).norm() / cr.norm()).item() <= 1e-3)

    # ------------------------------------------------ report (rank 0)
    if rank == 0:
        peak, _hbm, peak_src = _peaks()
        achieved = flops_step / (kernel_ms * 1e-3) / 1e12
        workload = "4096x4096x4096 slab"
        traffic = _traffic(workload)
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            ref = CpuReference(1)
            rows = ref.rows_for(12.0)
            dt = ref.run(rows)
            cpu = {"value": ref.tflops(rows, dt), "unit": UNIT, "cores": ref.threads,
                   "kind": ref.kind, "sample": ref.sample_text(rows, dt)}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": kernel_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic: reference LCG mapped to U(-1,1), seed 0, A then B (device fill)",
            "config": {
                "workload": "%dx%dx%d FP16 GEMM per rank (N-slab of %dx%dx%d, A replicated)"
                            % (M, N_SLAB, K, M, N_SLAB * world, K),
                "tile": cfg.as_dict(), "layout": "A row-major, B column-major, C row-major FP16",
                "accumulate": "fp32", "parallelism": "n-slab x%d" % world,
                "l2": "flushed before every timed launch (256 MiB write), inputs 96 MiB < L2",
                "timing": "CUDA events around each launch, summed; max over ranks",
            },
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_source": peak_src + " bf16 dense (burst)",
                         "traffic": traffic},
            "clocks": clocks.summary(),
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": (M * K + N_SLAB * K) * 2,
                    "d2h_bytes_per_step": M * N_SLAB * 2},
            "gpu_launches": args.steps,
            "e2e_result_matches": ok,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ridge", "reference"], default="ridge")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--panels", type=int, default=0,
                    help="M-panels of the end-to-end host-buffer call (0 = its default)")
    ap.add_argument("--config", default=None,
                    help="BM,BN,BK,stages,warps,groupM,cta_group instead of the default tile")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ridge(args)


if __name__ == "__main__":
    sys.exit(main())
