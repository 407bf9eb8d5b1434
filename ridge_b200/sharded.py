"""N-slab sharding of one large GEMM across the GPUs of a node.

C = A * B is split by N-column slabs of B with A replicated: rank r of P owns
rows [n0, n0 + n_slab) of B's N x K storage (a contiguous block, since B is
column-major) and computes C[:, n0:n0+n_slab] with an ordinary local launch --
no collective on the data path. Slab bounds come from ridge_slab_bounds (slab
width ceil(N / P) rounded up to a multiple of `align`, so every slab but the
last is tile-aligned).

When the caller wants the full C on every rank, `gather=True` all-gathers the
slabs over NCCL (NVLink / NVSwitch) into a slab-major buffer of P equal-size
slabs and re-lays it out into row-major C with ridge_slabs_to_rowmajor.

One process per GPU (torchrun); the reference is single-GPU, so this is the
B200 build's own multi-GPU mode.

    torchrun --nproc-per-node 8 -m ridge_b200.sharded --shape 16384x16384x16384 [--gather]
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import sys

from ._native import check, lib
from .gemm import TileConfig, _stream_handle, launch_raw

SLAB_ALIGN = 256


def slab_bounds(N: int, nranks: int, rank: int, align: int = SLAB_ALIGN):
    n0, ns = C.c_int64(), C.c_int64()
    check(lib.ridge_slab_bounds(N, nranks, rank, align, C.byref(n0), C.byref(ns)),
          "ridge_slab_bounds")
    return n0.value, ns.value


def slab_width(N: int, nranks: int, align: int = SLAB_ALIGN) -> int:
    """Columns every slab buffer holds in the gather (the first slab's width)."""
    return slab_bounds(N, nranks, 0, align)[1] if nranks > 1 else N


def slab_gemm(a, b_slab, c_slab, config: TileConfig, stream=None):
    """This rank's slab: c_slab (M x n_slab, leading dim >= n_slab) = a (M x K)
    times b_slab^T (b_slab = n_slab x K rows of B's storage)."""
    M, K = a.shape
    ns = b_slab.shape[0]
    if ns == 0 or M == 0:
        return c_slab
    st = launch_raw(config, a.data_ptr(), b_slab.data_ptr(), c_slab.data_ptr(), M, ns, K,
                    a.stride(0), b_slab.stride(0), c_slab.stride(0), _stream_handle(stream))
    check(st, "slab GEMM %dx%dx%d" % (M, ns, K))
    return c_slab


def slabs_to_rowmajor(slabs, C_out, M: int, N: int, nranks: int, slab_cols: int, stream=None):
    """Device re-layout of P contiguous (M x slab_cols) slabs into row-major C."""
    check(lib.ridge_slabs_to_rowmajor(slabs.data_ptr(), C_out.data_ptr(), M, N, nranks,
                                      slab_cols, C_out.stride(0), _stream_handle(stream)),
          "ridge_slabs_to_rowmajor")
    return C_out


def sharded_gemm(a, b, config: TileConfig, gather: bool = False, group=None, rank=None,
                 world=None):
    """Rank-local part of the N-slab GEMM. `b` is either the full N x K
    storage of B (this rank slices its rows) or already this rank's slab (then
    pass the full N as b.full_n). Returns (c_slab, full_c or None)."""
    import torch
    import torch.distributed as dist
    if world is None:
        world = dist.get_world_size(group) if dist.is_initialized() else 1
    if rank is None:
        rank = dist.get_rank(group) if dist.is_initialized() else 0
    N = getattr(b, "full_n", b.shape[0])
    n0, ns = slab_bounds(N, world, rank)
    b_slab = b if getattr(b, "full_n", None) is not None else b[n0:n0 + ns]
    M = a.shape[0]
    per = slab_width(N, world)
    # The gather needs equal-size slabs: compute into a per-column-wide buffer.
    c_slab = torch.empty((M, max(per, 1)), dtype=torch.float16, device=a.device)
    slab_gemm(a, b_slab, c_slab, config)
    if not gather or world == 1:
        return c_slab[:, :ns], (c_slab[:, :N] if world == 1 and gather else None)
    slabs = torch.empty((world, M, per), dtype=torch.float16, device=a.device)
    dist.all_gather_into_tensor(slabs.view(-1), c_slab.view(-1), group=group)
    full = torch.empty((M, N), dtype=torch.float16, device=a.device)
    slabs_to_rowmajor(slabs, full, M, N, world, per)
    return c_slab[:, :ns], full


def main(argv=None):
    """Whole-node TFLOP/s of an N-slab GEMM: device time of `steps` slab GEMMs
    per rank (CUDA events), max over ranks; optionally the gather separately."""
    import torch
    import torch.distributed as dist

    from .gemm import fill_lcg
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", default="16384x16384x16384", help="MxNxK")
    ap.add_argument("--config", default="256,256,64,5,4,8,2",
                    help="BM,BN,BK,stages,warps,groupM,cta_group")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--gather", action="store_true")
    a = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    cfg = TileConfig(*[int(x) for x in a.config.split(",")])
    M, N, K = (int(x) for x in a.shape.lower().split("x"))
    n0, ns = slab_bounds(N, world, rank)
    A = torch.empty((M, K), dtype=torch.float16, device=dev)
    st = fill_lcg(A, 0)
    B = torch.empty((ns, K), dtype=torch.float16, device=dev)
    # B rows [n0, n0+ns) of the LCG stream that continues after A
    if n0:
        skip = torch.empty((n0, K), dtype=torch.float16, device=dev)
        st = fill_lcg(skip, st)
        del skip
    fill_lcg(B, st)
    per = slab_width(N, world)
    Cs = torch.empty((M, per), dtype=torch.float16, device=dev)
    for _ in range(a.warmup):
        slab_gemm(A, B, Cs, cfg)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        slab_gemm(A, B, Cs, cfg)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    gather_ms = None
    if a.gather and world > 1:
        slabs = torch.empty((world, M, per), dtype=torch.float16, device=dev)
        full = torch.empty((M, N), dtype=torch.float16, device=dev)
        for _ in range(2):
            dist.all_gather_into_tensor(slabs.view(-1), Cs.view(-1))
        torch.cuda.synchronize()
        dist.barrier()
        e0.record()
        for _ in range(a.steps):
            dist.all_gather_into_tensor(slabs.view(-1), Cs.view(-1))
            slabs_to_rowmajor(slabs, full, M, N, world, per)
        e1.record()
        torch.cuda.synchronize()
        g = torch.tensor([e0.elapsed_time(e1) / a.steps], dtype=torch.float64, device=dev)
        dist.all_reduce(g, op=dist.ReduceOp.MAX)
        gather_ms = float(g.item())
    if rank == 0:
        tflops = 2.0 * M * N * K / (float(t.item()) * 1e-3) / 1e12
        print(json.dumps({"workload": "%dx%dx%d N-slab over %d GPU(s)" % (M, N, K, world),
                          "config": cfg.tag(), "ms_per_gemm_max_over_ranks": float(t.item()),
                          "tflops_whole_node": tflops, "gather_ms": gather_ms}))
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
