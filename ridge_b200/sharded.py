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
from datetime import timedelta

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


def nccl_comm_ptr(group=None) -> int:
    """The ncclComm_t behind a torch.distributed NCCL process group (default:
    the world group), for ridge_gemm_sharded's gather."""
    import torch
    import torch.distributed as dist
    pg = group if group is not None else dist.distributed_c10d._get_default_group()
    return pg._get_backend(torch.device("cuda"))._comm_ptr()


def sharded_gemm(a, b, config: TileConfig, gather: bool = False, group=None, rank=None,
                 world=None, stream=None):
    """Rank-local part of the N-slab GEMM through ridge_gemm_sharded. `b` is
    either the full N x K storage of B (this rank slices its rows) or already
    this rank's slab (then pass the full N as b.full_n). With gather=True the
    slabs are all-gathered over the group's NCCL communicator and re-laid out
    into the full row-major C on every rank. Returns (c_slab, full_c or None)."""
    import torch
    import torch.distributed as dist
    if world is None:
        world = dist.get_world_size(group) if dist.is_initialized() else 1
    if rank is None:
        rank = dist.get_rank(group) if dist.is_initialized() else 0
    N = getattr(b, "full_n", b.shape[0])
    n0, ns = slab_bounds(N, world, rank)
    b_slab = b if getattr(b, "full_n", None) is not None else b[n0:n0 + ns]
    M, K = a.shape
    per = slab_width(N, world)
    # the gather needs equal-size slabs: compute into a slab-width buffer
    c_slab = torch.empty((M, max(per, 1)), dtype=torch.float16, device=a.device)
    slabs = full = None
    comm = None
    if gather:
        full = torch.empty((M, N), dtype=torch.float16, device=a.device)
        if world > 1:
            slabs = torch.empty((world, M, per), dtype=torch.float16, device=a.device)
            comm = nccl_comm_ptr(group)
    cc = config.to_c()
    b_ptr = b_slab.data_ptr() if ns else a.data_ptr()   # unused when the slab is empty
    st = lib.ridge_gemm_sharded(C.byref(cc), a.data_ptr(), b_ptr, c_slab.data_ptr(), M, N, K,
                                max(a.stride(0), 1), max(b_slab.stride(0), 1) if ns else K,
                                world, rank, 1 if gather else 0, comm,
                                slabs.data_ptr() if slabs is not None else None,
                                full.data_ptr() if full is not None else None,
                                full.stride(0) if full is not None else N,
                                _stream_handle(stream))
    check(st, "ridge_gemm_sharded %dx%dx%d rank %d/%d" % (M, N, K, rank, world))
    return c_slab[:, :ns], full


class PeerC:
    """Every rank's full M x N C, mapped into every rank's process: allocated
    here with ridge_device_alloc (CUDA IPC needs a whole allocation),
    handles exchanged over the process group, peers' buffers opened with
    ridge_ipc_open. `ptrs` is the device-pointer array ridge_gemm_sharded_p2p
    takes; `local` is this rank's C as a torch tensor (no copy)."""

    def __init__(self, M: int, N: int, group=None):
        import torch
        import torch.distributed as dist
        self.M, self.N = M, N
        self.ldc = max(8, (N + 7) // 8 * 8)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        base = C.c_void_p()
        check(lib.ridge_device_alloc(M * self.ldc * 2, C.byref(base)), "ridge_device_alloc")
        self._base = base.value
        nb = lib.ridge_ipc_handle_bytes()
        h = (C.c_char * nb)()
        check(lib.ridge_ipc_export(self._base, h), "ridge_ipc_export")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(h), group=group)
        self._opened = []
        ptrs = []
        for r, hb in enumerate(handles):
            if r == self.rank:
                ptrs.append(self._base)
                continue
            p = C.c_void_p()
            check(lib.ridge_ipc_open(C.create_string_buffer(hb, nb), C.byref(p)),
                  "ridge_ipc_open rank %d" % r)
            self._opened.append(p.value)
            ptrs.append(p.value)
        self.ptrs = (C.c_void_p * self.world)(*ptrs)
        buf = self

        class _View:
            __cuda_array_interface__ = {"shape": (M, N), "strides": (self.ldc * 2, 2),
                                        "typestr": "<f2", "data": (buf._base, False),
                                        "version": 3}
        self.local = torch.as_tensor(_View(), device=torch.device("cuda",
                                                                  torch.cuda.current_device()))

    def close(self, group=None):
        """Collective: unmap the peers' buffers, wait until every rank has
        unmapped this rank's, then free it."""
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        for p in self._opened:
            lib.ridge_ipc_close(p)
        self._opened = []
        dist.barrier(group=group)
        if self._base:
            lib.ridge_device_free(self._base)
            self._base = None


def sharded_gemm_p2p(a, b_slab, config: TileConfig, peer_c: PeerC, group=None, barrier=True,
                     stream=None):
    """This rank's slab GEMM with the gather fused into its epilogue: every
    tile lands in every rank's C (peer_c) directly. With barrier=True the call
    is fenced by one-element all-reduces on `stream`: before the kernel (no
    rank writes into a peer's C until every rank has reached the call, so
    whatever a rank enqueued on `stream` earlier -- reading its previous C --
    is done) and after it (this rank's C then holds every rank's slab). A rank
    that reads its C on the host or on another stream must finish before its
    next call."""
    M, K = a.shape
    N = peer_c.N
    cc = config.to_c()
    comm = nccl_comm_ptr(group) if barrier and peer_c.world > 1 else None
    ns = b_slab.shape[0]
    st = lib.ridge_gemm_sharded_p2p(C.byref(cc), a.data_ptr(),
                                    b_slab.data_ptr() if ns else a.data_ptr(), M, N, K,
                                    max(a.stride(0), 1), max(b_slab.stride(0), 1) if ns else K,
                                    peer_c.world, peer_c.rank, peer_c.ptrs, peer_c.ldc, comm,
                                    _stream_handle(stream))
    check(st, "ridge_gemm_sharded_p2p %dx%dx%d rank %d/%d" % (M, N, K, peer_c.rank, peer_c.world))
    return peer_c.local


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
    ap.add_argument("--fused", action="store_true",
                    help="also time the GEMM with the gather fused into its epilogue (P2P)")
    ap.add_argument("--timeout", type=float, default=120.0,
                    help="seconds before a stuck collective is aborted")
    a = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        # a rank that never arrives ends the others' collectives with an error
        # after the deadline instead of hanging them
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=a.timeout))
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
    gather_ms = step_ms = None
    if a.gather and world > 1:
        # the whole step through the C ABI: slab GEMM + NCCL all-gather + re-layout
        B.full_n = N

        def step():
            sharded_gemm(A, B, cfg, gather=True, rank=rank, world=world)

        for _ in range(2):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        e0.record()
        for _ in range(a.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        g = torch.tensor([e0.elapsed_time(e1) / a.steps], dtype=torch.float64, device=dev)
        dist.all_reduce(g, op=dist.ReduceOp.MAX)
        step_ms = float(g.item())
        gather_ms = step_ms - float(t.item())
    fused_ms = None
    if a.fused and world > 1:
        pc = PeerC(M, N)
        Bv = B  # this rank's slab rows

        def fstep():
            sharded_gemm_p2p(A, Bv, cfg, pc)

        for _ in range(2):
            fstep()
        torch.cuda.synchronize()
        dist.barrier()
        e0.record()
        for _ in range(a.steps):
            fstep()
        e1.record()
        torch.cuda.synchronize()
        g = torch.tensor([e0.elapsed_time(e1) / a.steps], dtype=torch.float64, device=dev)
        dist.all_reduce(g, op=dist.ReduceOp.MAX)
        fused_ms = float(g.item())
        pc.close()
    if rank == 0:
        tflops = 2.0 * M * N * K / (float(t.item()) * 1e-3) / 1e12
        print(json.dumps({"workload": "%dx%dx%d N-slab over %d GPU(s)" % (M, N, K, world),
                          "config": cfg.tag(), "ms_per_gemm_max_over_ranks": float(t.item()),
                          "tflops_whole_node": tflops, "ms_gemm_plus_gather": step_ms,
                          "gather_ms": gather_ms, "ms_gemm_fused_gather": fused_ms,
                          "tflops_fused_with_gather": (2.0 * M * N * K / (fused_ms * 1e-3) / 1e12
                                                       if fused_ms else None)}))
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
