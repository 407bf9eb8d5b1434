"""Python face of the GEMM family: tile configs, the variant table, and the
launcher on torch CUDA tensors.

Mirrors the reference's kernel interface (bench/kernels/gemm-mma.cuh:368-387):
`variants()` is the KernelVariant table, `launch(config, A, B, C, ...)` is
KernelVariant::launch, and errors surface as RidgeError carrying the status
instead of a cudaError_t return value.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import asdict, dataclass

from ._native import (RIDGE_OK, TileConfigC, VariantInfoC, check, lib)


@dataclass(frozen=True)
class TileConfig:
    """One tile configuration (include/ridge_b200.h: ridge_tile_config)."""

    BM: int = 128
    BN: int = 256
    BK: int = 64
    stages: int = 4
    warps: int = 4
    groupM: int = 8
    cta_group: int = 0  # 0 = library default for this BM
    split_k: int = 0    # 0 = automatic split-K tail, 1 = never split

    def to_c(self) -> TileConfigC:
        return TileConfigC(self.BM, self.BN, self.BK, self.stages, self.warps, self.groupM,
                           self.cta_group, self.split_k)

    @staticmethod
    def from_c(c: TileConfigC) -> "TileConfig":
        return TileConfig(c.BM, c.BN, c.BK, c.stages, c.warps, c.groupM, c.cta_group, c.split_k)

    def tag(self) -> str:
        return "%dx%dx%d_s%d_w%d_g%d_c%d%s" % (self.BM, self.BN, self.BK, self.stages, self.warps,
                                               self.groupM, self.cta_group,
                                               "_nosplit" if self.split_k == 1 else "")

    def as_dict(self):
        return asdict(self)


@dataclass(frozen=True)
class VariantInfo:
    config: TileConfig
    smem_bytes: int
    threads: int
    regs_per_thread: int
    cluster_size: int
    tmem_cols: int
    acc_buffers: int
    kernel_name: str


def _info(v: VariantInfoC) -> VariantInfo:
    return VariantInfo(TileConfig.from_c(v.cfg), v.smem_bytes, v.threads, v.regs_per_thread,
                       v.cluster_size, v.tmem_cols, v.acc_buffers, v.kernel_name.decode())


DEFAULT_CONFIG = TileConfig()


def num_variants() -> int:
    return lib.ridge_num_variants()


def variant(i: int) -> VariantInfo:
    v = VariantInfoC()
    check(lib.ridge_variant(i, C.byref(v)), "variant %d" % i)
    return _info(v)


def variants() -> list[VariantInfo]:
    return [variant(i) for i in range(num_variants())]


def config_info(cfg: TileConfig) -> VariantInfo:
    v = VariantInfoC()
    c = cfg.to_c()
    check(lib.ridge_config_check(C.byref(c), C.byref(v)), "config %s" % cfg.tag())
    return _info(v)


def config_ok(cfg: TileConfig) -> bool:
    c = cfg.to_c()
    return lib.ridge_config_check(C.byref(c), None) == RIDGE_OK


def valid_for_shape(cfg: TileConfig, M: int, N: int, K: int, lda=None, ldb=None, ldc=None) -> bool:
    c = cfg.to_c()
    return lib.ridge_config_valid_for_shape(C.byref(c), M, N, K, K if lda is None else lda,
                                            K if ldb is None else ldb,
                                            N if ldc is None else ldc) == RIDGE_OK


def launch_raw(cfg: TileConfig, a_ptr: int, b_ptr: int, c_ptr: int, M: int, N: int, K: int,
               lda: int, ldb: int, ldc: int, stream: int = 0) -> int:
    """Launches on raw device pointers; returns the status (no raise)."""
    c = cfg.to_c()
    return lib.ridge_gemm_launch(C.byref(c), a_ptr, b_ptr, c_ptr, M, N, K, lda, ldb, ldc,
                                 stream or None)


def _stream_handle(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def gemm(a, b, out=None, config: TileConfig | None = None, stream=None):
    """C = A @ B for torch tensors: a (M, K) fp16, b (N, K) fp16 (i.e. B is
    column-major K x N), returns / fills out (M, N) fp16. Inner dimensions must
    be contiguous (stride 1). Asynchronous on `stream` (default: torch's
    current stream)."""
    import torch
    if a.dtype != torch.float16 or b.dtype != torch.float16:
        raise TypeError("ridge_b200.gemm takes float16 operands")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError("expected a (M, K) and b (N, K), got %s and %s" % (tuple(a.shape),
                                                                         tuple(b.shape)))
    if not (a.is_cuda and b.is_cuda):
        raise ValueError("ridge_b200.gemm operates on CUDA tensors")
    M, K = a.shape
    N = b.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=a.device)
    if a.stride(1) != 1 or b.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("inner dimensions must be contiguous")
    cfg = config or DEFAULT_CONFIG
    st = launch_raw(cfg, a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K,
                    max(a.stride(0), 1), max(b.stride(0), 1), max(out.stride(0), 1),
                    _stream_handle(stream))
    check(st, "ridge_gemm_launch %dx%dx%d %s" % (M, N, K, cfg.tag()))
    return out


def gemm_host(a, b, out=None, config: TileConfig | None = None, panels: int = 0, stream=None,
              device=None):
    """C = A @ B for HOST tensors (a (M, K), b (N, K), fp16, CPU; page-locked
    for copy/compute overlap): ridge_gemm_host pipelines the copies in, the
    kernel and the copy of C out by M-panels on `device` (default: torch's
    current device). Asynchronous on `stream`: synchronise before reading out."""
    import torch
    if a.dtype != torch.float16 or b.dtype != torch.float16:
        raise TypeError("ridge_b200.gemm_host takes float16 operands")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError("expected a (M, K) and b (N, K), got %s and %s" % (tuple(a.shape),
                                                                         tuple(b.shape)))
    if a.is_cuda or b.is_cuda or (out is not None and out.is_cuda):
        raise ValueError("ridge_b200.gemm_host takes host (CPU) tensors; use gemm on CUDA ones")
    M, K = a.shape
    N = b.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, pin_memory=a.is_pinned())
    if a.stride(1) != 1 or b.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("inner dimensions must be contiguous")
    cfg = config or DEFAULT_CONFIG
    c = cfg.to_c()
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        st = lib.ridge_gemm_host(C.byref(c), a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K,
                                 max(a.stride(0), K, 1), max(b.stride(0), K, 1),
                                 max(out.stride(0), N, 1), panels, _stream_handle(stream))
    check(st, "ridge_gemm_host %dx%dx%d %s" % (M, N, K, cfg.tag()))
    return out


def device_error(clear: bool = True) -> int:
    """Synchronises the current device and returns its kernel error word
    (0 = no bounded wait expired)."""
    code = C.c_int32(0)
    check(lib.ridge_device_error(1 if clear else 0, C.byref(code)), "ridge_device_error")
    return code.value


def fill_lcg(out, seed_state: int = 0, unit: bool = True, stream=None) -> int:
    """Fills the fp16 CUDA tensor `out` (contiguous) with the reference's LCG
    sequence starting from `seed_state`; returns the state after the fill so a
    second call continues the stream (A then B)."""
    import torch
    if out.dtype != torch.float16 or not out.is_contiguous() or not out.is_cuda:
        raise ValueError("fill_lcg needs a contiguous float16 CUDA tensor")
    st = C.c_uint32(seed_state)
    check(lib.ridge_fill_lcg(out.data_ptr(), out.numel(), C.byref(st), 1 if unit else 0,
                             _stream_handle(stream)), "ridge_fill_lcg")
    return st.value


def lcg_advance(state: int, n: int) -> int:
    """The LCG state after n more draws from `state` (s -> 1664525 s +
    1013904223 mod 2^32, applied n times by repeated squaring of the affine
    map), so a rank can start its slab of B without drawing the rows before it."""
    a, c = 1664525, 1013904223
    ra, rc = 1, 0                      # the identity map
    while n > 0:
        if n & 1:
            ra, rc = (a * ra) & 0xFFFFFFFF, (a * rc + c) & 0xFFFFFFFF
        a, c = (a * a) & 0xFFFFFFFF, (a * c + c) & 0xFFFFFFFF
        n >>= 1
    return (ra * state + rc) & 0xFFFFFFFF


def synthetic_inputs(M: int, N: int, K: int, seed: int = 0, device=None):
    """The benchmark operands: A (M, K) then B (N, K) drawn U(-1, 1) from one
    LCG stream seeded `seed` (B is the N x K storage of a column-major B)."""
    import torch
    a = torch.empty((M, K), dtype=torch.float16, device=device or "cuda")
    b = torch.empty((N, K), dtype=torch.float16, device=device or "cuda")
    st = fill_lcg(a, seed)
    fill_lcg(b, st)
    return a, b
