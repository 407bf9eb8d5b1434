"""CPU oracle for the ridge GEMM hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py (its CPU baseline and its
reference arm) may import this package; it is the checker, never the thing
measured or shipped. Two libraries back it:

  * libridge_oracle.so -- this repo's plain-C restatement (ridge_oracle.c) of
    the reference's fill, FP64 host GEMM and error statistics
    (bench/check-gemm.cu:98-145 in the reference).
  * _ref/libridge_ref.so -- the reference's own code compiled from its sources
    by oracle/Makefile (optional: present only where the reference was
    available at build time, and shipped with the tree to GPU boxes).
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libridge_oracle.so"
REF_PATH = HERE / "_ref" / "libridge_ref.so"

_vp = C.c_void_p
_i64 = C.c_int64


def build(reference: str | None = None) -> None:
    """Builds libridge_oracle.so, and _ref/libridge_ref.so when the reference
    sources are found at `reference` or, if that is not given, at the path in
    the RIDGE_REFERENCE environment variable (no default location)."""
    targets = ["liboracle"]
    ref = reference or os.environ.get("RIDGE_REFERENCE", "")
    if ref and Path(ref, "bench", "check-gemm.cu").exists():
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", str(HERE)] + (["REF=%s" % ref] if ref else []) + targets,
                   check=True)


def _load():
    if not LIB_PATH.exists():
        build()
    lib = C.CDLL(str(LIB_PATH))
    lib.oracle_f32_to_f16.restype = C.c_uint16
    lib.oracle_f32_to_f16.argtypes = [C.c_float]
    lib.oracle_f16_to_f32.restype = C.c_float
    lib.oracle_f16_to_f32.argtypes = [C.c_uint16]
    lib.oracle_fill_reference.argtypes = [_vp, C.c_size_t, C.c_uint32]
    lib.oracle_fill_unit.argtypes = [_vp, C.c_size_t, C.POINTER(C.c_uint32)]
    lib.oracle_gemm_f64_rows.argtypes = [_vp, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64,
                                         _i64]
    lib.oracle_gemm_f64_fast.argtypes = [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp,
                                         _i64, _vp]
    lib.oracle_error_stats.argtypes = [_vp, _vp, C.c_size_t, C.POINTER(C.c_double),
                                       C.POINTER(C.c_double)]
    lib.oracle_fp16_stats.argtypes = [_vp, _i64, _vp, _i64, _i64, _i64, C.POINTER(C.c_double),
                                      C.POINTER(C.c_double), C.POINTER(C.c_double)]
    for n in ("oracle_f32_to_f16_array", "oracle_f16_to_f32_array", "oracle_f64_to_f16_array"):
        getattr(lib, n).argtypes = [_vp, _vp, C.c_size_t]
    return lib


lib = _load()


def _p(a: np.ndarray):
    return a.ctypes.data_as(_vp)


# ---------------------------------------------------------------- fills

def fill_reference(n: int, seed: int) -> np.ndarray:
    """check-gemm.cu:139-145 fill: n FP16 values (as uint16 bits) in U(-0.5, 0.5)."""
    out = np.empty(n, np.uint16)
    lib.oracle_fill_reference(_p(out), n, seed)
    return out


def unit_inputs(M: int, N: int, K: int, seed: int = 0):
    """The benchmark inputs: A (M x K) then B (N x K storage of a column-major
    K x N B) from one LCG stream seeded `seed`, values U(-1, 1), FP16 bits."""
    st = C.c_uint32(seed)
    a = np.empty(M * K, np.uint16)
    lib.oracle_fill_unit(_p(a), a.size, C.byref(st))
    b = np.empty(N * K, np.uint16)
    lib.oracle_fill_unit(_p(b), b.size, C.byref(st))
    return a.reshape(M, K), b.reshape(N, K)


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    lib.oracle_f16_to_f32_array(_p(h), _p(out), h.size)
    return out


def f32_to_f16(f: np.ndarray) -> np.ndarray:
    f = np.ascontiguousarray(f, np.float32)
    out = np.empty(f.shape, np.uint16)
    lib.oracle_f32_to_f16_array(_p(f), _p(out), f.size)
    return out


# ---------------------------------------------------------------- GEMM

def gemm_f64_reference_loop(a: np.ndarray, b_kn: np.ndarray) -> np.ndarray:
    """The reference's loop order exactly (check-gemm.cu:98-108): a (M, K),
    b_kn row-major (K, N). Slow; small shapes only."""
    a = np.ascontiguousarray(a, np.uint16)
    b_kn = np.ascontiguousarray(b_kn, np.uint16)
    M, K = a.shape
    N = b_kn.shape[1]
    c = np.empty((M, N), np.float64)
    lib.oracle_gemm_f64_rows(_p(a), K, _p(b_kn), N, 1, _p(c), N, N, K, 0, M)
    return c


def gemm_f64(a: np.ndarray, b_nk: np.ndarray, rows=None) -> np.ndarray:
    """FP64 C = A * B for a (M, K) and b_nk the (N, K) storage of a column-major
    B; same products and summation order as the reference loop. `rows`
    restricts the output to those row indices (sampled check)."""
    a = np.ascontiguousarray(a, np.uint16)
    b_nk = np.ascontiguousarray(b_nk, np.uint16)
    M, K = a.shape
    N = b_nk.shape[0]
    scratch = np.empty(max(N * K, 1), np.float64)
    if rows is None:
        c = np.empty((M, N), np.float64)
        lib.oracle_gemm_f64_fast(_p(a), K, _p(b_nk), K, _p(c), N, M, N, K, None, 0, _p(scratch))
    else:
        r = np.ascontiguousarray(rows, np.int64)
        c = np.empty((r.size, N), np.float64)
        lib.oracle_gemm_f64_fast(_p(a), K, _p(b_nk), K, _p(c), N, M, N, K, _p(r), r.size,
                                 _p(scratch))
    return c


# ---------------------------------------------------------------- checking

def error_stats(got: np.ndarray, ref: np.ndarray):
    """check-gemm.cu:121-135: (relative Frobenius, max|d| / max|ref|)."""
    g = np.ascontiguousarray(got, np.float32).ravel()
    r = np.ascontiguousarray(ref, np.float64).ravel()
    fr, mr = C.c_double(), C.c_double()
    lib.oracle_error_stats(_p(g), _p(r), g.size, C.byref(fr), C.byref(mr))
    return fr.value, mr.value


def fp16_stats(got_f16: np.ndarray, ref: np.ndarray):
    """(relative Frobenius, max |dC|, max(|dC| - half FP16 ulp of ref)) for an
    FP16 result against an FP64 reference."""
    g = np.ascontiguousarray(got_f16, np.uint16)
    r = np.ascontiguousarray(ref, np.float64)
    M, N = r.shape
    a, b, c = C.c_double(), C.c_double(), C.c_double()
    lib.oracle_fp16_stats(_p(g), N, _p(r), N, M, N, C.byref(a), C.byref(b), C.byref(c))
    return a.value, b.value, c.value


# Acceptance thresholds for the FP16-output GEMM against the FP64 oracle, on
# U(-1,1) inputs: relative Frobenius error of C at most 1e-3, and the largest
# elementwise |dC| at most 2e-2 beyond the half-ulp rounding of the FP16 output
# itself (|C| exceeds 64 for large K, where one FP16 half-ulp alone is 0.031).
REL_FROB_TOL = 1e-3
MAX_ABS_EXCESS_TOL = 2e-2


# ---------------------------------------------------------------- reference library

class Reference:
    """The reference's own code (oracle/_ref/libridge_ref.so)."""

    def __init__(self, path: Path = REF_PATH):
        if not path.exists():
            raise FileNotFoundError("reference parity library %s not built" % path)
        L = C.CDLL(str(path))
        L.ref_fill.argtypes = [_vp, C.c_size_t, C.c_uint]
        L.ref_gemm_f64.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int]
        L.ref_error_stats.argtypes = [_vp, _vp, C.c_size_t, C.POINTER(C.c_double),
                                      C.POINTER(C.c_double)]
        L.ref_num_variants.restype = C.c_int
        L.ref_variant_info.argtypes = [C.c_int, _vp]
        L.ref_launch_variant.argtypes = [C.c_int, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp]
        L.ref_launch_variant.restype = C.c_int
        L.ref_predict_a100.argtypes = [C.POINTER(C.c_longlong), C.c_char_p, _vp]
        L.ref_predict_a100.restype = C.c_int
        self.lib = L

    def fill(self, n: int, seed: int) -> np.ndarray:
        out = np.empty(n, np.uint16)
        self.lib.ref_fill(_p(out), n, seed)
        return out

    def gemm_f64(self, a: np.ndarray, b_kn: np.ndarray, threads: int = 1) -> np.ndarray:
        a = np.ascontiguousarray(a, np.uint16)
        b_kn = np.ascontiguousarray(b_kn, np.uint16)
        M, K = a.shape
        N = b_kn.shape[1]
        c = np.empty((M, N), np.float64)
        self.lib.ref_gemm_f64(_p(a), _p(b_kn), _p(c), M, N, K, threads)
        return c

    def error_stats(self, got, ref):
        g = np.ascontiguousarray(got, np.float32).ravel()
        r = np.ascontiguousarray(ref, np.float64).ravel()
        fr, mr = C.c_double(), C.c_double()
        self.lib.ref_error_stats(_p(g), _p(r), g.size, C.byref(fr), C.byref(mr))
        return fr.value, mr.value

    def variants(self):
        out = []
        for i in range(self.lib.ref_num_variants()):
            v = np.zeros(10, np.int32)
            self.lib.ref_variant_info(i, _p(v))
            out.append(dict(zip(["BM", "BN", "BK", "WM", "WN", "stages", "groupM", "smemBytes",
                                 "threads", "regsPerThread"], map(int, v))))
        return out

    def launch(self, i, a_ptr, b_ptr, c_ptr, M, N, K, stream=0) -> int:
        return self.lib.ref_launch_variant(i, a_ptr, b_ptr, c_ptr, M, N, K, stream or None)

    def predict_a100(self, M, N, K, BM, BN, BK, WM, WN, stages, regs, hw_json: str = ""):
        cfg = (C.c_longlong * 10)(M, N, K, BM, BN, BK, WM, WN, stages, regs)
        out = np.zeros(24, np.float64)
        if self.lib.ref_predict_a100(cfg, hw_json.encode(), _p(out)) != 0:
            raise RuntimeError("reference model refused " + hw_json)
        keys = ["predictedTFLOPS", "bottleneck", "computeTFLOPS", "hbmTFLOPS", "peakTensorTFLOPS",
                "smEfficiency", "occFactor", "arithmeticIntensity", "baseIntensity",
                "l2ReuseFactor", "waveEfficiency", "totalCtas", "ctaSlots", "wavesExact",
                "envelopeEfficiency", "tPrologueCycles", "tEpilogueCycles", "tBodyCycles",
                "kSteps", "numWarps", "ctasPerSM", "tComputeCycles", "tSmemCycles",
                "tStepCycles"]
        return dict(zip(keys, out.tolist()))


def reference_available() -> bool:
    return REF_PATH.exists()
