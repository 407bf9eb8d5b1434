"""ctypes binding of libridge_b200.so (the C ABI in include/ridge_b200.h).

The library is loaded from ridge_b200/lib/. There is no fallback: if the
native library is missing, importing ridge_b200 raises ImportError telling the
user to build it (python ridge_b200/build.py).
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libridge_b200.so"

RIDGE_OK = 0
RIDGE_EINVAL = -1
RIDGE_EDEVICE = -2
RIDGE_ENOTSUP = -3
RIDGE_EIO = -4
RIDGE_ERANGE = -5
RIDGE_ENOSCRATCH = -6
RIDGE_ECOMM = -7

BOTTLENECKS = ["TENSOR_CORE", "SMEM", "HBM", "OCC", "WAVES", "ENVELOPE", "DOES_NOT_FIT",
               "EPILOGUE", "L2"]


class TileConfigC(C.Structure):
    _fields_ = [("BM", C.c_int32), ("BN", C.c_int32), ("BK", C.c_int32), ("stages", C.c_int32),
                ("warps", C.c_int32), ("groupM", C.c_int32), ("cta_group", C.c_int32),
                ("split_k", C.c_int32)]


class VariantInfoC(C.Structure):
    _fields_ = [("cfg", TileConfigC), ("smem_bytes", C.c_int32), ("threads", C.c_int32),
                ("regs_per_thread", C.c_int32), ("cluster_size", C.c_int32),
                ("tmem_cols", C.c_int32), ("acc_buffers", C.c_int32),
                ("kernel_name", C.c_char * 96)]


class HwC(C.Structure):
    _fields_ = [("name", C.c_char * 64), ("num_sms", C.c_int32), ("clock_hz", C.c_double),
                ("umma_cycles_128x256", C.c_double), ("umma_m64_ratio", C.c_double),
                ("smem_bytes_per_cycle", C.c_double), ("smem_mma_overlap", C.c_double),
                ("l2_bytes_per_sec", C.c_double), ("hbm_bytes_per_sec", C.c_double),
                ("tma_box_cycles", C.c_double), ("tma_box2_ratio", C.c_double),
                ("tma_box32_ratio", C.c_double),
                ("pipeline_efficiency", C.c_double),
                ("tile_overhead_cycles", C.c_double), ("pair_tile_overhead_cycles", C.c_double),
                ("c_write_bytes_per_sec", C.c_double),
                ("epi_bytes_per_cycle_w4", C.c_double), ("epi_bytes_per_cycle_w8", C.c_double),
                ("tma_latency_cycles", C.c_double),
                ("tma_latency_hbm_cycles", C.c_double), ("launch_overhead_sec", C.c_double),
                ("l2_bytes", C.c_double), ("smem_bytes_per_sm", C.c_int32),
                ("tmem_cols_per_sm", C.c_int32), ("max_ctas_per_sm", C.c_int32),
                ("calibrated", C.c_int32)]


class GemmConfigC(C.Structure):
    _fields_ = [("M", C.c_int64), ("N", C.c_int64), ("K", C.c_int64), ("tile", TileConfigC)]


PREDICTION_FIELDS = [
    "predicted_tflops", "bottleneck", "compute_tflops", "hbm_tflops", "peak_tensor_tflops",
    "smem_efficiency", "l2_efficiency", "occ_factor", "wave_efficiency", "envelope_efficiency",
    "epilogue_efficiency", "arithmetic_intensity", "dram_bytes", "total_tiles", "tile_slots",
    "waves_exact", "k_blocks", "t_mma_cycles", "t_smem_cycles", "t_l2_cycles", "t_step_cycles",
    "t_period_cycles", "t_epilogue_cycles", "t_tile_cycles", "t_prologue_cycles",
    "predicted_seconds", "ctas_per_sm", "acc_buffers"]
_INT_PRED = {"bottleneck", "ctas_per_sm", "acc_buffers"}


class PredictionC(C.Structure):
    _fields_ = [(n, C.c_int32 if n in _INT_PRED else C.c_double) for n in PREDICTION_FIELDS]


class TuneEntryC(C.Structure):
    _fields_ = [("tile", TileConfigC), ("predicted_tflops", C.c_double),
                ("measured_tflops", C.c_double), ("device", C.c_int32), ("status", C.c_int32)]


class TuneResultC(C.Structure):
    _fields_ = [("M", C.c_int64), ("N", C.c_int64), ("K", C.c_int64), ("best", TileConfigC),
                ("best_tflops", C.c_double), ("benchmarked", C.c_int32),
                ("candidates", C.c_int32)]


# Every symbol the header declares, with its ctypes signature. The CPU test
# suite checks that the built library exports each of these.
_i64 = C.c_int64
_i32 = C.c_int32
_vp = C.c_void_p
SIGNATURES = {
    "ridge_status_string": (C.c_char_p, [C.c_int]),
    "ridge_num_variants": (C.c_int, []),
    "ridge_variant": (C.c_int, [C.c_int, C.POINTER(VariantInfoC)]),
    "ridge_print_variant_table": (None, []),
    "ridge_config_check": (C.c_int, [C.POINTER(TileConfigC), C.POINTER(VariantInfoC)]),
    "ridge_config_valid_for_shape": (C.c_int, [C.POINTER(TileConfigC), _i64, _i64, _i64, _i64,
                                              _i64, _i64]),
    "ridge_gemm_launch": (C.c_int, [C.POINTER(TileConfigC), _vp, _vp, _vp, _i64, _i64, _i64,
                                    _i64, _i64, _i64, _vp]),
    "ridge_gemm_workspace_size": (C.c_int, [C.POINTER(TileConfigC), _i64, _i64, _i64,
                                            C.POINTER(_i64)]),
    "ridge_gemm_launch_ws": (C.c_int, [C.POINTER(TileConfigC), _vp, _vp, _vp, _i64, _i64, _i64,
                                       _i64, _i64, _i64, _vp, _i64, _vp]),
    "ridge_gemm_launch_noalloc": (C.c_int, [C.POINTER(TileConfigC), _vp, _vp, _vp, _i64, _i64,
                                            _i64, _i64, _i64, _i64, _vp]),
    "ridge_gemm_noalloc_scratch_bytes": (_i64, []),
    "ridge_gemm_sharded": (C.c_int, [C.POINTER(TileConfigC), _vp, _vp, _vp, _i64, _i64, _i64,
                                     _i64, _i64, C.c_int32, C.c_int32, C.c_int32, _vp, _vp, _vp,
                                     _i64, _vp]),
    "ridge_selftest_wait_timeout": (C.c_int, [_i64, C.POINTER(C.c_int32), C.POINTER(_i64)]),
    "ridge_selftest_stale_counters": (C.c_int, [C.c_int32]),
    "ridge_gemm_launch_multi": (C.c_int, [C.POINTER(TileConfigC), _vp, _vp, _vp, _i64, _i64, _i64,
                                          _i64, _i64, _i64, C.POINTER(_vp), C.c_int32, _vp]),
    "ridge_gemm_sharded_p2p": (C.c_int, [C.POINTER(TileConfigC), _vp, _vp, _i64, _i64, _i64, _i64,
                                         _i64, C.c_int32, C.c_int32, C.POINTER(_vp), _i64, _vp,
                                         _vp]),
    "ridge_ipc_handle_bytes": (_i64, []),
    "ridge_device_alloc": (C.c_int, [_i64, C.POINTER(_vp)]),
    "ridge_device_free": (C.c_int, [_vp]),
    "ridge_ipc_export": (C.c_int, [_vp, _vp]),
    "ridge_ipc_open": (C.c_int, [_vp, C.POINTER(_vp)]),
    "ridge_ipc_close": (C.c_int, [_vp]),
    "ridge_gemm_host": (C.c_int, [C.POINTER(TileConfigC), _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                  _i64, _i64, C.c_int32, _vp]),
    "ridge_gemm_launch_variant": (C.c_int, [C.c_int, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                            _i64, _i64, _vp]),
    "ridge_device_error": (C.c_int, [C.c_int, C.POINTER(_i32)]),
    "ridge_fill_lcg": (C.c_int, [_vp, _i64, C.POINTER(C.c_uint32), _i32, _vp]),
    "ridge_bottleneck_string": (C.c_char_p, [_i32]),
    "ridge_hw_b200": (C.c_int, [C.POINTER(HwC)]),
    "ridge_hw_load_json": (C.c_int, [C.c_char_p, C.POINTER(HwC), C.c_char_p, _i32]),
    "ridge_predict": (C.c_int, [C.POINTER(GemmConfigC), C.POINTER(HwC), C.POINTER(PredictionC)]),
    "ridge_autotune": (C.c_int, [C.POINTER(_i64), _i32, _i32, C.POINTER(_i32), _i32,
                                 C.POINTER(HwC), _i32, _i32, C.POINTER(TuneResultC),
                                 C.POINTER(TuneEntryC), _i32]),
    "ridge_farm_selftest": (C.c_int, [_i32, _i32, _i32, _i32, _i32, C.POINTER(_i32),
                                      C.POINTER(_i32)]),
    "ridge_time_gemm": (C.c_int, [C.POINTER(TileConfigC), _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                  _i64, _i64, _i32, _i32, _vp, C.POINTER(C.c_double)]),
    "ridge_time_gemm_cold": (C.c_int, [C.POINTER(TileConfigC), _vp, _vp, _vp, _i64, _i64, _i64,
                                       _i64, _i64, _i64, _vp, _i64, _i32, _i32, _vp,
                                       C.POINTER(C.c_double)]),
    "ridge_cal_umma": (C.c_int, [_i32, _i32, _i32, C.POINTER(C.c_double),
                                 C.POINTER(C.c_double)]),
    "ridge_cal_tma": (C.c_int, [_i64, _i32, _i32, _i32, _i32, _i32, _i32, C.POINTER(C.c_double),
                                C.POINTER(C.c_double)]),
    "ridge_cal_epi": (C.c_int, [_i32, _i64, _i32, C.POINTER(C.c_double),
                                C.POINTER(C.c_double)]),
    "ridge_cal_write": (C.c_int, [_i64, C.POINTER(C.c_double)]),
    "ridge_cal_copy": (C.c_int, [_i64, C.POINTER(C.c_double)]),
    "ridge_cal_launch": (C.c_int, [C.POINTER(C.c_double)]),
    "ridge_cal_clock": (C.c_int, [C.POINTER(C.c_double)]),
    "ridge_slab_bounds": (C.c_int, [_i64, _i32, _i32, _i64, C.POINTER(_i64), C.POINTER(_i64)]),
    "ridge_slabs_to_rowmajor": (C.c_int, [_vp, _vp, _i64, _i64, _i32, _i64, _i64, _vp]),
}


def _load():
    if not LIB_PATH.exists():
        raise ImportError(
            "ridge_b200: native library %s is missing; build it with "
            "`python ridge_b200/build.py` (there is no non-native fallback)" % LIB_PATH)
    lib = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | getattr(os, "RTLD_GLOBAL", 0))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue  # reported by exported_symbols(); calling it raises AttributeError
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def exported_symbols():
    """Names from SIGNATURES that the loaded library actually exports."""
    return [n for n in SIGNATURES if hasattr(lib, n)]


class RidgeError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = lib.ridge_status_string(status).decode()
        super().__init__("%s%s (status %d)" % (what + ": " if what else "", msg, status))


def check(status: int, what: str = "") -> None:
    if status != RIDGE_OK:
        raise RidgeError(status, what)
