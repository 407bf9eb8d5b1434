"""ridge_b200 -- B200-native (sm_100a) rebuild of ridge's FP16 tensor-core GEMM
hot path: the tcgen05/TMA GEMM family behind ridge's tile-config interface,
its Blackwell cost model, and the model-pruned autotuner.

The compute path is the native library libridge_b200.so (CUDA kernels + C ABI,
include/ridge_b200.h); this package is a thin host-side mirror of the
reference's interfaces on top of it. Importing it without the built library
raises ImportError -- there is no CPU fallback.
"""

from ._native import RidgeError, exported_symbols, lib  # noqa: F401
from .gemm import (DEFAULT_CONFIG, TileConfig, VariantInfo, config_info, config_ok,  # noqa: F401
                   device_error, fill_lcg, gemm, gemm_host, launch_raw, lcg_advance, synthetic_inputs, num_variants, valid_for_shape, variant,
                   variants)

__all__ = [
    "RidgeError", "TileConfig", "VariantInfo", "DEFAULT_CONFIG", "gemm", "gemm_host", "launch_raw",
    "variants", "variant", "num_variants", "config_info", "config_ok", "valid_for_shape",
    "device_error", "exported_symbols", "lib", "fill_lcg", "lcg_advance", "synthetic_inputs",
]
