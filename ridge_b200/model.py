"""The B200 cost model from Python: hardware constants and ridge_predict.

Mirrors the reference's model interface (include/ridge/model.h:10,
hardware.h:9-54): `predict(M, N, K, config, hw)` returns a Prediction with the
throughput, the bottleneck label and the terms that explain it; `b200()` is
the built-in placeholder model and `load_hw(path)` the all-or-nothing loader
for a calibration JSON.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

from ._native import (BOTTLENECKS, PREDICTION_FIELDS, GemmConfigC, HwC, PredictionC, check, lib)
from .gemm import TileConfig

DATA = Path(__file__).resolve().parent.parent / "data" / "hardware"
DEFAULT_HW_JSON = DATA / "b200.json"

HW_KEYS = {  # JSON key -> struct field
    "numSMs": "num_sms", "clockHz": "clock_hz", "ummaCycles128x256": "umma_cycles_128x256",
    "ummaM64Ratio": "umma_m64_ratio", "smemBytesPerCycle": "smem_bytes_per_cycle",
    "smemMmaOverlap": "smem_mma_overlap", "l2BytesPerSec": "l2_bytes_per_sec",
    "hbmBytesPerSec": "hbm_bytes_per_sec", "tmaBoxCycles": "tma_box_cycles",
    "tmaBoxCycles128Ratio": "tma_box2_ratio", "tmaBoxCycles32Ratio": "tma_box32_ratio",
    "pipelineEfficiency": "pipeline_efficiency",
    "tileOverheadCycles": "tile_overhead_cycles",
    "pairTileOverheadCycles": "pair_tile_overhead_cycles",
    "cWriteBytesPerSec": "c_write_bytes_per_sec", "epiBytesPerCycleW4": "epi_bytes_per_cycle_w4",
    "epiBytesPerCycleW8": "epi_bytes_per_cycle_w8", "tmaLatencyCycles": "tma_latency_cycles",
    "tmaLatencyHbmCycles": "tma_latency_hbm_cycles",
    "launchOverheadSec": "launch_overhead_sec", "l2Bytes": "l2_bytes",
    "smemBytesPerSM": "smem_bytes_per_sm", "tmemColsPerSM": "tmem_cols_per_sm",
    "maxCtasPerSM": "max_ctas_per_sm",
}


def b200() -> HwC:
    hw = HwC()
    check(lib.ridge_hw_b200(C.byref(hw)), "ridge_hw_b200")
    return hw


def load_hw(path) -> HwC:
    hw = HwC()
    err = C.create_string_buffer(512)
    check(lib.ridge_hw_load_json(str(path).encode(), C.byref(hw), err, 512),
          "ridge_hw_load_json: " + err.value.decode())
    return hw


def default_hw() -> HwC:
    """The committed calibration (data/hardware/b200.json) if present, else
    the placeholders."""
    return load_hw(DEFAULT_HW_JSON) if DEFAULT_HW_JSON.exists() else b200()


def hw_to_dict(hw: HwC) -> dict:
    d = {"name": hw.name.decode()}
    for k, f in HW_KEYS.items():
        d[k] = getattr(hw, f)
    return d


class Prediction(dict):
    """dict of every ridge_prediction field, plus .label."""

    @property
    def label(self) -> str:
        b = int(self["bottleneck"])
        return BOTTLENECKS[b] if 0 <= b < len(BOTTLENECKS) else "UNKNOWN"


def predict(M: int, N: int, K: int, config: TileConfig, hw: HwC | None = None) -> Prediction:
    hw = hw if hw is not None else default_hw()
    g = GemmConfigC(M, N, K, config.to_c())
    p = PredictionC()
    check(lib.ridge_predict(C.byref(g), C.byref(hw), C.byref(p)), "ridge_predict")
    return Prediction({f: getattr(p, f) for f in PREDICTION_FIELDS})


def bottleneck_name(code: int) -> str:
    return lib.ridge_bottleneck_string(code).decode()
