"""The calibration fit (ridge_b200.fit): recovers a constant that was perturbed
in synthetic 'measurements', never leaves its band, and the committed
calibration records where its fitted constants came from."""

import json

from ridge_b200 import TileConfig
from ridge_b200.autotune import REGISTERED, load_sweep
from ridge_b200.fit import ABS_BANDS, CAL_SWEEP, FIT_BANDS, MICRO, fit
from ridge_b200.model import DEFAULT_HW_JSON, HW_KEYS, load_hw, predict


def _rows(hw, shapes, configs):
    rows = []
    for (M, N, K) in shapes:
        for c in configs:
            rows.append({"M": M, "N": N, "K": K, "config": c,
                         "tflops": predict(M, N, K, c, hw)["predicted_tflops"]})
    return rows


def test_fit_recovers_a_perturbed_constant(tmp_path):
    base = {k: v for k, v in json.loads(DEFAULT_HW_JSON.read_text()).items()
            if k in HW_KEYS or k == "name"}
    truth = dict(base)
    truth["tmaBoxCycles"] = base["tmaBoxCycles"] * 1.3
    p = tmp_path / "truth.json"
    p.write_text(json.dumps(truth))
    configs = [TileConfig(128, 256, 64, 4, 4, 8, 1), TileConfig(256, 256, 64, 3, 4, 8, 2),
               TileConfig(128, 128, 32, 5, 4, 8, 1), TileConfig(64, 256, 128, 2, 8, 8, 1)]
    rows = _rows(load_hw(p), [(2048, 2048, 2048), (4096, 4096, 1024), (1024, 8192, 4096)], configs)
    fitted, obj = fit(rows, base, passes=3, steps=7, log=lambda *_: None)
    assert obj < 0.02
    assert abs(fitted["tmaBoxCycles"] / truth["tmaBoxCycles"] - 1.0) < 0.05
    for k, (lo, hi) in FIT_BANDS.items():
        assert lo * base[k] * (1 - 1e-9) <= fitted[k] <= hi * base[k] * (1 + 1e-9), k
    for k, (lo, hi) in ABS_BANDS.items():
        assert lo <= fitted[k] <= hi, k


def test_committed_fit_is_traceable_and_disjoint_from_validation():
    doc = json.loads(DEFAULT_HW_JSON.read_text())
    for k in list(FIT_BANDS) + list(ABS_BANDS):
        assert MICRO + k in doc, k
    assert doc["fitSource"] == "data/measured/b200-calibration.csv"
    cal = {s[:3] for s in load_sweep(CAL_SWEEP)}
    val = {s[:3] for s in load_sweep(REGISTERED)}
    assert cal and val and not (cal & val)
