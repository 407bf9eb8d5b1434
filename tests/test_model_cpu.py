"""The B200 cost model (ridge_predict) and its hardware loader, on CPU.

Like the reference's test/test-model.cpp, the worked example below is derived
by hand from the model's formulas on the built-in placeholder constants, value
by value; if a model change breaks it, re-derive the example, do not paste the
new output in."""

import ctypes as C
import json
import math

import pytest

import ridge_b200 as rb
from ridge_b200._native import HwC, lib
from ridge_b200.model import b200, load_hw, predict


def smax(a, b, p=4.0):
    m = max(a, b)
    return m * ((a / m) ** p + (b / m) ** p) ** (1 / p)


def test_worked_example_4096_cubed_256x256x64_one_cta():
    hw = b200()
    # placeholders: clock 1.4 GHz, 128 cycles per 128x256x16 MMA, smem 128 B/cycle
    # (reads overlap), TMA box 320 cycles, L2 fill cap 20 TB/s (96.53
    # B/cycle/SM at 1.4 GHz on 148 SMs), pipeline efficiency 0.9, TMA latency
    # 1000 cycles, epilogue 32 B/cycle (4 warps), HBM 6.5 TB/s read and write,
    # launch 4 us, no tile turnover cost.
    p = predict(4096, 4096, 4096, rb.TileConfig(256, 256, 64, 3, 4, 8, 1), hw)
    # One CTA holds 256 rows: 2 M-halves x BK/16 = 8 MMAs per stage, each
    # max(128 * 256/256, (128 + 256) * 32 / 128 = 96) = 128 cycles.
    assert p["t_mma_cycles"] == pytest.approx(1024.0)
    assert p["t_smem_cycles"] == pytest.approx(8 * 96.0)
    # fill: the one producer thread issues the stage's A box and B box, 2 x
    # 320 = 640 cycles; bytes term: a stage is (256 + 256) x 64 x 2 =
    # 65,536 B at 96.53 B/cycle = 678.9 cycles
    l2_bpc = 20e12 / 148 / 1.4e9
    t_fill = smax(640.0, 65536 / l2_bpc)
    assert 65536 / l2_bpc == pytest.approx(678.9, abs=0.1)
    assert p["t_l2_cycles"] == pytest.approx(t_fill, rel=1e-9)
    # 214,272 B of shared memory and all 512 TMEM columns: one CTA per SM,
    # one accumulator (no epilogue overlap).
    assert p["ctas_per_sm"] == 1 and p["acc_buffers"] == 1
    t_stage = smax(1024.0, t_fill) / 0.9
    assert p["t_step_cycles"] == pytest.approx(t_stage, rel=1e-9)
    # latency check: (1000 + t_fill + t_stage) / 3 stages < t_stage
    assert (1000 + t_fill + t_stage) / 3 < t_stage
    assert p["t_period_cycles"] == pytest.approx(t_stage, rel=1e-9)
    t_main = 64 * t_stage                                    # 64 K-blocks
    t_epi = 256 * 256 * 2 / 32.0                             # 4096 cycles
    assert p["t_epilogue_cycles"] == pytest.approx(t_epi)
    assert p["t_tile_cycles"] == pytest.approx(t_main + t_epi, rel=1e-9)
    # 256 tiles on 148 units: remainder 108 cannot split (148 // 108 = 1),
    # so the busiest unit runs 2 whole tiles, then one prologue latency.
    assert p["total_tiles"] == 256 and p["tile_slots"] == 148
    t_unit = 2 * (t_main + t_epi) + 1000
    compute = t_unit / 1.4e9
    # A and B (64 MiB) fit in L2: read once; C written once.
    hbm = (2 * 4096 * 4096 * 2) / 6.5e12 + (4096 * 4096 * 2) / 6.5e12
    assert p["dram_bytes"] == pytest.approx(3 * 4096 * 4096 * 2)
    # the two limits overlap (sharper smooth maximum, p = 8); the launch
    # overhead is paid once on top
    seconds = smax(compute, hbm, 8.0) + 4e-6
    assert p["predicted_seconds"] == pytest.approx(seconds, rel=1e-9)
    assert p["predicted_tflops"] == pytest.approx(2 * 4096 ** 3 / seconds / 1e12, rel=1e-9)
    # by hand: t_fill 785.3, t_stage 1225.5, unit 166,054 cycles = 118.6 us,
    # + 4 us launch = 122.6 us
    assert p["predicted_tflops"] == pytest.approx(1120.9, abs=0.2)
    # the worst factor is the partial second round: 256*64*t_stage / (148 * 2
    # tiles) = 0.82, just below the fill (1024 of 1225.5 cycles, 0.84)
    assert p["wave_efficiency"] == pytest.approx(256 * 64 * t_stage / (148 * (t_unit - 1000)),
                                                 rel=1e-9)
    assert p["l2_efficiency"] == pytest.approx(1024.0 / t_stage, rel=1e-9)
    assert p.label == "WAVES"


def test_split_k_tail_and_pairs_change_the_walk():
    hw = b200()
    # 16 x 8192 x 8192 with 128 x 256 tiles: 32 tiles on 148 units -> split 4 ways
    # (148 // 32 = 4, 128 K-blocks / 4 >= 4)
    split = predict(16, 8192, 8192, rb.TileConfig(128, 256, 64, 4, 8, 8, 1), hw)
    whole = predict(16, 8192, 8192, rb.TileConfig(128, 256, 64, 4, 8, 8, 1, 1), hw)
    assert split["predicted_tflops"] > whole["predicted_tflops"]
    pair = predict(4096, 4096, 4096, rb.TileConfig(256, 256, 64, 5, 4, 8, 2), hw)
    assert pair["tile_slots"] == 74 and pair["acc_buffers"] == 2


def test_invariants_large_square():
    hw = b200()
    for cfg in (rb.TileConfig(128, 256, 64, 4, 4, 8), rb.TileConfig(256, 256, 64, 5, 8, 8, 2),
                rb.TileConfig(64, 64, 32, 2, 4, 1)):
        p = predict(8192, 8192, 8192, cfg, hw)
        assert 0 < p["predicted_tflops"] <= min(p["compute_tflops"], p["hbm_tflops"]) + 1e-6
        assert p["predicted_tflops"] < p["peak_tensor_tflops"]
        for k in ("smem_efficiency", "l2_efficiency", "occ_factor", "wave_efficiency",
                  "envelope_efficiency", "epilogue_efficiency"):
            assert 0 < p[k] <= 1 + 1e-9, k


def test_groupm_matters_when_operands_exceed_l2():
    """The grouped-M walk changes modelled DRAM traffic once A and B no longer
    fit in L2 (the reference model had no term for it)."""
    hw = b200()
    g1 = predict(16384, 16384, 16384, rb.TileConfig(128, 256, 64, 4, 4, 1), hw)
    g8 = predict(16384, 16384, 16384, rb.TileConfig(128, 256, 64, 4, 4, 8), hw)
    assert g1["dram_bytes"] > g8["dram_bytes"]


def test_short_k_is_hbm_or_epilogue_bound():
    hw = b200()
    p = predict(8192, 8192, 128, rb.TileConfig(128, 256, 64, 4, 8, 8), hw)
    assert p.label in ("HBM", "EPILOGUE", "WAVES", "ENVELOPE")
    assert p["arithmetic_intensity"] < 200


def test_does_not_fit():
    p = predict(4096, 4096, 4096, rb.TileConfig(256, 256, 64, 5, 8, 8, 1), b200())
    assert p.label == "DOES_NOT_FIT"


def test_committed_calibration_loads_and_is_calibrated():
    from ridge_b200.model import DEFAULT_HW_JSON
    hw = load_hw(DEFAULT_HW_JSON)
    assert hw.calibrated == 1 and hw.num_sms == 148
    assert 0.8e9 < hw.clock_hz < 2.1e9


def test_loader_is_all_or_nothing(tmp_path):
    from ridge_b200.model import DEFAULT_HW_JSON
    good = json.loads(DEFAULT_HW_JSON.read_text())
    out = HwC()
    lib.ridge_hw_b200(C.byref(out))
    before = bytes(out)
    for mutate in ("missing", "nan", "zero", "nested", "garbage"):
        d = dict(good)
        text = None
        if mutate == "missing":
            d.pop("tmaBoxCycles")
        elif mutate == "nan":
            d["clockHz"] = "abc"
        elif mutate == "zero":
            d["hbmBytesPerSec"] = 0
        elif mutate == "nested":
            text = json.dumps(d)[:-1] + ', "x": {"y": 1}}'
        else:
            text = "{ not json"
        f = tmp_path / ("hw_%s.json" % mutate)
        f.write_text(text if text is not None else json.dumps(d))
        err = C.create_string_buffer(256)
        assert lib.ridge_hw_load_json(str(f).encode(), C.byref(out), err, 256) != 0, mutate
        assert err.value, mutate
        assert bytes(out) == before, mutate
    err = C.create_string_buffer(256)
    assert lib.ridge_hw_load_json(b"/nonexistent.json", C.byref(out), err, 256) != 0
    assert b"cannot open" in err.value


def test_cli_batch_keeps_rows_and_appends_predictions(tmp_path):
    import subprocess
    from pathlib import Path
    exe = Path(rb.__file__).parent / "lib" / "ridge-predict"
    src = tmp_path / "in.csv"
    src.write_text("# comment\nM,N,K,tag,BM,BN,BK,stages,warps\n4096,4096,4096,a,256,256,64,3,4\n"
                   "1024,1024,1024,b,128,128,64,4,8\n")
    dst = tmp_path / "out.csv"
    r = subprocess.run([str(exe), "--batch", str(src), "--out", str(dst)], capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stderr
    lines = dst.read_text().splitlines()
    assert lines[0] == "# comment"
    assert lines[1].endswith("pred_arith_intensity,pred_ctas_per_sm")
    row = lines[2].split(",")
    p = predict(4096, 4096, 4096, rb.TileConfig(256, 256, 64, 3, 4, 8, 0), b200())
    assert float(row[9]) == pytest.approx(p["predicted_tflops"], rel=1e-5)
    assert len(lines) == 4


def test_sweep_file_appends_and_resume(tmp_path):
    """The exhaustive sweep appends shape by shape; a shape whose every variant
    is in the file counts as done on resume, a partial one does not."""
    from ridge_b200.autotune import append_meta, append_rows, completed_shapes, load_measured, \
        write_header
    from ridge_b200.model import default_hw
    hw = default_hw()
    p = tmp_path / "sweep.csv"
    write_header(p, hw, "test")
    table = [v.config for v in rb.variants()]
    append_rows(p, (256, 256, 256, "a"), [{"config": c, "tflops": 1.0, "device": 0}
                                          for c in table], hw)
    append_rows(p, (512, 256, 256, "b"), [{"config": c, "tflops": 1.0, "device": 1}
                                          for c in table[:5]], hw)
    append_meta(p, "canary_tflops", "1400.0")
    assert completed_shapes(p) == {(256, 256, 256)}
    rows = load_measured(p)
    assert len(rows) == len(table) + 5 and rows[-1]["device"] == "1"


def test_merge_best_of_sweeps(tmp_path):
    """Merging sweeps keeps, per configuration, the highest throughput."""
    from ridge_b200.autotune import append_rows, load_measured, merge_best, write_header
    from ridge_b200.model import default_hw
    hw = default_hw()
    table = [v.config for v in rb.variants()][:3]
    paths = []
    for i, vals in enumerate(([1.0, 5.0, 3.0], [2.0, 4.0, 6.0])):
        p = tmp_path / ("s%d.csv" % i)
        write_header(p, hw, "run %d" % i)
        append_rows(p, (256, 256, 256, "a"), [{"config": c, "tflops": v, "device": i}
                                              for c, v in zip(table, vals)], hw)
        paths.append(p)
    out = tmp_path / "m.csv"
    assert merge_best(out, paths) == 3
    assert [r["tflops"] for r in load_measured(out)] == [2.0, 5.0, 6.0]
