"""The registered counters-to-label table (ridge_b200.ncu_validate) on
hand-made counter rows, one per rule, and the scorer's pass criterion."""

import csv

from ridge_b200.ncu_validate import CONFIGS, METRICS, PASS_AGREE, label_from_counters, \
    load_configs, score


def _c(dram=10.0, active=95.0, tensor=70.0, fill=40.0, write=5.0, cycles=1e6):
    return {METRICS[0]: dram, METRICS[1]: active, METRICS[2]: tensor,
            METRICS[3]: fill * cycles, METRICS[4]: write * cycles, METRICS[5]: cycles}


def test_each_rule_in_registered_order():
    assert label_from_counters(_c(dram=75, active=50)) == "HBM"        # rule 1 before 2
    assert label_from_counters(_c(active=79.9, tensor=90)) == "WAVES"  # rule 2 before 3
    assert label_from_counters(_c(tensor=85, fill=60)) == "TENSOR_CORE"
    assert label_from_counters(_c(tensor=70, fill=54)) == "L2"
    assert label_from_counters(_c(tensor=45, fill=30, write=12)) == "EPILOGUE"
    assert label_from_counters(_c(tensor=55, fill=30, write=5)) == "OCC"
    assert label_from_counters(_c(tensor=70, fill=30)) == "ENVELOPE"


def test_registered_configs_and_score(tmp_path):
    rows = load_configs(CONFIGS)
    assert len(rows) == 16
    assert {r["predicted_label"] for r in rows} == {"L2", "WAVES", "OCC", "HBM"}
    p = tmp_path / "labels.csv"
    with open(p, "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(["predicted_label", "tag", "M", "N", "K", "BM", "BN", "BK", "stages", "warps",
                    "groupM", "cta_group", *METRICS])
        for i, r in enumerate(rows):
            c = _c(tensor=70, fill=60) if i < PASS_AGREE else _c(dram=90)
            w.writerow([r["predicted_label"], r["tag"], r["M"], r["N"], r["K"], r["BM"], r["BN"],
                        r["BK"], r["stages"], r["warps"], r["groupM"], r["cta_group"],
                        *[c[m] for m in METRICS]])
    agree, n, verdict = score(p, log=lambda *_: None)
    # rows 0-3 are L2 (agree), 4-11 get L2 (disagree), 12-15 are HBM (agree)
    assert (agree, n, verdict) == (8, 16, "FAIL")
