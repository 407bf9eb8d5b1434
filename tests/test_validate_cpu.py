"""The validation report (ridge_b200.validate): its rank statistics on small
hand-checked cases, and the committed model against the committed B200 sweep
(registered cross product complete, MAPE within the gate, top-10 autotune
regret within 1%)."""

import math

from ridge_b200.validate import (average_ranks, best_rank_range, regret1_range, report,
                                 spearman, topk_regret)


def test_average_ranks_and_spearman_with_ties():
    assert average_ranks([3.0, 1.0, 3.0, 2.0]) == [1.5, 4.0, 1.5, 3.0]
    assert spearman([1, 2, 3, 4], [10, 20, 30, 40]) == 1.0
    assert spearman([1, 2, 3, 4], [40, 30, 20, 10]) == -1.0
    assert math.isnan(spearman([1, 1, 1], [1, 2, 3]))


def test_best_rank_and_regret_under_ties():
    pred = [5.0, 5.0, 3.0, 1.0]
    meas = [90.0, 100.0, 80.0, 70.0]
    assert best_rank_range(pred, meas) == (1, 2)
    worst, best, n = regret1_range(pred, meas)
    assert (round(worst, 3), best, n) == (0.1, 0.0, 2)
    assert topk_regret([1.0, 2.0, 3.0], [100.0, 50.0, 60.0], 1) == 0.4
    assert topk_regret([1.0, 2.0, 3.0], [100.0, 50.0, 60.0], 3) == 0.0


def test_committed_model_passes_on_the_committed_sweep():
    res = report(out=lambda *_: None)
    assert res["failures"] == []
    assert res["mape"] <= 20.0
    assert res["topk_regret_mean"] <= 0.01
