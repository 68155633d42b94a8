"""The statistical plan's machinery on CPU: the batched oracle runner gives
the reference's own counts on the plan's first trials (golden fixture made
by the reference's runner), the analysis behaves as specified, and the
plan has the power it claims."""
import json
from pathlib import Path

import numpy as np
import pytest

from tests.stat.analysis import g_test, holm, power_bound
from tests.stat.plan import PLAN
from tests.stat.run import oracle_counts

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "stat_counts.json").read_text())


@pytest.mark.parametrize("cell", PLAN["cells"], ids=lambda c: c["name"])
def test_oracle_runner_counts_equal_the_reference_runners(cell):
    assert GOLDEN["seed_start"] == PLAN["seed_start"] and GOLDEN["stream_id"] == PLAN["stream_id"]
    # Batches of 128 trials: the split into calls must not matter.
    assert oracle_counts(cell, GOLDEN["trials_per_cell"], PLAN["seed_start"], 128) == GOLDEN["counts"][cell["name"]]


def test_g_test():
    assert g_test([50, 50], [0.5, 0.5]) == {"g": 0.0, "p_value": 1.0, "hard_failure": None}
    far = g_test([900, 100], [0.5, 0.5])
    assert far["g"] > 600 and far["p_value"] < 1e-100
    assert g_test([5, 1], [1.0, 0.0])["hard_failure"] == "observed forbidden category"
    assert g_test([7, 0], [1.0, 0.0])["p_value"] == 1.0  # a single supported category
    with pytest.raises(ValueError):
        g_test([1, 2], [0.6, 0.6])


def test_holm_steps_down_and_stops_at_the_first_acceptance():
    assert holm([0.001, 0.04, 0.03, 0.5], 0.05) == [True, False, False, False]
    assert holm([0.001, 0.012, 0.02, 0.5], 0.05) == [True, True, True, False]
    assert holm([0.2] * 10, 0.01) == [False] * 10


def test_plan_power():
    power = power_bound(PLAN)
    assert power["minimum_alternative_g"] == pytest.approx(50.0)
    assert power["minimum_alternative_g"] > power["worst_critical_g"] and power["power_lower_bound"] > 0.9
    assert all(np.isclose(sum(c["expected"]), 1) for c in PLAN["cells"]) and len(PLAN["cells"]) == 10
