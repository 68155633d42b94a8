"""The statistical plan on the B200 kernels at a smoke size: on the plan's
first 10,000 trials per cell the kernels' counts equal the CPU oracle's
exactly (every trial is bit-exact), with lists on and off. The full plan
(2,000,000 trials per cell, G tests with Holm's step-down) runs with
``python -m tests.stat.run --backend cuda``."""
import pytest

from tests.stat.plan import PLAN
from tests.stat.run import cuda_counts, oracle_counts

pytestmark = pytest.mark.gpu
TRIALS = 10_000


@pytest.mark.parametrize("cell", PLAN["cells"], ids=lambda c: c["name"])
def test_kernel_counts_equal_the_oracles(cell):
    expected = oracle_counts(cell, TRIALS, PLAN["seed_start"], 2500)
    for list_max in [256, 0]:
        assert cuda_counts(cell, TRIALS, PLAN["seed_start"], 4096, list_max) == expected, list_max
