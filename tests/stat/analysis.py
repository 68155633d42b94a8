"""Decision rules of the statistical plan.

The plan (the reference's preregistered tests/stat_plan.json) tests each
cell's observed counts against its exact distribution with a multinomial
likelihood-ratio test, controls the family of cells with Holm's step-down
procedure, and states a lower bound on the power of the whole family. This
module computes those three things; the plan's constants live in
tests/stat/plan.py.
"""
import math

import numpy as np


def g_test(counts, probabilities):
    """Likelihood-ratio test of observed counts against a distribution.

    G = 2 * sum_i n_i * ln(n_i / E_i) with E_i = N * p_i, referred to the
    chi-square distribution whose degrees of freedom are the categories with
    positive probability, less one. A count in a category of probability zero
    cannot happen under the hypothesis, so it fails outright (p-value 0).
    Returns {"g", "p_value", "hard_failure"}.
    """
    from scipy.special import xlogy
    from scipy.stats import chi2

    n = np.asarray(counts, dtype=float)
    p = np.asarray(probabilities, dtype=float)
    if n.shape != p.shape or n.ndim != 1 or n.size == 0 or n.sum() <= 0:
        raise ValueError("nonempty matching counts/probabilities required")
    if np.any(n < 0) or np.any(n != np.floor(n)):
        raise ValueError("counts must be nonnegative integers")
    if np.any(p < 0) or not math.isclose(float(p.sum()), 1.0):
        raise ValueError("probabilities must sum to one")
    if np.any((n > 0) & (p == 0)):
        return {"g": None, "p_value": 0.0, "hard_failure": "observed forbidden category"}
    observed = n > 0
    expected = n.sum() * p[observed]
    # xlogy(n, n) - xlogy(n, E) = n ln(n / E); rounding can make the sum a
    # hair negative when the fit is perfect.
    statistic = 2.0 * float(np.sum(xlogy(n[observed], n[observed]) - xlogy(n[observed], expected)))
    statistic = statistic if statistic > 0 else 0.0
    dof = int(np.count_nonzero(p)) - 1
    p_value = 1.0 if dof == 0 else float(chi2.sf(statistic, dof))
    return {"g": statistic, "p_value": p_value, "hard_failure": None}


def holm(p_values, alpha):
    """Holm's step-down procedure at family error rate ``alpha``, through its
    adjusted p-values: with the m p-values sorted ascending, the adjusted value
    of the j-th (0-based) is the running maximum of (m - i) * p_(i) over i <= j;
    a hypothesis is rejected when its adjusted value is at most alpha. Returns
    one rejection flag per input, in input order."""
    m = len(p_values)
    order = np.argsort(np.asarray(p_values, dtype=float), kind="stable")
    adjusted = np.maximum.accumulate(np.asarray(p_values, dtype=float)[order] * (m - np.arange(m)))
    flags = np.zeros(m, dtype=bool)
    flags[order] = adjusted <= alpha
    return flags.tolist()


def power_bound(plan):
    """The plan's power statement for one cell of at most m categories.

    If the true distribution is at total variation delta or more from the
    hypothesis, Pinsker's inequality puts its Kullback-Leibler divergence at
    2 delta^2 or more, so N samples give an expected G of at least N delta^2.
    The empirical distribution strays from the true one by delta in total
    variation with probability at most 2^m exp(-N delta^2 / 2) (a union over
    the 2^m events of a Hoeffding bound), so the family catches the
    alternative with probability at least one minus that, provided N delta^2
    exceeds the largest critical value of the Holm family (the first step,
    alpha / cells). Returns {"minimum_alternative_g", "worst_critical_g",
    "power_lower_bound"}.
    """
    from scipy.stats import chi2

    samples = plan["samples_per_cell"]
    delta = plan["target_total_variation"]
    categories = plan["max_categories"]
    first_step = plan["family_error_rate"] / len(plan["cells"])
    critical = float(chi2.isf(first_step, categories - 1))
    separation = samples * delta ** 2
    log_miss = categories * math.log(2.0) - separation / 2.0
    miss = math.exp(min(0.0, log_miss))
    return {"minimum_alternative_g": separation, "worst_critical_g": critical,
            "power_lower_bound": 1.0 - miss if separation > critical else 0.0}
