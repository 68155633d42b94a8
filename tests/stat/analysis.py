"""The plan's analysis: a multinomial likelihood-ratio (G) test per cell,
Holm's step-down across the family, and the plan's power bound (restating
the reference's tests/stat/analysis.py methods)."""
import math


def g_test(counts, probabilities):
    """G = 2 sum n_i ln(n_i / (N p_i)), against chi-square with (support - 1)
    degrees of freedom. A count in a zero-probability category is a hard
    failure (p-value 0)."""
    from scipy.stats import chi2

    if len(counts) != len(probabilities) or sum(counts) <= 0:
        raise ValueError("nonempty matching counts/probabilities required")
    if any(n < 0 or int(n) != n for n in counts):
        raise ValueError("counts must be nonnegative integers")
    if any(p < 0 for p in probabilities) or not math.isclose(sum(probabilities), 1):
        raise ValueError("probabilities must sum to one")
    if any(n and not p for n, p in zip(counts, probabilities)):
        return {"g": None, "p_value": 0.0, "hard_failure": "observed forbidden category"}
    total = sum(counts)
    support = sum(p > 0 for p in probabilities)
    g = max(0.0, 2 * math.fsum(n * math.log(n / (total * p)) for n, p in zip(counts, probabilities) if n))
    return {"g": g, "p_value": 1.0 if support == 1 else float(chi2.sf(g, support - 1)), "hard_failure": None}


def holm(p_values, alpha):
    """Holm's step-down: which hypotheses are rejected at family error rate alpha."""
    rejected = [False] * len(p_values)
    for rank, i in enumerate(sorted(range(len(p_values)), key=p_values.__getitem__)):
        if p_values[i] > alpha / (len(p_values) - rank):
            break
        rejected[i] = True
    return rejected


def power_bound(plan):
    """Pinsker and Hoeffding: against any alternative at total variation
    >= delta, G exceeds N delta^2, which is above every cell's critical value,
    except with probability at most 2^m exp(-N delta^2 / 2)."""
    from scipy.stats import chi2

    n, delta, m = plan["samples_per_cell"], plan["target_total_variation"], plan["max_categories"]
    critical = float(chi2.isf(plan["family_error_rate"] / len(plan["cells"]), m - 1))
    g_alternative = n * delta * delta
    miss = min(1.0, 2 ** m * math.exp(-n * delta * delta / 2))
    return {"minimum_alternative_g": g_alternative, "worst_critical_g": critical,
            "power_lower_bound": 1 - miss if g_alternative > critical else 0.0}
