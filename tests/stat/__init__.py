"""The statistical plan: the reference's preregistered distribution checks
(tests/stat_plan.json, tests/stat/run.py, tests/stat/analysis.py of the
reference), run on the CPU oracle and on the B200 kernels."""
