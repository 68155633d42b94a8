"""TEST INFRASTRUCTURE ONLY: the CPU oracle for exactsample's sampling and
speculative-verification contract.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package. The product package ``exactsample_b200`` never
imports, links or calls it, and has no CPU fallback.

``oracle.reference`` restates the reference's FP64 NumPy oracle
(``python/exactsample/reference.py`` and ``rng.py``) operation for operation;
its Python-level loops (Philox, the Gumbel argmax, ``math.fsum`` prefix sums)
run in ``oracle_c.c``. Parity is pinned: ``tests/golden/make_golden.py`` runs
the reference's own oracle on fixed inputs and ``tests/test_oracle.py``
requires identical tokens, statuses and accept counts from this oracle.
"""
from .reference import (PathUsed, RequestParams, RngKey, Status, VerifyOutput, distribution, gumbel,
                        philox4x32, proposal_distribution, random_word, sample_distribution, uniform,
                        verify_reference)

__all__ = ["PathUsed", "RequestParams", "RngKey", "Status", "VerifyOutput", "distribution", "gumbel",
           "philox4x32", "proposal_distribution", "random_word", "sample_distribution", "uniform",
           "verify_reference"]
