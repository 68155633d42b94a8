"""The checked build: the GPU parity suite's C-ABI tests run once more on
libexactsample_b200_checked.so (built with -DES_CHECKS), whose device bounds
checks on shared-memory, distributed-shared-memory, candidate and tile
indices count failures in the workspace instead of trapping. Every call of
that run starts from a poisoned workspace and must leave the bytes past its
records untouched (tests/gpu_helpers.run_abi), with no failed check.

This stands in for the reference's sanitizer runs (memcheck, racecheck,
initcheck and synccheck over its suites, tests/sanitizer/run.py:32-46),
since compute-sanitizer does not run on this pool."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

pytestmark = pytest.mark.gpu


def test_parity_suite_passes_on_the_checked_build():
    from exactsample_b200 import build

    library = build.CHECKED_LIB
    assert library.is_file(), "build it with python -m exactsample_b200.build"
    env = dict(os.environ, EXACTSAMPLE_ABI_LIBRARY=str(library))
    selection = ("small_golden_through_abi or large_golden or full_size or cluster_split or row_mode or ring_depth "
                 "or every_mask or near_tie or near_threshold or min_p_threshold or top_k_selection or top_p")
    result = subprocess.run([sys.executable, "-m", "pytest", "tests/test_gpu_parity.py", "tests/test_real_logits.py",
                             "-q", "-x", "-m", "gpu", "-k", selection, "-p", "no:cacheprovider"],
                            cwd=ROOT, env=env, capture_output=True, text=True, timeout=1500)
    print(result.stdout[-3000:])
    assert result.returncode == 0, result.stdout[-6000:] + result.stderr[-3000:]
    assert " passed" in result.stdout
