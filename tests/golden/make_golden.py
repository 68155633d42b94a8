"""Generates the golden fixtures by running the reference's own FP64 oracle.

    PYTHONPATH=. python tests/golden/make_golden.py --reference /path/to/exactsample/python

It imports ``exactsample.verify_reference`` from the reference checkout (the
only place the reference runs) on every case of ``tests/cases.py``, and
writes:

* ``golden_small.npz``: the small cases, inputs and outputs;
* ``golden_large.npz``: benchmark configurations (``workloads.py``) named by
  configuration, request subset and input digest, with outputs only; the
  tests regenerate the inputs from their seeds and check the digest.

The fixtures are committed; the tests never need the reference itself.
"""
from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path[:0] = [str(ROOT)]

from tests import cases as C  # noqa: E402

# (configuration, request subset): each C4 subset covers every filter x
# temperature pair once, bf16-rounded rows and near-threshold rows.
LARGE = [
    ("C1", None),
    ("C2a", list(range(16))),
    ("C2b", list(range(4))),
    ("C3a", list(range(8))),
    ("C3b", list(range(4))),
    ("C3b_ratio_full", list(range(6))),
    ("C3b_coupled_onehot", list(range(8))),
]


def c4_subset():
    w = __import__("workloads").config("C4")
    picked = list(range(12))  # every (filter, temperature) combination once
    extra = [r for r in w.notes["bf16_rows"][:3] + w.notes["near_threshold_rows"][:6] if r not in picked]
    return picked + extra


def outputs(case, ref):
    out = ref.verify_reference(**C.oracle_inputs(case, ref))
    return np.asarray(out.tokens), np.asarray(out.accepted_len), np.asarray(out.status)


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", required=True, help="the reference's python/ directory")
    parser.add_argument("--only", choices=["small", "large"], default=None)
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    import exactsample as ref

    if args.only in (None, "small"):
        small = C.small_cases() + C.random_cases()
        store = {"names": np.array([c["name"] for c in small])}
        for i, case in enumerate(small):
            tokens, accepted, status = outputs(case, ref)
            for key, value in case.items():
                if key == "name" or value is None:
                    continue
                value = np.asarray(value)
                if value.dtype == np.float64 and np.array_equal(value.astype(np.float32).astype(np.float64), value,
                                                                equal_nan=True):
                    value = value.astype(np.float32)  # lossless; loaders widen to float64
                store[f"{i}/{key}"] = value
            store[f"{i}/out_tokens"], store[f"{i}/out_accepted"], store[f"{i}/out_status"] = tokens, accepted, status
        np.savez_compressed(HERE / "golden_small.npz", **store)
        print(f"small: {len(small)} cases")

    if args.only in (None, "large"):
        store, names = {}, []
        for name, subset in LARGE + [("C4", c4_subset())]:
            start = time.time()
            case = C.workload_case(name, subset)
            tokens, accepted, status = outputs(case, ref)
            i = len(names)
            names.append(name)
            store[f"{i}/subset"] = np.array(subset if subset is not None else [], np.int64)
            store[f"{i}/whole"] = np.array(subset is None)
            store[f"{i}/digest"] = np.array(C.digest(case))
            store[f"{i}/out_tokens"], store[f"{i}/out_accepted"], store[f"{i}/out_status"] = tokens, accepted, status
            print(f"{case['name']}: {time.time() - start:.1f}s statuses={np.bincount(status, minlength=4).tolist()}",
                  flush=True)
        store["names"] = np.array(names)
        np.savez_compressed(HERE / "golden_large.npz", **store)


if __name__ == "__main__":
    main()
