"""Generates tests/golden/stat_counts.json: the statistical plan's first 500
trials per cell, counted by the reference's own statistical runner.

    python tests/golden/make_stat_golden.py --reference /path/to/exactsample

It imports the reference checkout's ``tests.stat.run.reference_counts``
(its per-trial loop over its own FP64 oracle) and records the counts per
cell; ``tests/test_stat_plan.py`` requires this repository's batched oracle
runner to give the same counts on the same seeds. The fixture is committed;
the tests never need the reference itself.
"""
import argparse
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
TRIALS = 500


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--reference", type=Path, required=True, help="the reference checkout (its root)")
    args = parser.parse_args()
    sys.path[:0] = [str(args.reference / "python"), str(args.reference)]
    from tests.stat.run import reference_counts  # the reference's module of this name
    plan = json.loads((args.reference / "tests" / "stat_plan.json").read_text())
    counts = {cell["name"]: reference_counts(cell, TRIALS, plan["seed_start"], plan["stream_id"], plan["position"])
              for cell in plan["cells"]}
    record = {"trials_per_cell": TRIALS, "seed_start": plan["seed_start"], "stream_id": plan["stream_id"],
              "position": plan["position"], "counts": counts}
    (HERE / "stat_counts.json").write_text(json.dumps(record, indent=1) + "\n")
    print(json.dumps(record))


if __name__ == "__main__":
    main()
