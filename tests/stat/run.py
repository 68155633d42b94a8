"""Runs the statistical plan on the CPU oracle or on the B200 kernels and
writes a report (the reference's tests/stat/run.py, with this repository's
two backends).

    python -m tests.stat.run --backend cuda --output OUT.json                 # the preregistered 2,000,000 per cell
    python -m tests.stat.run --backend cuda --list-max 0 --output OUT.json    # every row on the whole-row path
    python -m tests.stat.run --backend oracle --samples 20000 --output OUT.json   # smaller: not qualification

A run qualifies only at the plan's sample count with no cell rejected; a
rejection triggers one full rerun of the family on disjoint seeds, reported
beside the initial failure (which stands).
"""
import argparse
import json
import platform
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from tests.stat.analysis import g_test, holm, power_bound  # noqa: E402
from tests.stat.plan import PLAN, observations, trial_inputs  # noqa: E402


def oracle_counts(cell, samples, seed_start, batch):
    import oracle

    proposals = np.random.Generator(np.random.PCG64(seed_start ^ 0x51A7))
    counts = np.zeros(len(cell["expected"]), np.int64)
    for first in range(0, samples, batch):
        size = min(batch, samples - first)
        rows, offsets, ids, params, seeds, positions, q, mode = trial_inputs(cell, first, size, seed_start, proposals)
        out = oracle.verify_reference(
            rows, offsets, ids, params=oracle.RequestParams(**params, draft_kind="full" if q is not None else "one_hot"),
            rng=oracle.RngKey([int(s) for s in seeds], PLAN["stream_id"], positions), draft_logits=q, mode=mode)
        if np.any(out.status != 0):
            raise RuntimeError(f"unexpected status in {cell['name']}")
        counts += np.bincount(observations(cell, out.tokens, out.accepted_len), minlength=counts.size)[:counts.size]
    return counts.tolist()


def cuda_counts(cell, samples, seed_start, batch, list_max):
    import torch

    from exactsample_b200.cuda import CudaRequestParams, CudaRngKey, plan, verify

    proposals = np.random.Generator(np.random.PCG64(seed_start ^ 0x51A7))
    drafts = {"sample": 0, "accepted": 3}.get(cell["kind"], 1)
    vocab = len(cell["weights"])
    work = plan(batch * (drafts + 1), batch, max(drafts, 1), vocab)
    work.list_max = list_max
    out = work.allocate_output()
    counts = torch.zeros(len(cell["expected"]), dtype=torch.int64, device="cuda")
    bad = torch.zeros((), dtype=torch.int64, device="cuda")
    t = lambda a, dt: torch.as_tensor(np.ascontiguousarray(a)).to("cuda", dt)
    for first in range(0, samples, batch):
        size = min(batch, samples - first)
        rows, offsets, ids, params, seeds, positions, q, mode = trial_inputs(cell, first, size, seed_start, proposals)
        full = lambda v, dt: torch.full((size,), v, dtype=dt, device="cuda")
        verify(t(rows, torch.float64), t(offsets, torch.int64), t(ids, torch.int64),
               params=CudaRequestParams(full(params["temperature"], torch.float64), full(params["top_k"], torch.int64),
                                        full(params["top_p"], torch.float64), full(params["min_p"], torch.float64),
                                        full(1 if q is not None else 0, torch.int64)),
               rng=CudaRngKey(t(seeds.view(np.int64), torch.int64), full(PLAN["stream_id"], torch.int64),
                              t(positions, torch.int64)),
               plan=work, out=out, draft_logits=None if q is None else t(q, torch.float64), mode=mode)
        seen = out.accepted_len[:size] if cell["kind"] == "accepted" else out.tokens[:size, 0]
        bad += (out.status[:size] != 0).sum() + ((seen < 0) | (seen >= counts.numel())).sum()
        counts += torch.bincount(seen.clamp(0, counts.numel() - 1).to(torch.int64), minlength=counts.numel())
    work.synchronize()
    if bad.item():
        raise RuntimeError(f"failed statuses or out-of-range categories in {cell['name']}")
    return counts.tolist()


def run_family(samples, seed_start, backend, batch, list_max=256, log=print):
    results = []
    for cell in PLAN["cells"]:
        counts = (oracle_counts(cell, samples, seed_start, batch) if backend == "oracle" else
                  cuda_counts(cell, samples, seed_start, batch, list_max))
        results.append({"cell": cell["name"], "counts": counts, "expected": cell["expected"],
                        **g_test(counts, cell["expected"])})
        log(json.dumps({"cell": cell["name"], "samples": samples, "p_value": results[-1]["p_value"]}))
    for result, rejected in zip(results, holm([r["p_value"] for r in results], PLAN["family_error_rate"])):
        result["rejected"] = rejected
    return results


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--backend", choices=["oracle", "cuda"], default="cuda")
    parser.add_argument("--samples", type=int, default=PLAN["samples_per_cell"])
    parser.add_argument("--batch-size", type=int, default=8192)
    parser.add_argument("--list-max", type=int, default=256, help="cuda: 0 sends every row through the whole-row path")
    parser.add_argument("--output", type=Path, required=True)
    args = parser.parse_args()
    if args.samples <= 0 or args.batch_size <= 0:
        parser.error("samples and batch size must be positive")
    if args.output.exists():
        parser.error("refusing to overwrite an existing report")
    started = time.time()
    results = run_family(args.samples, PLAN["seed_start"], args.backend, args.batch_size, args.list_max)
    failed = any(r["rejected"] for r in results)
    report = {"scope": "CPU FP64 oracle" if args.backend == "oracle" else
              f"exactsample_b200 kernels, float64 inputs, list_max={args.list_max}",
              "samples_per_cell": args.samples,
              "qualification": args.samples == PLAN["samples_per_cell"] and not failed,
              "rng": {"seed_start": PLAN["seed_start"], "stream_id": PLAN["stream_id"], "position": PLAN["position"]},
              "power": power_bound(PLAN), "cells": results, "initial_failure": failed,
              "environment": {"python": platform.python_version(), "numpy": np.__version__}}
    if args.backend == "cuda":
        import torch
        report["environment"].update(torch=torch.__version__, gpu=torch.cuda.get_device_name())
    if failed:
        report["diagnostic_retry"] = run_family(args.samples, PLAN["retry_seed_start"], args.backend, args.batch_size,
                                                args.list_max)
    report["elapsed_seconds"] = time.time() - started
    args.output.parent.mkdir(parents=True, exist_ok=True)
    args.output.write_text(json.dumps(report, indent=2) + "\n")
    print(json.dumps({"output": str(args.output), "qualification": report["qualification"], "failed": failed}))
    return int(failed)


if __name__ == "__main__":
    raise SystemExit(main())
