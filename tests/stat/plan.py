"""The fixed statistical plan and the inputs of its trials.

The plan's values are the reference's preregistered ones
(tests/stat_plan.json of the reference): ten cells, each a tiny row whose
sampled token (or accepted length) has a known distribution, 2,000,000
samples per cell, a multinomial likelihood-ratio G test per cell and Holm's
step-down over the ten at family error rate 0.01. Trial t of a cell uses
the Philox key (seed_start + t, stream 19) at positions 101, 102, ...; the
"full" cell draws its proposal token from NumPy's PCG64 seeded with
seed_start XOR 0x51A7 (0 with probability 1/4), independent of Philox.

Trials are independent requests, so a batch of trials is one call with one
request per trial; that gives the same outputs as one call per trial.
"""
import numpy as np

PLAN = {
    "samples_per_cell": 2_000_000,
    "family_error_rate": 0.01,
    "target_total_variation": 0.005,
    "max_categories": 8,
    "seed_start": 65536,
    "retry_seed_start": 1099511693312,
    "stream_id": 19,
    "position": 101,
    "cells": [
        dict(name="uniform4", kind="sample", weights=[1, 1, 1, 1], expected=[0.25, 0.25, 0.25, 0.25]),
        dict(name="skew4", kind="sample", weights=[97, 1, 1, 1], expected=[0.97, 0.01, 0.01, 0.01]),
        dict(name="temperature2", kind="sample", weights=[16, 4, 1], params=dict(temperature=2.0),
             expected=[4 / 7, 2 / 7, 1 / 7]),
        dict(name="topk2", kind="sample", weights=[8, 4, 2, 1], params=dict(top_k=2), expected=[2 / 3, 1 / 3, 0, 0]),
        dict(name="topp_boundary", kind="sample", weights=[1, 1, 1, 1], params=dict(top_p=0.5),
             expected=[0.5, 0.5, 0, 0]),
        dict(name="minp", kind="sample", weights=[8, 4, 2, 1], params=dict(min_p=0.4), expected=[2 / 3, 1 / 3, 0, 0]),
        dict(name="onehot_ratio", kind="onehot", weights=[1, 3], expected=[0.25, 0.75]),
        dict(name="onehot_coupled", kind="coupled", weights=[1, 3], expected=[0.25, 0.75]),
        dict(name="fullq_ratio", kind="full", weights=[3, 1], expected=[0.75, 0.25]),
        dict(name="accepted_length3", kind="accepted", weights=[1, 1], expected=[0.5, 0.25, 0.125, 0.125]),
    ],
}


def drafts_of(cell) -> int:
    return {"sample": 0, "accepted": 3}.get(cell["kind"], 1)


def trial_inputs(cell, first_trial: int, size: int, seed_start: int, proposals: np.random.Generator):
    """NumPy inputs of trials [first_trial, first_trial + size) of a cell:
    (rows, offsets, draft_ids, params dict, seeds, positions, draft_logits,
    mode). ``proposals`` is the cell's PCG64 stream, consumed in trial order."""
    kind, drafts = cell["kind"], drafts_of(cell)
    ids = np.zeros((size, max(drafts, 1)), np.int64)
    if drafts == 0:
        ids[:] = -1
    if kind == "full":
        ids[:, 0] = (proposals.random(size) >= 0.25).astype(np.int64)
    rows = np.tile(np.log(np.asarray(cell["weights"], np.float64)), (size * (drafts + 1), 1))
    offsets = np.arange(size + 1, dtype=np.int64) * (drafts + 1)
    seeds = (np.uint64(seed_start) + np.arange(first_trial, first_trial + size, dtype=np.uint64))
    positions = np.tile(np.arange(PLAN["position"], PLAN["position"] + drafts + 1, dtype=np.int64), size)
    q = np.tile(np.log([1.0, 3.0]), (size * 2, 1)) if kind == "full" else None
    params = dict(temperature=1.0, top_k=0, top_p=1.0, min_p=0.0)
    params.update(cell.get("params", {}))
    mode = "coupled" if kind == "coupled" else "ratio"
    return rows, offsets, ids, params, seeds, positions, q, mode


def observations(cell, tokens, accepted):
    """The observed category of each trial: the accepted length (accepted
    cell) or the first emitted token."""
    return np.asarray(accepted if cell["kind"] == "accepted" else tokens[:, 0])
