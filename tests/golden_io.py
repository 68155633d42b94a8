"""Loads the golden fixtures written by ``tests/golden/make_golden.py``."""
from __future__ import annotations

from pathlib import Path

import numpy as np

from tests import cases as C

GOLDEN = Path(__file__).resolve().parent / "golden"
_FIELDS = ["logits", "cu_rows", "draft_ids", "temperature", "top_k", "top_p", "min_p", "draft_kind", "seed",
           "stream_id", "positions", "mask", "draft_logits", "mode", "logit_dtype"]


def small():
    """[(case dict, (tokens, accepted, status))] of the small fixtures."""
    data = np.load(GOLDEN / "golden_small.npz")
    out = []
    for i, name in enumerate(data["names"]):
        case = {"name": str(name)}
        for key in _FIELDS:
            k = f"{i}/{key}"
            case[key] = data[k] if k in data else None
            if key in ("logits", "draft_logits", "temperature", "top_p", "min_p") and case[key] is not None:
                case[key] = case[key].astype(np.float64)
        case["mode"], case["logit_dtype"] = str(case["mode"]), str(case["logit_dtype"])
        out.append((case, (data[f"{i}/out_tokens"], data[f"{i}/out_accepted"], data[f"{i}/out_status"])))
    return out


def large_entries():
    """[(name, subset or None, digest, (tokens, accepted, status))] of the large fixtures."""
    data = np.load(GOLDEN / "golden_large.npz")
    out = []
    for i, name in enumerate(data["names"]):
        subset = None if bool(data[f"{i}/whole"]) else [int(x) for x in data[f"{i}/subset"]]
        out.append((str(name), subset, str(data[f"{i}/digest"]),
                    (data[f"{i}/out_tokens"], data[f"{i}/out_accepted"], data[f"{i}/out_status"])))
    return out


def large_case(name, subset, digest):
    case = C.workload_case(name, subset)
    if C.digest(case) != digest:
        raise AssertionError(f"regenerated inputs of {name} differ from the golden fixture's (generator drift)")
    return case


# The reference's agreement benchmark on real logits (bench/agreement.py:27-28,
# "8x8" variant): (sampling settings, requests, drafts) per cell, over the
# 64-row Qwen3-8B capture (8 sequences x 8 decode steps).
REAL_SETTINGS = {
    "qwen": dict(temperature=0.6, top_k=20, top_p=0.95),
    "temperature": dict(temperature=1.0, top_k=0, top_p=1.0),
    "top_p": dict(temperature=0.7, top_k=0, top_p=0.9),
}
REAL_CELLS = [("qwen", 64, 0), ("qwen", 16, 4), ("top_p", 64, 0), ("top_p", 16, 4), ("temperature", 24, 0),
              ("temperature", 8, 4)]


def real_logit_cells():
    """[(cell name, case, {gpu: (tokens, accepted_len, status)})] of the real-logit
    cells. The cell layout restates the reference's workload builder
    (bench/sampler.py:45-78): request i takes the capture rows of sequence
    i mod 8 from decode step (i div 8) (D + 1) mod (8 - D) on, D + 1
    consecutive steps, with the steps' sampled tokens as its D drafts; seeds
    1000 + i, stream i, positions from the capture, no min-p, one-hot drafts.
    The logits are the capture's bf16 values (exact in float64)."""
    capture = np.load(GOLDEN / "qwen3_8b_8x8.npz")
    bits = capture["logits_bf16"].astype(np.uint16).astype(np.uint32) << 16
    values = bits.view(np.float32).astype(np.float64)
    steps, sequences = int(capture["step"].max()) + 1, int(capture["sequence"].max()) + 1
    saved = {gpu: np.load(GOLDEN / f"reference_outputs_8x8_{gpu}.npz") for gpu in ("rtx4090", "a10")}
    cells = []
    for setting, requests, drafts in REAL_CELLS:
        rows = []
        ids = np.full((requests, max(drafts, 1)), -1, dtype=np.int64)
        for i in range(requests):
            start = (i // sequences) * (drafts + 1) % (steps - drafts)
            first = (i % sequences) * steps + start
            rows += range(first, first + drafts + 1)
            ids[i, :drafts] = capture["sampled"][first:first + drafts]
        rows = np.asarray(rows)
        p = REAL_SETTINGS[setting]
        name = f"{setting}-{requests}x{drafts}"
        case = dict(name=name, logits=values[rows], cu_rows=np.arange(requests + 1, dtype=np.int64) * (drafts + 1),
                    draft_ids=ids, temperature=np.full(requests, p["temperature"]),
                    top_k=np.full(requests, p["top_k"], np.int64), top_p=np.full(requests, p["top_p"]),
                    min_p=np.zeros(requests), draft_kind=np.zeros(requests, np.int64),
                    seed=(np.arange(requests) + 1000).astype(np.uint64), stream_id=np.arange(requests, dtype=np.int64),
                    positions=capture["position"][rows].astype(np.int64), mask=None, draft_logits=None, mode="ratio",
                    logit_dtype="bfloat16")
        outputs = {gpu: (f[f"{name}-tokens"], f[f"{name}-accepted_len"], f[f"{name}-status"]) for gpu, f in saved.items()}
        cells.append((name, case, outputs))
    return cells
