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
