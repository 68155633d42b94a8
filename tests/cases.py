"""Parity cases shared by the oracle tests and the GPU tests.

Each case is a dict of host arrays in the shapes of the reference's oracle
(``verify_reference``): target logits [M, V], cu_rows, draft_ids, the
per-request parameters, the RNG key, and optional mask / draft logits. The
small cases restate the scenarios of the reference's own test suites
(``tests/test_cuda.py``, ``tests/test_fused.py``, ``tests/edge``,
``tests/invariance``) as inputs; the large ones are benchmark configurations
(``workloads.py``), regenerated from their seeds.
"""
from __future__ import annotations

import hashlib

import numpy as np

import workloads

NEG_INF = -np.inf


def _case(name, logits, cu_rows, draft_ids, *, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0,
          draft_kind="one_hot", seed=1234, stream=3, positions=None, mask=None, draft_logits=None,
          mode="ratio", logit_dtype="float64"):
    logits = np.asarray(logits, dtype=np.float64)
    rows = logits.shape[0]
    cu_rows = np.asarray(cu_rows, dtype=np.int64)
    requests = cu_rows.size - 1

    def per(value, dtype):
        arr = np.asarray(value, dtype=object)
        return np.array([arr.item()] * requests if arr.ndim == 0 else list(arr), dtype=dtype)

    kinds = per(draft_kind, object)
    return dict(
        name=name, logits=logits, cu_rows=cu_rows,
        draft_ids=_drafts(draft_ids, requests),
        temperature=per(temperature, np.float64), top_k=per(top_k, np.int64), top_p=per(top_p, np.float64),
        min_p=per(min_p, np.float64),
        draft_kind=np.array([0 if k in ("one_hot", 0) else 1 for k in kinds], np.int64),
        seed=per(seed, object).astype(np.uint64), stream_id=per(stream, np.int64),
        positions=np.arange(rows, dtype=np.int64) if positions is None else np.asarray(positions, np.int64),
        mask=None if mask is None else np.asarray(mask, np.int32),
        draft_logits=None if draft_logits is None else np.asarray(draft_logits, np.float64),
        mode=mode, logit_dtype=logit_dtype)


def _drafts(draft_ids, requests):
    ids = np.asarray(draft_ids, dtype=np.int64)
    return ids if ids.ndim == 2 else ids.reshape(requests, -1)


def round_to(values, dtype):
    """Round float64 values to a narrower float type and back (what a device tensor of that type holds)."""
    values = np.asarray(values, dtype=np.float64)
    if dtype == "float64":
        return values
    if dtype == "float32":
        return values.astype(np.float32).astype(np.float64)
    if dtype == "float16":
        return values.astype(np.float16).astype(np.float64)
    if dtype == "bfloat16":
        f = values.astype(np.float32)
        bits = f.view(np.uint32).astype(np.uint64)
        finite = np.isfinite(f)
        rounded = np.where(finite, (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16 << 16, bits & 0xFFFF0000)
        nan = np.isnan(f)
        rounded = np.where(nan, 0x7FC00000, rounded)
        return rounded.astype(np.uint32).view(np.float32).astype(np.float64)
    raise ValueError(dtype)


def small_cases():
    """Restatements of the reference suites' scenarios (small vocabularies)."""
    cases = []
    g = np.random.default_rng(42)
    rows = g.normal(size=(6, 35))
    for dtype in ["float16", "bfloat16", "float32", "float64"]:
        for k in [0, 1, 20, 35]:
            cases.append(_case(f"dtype_{dtype}_k{k}", round_to(rows, dtype), [0, 1, 3, 6],
                               [[-1, -1], [2, -1], [3, 4]], top_k=k, logit_dtype=dtype))
    for p in [.5, float(np.nextafter(.5, 1)), 1.]:
        cases.append(_case(f"boundary_p{p!r}", np.zeros((4, 4)), [0, 4], [[0, 1, 2]], top_k=4, top_p=p))
    mask = np.array([[-2147483648, 1]] * 3, np.int32)
    cases.append(_case("mask_word_boundary", np.zeros((3, 35)), [0, 3], [[31, 32]], mask=mask, top_k=20))
    for bad in [float("nan"), float("inf"), -float("inf")]:
        cases.append(_case(f"status_{bad}", [[0., -np.inf], [bad, bad]], [0, 2], [[1]]))
    cases.append(_case("all_masked", np.zeros((2, 2)), [0, 2], [[0]], mask=np.zeros((2, 1), np.int32)))
    cases.append(_case("empty_segment", np.zeros((1, 2)), [0, 0, 1], np.empty((2, 0), np.int64)))
    cases.append(_case("full_q_top1", np.log([[3., 1.], [1., 1.]]), [0, 2], [[1]], top_k=1, draft_kind="full",
                       draft_logits=np.log([[1., 3.], [1., 1.]])))
    cases.append(_case("full_q_zero", [[0., 0.], [0., 0.]], [0, 2], [[1]], draft_kind="full",
                       draft_logits=[[0., -np.inf], [0., 0.]]))
    cases.append(_case("future_error_first", [[0., 0.], [np.nan, 0.]], [0, 2], [[1]], draft_kind="full",
                       draft_logits=[[0., -np.inf], [0., 0.]]))
    rows3 = np.array([[0., 1., 2.], [1., 0., 2.], [2., 1., 0.]])
    cases.append(_case("coupled_ordinary", rows3, [0, 1, 2, 3], np.empty((3, 0), np.int64),
                       seed=777, stream=7, positions=[20, 21, 22]))
    cases.append(_case("coupled_reordered", rows3[[2, 0, 1]], [0, 1, 2, 3], np.empty((3, 0), np.int64),
                       seed=777, stream=7, positions=[22, 20, 21]))
    for drafts in [[0, 0], [2, 1], [1, 2]]:
        cases.append(_case(f"coupled_{drafts}", rows3, [0, 3], [drafts], seed=777, stream=7, positions=[20, 21, 22],
                           mode="coupled"))
    cases.append(_case("large_k_fused", np.zeros((1, 100)), [0, 1], np.empty((1, 0), np.int64), top_k=65))
    cases.append(_case("rng_extremes", np.zeros((3, 80)), [0, 1, 2, 3], np.empty((3, 0), np.int64),
                       top_k=[0, 20, 65], seed=[0, 2**63, 2**64 - 1], stream=[0, 2**32 - 1, 9],
                       positions=[0, 2**32 - 1, 100]))
    cases.append(_case("noncontiguous_out", np.zeros((3, 4)), [0, 1, 3], [[-1], [2]]))
    for offsets in ([0, 1, 2],):
        cases.append(_case("two_requests", np.zeros((2, 4)), offsets, np.empty((2, 0), np.int64)))
    # Contract edges (tests/edge/test_contract_edges.py)
    cases.append(_case("reject_first", [[0., -np.inf], [0., 0.]], [0, 2], [[1]], seed=123, stream=0, positions=[4, 5]))
    cases.append(_case("reject_middle", [[0., -np.inf], [-np.inf, 0.], [0., 0.]], [0, 3], [[0, 0]], seed=456, stream=0,
                       positions=[4, 5, 6]))
    cases.append(_case("later_row_atomic", [[0., -np.inf], [np.nan, 0.]], [0, 2], [[1]], seed=5, stream=0,
                       positions=[0, 1]))
    for draft in [-1, 2]:
        cases.append(_case(f"invalid_draft_{draft}", np.zeros((2, 2)), [0, 2], [[draft]], seed=3, stream=0,
                           positions=[0, 1]))
    cases.append(_case("seed_extremes", np.zeros((2, 2)), [0, 1, 2], np.empty((2, 0), np.int64),
                       seed=[2**64 - 1, 0], stream=[2**32 - 1, 0], positions=[2**32 - 1, 0]))
    cases.append(_case("metadata_before_no_valid", [[-np.inf] * 2] * 2, [0, 2], [[2]], seed=0, stream=0,
                       positions=[0, 1]))
    for params in [dict(temperature=-1.), dict(temperature=np.nan), dict(top_p=0.), dict(top_p=1.1),
                   dict(min_p=-.1), dict(min_p=1.1), dict(top_k=-1)]:
        name = "invalid_" + "_".join(f"{k}{v}" for k, v in params.items())
        cases.append(_case(name, [[0., 1.]], [0, 1], np.empty((1, 0), np.int64), **params))
    cases.append(_case("greedy_tie", [[2., 2., 1.]], [0, 1], np.empty((1, 0), np.int64), temperature=0.))
    cases.append(_case("greedy_tie_mask", [[2., 2., 1.]], [0, 1], np.empty((1, 0), np.int64), temperature=0.,
                       mask=np.array([[6]], np.int32)))
    cases.append(_case("minp_equal_keeps", [[0., 0., -10.]], [0, 1], np.empty((1, 0), np.int64), min_p=1.))
    # Identity and permutation (tests/invariance/test_identity.py)
    rowsi = np.array([[1., 2., 3., 0.], [4., 0., 1., 2.], [0., 0., 0., 0.]])
    cases.append(_case("identity", rowsi, [0, 1, 2, 3], np.empty((3, 0), np.int64), seed=[12, 99, 123],
                       stream=[0, 1, 3], positions=[100, 5, 12]))
    rows4 = np.array([[0., 1., -1.], [1., 1., 0.], [2., -1., 0.], [-2., 0., 1.]])
    for seed in [0, 1, 0xFFFFFFFFFFFFFFFF]:
        for drafts in [(0, 0, 0), (1, 2, 0), (2, 2, 2)]:
            cases.append(_case(f"coupled_spec_{seed}_{drafts}", rows4, [0, 4], [drafts], seed=seed, stream=17,
                               positions=[10, 11, 12, 13], mode="coupled"))
    ragged = np.arange(28, dtype=float).reshape(7, 4) % 7
    cases.append(_case("ragged", ragged, [0, 3, 5, 7], [[0, 1, -1], [2, -1, -1], [1, -1, -1]], seed=[30, 40, 50],
                       stream=[2, 3, 4], positions=[0, 1, 2, 8, 9, 10, 11], mode="coupled"))
    # Hand-computed distributions (tests/exact/test_hand_examples.py), sampled
    for i, (w, kw) in enumerate([([1, 1, 1, 1], {}), ([97, 1, 1, 1], {}), ([8, 4, 2, 1], dict(min_p=.75)),
                                 ([1, 1, 1, 1], dict(top_p=.5)), ([1, 1, 1, 1], dict(top_p=float(np.nextafter(.5, 1)))),
                                 ([4, 2, 2, 1], dict(top_k=2)), ([8, 4, 2, 1], dict(min_p=.2, top_k=2, top_p=.7)),
                                 ([16, 4, 1], dict(temperature=2.))]):
        logits = np.log(np.asarray([w] * 8, dtype=np.float64))
        cases.append(_case(f"hand_{i}", logits, np.arange(9), np.empty((8, 0), np.int64), seed=list(range(8)),
                           stream=5, positions=np.arange(8) * 3, **kw))
    return cases


def random_cases(count=16, seed=2026):
    """Random batches as in the reference's fused-path test: vocabularies 37 / 300 / 2500,
    ties, -inf entries, masks, full-q and coupled requests, every filter."""
    g = np.random.default_rng(seed)
    cases = []
    for trial in range(count):
        vocab = int(g.choice([37, 300, 2500]))
        counts = g.integers(0, 4, size=6)
        offsets = np.concatenate([[0], np.cumsum(counts + 1)])
        rows = g.normal(scale=float(g.choice([1., 4.])), size=(offsets[-1], vocab))
        if trial % 2:
            rows = np.round(rows * 2) / 2
        rows[g.random(rows.shape) < .05] = -np.inf
        mask = workloads.packed_mask(g.random(rows.shape) < .8) if trial % 3 == 0 else None
        mode = "coupled" if trial % 4 == 3 else "ratio"
        kinds = ["one_hot" if mode == "coupled" or g.random() < .6 else "full" for _ in counts]
        top_k = [int(g.choice([0, 1, 3, vocab // 3, vocab])) for _ in counts]
        temperature = [float(g.choice([0., .4, 1., 1.7])) for _ in counts]
        min_p = [float(g.choice([0., 0., .02, .3])) for _ in counts]
        top_p = [float(g.choice([1., .9, .6])) for _ in counts]
        ids = g.integers(0, vocab, size=(len(counts), 3))
        seeds = g.integers(0, 2**63, size=len(counts), dtype=np.int64).astype(np.uint64) * np.uint64(2) + np.uint64(1)
        streams = g.integers(0, 2**32, size=len(counts))
        positions = g.integers(0, 2**32, size=offsets[-1])
        q = g.normal(scale=2., size=rows.shape) if "full" in kinds else None
        for dtype in ["float32", "bfloat16"]:
            cases.append(_case(f"random_{trial}_{dtype}", round_to(rows, dtype), offsets, ids, temperature=temperature,
                               top_k=top_k, top_p=top_p, min_p=min_p, draft_kind=kinds, seed=list(seeds),
                               stream=list(streams), positions=positions, mask=mask,
                               draft_logits=None if q is None else round_to(q, dtype), mode=mode, logit_dtype=dtype))
    return cases


def workload_case(name, requests=None, **kw):
    """A benchmark configuration (workloads.config) as a case, optionally a subset of requests."""
    w = workloads.config(name, **kw)
    if requests is not None:
        w = w.subset(requests)
    return case_of(w, f"{name}" + ("" if requests is None else f"_{len(list(requests))}req"))


def case_of(w, name):
    """A workloads.Workload as a case."""
    return dict(name=name,
                logits=w.logits, cu_rows=w.cu_rows, draft_ids=w.draft_ids, temperature=w.temperature,
                top_k=w.top_k, top_p=w.top_p, min_p=w.min_p, draft_kind=w.draft_kind, seed=w.seed,
                stream_id=w.stream_id, positions=w.positions, mask=w.mask, draft_logits=w.draft_logits,
                mode=w.mode, logit_dtype=str(w.logits.dtype))


def digest(case):
    """sha256 over a case's inputs (guards regenerated inputs against generator drift)."""
    h = hashlib.sha256()
    for key in ["logits", "cu_rows", "draft_ids", "temperature", "top_k", "top_p", "min_p", "draft_kind", "seed",
                "stream_id", "positions", "mask", "draft_logits"]:
        value = case.get(key)
        h.update(key.encode())
        if value is not None:
            h.update(np.ascontiguousarray(value).tobytes())
    return h.hexdigest()


def oracle_inputs(case, module):
    """Keyword arguments for ``module.verify_reference`` (the oracle or the reference's own)."""
    params = module.RequestParams(
        temperature=list(case["temperature"]), top_k=[int(k) for k in case["top_k"]], top_p=list(case["top_p"]),
        min_p=list(case["min_p"]), draft_kind=["one_hot" if k == 0 else "full" for k in case["draft_kind"]])
    rng = module.RngKey([int(s) for s in case["seed"]], [int(s) for s in case["stream_id"]], case["positions"])
    logits = np.asarray(case["logits"], dtype=np.float64)
    q = case.get("draft_logits")
    return dict(target_logits=logits, cu_rows=case["cu_rows"], draft_ids=case["draft_ids"], params=params, rng=rng,
                mask=case.get("mask"), draft_logits=None if q is None else np.asarray(q, dtype=np.float64),
                mode=case["mode"])
