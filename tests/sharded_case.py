"""Runs one parity case as a vocabulary-sharded call (test infrastructure):
either as N shards emulated on one GPU (N plans in one process, the four
steps of a call issued shard by shard), or as this process's shard of a
torch.distributed job. Returns numpy outputs in the order of run_abi."""
from __future__ import annotations

import numpy as np


def _inputs(case, dtype=None, device="cuda"):
    from tests.gpu_helpers import device_inputs
    return device_inputs(case, dtype=dtype, device=device)


def _fill(plan, t, rows):
    cols = plan.cols
    lo = plan.rank * cols
    plan.logits[:rows].copy_(t["target_logits"][:, lo:lo + plan.width])
    if plan.full_q:
        plan.draft_logits[:rows].copy_(t["draft_logits"][:, lo:lo + plan.width])


def _call_args(t, case):
    from exactsample_b200.cuda import CudaRequestParams, CudaRngKey
    params = CudaRequestParams(t["temperature"], t["top_k"], t["top_p"], t["min_p"], t["draft_kind"])
    rng = CudaRngKey(t["seeds"], t["stream_ids"], t["positions"])
    return dict(params=params, rng=rng, mask=t.get("mask"), mode=case["mode"])


def _outputs(plan, requests):
    o = plan.out
    return (o.tokens[:requests].cpu().numpy(), o.accepted_len[:requests].cpu().numpy(),
            o.status[:requests].cpu().numpy(), o.path_used[:requests].cpu().numpy())


def emulated(case, shards, *, dtype=None, calls=1):
    """Every shard's outputs (a list of run_abi-like tuples) after `calls` calls."""
    import torch
    from exactsample_b200.sharded import ShardedPlan

    t = _inputs(case, dtype)
    rows, vocab = t["target_logits"].shape
    requests = case["cu_rows"].size - 1
    full_q = t.get("draft_logits") is not None
    # Column-pulling mode only: per-phase kernels wait on one another, so
    # they never run as separate launches on one GPU.
    plans = [ShardedPlan(rows, requests, t["_max_draft"], vocab, shards=shards, rank=g,
                         dtype=t["target_logits"].dtype, full_q=full_q, connect=False, phases=False)
             for g in range(shards)]
    try:
        entries = [p.entry for p in plans]
        for p in plans:
            p.connect(entries)
        kw = _call_args(t, case)
        for _ in range(calls):
            for p in plans:
                _fill(p, t, rows)
                p.out.tokens.fill_(-777)
                p.epoch += 1
                p.signal_ready()
            for p in plans:
                p.launch(rows, t["cu_rows"], t["draft_ids"], **kw)
            for p in plans:
                p.signal_done()
            for p in plans:
                p.wait_done()
        torch.cuda.synchronize()
        assert sum(p.timeouts() for p in plans) == 0
        return [_outputs(p, requests) for p in plans]
    finally:
        for p in plans:
            p.close()


def distributed(case, group=None, *, dtype=None, phases=True, calls=1):
    """This rank's outputs of a sharded call (per-phase or column-pulling)
    over the torch.distributed job, after `calls` calls on the same plan."""
    import torch
    import torch.distributed as dist
    from exactsample_b200.sharded import ShardedPlan, verify_sharded

    t = _inputs(case, dtype, device=torch.device("cuda", torch.cuda.current_device()))
    rows, vocab = t["target_logits"].shape
    requests = case["cu_rows"].size - 1
    full_q = t.get("draft_logits") is not None
    plan = ShardedPlan(rows, requests, t["_max_draft"], vocab, shards=dist.get_world_size(group),
                       rank=dist.get_rank(group), dtype=t["target_logits"].dtype, full_q=full_q, group=group,
                       phases=phases)
    try:
        _fill(plan, t, rows)
        for _ in range(calls):
            plan.out.tokens.fill_(-777)
            verify_sharded(plan, rows, t["cu_rows"], t["draft_ids"], **_call_args(t, case))
        torch.cuda.synchronize()
        assert plan.timeouts() == 0
        return _outputs(plan, requests)
    finally:
        dist.barrier(group)
        plan.close()
