"""C5a at full size on one GPU: 4,096 requests of fp32 [4096, 151936] logits
with Qwen3 settings (2.49 GB), bit-exact against the CPU oracle, and the same
outputs when the requests are split into 2, 4 or 8 contiguous ranges and
each range is its own call, as N GPUs sharding by request rows take them
(the contract's slot and shard independence, reference docs/rng.md; the
reference's large-batch check, tests/invariance/large_gpu.py:35-44)."""
import numpy as np
import pytest

import oracle
import workloads
from tests import cases as C

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _device_call(w, r0, r1):
    """One call over requests [r0, r1) of a one-row-per-request workload
    through the C ABI; returns (tokens, accepted_len, status) on the host."""
    import torch
    from exactsample_b200 import capi

    n = r1 - r0
    dev = "cuda"
    t = lambda a, dt: torch.as_tensor(np.ascontiguousarray(a), dtype=dt, device=dev)
    tensors = dict(
        target_logits=torch.as_tensor(w.logits[r0:r1], device=dev),
        cu_rows=torch.arange(n + 1, dtype=torch.int64, device=dev),
        draft_ids=torch.full((n, 1), -1, dtype=torch.int64, device=dev),
        temperature=t(w.temperature[r0:r1], torch.float64), top_k=t(w.top_k[r0:r1], torch.int64),
        top_p=t(w.top_p[r0:r1], torch.float64), min_p=t(w.min_p[r0:r1], torch.float64),
        draft_kind=t(w.draft_kind[r0:r1], torch.int64), seeds=t(w.seeds_int64()[r0:r1], torch.int64),
        stream_ids=t(w.stream_id[r0:r1], torch.int64), positions=t(w.positions[r0:r1], torch.int64),
        workspace=torch.zeros(capi.workspace_bytes(n, w.vocab), dtype=torch.uint8, device=dev),
        tokens=torch.full((n, 2), -777, dtype=torch.int64, device=dev),
        accepted_len=torch.full((n,), -777, dtype=torch.int32, device=dev),
        status=torch.full((n,), -777, dtype=torch.int32, device=dev),
        path_used=torch.full((n,), -777, dtype=torch.int32, device=dev))
    capi.call(tensors, max_draft=1)
    torch.cuda.synchronize()
    return tuple(tensors[k].cpu().numpy() for k in ("tokens", "accepted_len", "status"))


def test_c5a_full_size_matches_the_oracle_and_any_request_split():
    w = workloads.config("C5a")
    assert w.logits.shape == (4096, workloads.VOCAB) and w.logits.dtype == np.float32
    whole = _device_call(w, 0, w.requests)
    assert (whole[2] == 0).all()
    for shards in (2, 4, 8):
        bounds = np.linspace(0, w.requests, shards + 1).astype(int)
        parts = [_device_call(w, int(a), int(b)) for a, b in zip(bounds[:-1], bounds[1:])]
        for field, name in enumerate(("tokens", "accepted_len", "status")):
            np.testing.assert_array_equal(np.concatenate([p[field] for p in parts]), whole[field],
                                          err_msg=f"{name} with {shards} request ranges")
    case = C.case_of(w, "C5a")
    expected = oracle.verify_reference(**C.oracle_inputs(case, oracle))
    np.testing.assert_array_equal(whole[2], expected.status)
    np.testing.assert_array_equal(whole[0][:, :1], expected.tokens[:, :1])
    np.testing.assert_array_equal(whole[1], expected.accepted_len)
