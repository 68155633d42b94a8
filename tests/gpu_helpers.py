"""Device-side helpers for the GPU tests: move a parity case (tests/cases.py)
to the GPU and run it through the C ABI (exactsample_b200.capi) or through the
drop-in Python API (exactsample_b200.cuda)."""
from __future__ import annotations

import numpy as np

TORCH_DTYPES = {}


def torch_dtype(name):
    import torch
    return {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32,
            "float64": torch.float64}[name]


def _tensor(value, dtype, strided, device="cuda"):
    import torch
    t = torch.as_tensor(np.array(value, copy=True), dtype=dtype, device=device)
    if strided and t.ndim and t.shape[-1]:
        backing = torch.empty((*t.shape[:-1], t.shape[-1] * 2), dtype=dtype, device=device)
        backing[..., ::2] = t
        t = backing[..., ::2]
    return t


def device_inputs(case, *, dtype=None, strided=False, max_draft=None, reference=False, device="cuda"):
    """es_args-named torch tensors for a case, with outputs and a workspace."""
    import torch
    from exactsample_b200 import capi

    dt = torch_dtype(dtype or case["logit_dtype"])
    logits = np.asarray(case["logits"], dtype=np.float64)
    rows, vocab = logits.shape
    requests = case["cu_rows"].size - 1
    ids = np.asarray(case["draft_ids"], dtype=np.int64)
    width = ids.shape[1] if max_draft is None else max_draft
    seeds = np.asarray(case["seed"], dtype=np.uint64).view(np.int64)
    t = dict(
        target_logits=_tensor(logits, dt, strided, device),
        cu_rows=_tensor(case["cu_rows"], torch.int64, strided, device),
        draft_ids=_tensor(ids, torch.int64, strided, device),
        temperature=_tensor(case["temperature"], torch.float64, strided, device),
        top_k=_tensor(case["top_k"], torch.int64, strided, device),
        top_p=_tensor(case["top_p"], torch.float64, strided, device),
        min_p=_tensor(case["min_p"], torch.float64, strided, device),
        draft_kind=_tensor(case["draft_kind"], torch.int64, strided, device),
        seeds=_tensor(seeds, torch.int64, strided, device),
        stream_ids=_tensor(case["stream_id"], torch.int64, strided, device),
        positions=_tensor(case["positions"], torch.int64, strided, device),
    )
    if case.get("mask") is not None:
        t["mask"] = _tensor(case["mask"], torch.int32, strided, device)
    if case.get("draft_logits") is not None:
        t["draft_logits"] = _tensor(np.asarray(case["draft_logits"], np.float64), dt, strided, device)
    t["workspace"] = torch.zeros(capi.workspace_bytes(rows, vocab, reference), dtype=torch.uint8, device=device)
    t["tokens"] = torch.full((requests, width + 1), -777, dtype=torch.int64, device=device)
    for name in ["accepted_len", "status", "path_used"]:
        t[name] = torch.full((requests,), -777, dtype=torch.int32, device=device)
    t["_max_draft"] = width
    return t


# Workspace poison: every call through run_abi starts from a workspace filled
# with this byte (the kernels must initialise whatever they read), and after
# the call the bytes past the records the call may use must still hold it.
POISON = 0xA5


def workspace_records(rows: int) -> int:
    """An upper bound on the workspace bytes a call over `rows` target rows
    uses: the 8-byte header, a 32-byte result and a 4-byte arrival counter
    per row, 64 bytes of diagnostics, up to 15 bytes of alignment and an
    80-byte context record per row (exactsample_b200/csrc/es_layout.cuh)."""
    return 8 if rows == 0 else 8 + rows * 36 + 64 + 15 + rows * 80


def diagnostics(t):
    """The workspace's diagnostic counters: near_ties, wait_timeouts,
    check_failures and first_site (checked builds count failed bounds checks)."""
    rows = t["target_logits"].shape[0]
    at = 8 + rows * 36
    d = t["workspace"][at:at + 16].cpu().numpy().view(np.uint32)
    return dict(near_ties=int(d[0]), wait_timeouts=int(d[1]), check_failures=int(d[2]), first_site=int(d[3]))


def run_abi(t, *, mode="ratio", dispatch="fused", list_max=256):
    """One call through the C ABI on a poisoned workspace; checks that nothing
    was written past the call's records and that no bounds check failed
    (in a checked build); returns numpy (tokens, accepted, status, path)."""
    import torch
    from exactsample_b200 import capi

    ws = t["workspace"]
    ws.fill_(POISON)
    capi.call({k: v for k, v in t.items() if not k.startswith("_")}, mode={"ratio": 0, "coupled": 1}[mode],
              dispatch={"auto": 0, "reference": 1, "fused": 2}[dispatch], max_draft=t["_max_draft"],
              list_max=list_max)
    torch.cuda.synchronize()
    rows, vocab = t["target_logits"].shape
    used = workspace_records(rows)
    if dispatch == "reference":  # the FP64 kernel's scratch: 16 bytes per token per row, 16-byte aligned
        used = (used + 15) // 16 * 16 + rows * vocab * 16
    tail = ws[used:]
    assert bool((tail == POISON).all()), "a call wrote past its workspace records"
    if t["cu_rows"].numel() > 1 and t["target_logits"].shape[0] > 0:
        d = diagnostics(t)
        assert d["check_failures"] == 0 and d["wait_timeouts"] == 0, d
    return outputs(t)


def outputs(t):
    return (t["tokens"].cpu().numpy(), t["accepted_len"].cpu().numpy(), t["status"].cpu().numpy(),
            t["path_used"].cpu().numpy())


def run_api(case, *, dtype=None, strided=False, mode=None, dispatch="auto", list_max=256, top_k_top_p=True):
    """One call through exactsample_b200.cuda (the drop-in API); returns (out, plan)."""
    from exactsample_b200.cuda import CudaRequestParams, CudaRngKey, plan, verify

    t = device_inputs(case, dtype=dtype, strided=strided, reference=dispatch == "reference")
    rows, vocab = case["logits"].shape
    requests = case["cu_rows"].size - 1
    work = plan(rows, requests, t["_max_draft"], vocab, reference=dispatch == "reference")
    work.list_max = list_max
    out = work.allocate_output()
    params = CudaRequestParams(t["temperature"], t["top_k"], t["top_p"], t["min_p"], t["draft_kind"])
    rng = CudaRngKey(t["seeds"], t["stream_ids"], t["positions"])
    verify(t["target_logits"], t["cu_rows"], t["draft_ids"], params=params, rng=rng, plan=work, out=out,
           draft_logits=t.get("draft_logits"), mask=t.get("mask"), mode=mode or case["mode"], dispatch=dispatch,
           top_k_top_p=top_k_top_p)
    work.synchronize()
    return out, work


def assert_same(got, expected, requests=None, context=""):
    """tokens / accepted_len / status equal to (tokens, accepted, status)."""
    tokens, accepted, status = (np.asarray(x) for x in expected)
    n = len(status) if requests is None else requests
    g_tokens, g_accepted, g_status = (np.asarray(x)[:n] for x in got[:3])
    np.testing.assert_array_equal(g_status, status[:n], err_msg=f"status {context}")
    np.testing.assert_array_equal(g_tokens[:, :tokens.shape[1]], tokens[:n], err_msg=f"tokens {context}")
    np.testing.assert_array_equal(g_accepted, accepted[:n], err_msg=f"accepted_len {context}")
