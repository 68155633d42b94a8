"""The drop-in Python API on the GPU: ownership, capacity, aliasing, strided
outputs, malformed offsets and refusals, as the reference's
tests/test_cuda.py:99-169 exercise them."""
import numpy as np
import pytest

from exactsample_b200 import Status
from tests import cases as C
from tests.gpu_helpers import device_inputs, run_api

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


def prepared(rows, offsets, ids, strided=False, **kw):
    """(verify keyword arguments, tensors) for a small case, like the reference's prepared_cuda."""
    from exactsample_b200.cuda import CudaRequestParams, CudaRngKey, plan
    case = C._case("api", np.asarray(rows, dtype=np.float64), offsets, C._drafts(ids, len(offsets) - 1), **kw)
    t = device_inputs(case, strided=strided)
    work = plan(case["logits"].shape[0], len(offsets) - 1, t["_max_draft"], case["logits"].shape[1], reference=True)
    args = dict(target_logits=t["target_logits"], cu_rows=t["cu_rows"], draft_ids=t["draft_ids"],
                params=CudaRequestParams(t["temperature"], t["top_k"], t["top_p"], t["min_p"], t["draft_kind"]),
                rng=CudaRngKey(t["seeds"], t["stream_ids"], t["positions"]), plan=work, out=work.allocate_output())
    return args


def test_workspace_conflict_and_separate_plans():
    import torch
    from exactsample_b200.cuda import verify
    args = prepared(np.zeros((1, 4)), [0, 1], np.empty((1, 0)))
    other = prepared(np.zeros((1, 4)), [0, 1], np.empty((1, 0)))
    # A first call loads the kernels (lazily, possibly for longer than the
    # sleep below); after it the first stream's call is still queued behind
    # the sleep when the second stream tries the same workspace.
    verify(**other)
    other["plan"].synchronize()
    first, second = torch.cuda.Stream(), torch.cuda.Stream()
    first.wait_stream(torch.cuda.current_stream())
    second.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(first):
        torch.cuda._sleep(1_000_000_000)  # about half a second
        verify(**args)
    with torch.cuda.stream(second):
        with pytest.raises(RuntimeError, match="in flight"):
            verify(**args)
        verify(**other)
    args["plan"].synchronize()
    other["plan"].synchronize()
    assert args["out"].tokens.cpu().tolist() == other["out"].tokens.cpu().tolist()


def test_capacity_and_large_k_on_fused_path():
    import torch
    from exactsample_b200.cuda import verify
    case = C._case("k65", np.zeros((1, 100)), [0, 1], np.empty((1, 0), np.int64), top_k=65)
    out, _ = run_api(case, dispatch="fused")
    assert out.path_used.cpu().tolist() == [1]
    args = prepared(np.zeros((1, 100)), [0, 1], np.empty((1, 0)))
    args["target_logits"] = torch.zeros((2, 100), device="cuda")
    with pytest.raises(ValueError, match="capacity"):
        verify(**args)


def test_output_alias_is_rejected():
    from exactsample_b200.cuda import verify
    args = prepared(np.zeros((1, 4)), [0, 1], np.empty((1, 0)))
    args["out"].tokens = args["rng"].seed.reshape(1, 1)
    with pytest.raises(RuntimeError, match="alias"):
        verify(**args)


def test_noncontiguous_outputs_keep_their_gaps():
    import torch
    from exactsample_b200.cuda import verify
    args = prepared(np.zeros((3, 4)), [0, 1, 3], [[-1], [2]], strided=True)
    out = args["out"]
    backing = torch.full((2, 4), -777, dtype=torch.int64, device="cuda")
    out.tokens = backing[:, ::2]
    for field in ["accepted_len", "status", "path_used"]:
        setattr(out, field, torch.empty(4, dtype=torch.int32, device="cuda")[::2])
    result = verify(**args)
    args["plan"].synchronize()
    assert torch.all(backing[:, 1::2] == -777).item()
    assert result.status.cpu().tolist() == [0, 0]


def test_invalid_offsets_do_not_write_tokens():
    from exactsample_b200.cuda import verify
    for offsets in [[1, 1, 2], [0, 2, 1], [0, -1, 2], [0, 1, 3]]:
        args = prepared(np.zeros((2, 4)), [0, 1, 2], np.empty((2, 0)))
        args["cu_rows"].copy_(__import__("torch").tensor(offsets, device="cuda"))
        out = verify(**args)
        args["plan"].synchronize()
        assert out.status.cpu().tolist() == [int(Status.INVALID_INPUT)] * 2
        assert out.tokens.cpu().tolist() == [[-1], [-1]]


def test_refusals():
    import torch
    from exactsample_b200.cuda import CudaRngKey, verify
    args = prepared(np.zeros((1, 4)), [0, 1], np.empty((1, 0)))
    with pytest.raises(ValueError, match="mode"):
        verify(**args, mode="other")
    with pytest.raises(TypeError):
        verify(**{**args, "rng": (1, 2, 3)})
    g = torch.cuda.CUDAGraph()
    with pytest.raises(RuntimeError, match="graph capture"):
        with torch.cuda.graph(g):
            verify(**args)
    args["plan"].synchronize()
    assert verify(**args).num_requests == 1


def test_fallback_counter_reads_zero_on_plain_rows():
    case = C.workload_case("C2a", list(range(8)))
    out, work = run_api(case)
    assert work.fallbacks() == 0
    assert (out.status[:8].cpu().numpy() == 0).all()


def test_capture_is_refused_by_default_and_replays_exactly_with_graphs():
    """The reference refuses graph capture (cuda.py:166-167); a plan made with
    graphs=True allows it, and replays of the captured call give what eager
    calls give on the same inputs, call after call."""
    import torch
    from exactsample_b200.cuda import CudaRequestParams, CudaRngKey, plan, verify
    cases = [C.workload_case("C2a", requests=range(8), master_seed=s) for s in (21, 22, 23)]
    t = device_inputs(cases[0])
    rows, vocab = cases[0]["logits"].shape
    requests = len(cases[0]["cu_rows"]) - 1
    params = CudaRequestParams(t["temperature"], t["top_k"], t["top_p"], t["min_p"], t["draft_kind"])
    rng = CudaRngKey(t["seeds"], t["stream_ids"], t["positions"])

    def call(work, out):
        verify(t["target_logits"], t["cu_rows"], t["draft_ids"], params=params, rng=rng, plan=work, out=out)

    refusing = plan(rows, requests, t["_max_draft"], vocab)
    refused_out = refusing.allocate_output()
    graph = torch.cuda.CUDAGraph()
    with pytest.raises(RuntimeError, match="graph capture"):
        with torch.cuda.graph(graph):
            call(refusing, refused_out)
    torch.cuda.synchronize()

    captured = plan(rows, requests, t["_max_draft"], vocab, graphs=True)
    out = captured.allocate_output()
    call(captured, out)  # an eager call first loads the kernels
    captured.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call(captured, out)
    eager = plan(rows, requests, t["_max_draft"], vocab)
    expected_out = eager.allocate_output()
    for case in cases:
        fresh = device_inputs(case)
        for name in ["target_logits", "seeds", "positions"]:
            t[name].copy_(fresh[name])
        out.tokens.fill_(-777)
        graph.replay()
        call(eager, expected_out)
        torch.cuda.synchronize()
        assert out.tokens[:requests].tolist() == expected_out.tokens[:requests].tolist()
        assert out.status[:requests].tolist() == expected_out.status[:requests].tolist()
    del graph


def test_a_workspace_aligned_to_8_bytes_only():
    """The C ABI asks for an 8-byte aligned workspace (bindings.cpp:106); the
    per-row records inside it are placed on 16-byte boundaries whatever its
    alignment, so a workspace at an odd multiple of 8 works the same."""
    import torch
    from exactsample_b200 import capi
    from tests.gpu_helpers import outputs
    case = C.workload_case("C3a", requests=range(6))
    t = device_inputs(case)
    tensors = {k: v for k, v in t.items() if not k.startswith("_")}
    capi.call(tensors, max_draft=t["_max_draft"])
    torch.cuda.synchronize()
    expected = outputs(t)
    backing = torch.zeros(t["workspace"].numel() + 8, dtype=torch.uint8, device="cuda")
    tensors["workspace"] = backing[8:]
    assert tensors["workspace"].data_ptr() % 16 == 8
    t["tokens"].fill_(-777)
    capi.call(tensors, max_draft=t["_max_draft"])
    torch.cuda.synchronize()
    for got, exp in zip(outputs(t), expected):
        np.testing.assert_array_equal(got, exp)
