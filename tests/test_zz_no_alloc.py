"""es_verify_static, the entry point that allocates nothing: its scratch is a
fixed area of static device memory in the library (one per device). It must
give exactly what es_verify gives with a caller-provided workspace, on two
calls in a row, and refuse batches beyond its scratch before enqueueing
anything.

The file name keeps it last in collection: it has to pass both in a fresh
process (where its first call does the scratch set-up) and after every other
test has run in the same process.
"""
import ctypes

import numpy as np
import pytest

from exactsample_b200 import capi
from tests import cases as C
from tests.gpu_helpers import device_inputs, outputs
from tests.test_abi import args as host_args

MODES = {"ratio": 0, "coupled": 1}


def test_batches_beyond_the_static_scratch_are_refused():
    lib = capi.load()
    a = host_args(rows=capi.STATIC_MAX_ROWS + 1, vocab=8, requests=1)
    a.workspace = capi.Tensor()
    assert lib.es_verify_static(ctypes.byref(a), None) == -2
    message = lib.es_last_error().decode()
    assert str(capi.STATIC_MAX_ROWS) in message and "es_verify with a workspace" in message


def test_a_caller_workspace_is_refused():
    lib = capi.load()
    a = host_args(rows=2, vocab=8, requests=1)  # carries a workspace
    assert lib.es_verify_static(ctypes.byref(a), None) == -1
    assert "leave workspace empty" in lib.es_last_error().decode()


def _reset(t):
    t["tokens"].fill_(-777)
    for name in ["accepted_len", "status", "path_used"]:
        t[name].fill_(-777)


def _cases():
    return [
        ("C1", C.workload_case("C1")),
        ("C3a_8", C.workload_case("C3a", requests=range(8))),
        ("C3b_ratio_full_4", C.workload_case("C3b_ratio_full", requests=range(4))),
        ("C4_19", C.workload_case("C4", requests=range(19))),
    ]


@pytest.mark.gpu
@pytest.mark.parametrize("dispatch", [2, 1], ids=["fused", "reference"])
def test_static_scratch_matches_es_verify_on_two_calls_in_a_row(dispatch):
    import torch

    for name, case in _cases():
        t = device_inputs(case, reference=dispatch == 1)
        tensors = {k: v for k, v in t.items() if not k.startswith("_")}
        kw = dict(mode=MODES[case["mode"]], dispatch=dispatch, max_draft=t["_max_draft"])
        capi.call(tensors, **kw)
        torch.cuda.synchronize()
        expected = outputs(t)
        assert (expected[2] != -777).all(), name
        for attempt in range(2):
            _reset(t)
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info()[0]
            allocations = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
            capi.call(tensors, static_scratch=True, **kw)
            torch.cuda.synchronize()
            if attempt == 1:  # set-up is done: the call itself takes no device memory
                assert torch.cuda.memory_stats().get("allocation.all.allocated", 0) == allocations, name
                # Device-wide free memory also sees other processes on the GPU:
                # only a decrease can point at this call.
                assert torch.cuda.mem_get_info()[0] >= free_before, \
                    f"{name}: device free memory fell during es_verify_static (this call, or another process)"
            got = outputs(t)
            for g, e, what in zip(got, expected, ["tokens", "accepted_len", "status", "path_used"]):
                np.testing.assert_array_equal(g, e, err_msg=f"{name} call {attempt + 1}: {what}")


@pytest.mark.gpu
def test_static_scratch_at_its_largest_batch():
    import torch

    rows = capi.STATIC_MAX_ROWS
    g = np.random.default_rng(7)
    logits = g.normal(0.0, 2.0, (rows, 1000)).astype(np.float32)
    case = C._case("static_max", logits, np.arange(rows + 1), C._drafts(np.empty((rows, 0), np.int64), rows),
                   temperature=0.7, top_k=20, top_p=0.9, logit_dtype="float32")
    t = device_inputs(case)
    tensors = {k: v for k, v in t.items() if not k.startswith("_")}
    capi.call(tensors, max_draft=0)
    torch.cuda.synchronize()
    expected = outputs(t)
    _reset(t)
    capi.call(tensors, max_draft=0, static_scratch=True)
    torch.cuda.synchronize()
    for g_, e in zip(outputs(t), expected):
        np.testing.assert_array_equal(g_, e)
    # One row more is refused before anything is enqueued: outputs untouched.
    bigger = device_inputs(C._case("static_over", np.zeros((rows + 1, 8), np.float32), np.arange(rows + 2),
                                   C._drafts(np.empty((rows + 1, 0), np.int64), rows + 1), logit_dtype="float32"))
    with pytest.raises(capi.AbiError, match="at most 4096 target rows"):
        capi.call({k: v for k, v in bigger.items() if not k.startswith("_")}, max_draft=0, static_scratch=True)
    torch.cuda.synchronize()
    assert (bigger["status"].cpu().numpy() == -777).all()
