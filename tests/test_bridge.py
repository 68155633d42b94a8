"""The engine-side step around a verify call (exactsample_b200.bridge), on
CPU tensors: grammar-mask densification (the reference's
tests/test_vllm_bridge.py:133-144 scenario of a reordered constrained
subset), parameter staging, the draft gather and the committed counts."""
import numpy as np
import pytest
import torch

from exactsample_b200 import bridge
from exactsample_b200.cuda import CudaOutput


def test_constrained_requests_in_their_own_order_keep_every_row():
    # Requests own rows [0,3) [3,4) [4,6) [6,10); "d" and "a" are constrained,
    # their bitmask rows listed in that order.
    ids = ["a", "b", "c", "d"]
    offsets = np.array([0, 3, 4, 6, 10])
    bitmask = (np.arange(14, dtype=np.int32) * 7).reshape(7, 2)
    dense = bridge.grammar_mask_rows(ids, offsets, ["d", "a"], bitmask, 40)
    np.testing.assert_array_equal(dense[6:10], bitmask[:4])
    np.testing.assert_array_equal(dense[0:3], bitmask[4:7])
    np.testing.assert_array_equal(dense[3:6], np.full((3, 2), -1, np.int32))
    sources = bridge.grammar_row_sources(ids, offsets, ["d", "a"], 7)
    assert sources.tolist() == [4, 5, 6, -1, -1, -1, 0, 1, 2, 3]
    # The device form gives the same mask.
    out = torch.zeros((10, 2), dtype=torch.int32)
    bridge.densify_grammar_mask(torch.as_tensor(bitmask), sources, out)
    np.testing.assert_array_equal(out.numpy(), dense)
    # Into a caller's buffer.
    buffer = np.zeros((10, 2), np.int32)
    assert bridge.grammar_mask_rows(ids, offsets, ["d", "a"], bitmask, 40, out=buffer) is buffer


@pytest.mark.parametrize("ids,grammar,rows,message", [
    (["a", "a"], ["a"], 1, "duplicate"),
    (["a", "b"], ["b", "b"], 2, "duplicate"),
    (["a", "b"], ["c"], 1, "missing"),
    (["a", "b"], ["a", "b"], 1, "fewer rows"),
    (["a", "b"], ["a"], 2, "unused rows"),
])
def test_grammar_layout_errors(ids, grammar, rows, message):
    with pytest.raises(ValueError, match=message):
        bridge.grammar_mask_rows(ids, [0, 1, 2], grammar, np.ones((rows, 1), np.int32), 8)


def test_grammar_bitmask_and_buffer_shapes_are_checked():
    with pytest.raises(ValueError, match="shape/dtype"):
        bridge.grammar_mask_rows(["a"], [0, 1], ["a"], np.ones((1, 2), np.int64), 40)
    with pytest.raises(ValueError, match="shape/dtype"):
        bridge.grammar_mask_rows(["a"], [0, 1], ["a"], np.ones((1, 2), np.int32), 100)
    with pytest.raises(ValueError, match="shape/dtype"):
        bridge.grammar_mask_rows(["a"], [0, 1], ["a"], np.ones((1, 2), np.int32), 40, out=np.zeros((2, 2), np.int32))


def test_staging_packs_parameters_and_draft_rows():
    staging = bridge.StepStaging(4, 3, 1000, device="cpu")
    offsets = np.array([0, 4, 5, 7])  # 3, 0 and 1 drafts
    step = staging.stage(offsets, temperature=[0.6, 1.0, 0.7], top_k=[20, 1000, 0], top_p=[0.95, 1.0, 1.0],
                         min_p=[0.0, 0.0, 0.05], seeds=np.array([2**64 - 1, 5, 7], np.uint64))
    assert step.params.temperature.tolist() == [0.6, 1.0, 0.7]
    assert step.params.top_k.tolist() == [20, 0, 0]  # top_k equal to the vocabulary means none
    assert step.params.min_p.tolist() == [0.0, 0.0, 0.05]
    assert step.params.draft_kind.tolist() == [0, 0, 0]
    assert step.seeds.tolist() == [-1, 5, 7]  # uint64 bits in int64 storage
    assert step.draft_index.tolist() == [[1, 2, 3], [-1, -1, -1], [6, -1, -1]]
    assert step.top_k_top_p and step.counts.tolist() == [3, 0, 1]
    plain = staging.stage(np.array([0, 1]), temperature=[1.0], top_k=[0], top_p=[1.0], min_p=[0.0], seeds=[3])
    assert not plain.top_k_top_p


def test_staging_rejects_layouts_beyond_its_capacity():
    staging = bridge.StepStaging(2, 1, 100, device="cpu")
    kw = dict(temperature=[1.0] * 2, top_k=[0] * 2, top_p=[1.0] * 2, min_p=[0.0] * 2, seeds=[1, 2])
    with pytest.raises(bridge.DecodeStepError, match="draft counts"):
        staging.stage([0, 3, 4], **kw)  # 2 drafts > 1
    with pytest.raises(bridge.DecodeStepError, match="draft counts"):
        staging.stage([0, 0, 1], **kw)  # a request without rows
    with pytest.raises(bridge.DecodeStepError, match="ragged"):
        staging.stage([0, 1, 2, 3], **{k: v * 2 for k, v in kw.items()})  # 3 requests > 2
    with pytest.raises(bridge.DecodeStepError, match="one value per request"):
        staging.stage([0, 1, 2], **{**kw, "seeds": [1]})


def test_drafts_are_read_from_the_rows_after_each_requests_first():
    row_tokens = torch.tensor([10, 11, 12, 13, 14, 15, 16], dtype=torch.int32)
    index = torch.tensor([[1, 2, 3], [-1, -1, -1], [6, -1, -1]])
    assert bridge.gather_drafts(row_tokens, index).tolist() == [[11, 12, 13], [-1, -1, -1], [16, -1, -1]]


def test_failed_requests_commit_nothing():
    out = CudaOutput(tokens=torch.tensor([[5, 6, 7], [8, -1, -1], [-1, -1, -1]]),
                     accepted_len=torch.tensor([2, 0, 0], dtype=torch.int32),
                     status=torch.tensor([0, 0, 2], dtype=torch.int32), path_used=torch.zeros(3, dtype=torch.int32))
    assert bridge.committed_counts(out, 3).tolist() == [3, 1, 0]
    status, committed = bridge.StatusCopy(out, 3).get()
    assert status.tolist() == [0, 0, 2] and committed == [[5, 6, 7], [8], []]
