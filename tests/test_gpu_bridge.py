"""The engine-side step (exactsample_b200.bridge.decode_step) on the GPU: the
staged parameters, gathered drafts and device-densified grammar mask give
exactly what a direct verify call with hand-built inputs gives, and the
status copy delivers the committed tokens."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_decode_step_equals_a_direct_call():
    import torch

    from exactsample_b200 import bridge
    from exactsample_b200.cuda import CudaRequestParams, CudaRngKey, plan, verify

    g = np.random.default_rng(8)
    vocab, max_draft = 1000, 3
    offsets = np.array([0, 3, 4, 6, 10])  # 2, 0, 1 and 3 drafts
    requests, rows = offsets.size - 1, int(offsets[-1])
    logits = torch.as_tensor(g.normal(0, 2, (rows, vocab)), dtype=torch.float32, device="cuda")
    row_tokens = torch.as_tensor(g.integers(0, vocab, rows), dtype=torch.int32, device="cuda")
    positions = torch.as_tensor(np.concatenate([100 * r + np.arange(offsets[r + 1] - offsets[r])
                                                for r in range(requests)]), device="cuda")
    params = dict(temperature=np.array([0.7, 1.0, 0.0, 0.9]), top_k=np.array([20, vocab, 0, 50]),
                  top_p=np.array([0.95, 1.0, 1.0, 0.8]), min_p=np.array([0.0, 0.0, 0.0, 0.02]),
                  seeds=np.array([11, 2**63 + 5, 13, 14], np.uint64))
    words = (vocab + 31) // 32
    # Requests "r3" and "r0" are grammar-constrained, their bitmask rows in that order.
    allowed = g.random((4 + 3, vocab)) < 0.3
    padded = np.zeros((allowed.shape[0], words * 32), bool)
    padded[:, :vocab] = allowed
    bitmask_np = np.packbits(padded, axis=1, bitorder="little").view("<u4").view(np.int32)
    grammar = (["r0", "r1", "r2", "r3"], ["r3", "r0"], torch.as_tensor(bitmask_np, device="cuda"))

    for mode in ["coupled", "ratio"]:
        work = plan(rows, requests, max_draft, vocab)
        out = work.allocate_output()
        staging = bridge.StepStaging(requests, max_draft, vocab)
        mask_buffer = torch.empty((rows, words), dtype=torch.int32, device="cuda")
        got, counts, copy = bridge.decode_step(logits, offsets, row_tokens, positions, staging=staging, plan=work,
                                               out=out, grammar=grammar, mask_buffer=mask_buffer, mode=mode,
                                               **params)
        status, committed = copy.get()

        # The same call built by hand.
        index = offsets[:-1, None] + 1 + np.arange(max_draft)
        index[np.arange(max_draft) >= (np.diff(offsets) - 1)[:, None]] = -1
        rt = row_tokens.cpu().numpy()
        drafts = np.where(index >= 0, rt[np.clip(index, 0, None)], -1)
        dense = bridge.grammar_mask_rows(grammar[0], offsets, grammar[1], bitmask_np, vocab)
        t = lambda a, dt: torch.as_tensor(np.asarray(a), dtype=dt, device="cuda")
        direct = plan(rows, requests, max_draft, vocab)
        expected = direct.allocate_output()
        verify(logits, t(offsets, torch.int64), t(drafts, torch.int64),
               params=CudaRequestParams(t(params["temperature"], torch.float64),
                                        t(np.where(params["top_k"] == vocab, 0, params["top_k"]), torch.int64),
                                        t(params["top_p"], torch.float64), t(params["min_p"], torch.float64),
                                        t(np.zeros(requests), torch.int64)),
               rng=CudaRngKey(t(params["seeds"].view(np.int64), torch.int64), t(np.zeros(requests), torch.int64),
                              positions),
               plan=direct, out=expected, mask=t(dense, torch.int32), mode=mode)
        torch.cuda.synchronize()
        assert got.tokens[:requests].tolist() == expected.tokens[:requests].tolist(), mode
        assert got.status[:requests].tolist() == expected.status[:requests].tolist() == status.tolist(), mode
        assert (status == 0).all()
        assert counts.tolist() == (expected.accepted_len[:requests] + 1).tolist()
        acc = expected.accepted_len[:requests].tolist()
        assert committed == [expected.tokens[r, :acc[r] + 1].tolist() for r in range(requests)]
        # The constrained requests' tokens are ones their grammar rows allow.
        for r, first_mask_row in [(3, 0), (0, 4)]:
            for i, token in enumerate(committed[r]):
                assert allowed[first_mask_row + i, token], (mode, r, i, token)
