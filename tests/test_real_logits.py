"""Parity on the reference's real logits: 64 rows of Qwen3-8B bf16 logits
and the six cells of its agreement benchmark (bench/agreement.py:27-28),
against the reference fused path's saved outputs on an RTX 4090 and an
A10 (tests/golden/reference_outputs_8x8_*.npz; the reference reports
192/192 requests identical to its oracle, with 0 FP64 fallbacks).

* CPU: the oracle reproduces both GPUs' saved outputs on every cell.
* GPU: the B200 kernels reproduce the oracle and the saved outputs, through
  the drop-in API and through the C ABI."""
import numpy as np
import pytest

import oracle
from tests import cases as C
from tests import golden_io

CELLS = golden_io.real_logit_cells()


def _oracle(case):
    out = oracle.verify_reference(**C.oracle_inputs(case, oracle))
    return out.tokens, out.accepted_len, out.status


def _same(got, want, context):
    tokens, accepted, status = (np.asarray(x) for x in want)
    np.testing.assert_array_equal(np.asarray(got[2])[:len(status)], status, err_msg=f"status {context}")
    np.testing.assert_array_equal(np.asarray(got[0])[:len(status), :tokens.shape[1]], tokens, err_msg=f"tokens {context}")
    np.testing.assert_array_equal(np.asarray(got[1])[:len(status)], accepted, err_msg=f"accepted_len {context}")


@pytest.mark.parametrize("cell", CELLS, ids=lambda c: c[0])
def test_oracle_reproduces_the_reference_gpus_on_real_logits(cell):
    name, case, saved = cell
    got = _oracle(case)
    assert (got[2] == 0).all()
    for gpu, outputs in saved.items():
        _same(got, outputs, f"{name} vs the reference on {gpu}")


@pytest.mark.gpu
@pytest.mark.parametrize("cell", CELLS, ids=lambda c: c[0])
def test_kernels_reproduce_the_oracle_and_the_reference_on_real_logits(cell):
    from tests.gpu_helpers import device_inputs, run_abi, run_api

    name, case, saved = cell
    expected = _oracle(case)
    out, work = run_api(case)
    got_api = (out.tokens.cpu().numpy(), out.accepted_len.cpu().numpy(), out.status.cpu().numpy())
    print(name, "fp64 fallbacks:", work.fallbacks())
    _same(got_api, expected, f"{name} (API) vs oracle")
    for gpu, outputs in saved.items():
        _same(got_api, outputs, f"{name} (API) vs the reference on {gpu}")
    for list_max in (256, 0):
        got = run_abi(device_inputs(case), mode="ratio", list_max=list_max)
        _same(got, expected, f"{name} (C ABI, list_max {list_max}) vs oracle")
