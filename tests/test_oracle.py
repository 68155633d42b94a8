"""The CPU oracle pinned against the reference: Random123 known answers, the
reference suites' hand-computed examples, and the golden fixtures that the
reference's own oracle produced (tests/golden/make_golden.py)."""
import math

import numpy as np
import pytest

import oracle
from oracle import RequestParams, RngKey, Status, distribution, verify_reference
from tests import cases as C
from tests import golden_io


def test_random123_known_answers():
    # Published Random123 Philox4x32-10 known-answer vectors (kat_vectors).
    cases = [((0, 0, 0, 0), (0, 0), (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)),
             ((0xffffffff,) * 4, (0xffffffff,) * 2, (0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd)),
             ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0xa4093822, 0x299f31d0),
              (0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1))]
    for counter, key, expected in cases:
        assert oracle.philox4x32(counter, key) == expected


def test_lane_addressing_and_open_interval():
    expected = (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)
    for token, word in enumerate(expected):
        u = oracle.uniform(0, 0, 0, 0, token)
        assert u == (word + .5) / 4294967296 and 0 < u < 1


def _check(weights, expected, **kw):
    p, status = distribution(np.log(np.asarray(weights, dtype=np.float64)), **kw)
    assert status == Status.OK
    np.testing.assert_allclose(p, expected, rtol=1e-13, atol=1e-15)


def test_hand_computed_distributions():
    _check([1, 1, 1, 1], [.25] * 4)
    _check([97, 1, 1, 1], [.97, .01, .01, .01])
    _check([8, 4, 2, 1], [1, 0, 0, 0], min_p=.75)
    _check([1, 1, 1, 1], [.5, .5, 0, 0], top_p=.5)
    _check([1, 1, 1, 1], [1 / 3] * 3 + [0], top_p=np.nextafter(.5, 1.0))
    _check([4, 2, 2, 1], [2 / 3, 1 / 3, 0, 0], top_k=2)
    _check([8, 4, 2, 1], [2 / 3, 1 / 3, 0, 0], min_p=.2, top_k=2, top_p=.7)
    _check([16, 4, 1], [4 / 7, 2 / 7, 1 / 7], temperature=2)


def test_contract_edges():
    assert distribution([0., math.nan], mask=np.array([1], np.int32))[1] == Status.INVALID_INPUT
    assert distribution([-math.inf] * 3)[1] == Status.NO_VALID_TOKEN
    p, _ = distribution([2., 2., 1.], temperature=0, mask=np.array([6], np.int32))
    np.testing.assert_array_equal(p, [0, 1, 0])
    p, _ = distribution(np.zeros(35), mask=np.array([-2147483648, 1], np.int32))
    assert np.flatnonzero(p).tolist() == [31, 32]
    from unittest.mock import patch
    with patch("oracle.reference.uniform", return_value=.5):
        out = verify_reference(np.zeros((2, 2)), [0, 2], [[0]], rng=RngKey(1, 0, [0, 1]))
    assert out.accepted_len.tolist() == [0] and out.tokens.tolist() == [[1, -1]]
    with patch("oracle.reference.uniform", return_value=np.nextafter(.5, 0)):
        out = verify_reference(np.zeros((2, 2)), [0, 2], [[0]], rng=RngKey(1, 0, [0, 1]))
    assert out.accepted_len.tolist() == [1]


def test_structural_errors_raise():
    with pytest.raises(ValueError):
        verify_reference(np.zeros((2, 2)), [0, 1], np.empty((1, 0), np.int64), rng=RngKey(1, 0, [0, 1]))
    with pytest.raises(ValueError):
        verify_reference(np.zeros((2, 2)), [0, 2], np.empty((1, 0), np.int64), rng=RngKey(1, 0, [0, 1]))


@pytest.mark.parametrize("entry", golden_io.small(), ids=lambda e: e[0]["name"])
def test_small_golden(entry):
    case, (tokens, accepted, status) = entry
    out = verify_reference(**C.oracle_inputs(case, oracle))
    np.testing.assert_array_equal(out.status, status)
    np.testing.assert_array_equal(out.tokens, tokens)
    np.testing.assert_array_equal(out.accepted_len, accepted)


def _large():
    try:
        return golden_io.large_entries()
    except FileNotFoundError:
        return []


@pytest.mark.parametrize("entry", _large(), ids=lambda e: e[0])
def test_large_golden(entry):
    name, subset, digest, (tokens, accepted, status) = entry
    case = golden_io.large_case(name, subset, digest)
    out = verify_reference(**C.oracle_inputs(case, oracle))
    np.testing.assert_array_equal(out.status, status)
    np.testing.assert_array_equal(out.tokens, tokens)
    np.testing.assert_array_equal(out.accepted_len, accepted)


def test_every_mask_of_a_uniform_row():
    """Every nonempty mask of uniform rows of 1 to 8 tokens, with top-k 0, 1 or
    V and top-p 1/4 ... 1: the kept set is the first ceil(kept * top_p)
    allowed IDs (ties break by ID), each with mass exactly 1/n (the
    reference's tests/exact/test_exhaustive_oracle.py:12-27 check)."""
    for vocab in range(1, 9):
        for bits in range(1, 1 << vocab):
            allowed = [t for t in range(vocab) if bits >> t & 1]
            for k in [0, 1, vocab]:
                kept = len(allowed) if k == 0 else min(k, len(allowed))
                for top_p in [0.25, 0.5, 0.75, 1.0]:
                    n = math.ceil(kept * top_p)
                    expected = np.zeros(vocab)
                    expected[allowed[:n]] = 1 / n
                    probs, status = oracle.distribution(np.zeros(vocab), top_k=k, top_p=top_p,
                                                        mask=np.array([bits], np.int32))
                    assert status == oracle.Status.OK
                    np.testing.assert_array_equal(probs, expected)
