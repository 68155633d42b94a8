"""TEST INFRASTRUCTURE ONLY: FP64 NumPy restatement of the reference oracle.

Each function follows the reference's Python oracle step by step, with the
same NumPy operations where a result's rounding depends on them (``np.exp``
for weights, stable ``np.argsort``, FP64 division), so that on one machine its
outputs are bit-identical to the reference's. The loops that the reference
runs in Python call ``oracle_c.c`` instead (Philox, the Gumbel argmax,
``math.fsum`` and the top-p prefix), which gives the same doubles.

Cited lines are ``python/exactsample/reference.py`` (``ref``) and
``python/exactsample/rng.py`` (``rng``) of the reference project.
"""
from __future__ import annotations

import ctypes
import operator
from dataclasses import dataclass
from enum import IntEnum
from typing import Any

import numpy as np

from .build import library_path, build as _build_library

_U32 = (1 << 32) - 1
_U64 = (1 << 64) - 1


class Status(IntEnum):  # python/exactsample/types.py:7-11
    OK = 0
    NO_VALID_TOKEN = 1
    INVALID_INPUT = 2
    DRAFT_ZERO_PROB = 3


class PathUsed(IntEnum):  # python/exactsample/types.py:14-16
    REFERENCE = 0
    FUSED = 1


@dataclass(frozen=True)
class RequestParams:  # python/exactsample/types.py:19-27
    temperature: Any = 1.0
    top_k: Any = 0
    top_p: Any = 1.0
    min_p: Any = 0.0
    draft_kind: Any = "one_hot"


@dataclass(frozen=True)
class RngKey:  # python/exactsample/types.py:30-36
    seed: Any
    stream_id: Any
    positions: Any


@dataclass
class VerifyOutput:  # python/exactsample/types.py:39-44
    tokens: Any
    accepted_len: Any
    status: Any
    path_used: Any


_lib = None


def _native():
    global _lib
    if _lib is None:
        path = library_path()
        if not path.is_file():
            _build_library()
        lib = ctypes.CDLL(str(path))
        u32, u64, i64, dptr = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int64, ctypes.POINTER(ctypes.c_double)
        u32ptr = ctypes.POINTER(ctypes.c_uint32)
        lib.es_oracle_philox.argtypes = [u32ptr, u32ptr, u32ptr]
        lib.es_oracle_philox.restype = None
        lib.es_oracle_word.argtypes = [u64, u32, u32, u32, u64]
        lib.es_oracle_word.restype = u32
        lib.es_oracle_words.argtypes = [u64, u32, u32, u32, i64, u32ptr]
        lib.es_oracle_words.restype = None
        lib.es_oracle_sample.argtypes = [dptr, i64, u64, u32, u32, u32]
        lib.es_oracle_sample.restype = i64
        lib.es_oracle_fsum.argtypes = [dptr, i64]
        lib.es_oracle_fsum.restype = ctypes.c_double
        lib.es_oracle_top_p_count.argtypes = [dptr, i64, ctypes.c_double]
        lib.es_oracle_top_p_count.restype = i64
        _lib = lib
    return _lib


def _dptr(array):
    return array.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def _uint(value, maximum, name):  # rng:12-19
    try:
        result = operator.index(value)
    except TypeError as exc:
        raise ValueError(f"{name} must be an integer") from exc
    if isinstance(value, bool) or not 0 <= result <= maximum:
        raise ValueError(f"{name} outside [0, {maximum}]")
    return result


def philox4x32(counter, key):  # rng:22-43
    """Four uint32 words of Random123 Philox4x32-10 for 4 counter and 2 key words."""
    if len(counter) != 4 or len(key) != 2:
        raise ValueError("Philox requires 4 counter and 2 key words")
    c = (ctypes.c_uint32 * 4)(*[_uint(x, _U32, "counter") for x in counter])
    k = (ctypes.c_uint32 * 2)(*[_uint(x, _U32, "key") for x in key])
    out = (ctypes.c_uint32 * 4)()
    _native().es_oracle_philox(c, k, out)
    return tuple(int(x) for x in out)


def random_word(seed, stream_id, position, substream=0, token=0):  # rng:46-56
    seed = _uint(seed, _U64, "seed")
    stream_id = _uint(stream_id, _U32, "stream_id")
    position = _uint(position, _U32, "position")
    substream = _uint(substream, _U32, "substream")
    token = _uint(token, (1 << 34) - 1, "token")
    return int(_native().es_oracle_word(seed, stream_id, position, substream, token))


def uniform(seed, stream_id, position, substream=0, token=0):  # rng:59-61
    return (random_word(seed, stream_id, position, substream, token) + 0.5) / (1 << 32)


def gumbel(seed, stream_id, position, substream=0, token=0):  # rng:64-65
    import math
    return -math.log(-math.log(uniform(seed, stream_id, position, substream, token)))


def _scalar_integer(value):  # ref:11-17
    if isinstance(value, (bool, np.bool_)):
        raise ValueError("booleans are not integer parameters")
    try:
        return operator.index(value)
    except TypeError as exc:
        raise ValueError("expected integer parameter") from exc


def _packed_mask(mask, vocab):  # ref:20-27, decoded with NumPy bit operations
    if mask is None:
        return np.ones(vocab, dtype=bool)
    words = np.asarray(mask)
    if words.shape != ((vocab + 31) // 32,) or words.dtype.kind not in "iu" or words.dtype.itemsize != 4:
        raise ValueError("mask must contain ceil(vocab/32) int32 or uint32 words")
    words = words.astype(np.uint32, copy=False)
    bits = np.unpackbits(words.astype("<u4").view(np.uint8), bitorder="little")
    return bits[:vocab].astype(bool)


def _fsum(values):
    array = np.ascontiguousarray(values, dtype=np.float64)
    return float(_native().es_oracle_fsum(_dptr(array), array.size))


def distribution(logits, *, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, mask=None):  # ref:30-86
    """(float64 probabilities, Status) of one target row.

    Order: mask, temperature, min-p, stable top-k, shortest top-p prefix by
    correctly rounded sums, normalization. NaN/+inf anywhere is invalid, even
    behind the mask; -inf has zero mass.
    """
    import math
    values = np.asarray(logits)
    if values.ndim != 1 or values.size == 0 or values.dtype.kind not in "fiu":
        raise ValueError("logits must be a nonempty real vector")
    values = values.astype(np.float64, copy=True)
    probs = np.zeros(values.size, dtype=np.float64)
    allowed = _packed_mask(mask, values.size)
    try:
        k = _scalar_integer(top_k)
        temperature, top_p, min_p = float(temperature), float(top_p), float(min_p)
        valid = (math.isfinite(temperature) and temperature >= 0 and 0 <= k <= values.size
                 and math.isfinite(top_p) and 0 < top_p <= 1
                 and math.isfinite(min_p) and 0 <= min_p <= 1)
    except (ValueError, TypeError, OverflowError):
        valid = False
    if not valid or np.isnan(values).any() or np.isposinf(values).any():
        return probs, Status.INVALID_INPUT
    active = allowed & np.isfinite(values)
    if not active.any():
        return probs, Status.NO_VALID_TOKEN
    if temperature == 0:
        probs[int(np.argmax(np.where(active, values, -np.inf)))] = 1.0
        return probs, Status.OK
    maximum = np.max(values[active])
    with np.errstate(over="ignore", under="ignore"):
        shifted = (values - maximum) / temperature
        weights = np.where(active, np.exp(shifted), 0.0)
    active &= weights >= min_p
    active &= weights > 0.0
    ordered = np.flatnonzero(active)
    ordered = ordered[np.argsort(-values[ordered], kind="stable")]
    if k:
        ordered = ordered[:k]
    selected = np.ascontiguousarray(weights[ordered])
    denominator = _fsum(selected)
    if top_p < 1:
        target = top_p * denominator
        count = int(_native().es_oracle_top_p_count(_dptr(selected), selected.size, target))
        ordered = ordered[:count]
        denominator = _fsum(weights[ordered])
    probs[ordered] = weights[ordered] / denominator
    return probs, Status.OK


def proposal_distribution(logits):  # ref:89-91
    return distribution(logits)


def sample_distribution(probs, *, seed, stream_id, position, substream=0):  # ref:94-104
    """Gumbel-max draw from probs with the addressable Philox noise."""
    probs = np.ascontiguousarray(probs, dtype=np.float64)
    if probs.ndim != 1 or probs.size == 0 or not np.isfinite(probs).all() or (probs < 0).any() or not (probs > 0).any():
        raise ValueError("probabilities must be nonnegative, finite, and have positive mass")
    seed = _uint(seed, _U64, "seed")
    return int(_native().es_oracle_sample(_dptr(probs), probs.size, seed, _uint(stream_id, _U32, "stream_id"),
                                          _uint(position, _U32, "position"), _uint(substream, _U32, "substream")))


def _per_request(value, count, name):  # ref:107-115
    arr = np.asarray(value, dtype=object)
    if arr.ndim == 0:
        return [arr.item()] * count
    if arr.shape != (count,):
        raise ValueError(f"{name} must be scalar or shape [{count}]")
    return list(arr)


def _bounded_int(value, bits):  # ref:118-122
    result = _scalar_integer(value)
    if not 0 <= result < (1 << bits):
        raise ValueError(f"integer outside uint{bits}")
    return result


def _field(obj, name):
    if not hasattr(obj, name):
        raise TypeError("params/RNG must be RequestParams/RngKey")
    return getattr(obj, name)


def verify_request(logits, begin, end, drafts_row, *, fields, seed, stream, positions, draft_logits, mask, mode):
    """Status, tokens, accepted count of one request (ref:177-254).

    ``fields`` holds this request's temperature, top_k, top_p, min_p and
    draft_kind; ``positions`` the whole batch's positions. Returns
    (status, tokens list of length D+1 or fewer, accepted).
    """
    count = end - begin - 1
    kind = fields["draft_kind"]
    if count < 0 or kind not in ("one_hot", "full") or (kind == "full" and mode == "coupled"):
        return Status.INVALID_INPUT, [], 0
    if count and kind == "full" and draft_logits is None:
        return Status.INVALID_INPUT, [], 0
    try:
        seed = _bounded_int(seed, 64)
        stream = _bounded_int(stream, 32)
        row_positions = [_bounded_int(pos, 32) for pos in positions[begin:end]]
    except (ValueError, TypeError, OverflowError):
        return Status.INVALID_INPUT, [], 0
    vocab = logits.shape[1]
    if any(not 0 <= int(drafts_row[index]) < vocab for index in range(count)):
        return Status.INVALID_INPUT, [], 0
    row_probs, proposal_probs = [], []
    status = Status.OK
    params = {name: fields[name] for name in ("temperature", "top_k", "top_p", "min_p")}
    for row in range(begin, end):
        probabilities, status = distribution(logits[row], mask=None if mask is None else mask[row], **params)
        if status != Status.OK:
            break
        row_probs.append(probabilities)
    if status == Status.OK:
        for index in range(count):
            token = int(drafts_row[index])
            if kind == "full":
                proposal, status = proposal_distribution(draft_logits[begin + index])
                if status != Status.OK:
                    break
                if proposal[token] == 0:
                    status = Status.DRAFT_ZERO_PROB
                    break
                proposal_probs.append(proposal)
    if status != Status.OK:
        return status, [], 0
    tokens = []
    for index in range(count):
        p = row_probs[index]
        token = int(drafts_row[index])
        address = dict(seed=seed, stream_id=stream, position=row_positions[index])
        if mode == "coupled":
            sampled = sample_distribution(p, **address, substream=0)
            accept = sampled == token
        else:
            q_token = 1.0 if kind == "one_hot" else float(proposal_probs[index][token])
            accept = uniform(seed, stream, row_positions[index], 1, 0) < min(1.0, float(p[token]) / q_token)
            if not accept:
                if kind == "one_hot":
                    residual = p.copy()
                    residual[token] = 0.0
                else:
                    residual = np.maximum(p - proposal_probs[index], 0.0)
                if not (residual > 0).any():
                    return Status.INVALID_INPUT, [], 0
                sampled = sample_distribution(residual, **address, substream=2)
        if not accept:
            tokens.append(sampled)
            return Status.OK, tokens, index
        tokens.append(token)
    tokens.append(sample_distribution(row_probs[count], seed=seed, stream_id=stream,
                                      position=row_positions[count], substream=0))
    return Status.OK, tokens, count


def verify_reference(target_logits, cu_rows, draft_ids, *, params=None, rng, draft_logits=None, mask=None,
                     mode="ratio", requests_subset=None):  # ref:125-255
    """Verify a ragged batch against the exactsample v1 contract.

    Structural errors raise ValueError/TypeError; request-local errors give a
    status with -1 tokens and zero accepted_len. ``requests_subset`` (an
    iterable of request indices) restricts the work to those requests; the
    others keep status OK and -1 tokens, which callers must ignore.
    """
    if mode not in ("ratio", "coupled"):
        raise ValueError("mode must be 'ratio' or 'coupled'")
    params = RequestParams() if params is None else params
    logits, offsets, drafts = map(np.asarray, (target_logits, cu_rows, draft_ids))
    if logits.ndim != 2 or logits.shape[1] == 0 or logits.dtype.kind not in "fiu":
        raise ValueError("target_logits must be a real [rows, vocab] array")
    rows, vocab = logits.shape
    if offsets.ndim != 1 or offsets.size == 0 or offsets.dtype.kind not in "iu":
        raise ValueError("cu_rows must be an integer [requests+1] vector")
    if int(offsets[0]) != 0 or int(offsets[-1]) != rows or any(int(b) < int(a) for a, b in zip(offsets[:-1], offsets[1:])):
        raise ValueError("cu_rows must be monotone, start at zero, and end at rows")
    requests = offsets.size - 1
    if drafts.ndim != 2 or drafts.shape[0] != requests or drafts.dtype.kind not in "iu":
        raise ValueError("draft_ids must be an integer [requests, max_draft] array")
    max_draft = drafts.shape[1]
    if any(int(b) - int(a) > max_draft + 1 for a, b in zip(offsets[:-1], offsets[1:])):
        raise ValueError("ragged segment exceeds draft_ids capacity")
    if mask is not None:
        mask = np.asarray(mask)
        if mask.shape != (rows, (vocab + 31) // 32) or mask.dtype.kind not in "iu" or mask.dtype.itemsize != 4:
            raise ValueError("mask must be packed int32 [rows, ceil(vocab/32)]")
    if draft_logits is not None:
        draft_logits = np.asarray(draft_logits)
        if draft_logits.shape != logits.shape or draft_logits.dtype.kind not in "fiu":
            raise ValueError("draft_logits must have target_logits shape and real dtype")
    positions = np.asarray(_field(rng, "positions"))
    if positions.shape != (rows,):
        raise ValueError("rng.positions must have shape [rows]")
    fields = {name: _per_request(_field(params, name), requests, name)
              for name in ("temperature", "top_k", "top_p", "min_p", "draft_kind")}
    seeds = _per_request(_field(rng, "seed"), requests, "seed")
    streams = _per_request(_field(rng, "stream_id"), requests, "stream_id")
    output = VerifyOutput(np.full((requests, max_draft + 1), -1, dtype=np.int64), np.zeros(requests, dtype=np.int32),
                          np.full(requests, int(Status.OK), dtype=np.int32),
                          np.full(requests, int(PathUsed.REFERENCE), dtype=np.int32))
    chosen = range(requests) if requests_subset is None else requests_subset
    for request in chosen:
        begin, end = int(offsets[request]), int(offsets[request + 1])
        status, tokens, accepted = verify_request(
            logits, begin, end, drafts[request], fields={name: fields[name][request] for name in fields},
            seed=seeds[request], stream=streams[request], positions=positions, draft_logits=draft_logits,
            mask=mask, mode=mode)
        output.status[request] = int(status)
        if status == Status.OK:
            output.tokens[request, :len(tokens)] = tokens
            output.accepted_len[request] = accepted
    return output
