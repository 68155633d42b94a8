"""Host logic of vocabulary-sharded calls, without a GPU: the shard widths
and request split, and the C ABI's checks of a shard table (host pointers
that are never dereferenced; a valid table reaches the device check)."""
import ctypes

import numpy as np
import pytest

from exactsample_b200 import capi
from exactsample_b200.sharded import request_range, shard_columns
from tests.test_abi import args


def test_shard_columns_are_multiples_of_16_covering_the_row():
    for vocab in [151936, 152064, 32000, 50257, 1000]:
        for n in range(2, 9):
            try:
                cols = shard_columns(vocab, n)
            except ValueError:
                assert vocab < 16 * n * 2
                continue
            assert cols % 16 == 0 and (n - 1) * cols < vocab <= n * cols
    assert shard_columns(151936, 2) == 75968 and shard_columns(151936, 8) == 18992
    with pytest.raises(ValueError):
        shard_columns(151936, 9)


def test_request_ranges_partition_the_batch():
    for requests in [0, 1, 7, 128, 4096]:
        for n in range(2, 9):
            ranges = [request_range(requests, n, g) for g in range(n)]
            assert ranges[0][0] == 0 and ranges[-1][1] == requests
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            assert max(e - b for b, e in ranges) - min(e - b for b, e in ranges) <= 1


def _table(a, n=2, rank=0, vocab=16, cols=16, **override):
    sh = capi.Shards()
    sh.count, sh.rank, sh.cols, sh.vocab = n, rank, cols, vocab
    sh.req_begin, sh.req_end, sh.epoch = 0, 1, 1
    h = a._host
    for g in range(n):
        own = g == rank
        sh.target[g] = a.target_logits.data if own else h.t((2, cols), np.float32, capi.ES_F32).data
        sh.tokens[g] = a.tokens.data if own else h.t((1, 2), np.int64, capi.ES_I64).data
        sh.accepted[g] = a.accepted_len.data if own else h.t((1,), np.int32, capi.ES_I32).data
        sh.status[g] = a.status.data if own else h.t((1,), np.int32, capi.ES_I32).data
        sh.path[g] = a.path_used.data if own else h.t((1,), np.int32, capi.ES_I32).data
        sh.ready[g] = h.t((8,), np.uint64, capi.ES_U8).data
    for k, v in override.items():
        setattr(sh, k, v)
    return sh


def _call(a, sh):
    lib = capi.load()
    return lib.es_verify_sharded(ctypes.byref(a), ctypes.byref(sh), None), lib.es_last_error().decode()


def test_a_valid_shard_table_reaches_the_device_check():
    a = args(rows=2, vocab=16, requests=1)  # this GPU's shard: 16 of 24 columns
    a.mask = a._host.t((2, 1), np.int32, capi.ES_I32)
    code, message = _call(a, _table(a, vocab=24))
    assert code == -7, message


@pytest.mark.parametrize("override,message", [
    (dict(count=1), "count must be in [2, 8]"),
    (dict(count=9), "count must be in [2, 8]"),
    (dict(rank=2), "rank in [0, count)"),
    (dict(cols=24, vocab=40), "multiple of 16"),
    (dict(vocab=33), "(count - 1) * cols < vocab <= count * cols"),
    (dict(vocab=16), "(count - 1) * cols < vocab <= count * cols"),
    (dict(req_end=2), "request range"),
])
def test_shard_table_errors(override, message):
    a = args(rows=2, vocab=16, requests=1)
    code, text = _call(a, _table(a, **{"vocab": 24, **override}))
    assert code == -1 and message in text


def test_the_shard_must_be_this_gpus_columns_and_tensors():
    a = args(rows=2, vocab=16, requests=1)
    code, text = _call(a, _table(a, rank=1, vocab=24))  # rank 1 holds 8 columns, not 16
    assert code == -1 and "this GPU's shard" in text
    b = args(rows=2, vocab=16, requests=1)
    sh = _table(b, vocab=24)
    sh.tokens[0] = sh.tokens[1]
    code, text = _call(b, sh)
    assert code == -1 and "own tensors" in text
    c = args(rows=2, vocab=16, requests=1)
    sh = _table(c, vocab=24)
    sh.ready[1] = None
    code, text = _call(c, sh)
    assert code == -1 and "every GPU needs" in text


def test_per_phase_tables():
    """A per-phase call finishes every request on every GPU and needs every
    GPU's exchange buffer and this GPU's scratch (16-byte aligned)."""
    def phased(a, **override):
        sh = _table(a, vocab=24, **override)
        sh.phases = 1
        for g in range(2):
            sh.exchange[g] = a._host.t((64,), np.uint64, capi.ES_U8).data
        sh.scratch = a._host.t((64,), np.uint64, capi.ES_U8).data
        return sh

    a = args(rows=2, vocab=16, requests=1)
    code, message = _call(a, phased(a))
    assert code == -7, message  # a valid table reaches the device check
    b = args(rows=2, vocab=16, requests=1)
    code, text = _call(b, phased(b, req_end=0))
    assert code == -1 and "every request on every GPU" in text
    c = args(rows=2, vocab=16, requests=1)
    sh = phased(c)
    sh.exchange[1] = None
    code, text = _call(c, sh)
    assert code == -1 and "exchange buffer" in text
    d = args(rows=2, vocab=16, requests=1)
    sh = phased(d)
    sh.scratch = None
    code, text = _call(d, sh)
    assert code == -1 and "scratch" in text
    size = ctypes.c_uint64()
    assert capi.load().es_shard_exchange_bytes(128, ctypes.byref(size)) == 0 and size.value % 16 == 0
    assert size.value >= 128 * (16 + 8 + 16 + 256 + 512 * 12)


def test_flag_and_ipc_entry_points_need_a_gpu():
    lib = capi.load()
    flag = (ctypes.c_uint64 * 1)()
    assert lib.es_shard_signal(ctypes.cast(flag, ctypes.c_void_p), 1, None) == -7
    flags = (ctypes.c_void_p * 1)(ctypes.cast(flag, ctypes.c_void_p))
    assert lib.es_shard_wait(flags, 1, 1, None, None) == -7
    assert lib.es_shard_wait(flags, 0, 1, None, None) == -1
    done = ctypes.cast(flag, ctypes.c_void_p)
    assert lib.es_shard_finish(done, flags, 1, 1, None, None) == -7
    assert lib.es_shard_finish(None, flags, 1, 1, None, None) == -1
    # This GPU's slot array must be one of every GPU's slot arrays.
    other = (ctypes.c_uint64 * 1)()
    assert lib.es_shard_finish(ctypes.cast(other, ctypes.c_void_p), flags, 1, 1, None, None) == -1
    assert b"slot arrays" in lib.es_last_error()
    ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
    assert lib.es_ipc_alloc(1024, ctypes.byref(ptr), handle) == -7
