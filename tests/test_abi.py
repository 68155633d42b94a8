"""The C ABI without a GPU: the library loads and exports every function the
header declares, the workspace formula matches the reference's, and the
argument checks (the reference binding's, csrc/bindings.cpp:50-119) reject
bad calls before any device work. Pointers here are host addresses that are
never dereferenced."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from exactsample_b200 import capi

ROOT = Path(__file__).resolve().parents[1]


def test_header_declarations_are_exported():
    header = (ROOT / "include" / "exactsample_b200.h").read_text()
    declared = sorted(set(re.findall(r"^\w[\w\s\*]*?\b(es_\w+)\s*\(", header, flags=re.M)))
    assert declared == sorted(capi.EXPORTS)
    lib = capi.load()
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.es_abi_version() == 1


def test_workspace_formula_matches_reference():
    for rows, vocab in [(0, 1), (1, 4), (128, 151936), (320, 151936), (7, 1000)]:
        assert capi.workspace_bytes(rows, vocab) == 8 + rows * (32 + 12288)
        assert capi.workspace_bytes(rows, vocab, True) == 8 + rows * (32 + max(12288, 20 * vocab))


class Host:
    """Host buffers standing in for device tensors (sizes/strides only matter)."""

    def __init__(self):
        self.keep = []

    def t(self, shape, dtype, code):
        arr = np.zeros(shape, dtype=dtype)
        self.keep.append(arr)
        d = capi.Tensor()
        d.data = arr.ctypes.data
        d.dtype = code
        d.ndim = len(shape)
        for i, n in enumerate(shape):
            d.size[i] = n
            d.stride[i] = arr.strides[i] // arr.itemsize
        return d


def args(rows=2, vocab=8, requests=1, max_draft=1, **override):
    h = Host()
    a = capi.Args()
    a.target_logits = h.t((rows, vocab), np.float32, capi.ES_F32)
    a.cu_rows = h.t((requests + 1,), np.int64, capi.ES_I64)
    a.draft_ids = h.t((requests, max(max_draft, 0)), np.int64, capi.ES_I64)
    for name in ["temperature", "top_p", "min_p"]:
        setattr(a, name, h.t((requests,), np.float64, capi.ES_F64))
    for name in ["top_k", "draft_kind", "seeds", "stream_ids"]:
        setattr(a, name, h.t((requests,), np.int64, capi.ES_I64))
    a.positions = h.t((rows,), np.int64, capi.ES_I64)
    a.workspace = h.t((capi.workspace_bytes(rows, vocab),), np.uint8, capi.ES_U8)
    a.tokens = h.t((requests, max(max_draft, 0) + 1), np.int64, capi.ES_I64)
    for name in ["accepted_len", "status", "path_used"]:
        setattr(a, name, h.t((requests,), np.int32, capi.ES_I32))
    a.max_draft, a.list_max = max_draft, 256
    for key in ("mode", "dispatch", "max_draft", "list_max"):
        if key in override:
            setattr(a, key, override.pop(key))
    for key, value in override.items():
        setattr(a, key, value(h, a) if callable(value) else value)
    a._host = h
    return a


def call(a):
    lib = capi.load()
    code = lib.es_verify(ctypes.byref(a), None)
    return code, lib.es_last_error().decode()


def test_valid_arguments_reach_the_device_check():
    code, message = call(args())
    assert code == -7 and ("GPU" in message or "device" in message)


@pytest.mark.parametrize("override,code,message", [
    (dict(list_max=257), -1, "list_max must be in [0, 256]"),
    (dict(mode=2), -1, "invalid mode/dispatch"),
    (dict(max_draft=-1), -1, "invalid max_draft"),
    (dict(workspace=lambda h, a: h.t((100,), np.uint8, capi.ES_U8)), -2, "workspace capacity exceeded"),
    (dict(tokens=lambda h, a: h.t((1, 1), np.int64, capi.ES_I64)), -2, "tokens capacity exceeded"),
    (dict(positions=lambda h, a: h.t((3,), np.int64, capi.ES_I64)), -1, "positions must be per target row"),
    (dict(temperature=lambda h, a: h.t((1,), np.float32, capi.ES_F32)), -1, "wrong device, dtype or rank"),
    (dict(mask=lambda h, a: h.t((2, 2), np.int32, capi.ES_I32)), -1, "mask shape mismatch"),
    (dict(draft_logits=lambda h, a: h.t((2, 8), np.float64, capi.ES_F64)), -1, "draft_logits must have the target_logits dtype"),
])
def test_argument_errors(override, code, message):
    got, text = call(args(**override))
    assert got == code and message in text


def test_output_aliasing_is_rejected():
    a = args()
    a.tokens = capi.Tensor(a.seeds.data, (1, 2), (2, 1), capi.ES_I64, 2)  # tokens over an input
    assert call(a) == (-4, "exactsample input/output aliasing is forbidden")
    b = args()
    b.status = b.accepted_len
    assert call(b) == (-4, "exactsample outputs alias")
    c = args()
    c.status = capi.Tensor(c.status.data, (2, 0), (0, 0), capi.ES_I32, 1)
    c.status.size[0], c.status.stride[0] = 2, 0
    assert call(c)[0] == -4


def test_workspace_alignment():
    a = args()
    a.workspace.data += 4
    a.workspace.size[0] -= 8
    code, text = call(a)
    assert code in (-2, -3)
    a = args(workspace=lambda h, w: h.t((capi.workspace_bytes(2, 8) + 16,), np.uint8, capi.ES_U8))
    a.workspace.data += 4
    assert call(a) == (-3, "workspace alignment must be 8 bytes")


def test_empty_batch_rules():
    a = args(rows=1, requests=0, max_draft=0)
    assert call(a) == (-1, "an empty request batch cannot contain target rows")
    ok = args(rows=0, requests=0, max_draft=0)
    assert call(ok) == (0, "")  # nothing to launch
