"""ctypes binding of the C ABI (include/exactsample_b200.h).

This is what a non-torch caller binds; the tests use it to call the kernels
through the C ABI directly. ``call`` takes torch tensors only to read their
device pointers, sizes and strides.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import os

# $EXACTSAMPLE_ABI_LIBRARY picks another build of the C ABI (the tests' checked
# run loads libexactsample_b200_checked.so this way).
LIBRARY = Path(os.environ.get("EXACTSAMPLE_ABI_LIBRARY") or Path(__file__).with_name("libexactsample_b200.so"))

ES_F32, ES_F64, ES_F16, ES_BF16, ES_I32, ES_I64, ES_U8 = range(7)
ERRORS = {0: "ES_SUCCESS", -1: "ES_ERR_ARGUMENT", -2: "ES_ERR_CAPACITY", -3: "ES_ERR_ALIGNMENT",
          -4: "ES_ERR_ALIAS", -5: "ES_ERR_UNSUPPORTED", -6: "ES_ERR_LAUNCH", -7: "ES_ERR_DEVICE"}
# Every function the header declares.
EXPORTS = ["es_workspace_bytes", "es_verify", "es_verify_timed", "es_verify_static", "es_verify_sharded",
           "es_shard_exchange_bytes", "es_shard_signal", "es_shard_wait", "es_shard_finish", "es_ipc_alloc", "es_ipc_open", "es_ipc_close", "es_ipc_free",
           "es_last_error", "es_abi_version"]
MAX_SHARDS = 8  # ES_MAX_SHARDS
STATIC_MAX_ROWS = 4096  # ES_STATIC_MAX_ROWS


class Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("size", ctypes.c_int64 * 2), ("stride", ctypes.c_int64 * 2),
                ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32)]


FIELDS = ["target_logits", "cu_rows", "draft_ids", "draft_logits", "temperature", "top_k", "top_p", "min_p",
          "draft_kind", "seeds", "stream_ids", "positions", "mask", "workspace", "tokens", "accepted_len",
          "status", "path_used"]


class Args(ctypes.Structure):
    _fields_ = [(name, Tensor) for name in FIELDS] + [
        ("mode", ctypes.c_int64), ("dispatch", ctypes.c_int64), ("max_draft", ctypes.c_int64),
        ("list_max", ctypes.c_int64)]


class Shards(ctypes.Structure):
    """es_shards: one GPU's view of a vocabulary-sharded call."""
    _fields_ = [("count", ctypes.c_int32), ("rank", ctypes.c_int32), ("cols", ctypes.c_int64),
                ("vocab", ctypes.c_int64), ("req_begin", ctypes.c_int64), ("req_end", ctypes.c_int64),
                ("epoch", ctypes.c_uint64)] + [
        (name, ctypes.c_void_p * MAX_SHARDS)
        for name in ["target", "draft", "tokens", "accepted", "status", "path", "ready"]] + [
        ("phases", ctypes.c_int32), ("pad", ctypes.c_int32), ("exchange", ctypes.c_void_p * MAX_SHARDS),
        ("scratch", ctypes.c_void_p)]


_lib = None


def load(path: str | Path | None = None) -> ctypes.CDLL:
    """The C ABI library (raises if it was not built)."""
    global _lib
    if _lib is None or path is not None:
        target = Path(path) if path else LIBRARY
        if not target.is_file():
            raise RuntimeError(f"{target} is missing; build it with `python -m exactsample_b200.build`")
        lib = ctypes.CDLL(str(target))
        lib.es_workspace_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                           ctypes.POINTER(ctypes.c_uint64)]
        lib.es_workspace_bytes.restype = ctypes.c_int
        lib.es_verify.argtypes = [ctypes.POINTER(Args), ctypes.c_void_p]
        lib.es_verify.restype = ctypes.c_int
        lib.es_verify_timed.argtypes = [ctypes.POINTER(Args), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.es_verify_timed.restype = ctypes.c_int
        lib.es_verify_static.argtypes = [ctypes.POINTER(Args), ctypes.c_void_p]
        lib.es_verify_static.restype = ctypes.c_int
        lib.es_verify_sharded.argtypes = [ctypes.POINTER(Args), ctypes.POINTER(Shards), ctypes.c_void_p]
        lib.es_verify_sharded.restype = ctypes.c_int
        lib.es_shard_exchange_bytes.argtypes = [ctypes.c_int64, ctypes.POINTER(ctypes.c_uint64)]
        lib.es_shard_exchange_bytes.restype = ctypes.c_int
        lib.es_shard_signal.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
        lib.es_shard_signal.restype = ctypes.c_int
        lib.es_shard_wait.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32, ctypes.c_uint64,
                                      ctypes.c_void_p, ctypes.c_void_p]
        lib.es_shard_wait.restype = ctypes.c_int
        lib.es_shard_finish.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32,
                                        ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]
        lib.es_shard_finish.restype = ctypes.c_int
        lib.es_ipc_alloc.argtypes = [ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]
        lib.es_ipc_alloc.restype = ctypes.c_int
        lib.es_ipc_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
        lib.es_ipc_open.restype = ctypes.c_int
        lib.es_ipc_close.argtypes = [ctypes.c_void_p]
        lib.es_ipc_close.restype = ctypes.c_int
        lib.es_ipc_free.argtypes = [ctypes.c_void_p]
        lib.es_ipc_free.restype = ctypes.c_int
        lib.es_last_error.argtypes = []
        lib.es_last_error.restype = ctypes.c_char_p
        lib.es_abi_version.argtypes = []
        lib.es_abi_version.restype = ctypes.c_int
        _lib = lib
    return _lib


def workspace_bytes(rows: int, vocab: int, reference: bool = False) -> int:
    out = ctypes.c_uint64()
    code = load().es_workspace_bytes(rows, vocab, int(reference), ctypes.byref(out))
    if code:
        raise ValueError(load().es_last_error().decode())
    return int(out.value)


_CODES: dict = {}


def describe(t) -> Tensor:
    """An es_tensor for a torch tensor (None: absent)."""
    d = Tensor()
    if t is None:
        return d
    if not _CODES:
        import torch

        _CODES.update({torch.float32: ES_F32, torch.float64: ES_F64, torch.float16: ES_F16,
                       torch.bfloat16: ES_BF16, torch.int32: ES_I32, torch.int64: ES_I64, torch.uint8: ES_U8})
    if t.numel():
        d.data = t.data_ptr()
    d.dtype = _CODES.get(t.dtype, -1)
    dims = t.dim()
    if dims == 1:
        d.ndim, d.size[0], d.stride[0] = 1, t.shape[0], t.stride(0)
    elif dims == 2:
        d.ndim = 2
        d.size[0], d.size[1] = t.shape
        d.stride[0], d.stride[1] = t.stride()
    else:
        d.ndim = -1
    return d


class AbiError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{ERRORS.get(code, code)}: {message}")
        self.code = code


def call(tensors: dict, *, mode: int = 0, dispatch: int = 0, max_draft: int = 0, list_max: int = 256,
         stream=None, events=None, static_scratch: bool = False) -> None:
    """es_verify (es_verify_timed with events=(before, after); es_verify_static
    with static_scratch=True, which ignores any workspace given) on torch tensors.

    ``tensors`` maps the es_args field names to torch tensors (optional ones may
    be absent or None). ``stream`` is a torch.cuda.Stream (default: current).
    """
    import torch

    args = Args()
    for name in FIELDS:
        if not (static_scratch and name == "workspace"):
            setattr(args, name, describe(tensors.get(name)))
    args.mode, args.dispatch, args.max_draft, args.list_max = mode, dispatch, max_draft, list_max
    s = (stream or torch.cuda.current_stream()).cuda_stream
    lib = load()
    if static_scratch:
        code = lib.es_verify_static(ctypes.byref(args), ctypes.c_void_p(s))
    elif events is None:
        code = lib.es_verify(ctypes.byref(args), ctypes.c_void_p(s))
    else:
        before, after = events
        code = lib.es_verify_timed(ctypes.byref(args), ctypes.c_void_p(s),
                                   ctypes.c_void_p(before.cuda_event if before is not None else 0),
                                   ctypes.c_void_p(after.cuda_event if after is not None else 0))
    if code != 0:
        raise AbiError(code, lib.es_last_error().decode())


def check(code: int) -> None:
    """Raises AbiError for a non-zero return code of the C ABI."""
    if code != 0:
        raise AbiError(code, load().es_last_error().decode())


def args_of(tensors: dict, *, mode: int = 0, dispatch: int = 0, max_draft: int = 0, list_max: int = 256) -> Args:
    """An es_args for torch tensors keyed by field name (absent or None: an empty descriptor)."""
    args = Args()
    for name in FIELDS:
        setattr(args, name, describe(tensors.get(name)))
    args.mode, args.dispatch, args.max_draft, args.list_max = mode, dispatch, max_draft, list_max
    return args
