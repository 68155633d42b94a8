"""Vocabulary-sharded verification: N GPUs (one process each, 2 to 8) hold
contiguous shards of the vocabulary of every row, as a tensor-parallel LM
head produces them, and every GPU gets the whole batch's outputs.

Two modes. Per-phase (``phases=True``, the default): every GPU streams only
its own shard of every row, and the GPUs exchange per-row partial results
over NVLink. Each GPU stores its results into its slot in every GPU's
exchange buffer, as 64-bit words that carry the call's tag beside each
datum, and reads the others' from its own buffer. They are the row
statistics with the tile-maximum bins (so every GPU knows the whole row's
maximum and the candidate window), then each GPU's best window candidates
(at most the top-k), which every GPU finishes alike (sort and FP64 finish),
writing every request's outputs into its own ``plan.out``. Rows this cannot
finish (no window, more than 64 candidates on a GPU that must cut them, or
a request off the top-k list path: greedy, full-q drafts, masks, lists over
256 tokens) are finished by the independent FP64 path on each GPU, reading
the whole row from every shard. Column-pulling (``phases=False``): the
description below.

Each process makes a ``ShardedPlan`` (collectively: the plans exchange the
handles of their registered buffers), writes its rows' logits shard into
``plan.logits[:rows]`` (and the proposal's into ``plan.draft_logits``), and
calls ``verify_sharded`` with the replicated inputs (offsets, drafts,
parameters, RNG key, optional whole-row mask). The GPUs split the requests:
each finishes a contiguous range, streaming its requests' full rows (its own
shard from HBM, the peers' over NVLink), and writes their outputs into every
GPU's ``plan.out``. Results are identical to ``exactsample_b200.cuda.verify``
on the unsharded rows.

The call is stream-ordered on each GPU: a flag tells the peers that this
GPU's shard is written, the kernels wait for every GPU's flag before reading
a shard, and a last step waits until every GPU has finished, so that
``plan.out`` is complete and the shard buffer may be rewritten when the
call's work on the stream is done. Every GPU must make the same calls in the
same order. Shard widths are multiples of 16 columns (``shard_columns``).
"""
from __future__ import annotations

import ctypes
import os
from typing import Any, Callable, Sequence

from . import capi
from .cuda import CudaOutput, CudaRequestParams, CudaRngKey, _DISPATCH, _MODES

_LOCAL_BLOCKS: dict[bytes, int] = {}  # handle -> pointer of blocks allocated by this process


def shard_columns(vocab: int, shards: int) -> int:
    """Columns per shard: vocab / shards rounded up to a multiple of 16 (the
    last shard holds the rest)."""
    if not 2 <= shards <= capi.MAX_SHARDS:
        raise ValueError(f"shards must be in [2, {capi.MAX_SHARDS}]")
    cols = -(-vocab // shards)
    cols = -(-cols // 16) * 16
    if (shards - 1) * cols >= vocab:
        raise ValueError(f"vocab {vocab} is too small for {shards} shards of multiples of 16 columns")
    return cols


def request_range(requests: int, shards: int, rank: int) -> tuple[int, int]:
    """The requests GPU `rank` finishes: a contiguous, balanced range."""
    return requests * rank // shards, requests * (rank + 1) // shards


class _DeviceArray:
    """A strided view of device memory, for torch.as_tensor (no copy)."""

    def __init__(self, ptr: int, shape, typestr: str, itemsize: int, row_stride: int | None = None):
        strides = None
        if row_stride is not None and len(shape) == 2:
            strides = (row_stride * itemsize, itemsize)
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 2, "strides": strides}


def _view(ptr: int, shape, dtype, row_stride: int | None = None):
    import torch

    codes = {torch.float32: ("<f4", 4), torch.float64: ("<f8", 8), torch.float16: ("<f2", 2),
             torch.bfloat16: ("<i2", 2), torch.int64: ("<i8", 8), torch.int32: ("<i4", 4), torch.uint64: ("<u8", 8)}
    typestr, size = codes[dtype]
    t = torch.as_tensor(_DeviceArray(ptr, shape, typestr, size, row_stride), device="cuda")
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


def _all_gather(group) -> Callable[[Any], list]:
    def gather(obj):
        import torch.distributed as dist

        out = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, obj, group=group)
        return out
    return gather


class ShardedPlan:
    """One GPU's part of a vocabulary-sharded plan (collective construction).

    ``exchange(obj) -> list`` gathers one object from every rank in rank order;
    by default ``torch.distributed.all_gather_object`` over ``group``. With
    ``connect=False`` the plan only allocates, and ``connect(entries)`` takes
    every rank's ``entry`` later (several ranks in one process, e.g. N shards
    on one GPU).
    """

    def __init__(self, max_rows: int, max_requests: int, max_draft: int, vocab: int, *, shards: int, rank: int,
                 dtype=None, full_q: bool = False, device: Any = None, group=None,
                 exchange: Callable[[Any], Sequence] | None = None, connect: bool = True, phases: bool = True):
        import torch

        if not 0 <= rank < shards:
            raise ValueError("rank must be in [0, shards)")
        self.max_rows, self.max_requests, self.max_draft, self.vocab = max_rows, max_requests, max_draft, vocab
        self.shards, self.rank, self.full_q, self.phases = shards, rank, full_q, phases
        self.dtype = dtype or torch.float32
        self.cols = shard_columns(vocab, shards)
        self.width = min(self.cols, vocab - rank * self.cols)
        self.list_max = 256
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else
                                   torch.device(device).index)
        self.epoch = 0
        item = torch.empty((), dtype=self.dtype).element_size()
        # Registered block: flags, shards, outputs (the same layout on every GPU).
        self._layout = layout = {}
        at = 256  # ready flag at 0, done flag at 64, wait timeouts at 128, done slots (one per GPU) at 192
        xbytes = ctypes.c_uint64()
        capi.check(capi.load().es_shard_exchange_bytes(max_rows, ctypes.byref(xbytes)))
        for name, nbytes in [("exchange", int(xbytes.value) if phases else 0),
                             ("logits", max_rows * self.cols * item),
                             ("draft", max_rows * self.cols * item if full_q else 0),
                             ("tokens", max_requests * (max_draft + 1) * 8), ("accepted", max_requests * 4),
                             ("status", max_requests * 4), ("path", max_requests * 4)]:
            layout[name] = at
            at = _align(at + max(nbytes, 1))
        self._bytes = at
        lib = capi.load()
        with torch.cuda.device(self.device):
            ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
            capi.check(lib.es_ipc_alloc(self._bytes, ctypes.byref(ptr), handle))
            self._base, self._handle = ptr.value, handle.raw
            _LOCAL_BLOCKS[self._handle] = self._base
            self.entry = (self._handle, os.getpid())
            self._bases, self._opened, self._sh = [], [], None
            self.logits = _view(self._base + layout["logits"], (max_rows, self.width), self.dtype, self.cols)
            self.draft_logits = (_view(self._base + layout["draft"], (max_rows, self.width), self.dtype, self.cols)
                                 if full_q else None)
            self.out = CudaOutput(
                _view(self._base + layout["tokens"], (max_requests, max_draft + 1), torch.int64),
                _view(self._base + layout["accepted"], (max_requests,), torch.int32),
                _view(self._base + layout["status"], (max_requests,), torch.int32),
                _view(self._base + layout["path"], (max_requests,), torch.int32))
            self._timeouts = _view(self._base + 128, (1,), torch.int32)
            self.workspace = torch.zeros(capi.workspace_bytes(max_rows, vocab, False), dtype=torch.uint8,
                                         device=self.device)
            # Per-phase mode: the FP64 path's scratch (16 bytes per token per row, this GPU only).
            self.scratch = (torch.empty(max_rows * vocab * 16, dtype=torch.uint8, device=self.device)
                            if phases else None)
        if connect:
            self.connect(list((exchange or _all_gather(group))(self.entry)))

    def connect(self, entries: Sequence) -> None:
        """Maps every rank's block (entries in rank order, from ``entry``)."""
        import torch

        if len(entries) != self.shards or tuple(entries[self.rank]) != self.entry:
            raise ValueError("connect needs one entry per shard, this plan's at its rank")
        lib = capi.load()
        with torch.cuda.device(self.device):
            for handle_g, _pid in entries:
                if handle_g in _LOCAL_BLOCKS:
                    self._bases.append(_LOCAL_BLOCKS[handle_g])
                else:
                    peer = ctypes.c_void_p()
                    capi.check(lib.es_ipc_open(handle_g, ctypes.byref(peer)))
                    self._bases.append(peer.value)
                    self._opened.append(peer.value)

    def _ptrs(self, name: str):
        arr = (ctypes.c_void_p * capi.MAX_SHARDS)()
        for g, base in enumerate(self._bases):
            arr[g] = base + self._layout[name] if name in self._layout else base + {"ready": 0, "done": 64, "slots": 192}[name]
        return arr

    def _shards(self):
        """The es_shards of this plan's calls; built once, since the peers'
        addresses do not change after connect (a call sets the request range
        and the epoch, and es_verify_sharded reads it only while enqueueing)."""
        if self._sh is None:
            sh = capi.Shards()
            sh.count, sh.rank, sh.cols, sh.vocab = self.shards, self.rank, self.cols, self.vocab
            if self.phases:
                sh.phases = 1
                sh.exchange = self._ptrs("exchange")
                sh.scratch = self.scratch.data_ptr()
            for name in ["target", "tokens", "accepted", "status", "path", "ready"]:
                setattr(sh, name, self._ptrs({"target": "logits"}.get(name, name)))
            if self.full_q:
                sh.draft = self._ptrs("draft")
            self._sh = sh
        return self._sh

    def timeouts(self) -> int:
        """Waits for peer GPUs that gave up so far (synchronizes)."""
        import torch

        torch.cuda.synchronize(self.device)
        return int(self._timeouts.item())

    # ---- the steps of a call: verify_sharded runs launch then finish;
    # several shards on one GPU need signal_ready, launch, signal_done and
    # wait_done, each issued for every shard before the next ----
    def signal_ready(self, stream=None) -> None:
        capi.check(capi.load().es_shard_signal(ctypes.c_void_p(self._base), self.epoch, self._stream(stream)))

    def launch(self, rows: int, cu_rows, draft_ids, *, params: CudaRequestParams, rng: CudaRngKey, mask=None,
               mode: str = "ratio", dispatch: str = "auto", top_k_top_p: bool = True, stream=None) -> None:
        requests = cu_rows.numel() - 1
        if rows > self.max_rows or requests > self.max_requests:
            raise ValueError("input exceeds plan capacity")
        if len(self._bases) != self.shards:
            raise RuntimeError("the plan is not connected to its peers")
        if mode not in _MODES or dispatch not in ("auto", "fused"):
            raise ValueError("mode must be ratio/coupled; dispatch must be auto/fused")
        tensors = dict(target_logits=self.logits[:rows], cu_rows=cu_rows, draft_ids=draft_ids,
                       draft_logits=self.draft_logits[:rows] if self.full_q else None,
                       temperature=params.temperature, top_k=params.top_k, top_p=params.top_p, min_p=params.min_p,
                       draft_kind=params.draft_kind, seeds=rng.seed, stream_ids=rng.stream_id,
                       positions=rng.positions, mask=mask, workspace=self.workspace, tokens=self.out.tokens,
                       accepted_len=self.out.accepted_len, status=self.out.status, path_used=self.out.path_used)
        args = capi.args_of(tensors, mode=_MODES[mode], dispatch=_DISPATCH[dispatch], max_draft=self.max_draft,
                            list_max=self.list_max if top_k_top_p else 0)
        sh = self._shards()
        sh.req_begin, sh.req_end = (0, requests) if self.phases else request_range(requests, self.shards, self.rank)
        sh.epoch = self.epoch
        capi.check(capi.load().es_verify_sharded(ctypes.byref(args), ctypes.byref(sh), self._stream(stream)))
        self.out.num_requests = requests

    def signal_done(self, stream=None) -> None:
        capi.check(capi.load().es_shard_signal(ctypes.c_void_p(self._base + 64), self.epoch, self._stream(stream)))

    def wait_done(self, stream=None) -> None:
        flags = self._ptrs("done")
        capi.check(capi.load().es_shard_wait(ctypes.cast(flags, ctypes.POINTER(ctypes.c_void_p)), self.shards,
                                             self.epoch, ctypes.c_void_p(self._base + 128), self._stream(stream)))

    def finish(self, stream=None) -> None:
        """The end of a call: this GPU's tag into its slot on every GPU, then
        every GPU's tag in this GPU's slots (one launch)."""
        flags = self._ptrs("slots")
        capi.check(capi.load().es_shard_finish(ctypes.c_void_p(self._base + 192),
                                               ctypes.cast(flags, ctypes.POINTER(ctypes.c_void_p)), self.shards,
                                               self.epoch, ctypes.c_void_p(self._base + 128), self._stream(stream)))

    def _stream(self, stream):
        import torch

        return ctypes.c_void_p((stream or torch.cuda.current_stream(self.device)).cuda_stream)

    def close(self) -> None:
        """Unmaps the peers' blocks and frees this GPU's (after synchronizing)."""
        import torch

        if getattr(self, "_base", None) is None:
            return
        torch.cuda.synchronize(self.device)
        lib = capi.load()
        for ptr in self._opened:
            lib.es_ipc_close(ctypes.c_void_p(ptr))
        _LOCAL_BLOCKS.pop(self._handle, None)
        lib.es_ipc_free(ctypes.c_void_p(self._base))
        self._base = None


def verify_sharded(plan: ShardedPlan, rows: int, cu_rows, draft_ids, *, params: CudaRequestParams, rng: CudaRngKey,
                   mask=None, mode: str = "ratio", dispatch: str = "auto", top_k_top_p: bool = True) -> CudaOutput:
    """One GPU's part of a sharded call over plan.logits[:rows]; returns plan.out
    (complete for every request once the stream reaches the end of the call)."""
    plan.epoch += 1
    plan.launch(rows, cu_rows, draft_ids, params=params, rng=rng, mask=mask, mode=mode, dispatch=dispatch,
                top_k_top_p=top_k_top_p)  # raises this GPU's ready flag first
    plan.finish()
    return plan.out
