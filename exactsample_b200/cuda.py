"""The device-side decode API: ``plan`` once, then ``verify`` every step.

This module replaces the reference's ``exactsample.cuda``
(python/exactsample/cuda.py:15-198) for callers such as a vLLM bridge: its
dataclasses, the signatures of ``plan`` / ``CudaPlan`` / ``verify``, the torch
op ``torch.ops.exactsample.verify_out`` (schema of csrc/bindings.cpp:139-146),
and its exception types and messages are kept. The op runs the B200 kernels of
``libexactsample_b200.so`` through that library's C ABI
(include/exactsample_b200.h).

A plan owns one workspace; the caller owns every input and output tensor and
makes them before the first step. A step (``verify``) launches kernels on
tensors that already live on the device: it neither allocates nor reads
anything from the host. If the native library is missing, the call raises;
nothing falls back to the CPU.
"""
from __future__ import annotations

import os
import threading
from dataclasses import dataclass
from pathlib import Path
from typing import Any

_MODES = {"ratio": 0, "coupled": 1}
_DISPATCH = {"auto": 0, "reference": 1, "fused": 2}


@dataclass(frozen=True)
class CudaRequestParams:
    temperature: Any  # CUDA float64 [R]
    top_k: Any  # CUDA int64 [R], 0 disables
    top_p: Any  # CUDA float64 [R]
    min_p: Any  # CUDA float64 [R]
    draft_kind: Any  # CUDA int64 [R], 0=one_hot, 1=full


@dataclass(frozen=True)
class CudaRngKey:
    seed: Any  # CUDA int64 [R]; signed storage of uint64 key bits
    stream_id: Any  # CUDA int64 [R], values in [0, 2**32)
    positions: Any  # CUDA int64 [rows], values in [0, 2**32)


@dataclass
class CudaOutput:
    tokens: Any
    accepted_len: Any
    status: Any
    path_used: Any
    num_requests: int = 0


def library_path(path: str | os.PathLike[str] | None = None) -> Path:
    """The torch-op library: ``path``, else $EXACTSAMPLE_LIBRARY, else next to this file."""
    chosen = path or os.environ.get("EXACTSAMPLE_LIBRARY")
    return Path(chosen) if chosen else Path(__file__).with_name("exactsample_cuda.so")


def load_library(path: str | os.PathLike[str] | None = None) -> None:
    """Register ``torch.ops.exactsample.verify_out`` from the prebuilt library (no JIT build)."""
    import torch

    if hasattr(torch.ops.exactsample, "verify_out"):
        return
    library = library_path(path)
    if not library.is_file():
        raise RuntimeError(f"exactsample CUDA library is missing: {library}. Build it with "
                           "`python -m exactsample_b200.build`, or set EXACTSAMPLE_LIBRARY.")
    torch.ops.load_library(str(library.resolve()))


def _check_count(name: str, value) -> None:
    if isinstance(value, bool) or not isinstance(value, int) or value < (1 if name == "vocab" else 0):
        raise ValueError(f"{name} must be a nonnegative integer (vocab must be positive)")
    if value >= 2**31:
        raise ValueError(f"{name} exceeds kernel int32 indexing")


class _Ownership:
    """Who may use a plan's workspace: one host call at a time (a non-blocking
    lock), and one stream until the last call's completion event has fired."""

    def __init__(self, device):
        import torch

        self.lock = threading.Lock()
        self.event = torch.cuda.Event(enable_timing=False)
        self.stream = None      # cuda_stream handle of the last call
        self.retained = ()      # tensors of the last call, alive until it completes
        # Create the event now, outside any decode step.
        self.event.record(torch.cuda.current_stream(device))
        self.event.synchronize()

    def claim(self, stream, capturing: bool = False) -> None:
        if not self.lock.acquire(blocking=False):
            raise RuntimeError("exactsample workspace is already in use by another host call")
        if capturing:  # events cannot be queried inside a capture
            return
        if self.stream is not None and self.stream != stream.cuda_stream and not self.event.query():
            self.lock.release()
            raise RuntimeError("exactsample workspace is in flight on another stream; synchronize or use a separate plan")

    def enqueued(self, stream, tensors) -> None:
        """Ties every tensor's allocation and the workspace to the launching stream."""
        for tensor in tensors:
            if tensor is not None:
                tensor.record_stream(stream)
        self.retained = tensors
        self.stream = stream.cuda_stream
        self.event.record(stream)

    def release(self) -> None:
        self.lock.release()

    def drain(self) -> None:
        with self.lock:
            self.event.synchronize()
            self.retained = ()
            self.stream = None


class CudaPlan:
    """A workspace sized for ``max_rows`` rows and its ownership rules.

    Calls queued on one stream run in order. A call from a second stream while
    the previous call is still running raises instead of racing on the
    workspace. A call's tensors belong to it until it has finished on the
    device (``synchronize``, or any later work on the same stream), so the
    caller must not overwrite them before then; each tensor is recorded on
    the launching stream, so the caching allocator cannot hand its memory to
    someone else early.

    CUDA graph capture is refused, as in the reference, unless the plan is
    made with ``graphs=True``: ``verify`` then may be captured (it allocates
    nothing and never synchronizes; its kernels and their programmatic
    dependency are recorded as graph nodes). A captured call reads and writes
    the tensors it was captured with, so a replay takes its inputs from those
    same tensors; the ownership checks between streams are skipped during
    capture, and replays of a plan's graphs must not overlap each other or
    eager calls on the plan.
    """

    def __init__(self, max_rows: int, max_requests: int, max_draft: int, vocab: int,
                 *, device: Any = "cuda", caps: dict | None = None, reference: bool = False,
                 graphs: bool = False):
        import torch

        if caps:
            raise ValueError("caps is reserved; v1 supports the default capabilities only")
        for name, value in (("max_rows", max_rows), ("max_requests", max_requests),
                            ("max_draft", max_draft), ("vocab", vocab)):
            _check_count(name, value)
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("CudaPlan requires a CUDA device")
        self.max_rows, self.max_requests, self.max_draft, self.vocab = max_rows, max_requests, max_draft, vocab
        # Kept sets of at most this many tokens are finished as an exact FP64
        # list; 0 sends every row to the full-row path (results are the same).
        self.list_max = 256
        self.graphs = graphs
        self.device = torch.device("cuda", torch.cuda.current_device() if device.index is None else device.index)
        self.reference = reference
        # The reference's sizing, so plans are interchangeable: 8 bytes of
        # header, then per row 32 bytes plus max(12288, 20 * vocab with reference=True).
        self.workspace_bytes = 8 + max_rows * (32 + max(12288, 20 * vocab if reference else 0))
        self.workspace = torch.zeros(self.workspace_bytes, dtype=torch.uint8, device=self.device)
        self._owner = _Ownership(self.device)

    def allocate_output(self) -> CudaOutput:
        import torch

        def ints(*shape, dtype=torch.int32):
            return torch.empty(shape, device=self.device, dtype=dtype)

        return CudaOutput(ints(self.max_requests, self.max_draft + 1, dtype=torch.int64), ints(self.max_requests),
                          ints(self.max_requests), ints(self.max_requests))

    def fallbacks(self) -> int:
        """How many times the last call had to settle a draw or a cut in FP64
        because the FP32 bounds left it open. Waits for that call to finish."""
        import torch

        self.synchronize()
        return int(self.workspace[4:8].view(torch.int32).item())

    def synchronize(self) -> None:
        """Blocks until this plan's last call has finished; after that any
        stream may use the workspace."""
        self._owner.drain()


def plan(max_rows: int, max_requests: int, max_draft: int, vocab: int,
         caps: dict | None = None, *, device: Any = "cuda", reference: bool = False,
         graphs: bool = False) -> CudaPlan:
    return CudaPlan(max_rows, max_requests, max_draft, vocab, device=device, caps=caps, reference=reference,
                    graphs=graphs)


def _check_call(target_logits, cu_rows, params, rng, plan: CudaPlan, mode: str, dispatch: str) -> int:
    """Host-side checks made before touching the device; returns the request count."""
    if mode not in _MODES or dispatch not in _DISPATCH:
        raise ValueError("mode must be ratio/coupled; dispatch must be auto/reference/fused")
    if dispatch == "reference" and not plan.reference:
        raise ValueError("dispatch='reference' needs a plan made with reference=True")
    if not isinstance(params, CudaRequestParams) or not isinstance(rng, CudaRngKey):
        raise TypeError("CUDA verify requires CudaRequestParams and CudaRngKey containing device tensors")
    if target_logits.ndim != 2 or cu_rows.ndim != 1 or cu_rows.numel() < 1:
        raise ValueError("target_logits must be 2D and cu_rows a nonempty 1D tensor")
    requests = cu_rows.numel() - 1
    rows, vocab = target_logits.shape
    if rows > plan.max_rows or requests > plan.max_requests or vocab != plan.vocab:
        raise ValueError("input exceeds plan capacity or has a different vocabulary")
    if target_logits.device != plan.device:
        raise ValueError("input and plan must be on the same CUDA device")
    return requests


def verify(target_logits, cu_rows, draft_ids, *, params: CudaRequestParams,
           rng: CudaRngKey, plan: CudaPlan, out: CudaOutput,
           draft_logits=None, mask=None, mode: str = "ratio", dispatch: str = "auto",
           top_k_top_p: bool = True) -> CudaOutput:
    """Samples or verifies a ragged batch and writes the results into ``out``.

    Request i owns rows ``cu_rows[i]:cu_rows[i + 1]`` of ``target_logits``:
    one row per draft token plus a final bonus row. Every tensor must already
    be on the plan's device. ``draft_logits`` (full-q drafts only) give the
    log weights of the distribution the drafter really sampled from, with its
    own processing already applied; the target's filters are not applied to
    them, and the bonus rows' entries are not read. The call writes output
    rows ``0 .. out.num_requests - 1`` and leaves the rest of ``out`` alone.
    Bad values inside device tensors (NaN logits, an out-of-range parameter)
    do not raise: they show up later as that request's status.

    ``top_k_top_p=False`` tells the kernels that no request has a top-k below
    the vocabulary or a top-p below 1 (a caller that keeps its sampling
    parameters on the host knows this). It never changes a result: a request
    that does filter is finished on the full-row path.
    """
    import torch

    requests = _check_call(target_logits, cu_rows, params, rng, plan, mode, dispatch)
    load_library()
    tensors = (target_logits, cu_rows, draft_ids, draft_logits, params.temperature, params.top_k, params.top_p,
               params.min_p, params.draft_kind, rng.seed, rng.stream_id, rng.positions, mask, plan.workspace,
               out.tokens, out.accepted_len, out.status, out.path_used)
    with torch.cuda.device(plan.device):
        capturing = torch.cuda.is_current_stream_capturing()
        if capturing and not plan.graphs:
            raise RuntimeError("exactsample v1 does not support CUDA graph capture")
        stream = torch.cuda.current_stream(plan.device)
        owner = plan._owner
        owner.claim(stream, capturing)
        try:
            if any(t is not None and not isinstance(t, torch.Tensor) for t in tensors):
                raise TypeError("all CUDA arguments must be preallocated tensors")
            if any(t is not None and t.requires_grad for t in tensors):
                raise ValueError("exactsample is an inference operator and does not support autograd")
            list_max = plan.list_max if top_k_top_p else 0
            try:
                torch.ops.exactsample.verify_out(*tensors, _MODES[mode], _DISPATCH[dispatch], plan.max_draft, list_max)
            finally:
                # Even a failed launch may have enqueued work: keep ownership
                # (a captured call enqueues nothing until its graph replays).
                if not capturing:
                    owner.enqueued(stream, [t for t in tensors if t is not None and t.device == plan.device])
            out.num_requests = requests
        finally:
            owner.release()
    return out
