"""The work around one verify call in a serving engine's decode step,
independent of the engine.

The reference's vLLM bridge (python/exactsample/vllm_bridge.py:53-327, with
vllm_async.py:43-85) surrounds exactsample.cuda.verify with four steps. This
module gives each as an engine-independent piece on torch tensors, so an
engine integration is the mapping of its own batch objects onto them:

* Grammar masks. An engine keeps packed grammar bitmasks only for its
  constrained requests: one row per logits row of each such request, in its
  own order. ``grammar_row_sources`` checks that layout against the step's
  offsets and maps every logits row to its bitmask row (-1: unconstrained).
  ``grammar_mask_rows`` builds the dense int32 mask on the host (the
  reference's function, vllm_bridge.py:117-152, with its errors);
  ``densify_grammar_mask`` builds it on the device from a bitmask already
  there, with one row copy, so the mask does not cross PCIe twice.
* Staging. ``StepStaging`` packs a step's per-request parameters and the
  positions of its draft rows into a pinned host slot (a ring of three, each
  rewritten only after its previous copy ran) and moves them with one
  asynchronous copy (vllm_bridge.py:62-83, 270-290).
* Drafts. ``gather_drafts`` reads request r's d-th proposal from the engine's
  per-row token vector at row offsets[r] + 1 + d (vllm_bridge.py:286-299).
* After the call. ``committed_counts`` gives accepted drafts plus one, zero
  for a failed request (vllm_bridge.py:312-320). ``StatusCopy`` snapshots the
  statuses and tokens, copies them to pinned host memory on a side stream
  behind one event, and gives a failed request no tokens when the host reads
  them (vllm_async.py:43-85).

``decode_step`` runs them in order around one verify call.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np

from .types import Status


class DecodeStepError(RuntimeError):
    """Malformed step metadata: the step cannot be submitted safely."""


# ---------------------------------------------------------------- grammar masks
def grammar_row_sources(req_ids, offsets, grammar_req_ids, bitmask_rows: int) -> np.ndarray:
    """For every logits row of the step, the row of the engine's grammar
    bitmask that constrains it, or -1.

    ``offsets`` (length R + 1) gives request r the logits rows
    [offsets[r], offsets[r + 1]); ``grammar_req_ids`` lists the constrained
    requests in the bitmask's order, each owning as many consecutive bitmask
    rows as it has logits rows. Raises ValueError when the bitmask does not
    describe exactly those rows.
    """
    offsets = np.asarray(offsets, dtype=np.int64)
    index_of = {request: i for i, request in enumerate(req_ids)}
    if len(index_of) != len(req_ids) or len(set(grammar_req_ids)) != len(grammar_req_ids):
        raise ValueError("duplicate request identity in grammar mapping")
    sources = np.full(int(offsets[-1]) if offsets.size else 0, -1, dtype=np.int64)
    used = 0
    for request in grammar_req_ids:
        if request not in index_of:
            raise ValueError("grammar request missing from sampled batch")
        r = index_of[request]
        begin, end = int(offsets[r]), int(offsets[r + 1])
        if used + (end - begin) > bitmask_rows:
            raise ValueError("grammar bitmask has fewer rows than scheduled logits")
        sources[begin:end] = np.arange(used, used + end - begin)
        used += end - begin
    if used != bitmask_rows:
        raise ValueError("grammar bitmask has unused rows; unsupported layout")
    return sources


def grammar_mask_rows(req_ids, offsets, grammar_req_ids, bitmask, vocab, out=None) -> np.ndarray:
    """The dense packed mask of the step on the host: int32 [rows, ceil(vocab / 32)],
    the constraining bitmask row for constrained logits rows and all ones
    (-1) for the others. ``out`` (e.g. a pinned buffer's NumPy view)
    receives it if given."""
    words = (vocab + 31) // 32
    bitmask = np.asarray(bitmask)
    if bitmask.ndim != 2 or bitmask.shape[1] != words or bitmask.dtype != np.int32:
        raise ValueError("grammar bitmask has unexpected shape/dtype")
    sources = grammar_row_sources(req_ids, offsets, grammar_req_ids, bitmask.shape[0])
    shape = (sources.size, words)
    if out is None:
        out = np.empty(shape, dtype=np.int32)
    elif out.shape != shape or out.dtype != np.int32:
        raise ValueError("grammar mask output has unexpected shape/dtype")
    out.fill(-1)
    rows = np.flatnonzero(sources >= 0)
    out[rows] = bitmask[sources[rows]]
    return out


def densify_grammar_mask(bitmask, sources: np.ndarray, out):
    """The dense mask built where the bitmask already is (a device tensor, as
    grammar backends fill it): ``out[i] = bitmask[sources[i]]`` for
    constrained rows, all ones elsewhere. ``sources`` comes from
    grammar_row_sources; ``out`` is int32 [len(sources), words]."""
    import torch

    if bitmask.dtype != torch.int32 or out.dtype != torch.int32 or bitmask.shape[1:] != out.shape[1:]:
        raise ValueError("grammar bitmask and mask must be int32 with the same words per row")
    if out.shape[0] != sources.size:
        raise ValueError("grammar mask output has unexpected shape/dtype")
    out.fill_(-1)
    rows = np.flatnonzero(sources >= 0)
    if rows.size:
        dst = torch.as_tensor(rows, dtype=torch.int64).to(out.device, non_blocking=True)
        src = torch.as_tensor(sources[rows], dtype=torch.int64).to(bitmask.device, non_blocking=True)
        out.index_copy_(0, dst, bitmask.index_select(0, src))
    return out


# ---------------------------------------------------------------- staging
@dataclass
class StagedStep:
    """One step's device-side parameters (views into the staging buffer)."""

    params: Any       # CudaRequestParams
    seeds: Any        # int64 [R], uint64 bits
    draft_index: Any  # int64 [R, max_draft]: logits row of each proposal, -1 past a request's drafts
    top_k_top_p: bool  # some request filters by top-k or top-p (the verify hint)
    counts: np.ndarray  # drafts per request (host)


class StepStaging:
    """Pinned host staging of per-step parameters, one copy per step.

    Each step's parameters ([temperature, top_k, top_p, min_p, seed] x R,
    then R x max_draft draft-row indices, as 8-byte words) are written into
    the next of ``depth`` pinned slots and copied to the device without
    blocking; a slot is rewritten only after the event recorded behind its
    last copy, so the host can run up to ``depth`` steps ahead of the GPU.
    On a CPU device the copies are plain.
    """

    FIELDS = ("temperature", "top_k", "top_p", "min_p", "seeds")
    FLOATS = ("temperature", "top_p", "min_p")

    def __init__(self, max_requests: int, max_draft: int, vocab: int, *, device="cuda", depth: int = 3):
        import torch

        self.max_requests, self.max_draft, self.vocab = int(max_requests), int(max_draft), int(vocab)
        self.device = torch.device(device)
        cuda = self.device.type == "cuda"
        words = self.max_requests * (len(self.FIELDS) + self.max_draft)
        self.slots = [torch.empty(words, dtype=torch.int64, pin_memory=cuda) for _ in range(depth)]
        self.events = [torch.cuda.Event() for _ in range(depth)] if cuda else None
        self.next = 0
        self.staged = torch.empty(words, dtype=torch.int64, device=self.device)
        self.kind = torch.zeros(self.max_requests, dtype=torch.int64, device=self.device)  # one-hot proposals

    def stage(self, offsets, *, temperature, top_k, top_p, min_p, seeds) -> StagedStep:
        """Stages one step. ``offsets`` (host, length R + 1) is the step's
        ragged row layout: request r has offsets[r + 1] - offsets[r] - 1
        drafts. Parameters are host arrays of length R; a top_k equal to the
        vocabulary means no top-k (as engines encode it) and becomes 0."""
        import torch

        from .cuda import CudaRequestParams

        offsets = np.asarray(offsets, dtype=np.int64)
        requests = offsets.size - 1
        if requests < 0 or requests > self.max_requests or (requests and offsets[0] != 0):
            raise DecodeStepError("ragged metadata does not describe the step's logits")
        counts = np.diff(offsets) - 1
        if np.any(counts < 0) or np.any(counts > self.max_draft):
            raise DecodeStepError("invalid draft counts for the staging capacity")
        slot = self.next
        self.next = (slot + 1) % len(self.slots)
        if self.events is not None:
            self.events[slot].synchronize()  # the slot's previous copy has run
        fields = len(self.FIELDS)
        words = requests * (fields + self.max_draft)
        host = self.slots[slot].numpy()[:words]
        values = dict(temperature=temperature, top_k=top_k, top_p=top_p, min_p=min_p, seeds=seeds)
        for i, name in enumerate(self.FIELDS):
            view = host[i * requests:(i + 1) * requests]
            given = np.asarray(values[name])
            if given.shape != (requests,):
                raise DecodeStepError(f"{name} must have one value per request")
            if name in self.FLOATS:
                view.view(np.float64)[:] = given.astype(np.float64)
            elif name == "seeds":
                view[:] = given.astype(np.uint64).view(np.int64) if given.dtype.kind == "u" else given.astype(np.int64)
            else:
                view[:] = given.astype(np.int64)
        top_k_view = host[requests:2 * requests]
        top_k_view[top_k_view == self.vocab] = 0
        draft_index = host[fields * requests:words].reshape(requests, self.max_draft)
        draft_index[:] = offsets[:-1, None] + 1 + np.arange(self.max_draft)
        draft_index[np.arange(self.max_draft) >= counts[:, None]] = -1
        hint = bool((top_k_view > 0).any() or (host[2 * requests:3 * requests].view(np.float64) < 1).any())
        staged = self.staged[:words]
        staged.copy_(self.slots[slot][:words], non_blocking=self.events is not None)
        if self.events is not None:
            self.events[slot].record()
        part = {name: staged[i * requests:(i + 1) * requests] for i, name in enumerate(self.FIELDS)}
        for name in self.FLOATS:
            part[name] = part[name].view(torch.float64)
        params = CudaRequestParams(part["temperature"], part["top_k"], part["top_p"], part["min_p"],
                                   self.kind[:requests])
        return StagedStep(params, part["seeds"], staged[fields * requests:].view(requests, self.max_draft), hint,
                          counts)


# ---------------------------------------------------------------- drafts and results
def gather_drafts(row_tokens, draft_index, out=None):
    """Request r's d-th proposal: ``row_tokens[draft_index[r, d]]`` (the
    engine's per-logits-row token vector), -1 where the index is -1."""
    gathered = row_tokens[draft_index.clamp(min=0)].to(draft_index.dtype)
    gathered.masked_fill_(draft_index < 0, -1)
    if out is None:
        return gathered
    out.copy_(gathered)
    return out


def committed_counts(out, requests: int):
    """Tokens each request commits this step: accepted drafts plus one (the
    residual or bonus token), zero for a failed request."""
    counts = out.accepted_len[:requests].to(out.tokens.dtype) + 1
    return counts.masked_fill_(out.status[:requests] != int(Status.OK), 0)


class StatusCopy:
    """The statuses, tokens and accepted lengths of a call, on their way to
    the host. Snapshots are taken on the current stream (the plan's output
    buffers are reused by the next call), copied to pinned host memory on
    ``copy_stream`` behind one event; nothing blocks until ``get``."""

    def __init__(self, out, requests: int, copy_stream=None):
        import torch

        self.requests = int(requests)
        snapshots = [out.status[:requests].clone(), out.tokens[:requests].clone(), out.accepted_len[:requests].clone()]
        self.event = None
        if snapshots[0].is_cuda:
            main = torch.cuda.current_stream(snapshots[0].device)
            side = copy_stream or main
            side.wait_stream(main)
            self.host = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in snapshots]
            with torch.cuda.stream(side):
                for h, t in zip(self.host, snapshots):
                    h.copy_(t, non_blocking=True)
                    t.record_stream(side)
                self.event = torch.cuda.Event()
                self.event.record(side)
        else:
            self.host = snapshots
        self._snapshots = snapshots  # kept alive until the copies ran

    def get(self):
        """(statuses, committed tokens per request): a failed request commits
        none, whatever its token row holds."""
        if self.event is not None:
            self.event.synchronize()
        status, tokens, accepted = (t.numpy() for t in self.host)
        committed = [[] if status[r] != int(Status.OK) else tokens[r, :int(accepted[r]) + 1].tolist()
                     for r in range(self.requests)]
        return status.copy(), committed


def decode_step(logits, offsets, row_tokens, positions, *, staging: StepStaging, plan, out, temperature, top_k,
                top_p, min_p, seeds, stream_ids=None, grammar=None, mask_buffer=None, mode: str = "coupled",
                dispatch: str = "auto", copy_stream=None):
    """One decode step around verify: stage the parameters, gather the drafts,
    densify the grammar mask, verify, and start the status copy.

    ``logits`` [rows, vocab] are the raw target logits of the step (request
    r's rows [offsets[r], offsets[r + 1]), its drafts first and its bonus
    row last); ``row_tokens`` [rows] holds the token each logits row's
    input carries, from which proposals are read; ``positions`` [rows] are
    the rows' sequence positions. ``grammar`` is (req_ids, grammar_req_ids,
    bitmask) with the bitmask on the device, and ``mask_buffer`` int32
    [>= rows, words] receives the dense mask. Returns (out, committed_counts,
    StatusCopy). The mode defaults to coupled verification, as proposals
    from a greedy draft model call for.
    """
    import torch

    from .cuda import CudaRngKey, verify

    offsets_np = np.asarray(offsets, dtype=np.int64)
    requests, rows = offsets_np.size - 1, int(logits.shape[0])
    if requests < 1 or offsets_np[0] != 0 or offsets_np[-1] != rows:
        raise DecodeStepError("ragged metadata does not describe the step's logits")
    step = staging.stage(offsets_np, temperature=temperature, top_k=top_k, top_p=top_p, min_p=min_p, seeds=seeds)
    drafts = gather_drafts(row_tokens, step.draft_index) if staging.max_draft else \
        torch.empty((requests, 0), dtype=torch.int64, device=logits.device)
    cu_rows = torch.as_tensor(offsets_np).to(logits.device, non_blocking=True)
    if stream_ids is None:
        streams = torch.zeros(requests, dtype=torch.int64, device=logits.device)
    else:
        streams = torch.as_tensor(np.asarray(stream_ids, dtype=np.int64)).to(logits.device, non_blocking=True)
    mask = None
    if grammar is not None and len(grammar[1]):
        req_ids, grammar_req_ids, bitmask = grammar
        if mask_buffer is None or mask_buffer.shape[0] < rows:
            raise DecodeStepError("a grammar needs a mask_buffer with a row per logits row")
        sources = grammar_row_sources(req_ids, offsets_np, grammar_req_ids, int(bitmask.shape[0]))
        mask = densify_grammar_mask(bitmask, sources, mask_buffer[:rows])
    rng = CudaRngKey(step.seeds, streams, positions.to(torch.int64))
    verify(logits, cu_rows, drafts, params=step.params, rng=rng, plan=plan, out=out, mask=mask, mode=mode,
           dispatch=dispatch, top_k_top_p=step.top_k_top_p)
    return out, committed_counts(out, requests), StatusCopy(out, requests, copy_stream)
