"""Seeded synthetic inputs for the benchmark configurations and the parity tests.

No public dataset is involved: the reference benchmarks captured Qwen3-8B
logits, which are not available here, so every configuration is generated
from a master seed with the shapes and value distributions the benchmark
plan names (vocabulary 151,936, fp32 logits):

* each row is N(0, 2^2) noise plus, on 64 uniformly chosen token IDs, a peak
  drawn from U(8, 16), built in float64 and rounded to float32;
* each request gets a uint64 seed (stored as int64 bits), stream = its
  index, and a first position drawn from U[0, 32768); a request's rows use
  consecutive positions.

Workloads are plain NumPy (host) arrays; callers move them to a device.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

VOCAB = 151_936
QWEN = dict(temperature=0.6, top_k=20, top_p=0.95, min_p=0.0)
TEMPERATURE_ONLY = dict(temperature=1.0, top_k=0, top_p=1.0, min_p=0.0)


@dataclass
class Workload:
    """One call's inputs. Per-request parameters are arrays of length R."""
    name: str
    logits: np.ndarray            # float32 or float64 [M, V]
    cu_rows: np.ndarray           # int64 [R + 1]
    draft_ids: np.ndarray         # int64 [R, D] (D >= 1 columns; unused entries -1)
    temperature: np.ndarray       # float64 [R]
    top_k: np.ndarray             # int64 [R]
    top_p: np.ndarray             # float64 [R]
    min_p: np.ndarray             # float64 [R]
    draft_kind: np.ndarray        # int64 [R], 0 one-hot, 1 full
    seed: np.ndarray              # uint64 [R]
    stream_id: np.ndarray         # int64 [R]
    positions: np.ndarray         # int64 [M]
    mode: str = "ratio"
    mask: np.ndarray | None = None          # int32 [M, ceil(V/32)]
    draft_logits: np.ndarray | None = None  # like logits
    notes: dict = field(default_factory=dict)

    @property
    def rows(self) -> int:
        return int(self.logits.shape[0])

    @property
    def requests(self) -> int:
        return int(self.cu_rows.size - 1)

    @property
    def vocab(self) -> int:
        return int(self.logits.shape[1])

    def seeds_int64(self) -> np.ndarray:
        return self.seed.astype(np.uint64).view(np.int64)

    def algorithmic_bytes(self) -> int:
        """One read of every input the call streams (logits, full-q rows, mask)."""
        total = self.logits.nbytes
        if self.draft_logits is not None:
            full_rows = 0
            for r in range(self.requests):
                if self.draft_kind[r] == 1:
                    full_rows += max(int(self.cu_rows[r + 1] - self.cu_rows[r]) - 1, 0)
            total += full_rows * self.vocab * self.draft_logits.itemsize
        if self.mask is not None:
            total += self.mask.nbytes
        return int(total)

    def subset(self, requests) -> "Workload":
        """The same inputs restricted to some requests, rows renumbered."""
        requests = list(requests)
        row_index = np.concatenate([np.arange(self.cu_rows[r], self.cu_rows[r + 1]) for r in requests]) \
            if requests else np.zeros(0, np.int64)
        sizes = [int(self.cu_rows[r + 1] - self.cu_rows[r]) for r in requests]
        pick = np.array(requests, dtype=np.int64)
        return Workload(
            name=self.name, logits=self.logits[row_index], cu_rows=np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64),
            draft_ids=self.draft_ids[pick], temperature=self.temperature[pick], top_k=self.top_k[pick],
            top_p=self.top_p[pick], min_p=self.min_p[pick], draft_kind=self.draft_kind[pick], seed=self.seed[pick],
            stream_id=self.stream_id[pick], positions=self.positions[row_index], mode=self.mode,
            mask=None if self.mask is None else self.mask[row_index],
            draft_logits=None if self.draft_logits is None else self.draft_logits[row_index], notes=dict(self.notes))


def packed_mask(allowed: np.ndarray) -> np.ndarray:
    """Pack a boolean [rows, V] array into xgrammar int32 words (bit t%32 of word t//32)."""
    allowed = np.asarray(allowed, dtype=bool)
    rows, vocab = allowed.shape
    padded = np.zeros((rows, (vocab + 31) // 32 * 32), dtype=bool)
    padded[:, :vocab] = allowed
    return np.packbits(padded, axis=1, bitorder="little").view("<u4").astype(np.uint32).view(np.int32)


def synthetic_rows(g: np.random.Generator, rows: int, vocab: int = VOCAB, peaks: int = 64) -> np.ndarray:
    """N(0, 2^2) noise plus U(8, 16) on `peaks` random token IDs per row, float64 then float32."""
    out = g.normal(0.0, 2.0, size=(rows, vocab))
    for r in range(rows):
        ids = g.choice(vocab, size=min(peaks, vocab), replace=False)
        out[r, ids] += g.uniform(8.0, 16.0, size=ids.size)
    return out.astype(np.float32)


def _rng_fields(g: np.random.Generator, requests: int, rows_per_request: list[int]):
    seed = g.integers(0, 2**64, size=requests, dtype=np.uint64)
    stream = np.arange(requests, dtype=np.int64)
    first = g.integers(0, 32768, size=requests)
    positions = np.concatenate([first[r] + np.arange(n) for r, n in enumerate(rows_per_request)]).astype(np.int64) \
        if requests else np.zeros(0, np.int64)
    return seed, stream, positions


def _params(requests: int, settings: dict):
    return (np.full(requests, settings["temperature"], np.float64), np.full(requests, settings["top_k"], np.int64),
            np.full(requests, settings["top_p"], np.float64), np.full(requests, settings.get("min_p", 0.0), np.float64))


def sampling(requests: int, settings: dict = QWEN, *, master_seed: int = 1, vocab: int = VOCAB,
             ties_rows: int = 0, name: str = "sampling") -> Workload:
    """One row per request (C1, C2a, C2b, C5a)."""
    g = np.random.default_rng(master_seed)
    logits = synthetic_rows(g, requests, vocab)
    for r in g.choice(requests, size=min(ties_rows, requests), replace=False) if ties_rows else []:
        top = np.argsort(-logits[r], kind="stable")[:3]
        others = g.choice(np.setdiff1d(np.arange(vocab), top), size=3, replace=False)
        logits[r, others] = logits[r, top]
    seed, stream, positions = _rng_fields(g, requests, [1] * requests)
    t, k, p, m = _params(requests, settings)
    return Workload(name, logits, np.arange(requests + 1, dtype=np.int64), np.full((requests, 1), -1, np.int64),
                    t, k, p, m, np.zeros(requests, np.int64), seed, stream, positions)


def _filtered_log_weights(row: np.ndarray, settings: dict) -> np.ndarray:
    """Log weights of a row after temperature, top-k and top-p (others -inf), in float64."""
    x = row.astype(np.float64) / settings["temperature"]
    order = np.argsort(-x, kind="stable")
    keep = order[:settings["top_k"]] if settings["top_k"] else order
    w = np.exp(x[keep] - x[keep[0]])
    if settings["top_p"] < 1:
        cum = np.cumsum(w) / w.sum()
        keep = keep[:int(np.searchsorted(cum, settings["top_p"]) + 1)]
    out = np.full(row.shape, -np.inf)
    out[keep] = x[keep] - x[keep[0]]
    return out


def verification(requests: int, drafts: int, settings: dict = QWEN, *, master_seed: int = 3, vocab: int = VOCAB,
                 mode: str = "ratio", full_q: bool = False, name: str = "verify") -> Workload:
    """Speculative verification (C3): R requests of D drafts plus a bonus row.

    Draft i of a request is drawn (NumPy generator) from the draft model's
    distribution: the target row i plus N(0, 0.5^2) noise, with the same
    temperature / top-k / top-p filters. With full_q, draft_logits holds
    that distribution's log weights (-inf outside its kept set); bonus rows
    of draft_logits are ignored by the contract and hold the noisy row.
    """
    g = np.random.default_rng(master_seed)
    rows = requests * (drafts + 1)
    logits = synthetic_rows(g, rows, vocab)
    noisy = (logits.astype(np.float64) + g.normal(0.0, 0.5, size=logits.shape))
    ids = np.full((requests, max(drafts, 1)), -1, np.int64)
    q = np.empty_like(logits) if full_q else None
    for r in range(requests):
        for i in range(drafts + 1):
            row = r * (drafts + 1) + i
            if i == drafts:
                if full_q:
                    q[row] = noisy[row].astype(np.float32)
                continue
            lw = _filtered_log_weights(noisy[row], settings)
            w = np.exp(lw - lw.max())
            ids[r, i] = int(g.choice(vocab, p=w / w.sum()))
            if full_q:
                q[row] = lw.astype(np.float32)
    seed, stream, positions = _rng_fields(g, requests, [drafts + 1] * requests)
    t, k, p, m = _params(requests, settings)
    kind = np.full(requests, 1 if full_q else 0, np.int64)
    cu = (np.arange(requests + 1) * (drafts + 1)).astype(np.int64)
    return Workload(name, logits, cu, ids, t, k, p, m, kind, seed, stream, positions, mode=mode, draft_logits=q,
                    notes={"draft_sampler": "numpy Generator.choice over the noisy row's filtered softmax"})


def fallback_stress(requests: int = 256, *, master_seed: int = 4, vocab: int = VOCAB, name: str = "stress") -> Workload:
    """C4: wide kept sets, a grammar mask, bf16-rounded rows and near-threshold logits.

    Request r takes filter (min-p 0.05, top-k 4096, top-p 0.99)[r % 3] and
    temperature (0.3, 0.7, 1.0, 1.5)[(r // 3) % 4]. The mask allows a random
    50% of tokens, except 1% of rows that allow all. 10% of rows are rounded
    to bf16-representable values (stored as fp32). In 5% of rows two logits
    are moved so that (l - max) / T is within one fp32 ulp of the row's cut:
    ln(min_p) for min-p rows; for top-k rows the 4096th token is duplicated
    with its neighbour; for top-p rows the logits are set so that the weights
    are exactly 1.0 and the target falls on a prefix boundary.
    """
    g = np.random.default_rng(master_seed)
    logits = synthetic_rows(g, requests, vocab).astype(np.float64)
    filters = [dict(min_p=0.05, top_k=0, top_p=1.0), dict(min_p=0.0, top_k=4096, top_p=1.0),
               dict(min_p=0.0, top_k=0, top_p=0.99)]
    temps = [0.3, 0.7, 1.0, 1.5]
    t = np.array([temps[(r // 3) % 4] for r in range(requests)], np.float64)
    k = np.array([filters[r % 3]["top_k"] for r in range(requests)], np.int64)
    p = np.array([filters[r % 3]["top_p"] for r in range(requests)], np.float64)
    m = np.array([filters[r % 3]["min_p"] for r in range(requests)], np.float64)
    allowed = g.random((requests, vocab)) < 0.5
    dense = g.choice(requests, size=max(1, requests // 100), replace=False)
    allowed[dense] = True
    bf16_rows = g.choice(requests, size=max(1, requests // 10), replace=False)
    for r in bf16_rows:
        as32 = logits[r].astype(np.float32)
        bits = as32.view(np.uint32).astype(np.uint64)
        rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16 << 16).astype(np.uint32)
        logits[r] = rounded.view(np.float32).astype(np.float64)
    near_rows = g.choice(np.setdiff1d(np.arange(requests), bf16_rows), size=max(1, requests // 20), replace=False)
    for r in near_rows:
        row = logits[r].astype(np.float32).astype(np.float64)
        valid = np.flatnonzero(allowed[r])
        top = valid[np.argmax(row[valid])]
        mx = row[top]
        if m[r] > 0:
            # Two logits with (l - max)/T within an ulp of ln(min_p), one on each side.
            target = mx + t[r] * np.log(m[r])
            a, b = g.choice(np.setdiff1d(valid, [top]), size=2, replace=False)
            row[a] = float(np.nextafter(np.float32(target), np.float32(np.inf)))
            row[b] = float(np.nextafter(np.float32(target), np.float32(-np.inf)))
        elif k[r] > 0:
            order = valid[np.argsort(-row[valid], kind="stable")]
            row[order[k[r]]] = row[order[k[r] - 1]]  # a tie across the top-k cut
            row[order[k[r] + 1]] = row[order[k[r] - 1]]
        else:
            # 50 tokens at the maximum (weight exactly 1), the rest far below:
            # every prefix sum is an integer, and top_p * total lands on one.
            chosen = g.choice(valid, size=50, replace=False)
            row[:] = g.normal(size=vocab) - 800.0
            row[chosen] = 0.0
            p[r] = 49.0 / 50.0
        logits[r] = row
    mask = packed_mask(allowed)
    seed, stream, positions = _rng_fields(g, requests, [1] * requests)
    return Workload(name, logits.astype(np.float32), np.arange(requests + 1, dtype=np.int64),
                    np.full((requests, 1), -1, np.int64), t, k, p, m, np.zeros(requests, np.int64), seed, stream,
                    positions, mask=mask, notes={"bf16_rows": sorted(int(x) for x in bf16_rows),
                                                 "near_threshold_rows": sorted(int(x) for x in near_rows)})


def config(name: str, **kw) -> Workload:
    """The named benchmark configuration (C1 ... C5a)."""
    if name == "C1":
        return sampling(8, QWEN, master_seed=kw.pop("master_seed", 11), ties_rows=2, name="C1", **kw)
    if name == "C2a":
        return sampling(kw.pop("requests", 128), QWEN, master_seed=kw.pop("master_seed", 21), name="C2a", **kw)
    if name == "C2b":
        return sampling(kw.pop("requests", 128), TEMPERATURE_ONLY, master_seed=kw.pop("master_seed", 22), name="C2b", **kw)
    if name == "C3a":
        return verification(kw.pop("requests", 64), 4, QWEN, master_seed=kw.pop("master_seed", 31), name="C3a", **kw)
    if name == "C3b":
        return verification(kw.pop("requests", 64), 4, QWEN, master_seed=kw.pop("master_seed", 32), mode="coupled",
                            full_q=True, name="C3b", **kw)
    if name == "C3b_ratio_full":
        return verification(kw.pop("requests", 64), 4, QWEN, master_seed=kw.pop("master_seed", 33), mode="ratio",
                            full_q=True, name="C3b_ratio_full", **kw)
    if name == "C3b_coupled_onehot":
        return verification(kw.pop("requests", 64), 4, QWEN, master_seed=kw.pop("master_seed", 34), mode="coupled",
                            name="C3b_coupled_onehot", **kw)
    if name == "C4":
        return fallback_stress(kw.pop("requests", 256), master_seed=kw.pop("master_seed", 41), name="C4", **kw)
    if name == "C5a":
        return sampling(kw.pop("requests", 4096), QWEN, master_seed=kw.pop("master_seed", 51), name="C5a", **kw)
    raise ValueError(f"unknown configuration {name}")
