// The row kernel's body (one cluster per row) and its launcher.
#pragma once
#include "es_reference.cuh"
#include "es_rows.cuh"

namespace es {

constexpr uint32_t WAIT_LIMIT = 1u << 22;  // mbarrier polls (about a second) before a copy is declared lost
constexpr uint32_t PEER_WAIT_LIMIT = 1u << 20;  // polls of a peer GPU's flag (about a second) before giving up

__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

template <int DT> __host__ __device__ constexpr size_t smem_head() {
  return align_up(sizeof(Smem<typename Types<DT>::W>), 128);
}
// Dynamic shared memory: the header, the slice's mask words (resident rows),
// its tile maxima, then the slice itself (resident) or the TMA ring (streamed).
template <int DT> __host__ __device__ constexpr size_t smem_tmax(int slice_words, bool stream) {
  return smem_head<DT>() + (stream ? 0 : align_up(4 * size_t(slice_words), 128));
}
template <int DT> __host__ __device__ constexpr size_t smem_slice(int slice_words, bool stream) {
  return smem_tmax<DT>(slice_words, stream) + align_up(size_t(slice_words) * sizeof(typename Types<DT>::W), 128);
}
template <int DT> __host__ __device__ constexpr size_t smem_bytes(int slice_words, int ring_stages) {
  const bool stream = ring_stages > 0;
  return smem_slice<DT>(slice_words, stream) +
         (stream ? size_t(ring_stages) * RING_CHUNK
                 : align_up(size_t(slice_words) * 32 * sizeof(typename Types<DT>::T), 128));
}

// The last request whose segment starts at or before `row` (empty segments
// share their start with the next request, which owns the row).
__device__ inline int request_of(const Params& p, int row) {
  int lo = 0, hi = p.requests - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) / 2;
    if (at(p.cu_rows, p.cu_s, mid) <= row) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

template <int DT> struct RowKernel {
  using R = Row<DT>;
  using T = typename R::T;
  using W = typename R::W;
  using Key = typename R::Key;

  // Target point mass at the greedy token (temperature 0).
  __device__ static void greedy(R& r, const RowCtx& c, bool verify, bool full_q, double sq, RowResult& res) {
    const int g = r.argmax_id();
    res.sample = g;
    if (!verify) return;
    res.accept = c.draft_id == g;
    if (res.accept) return;
    if (!full_q) {
      res.residual = g;
      return;
    }
    // max(p - q, 0) is positive only at the greedy token, unless q rounds to 1 there.
    const W y = r.q_value(g);
    const double q = y > W(-INFINITY) ? exp(double(y) - double(r.all.qmax)) / sq : 0.0;
    res.residual = 1.0 - q > 0 ? g : -1;
  }

  // q of the draft token (1 for one-hot drafts).
  __device__ static double q_of_draft(R& r, const RowCtx& c, bool full_q, double sq) {
    if (!full_q) return 1.0;
    const W y = r.q_value(c.draft_id);
    return y > W(-INFINITY) ? exp(double(y) - double(r.all.qmax)) / sq : 0.0;
  }

  // Warp 0 of rank 0 finishes a sorted list of n_keep <= 32 kept tokens,
  // one per lane: the steps and FP64 formulas of list_finish below, with
  // warp shuffles and ballots in place of block reductions and barriers.
  // Returns false, with nothing written, where list_finish does.
  __device__ static bool finish_small(R& r, const RowCtx& c, int n_keep, bool verify, bool full_q, double sq,
                                      RowResult& res, Interval open) {
    constexpr unsigned ALL = 0xffffffffu;
    const int i = lane_id();
    const bool in = i < n_keep;
    const int id = in ? r.s.u.cand.id[i] : INT_MAX;
    // The lane's Gumbel noise for the one draw this row can need (substream
    // 2 for a ratio test's residual, else 0), computed first so that it
    // overlaps the weight and prefix chain below.
    const uint32_t draw_sub = verify && !full_q ? 2u : 0u;
    const double noise = in ? noise64(r.addr.word(draw_sub, uint32_t(id))) : 0.0;
    ES_TRACE(r.p.workspace, r.p.rows, r.row, r.rank, 11);
    double w = 0;
    bool ok = false;
    if (in) {
      w = exp(r.x64(key_value(Key(r.s.u.cand.key[i]))));
      ok = w >= r.min_p && w > 0;
    }
    // min-p and positivity remove a suffix of the order.
    const unsigned out = __ballot_sync(ALL, in && !ok);
    const int n1 = out ? min(n_keep, __ffs(out) - 1) : n_keep;
    // Inclusive prefix sums of the exact weights; lanes from n1 on add zero.
    u128 prefix = i < n1 ? fx_of(w) : u128(0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t lo = __shfl_up_sync(ALL, uint64_t(prefix), o);
      const uint64_t hi = __shfl_up_sync(ALL, uint64_t(prefix >> 64), o);
      if (i >= o) prefix += (u128(hi) << 64) | lo;
    }
    // Every lane rounds its own prefix (of i + 1 weights) at once: the total
    // is lane n1 - 1's, the top-p normalizer lane n2 - 1's.
    bool near_i = false;
    const double rounded = i < n1 ? fx_round(prefix, uint32_t(i + 1), &near_i) : 0.0;
    const double d1 = __shfl_sync(ALL, rounded, n1 - 1);
    r.count_near_tie(__shfl_sync(ALL, near_i, n1 - 1));
    int n2 = n1;
    double denominator = d1;
    if (r.top_p < 1) {
      // The length of the shortest prefix whose rounded sum reaches t (0 if
      // none in the list); the first token's weight is exactly 1.
      auto first_reach = [&](double t) {
        if (t <= 1.0) return 1;
        bool nr = false;
        const unsigned hits = __ballot_sync(ALL, i < n1 && fx_reaches(prefix, uint32_t(i + 1), t, &nr));
        return hits ? __ffs(hits) : 0;
      };
      if (open.hi > 0 && n1 == n_keep) {
        // The kept set may run past the list: the boundary must be the same
        // for every target within the bounds.
        const int a = first_reach(open.lo), b = first_reach(open.hi);
        if (b == 0 || a != b) return false;
        n2 = b;
      } else {
        const int f = first_reach(r.top_p * d1);
        n2 = f ? f : n1;
      }
      denominator = __shfl_sync(ALL, rounded, n2 - 1);
      r.count_near_tie(__shfl_sync(ALL, near_i, n2 - 1));
    }
    const double prob = i < n2 ? w / denominator : 0.0;
    ES_TRACE(r.p.workspace, r.p.rows, r.row, r.rank, 12);
    // One draw over the list: argmax log(p) + G, lowest ID on ties.
    auto draw_list = [&](uint32_t sub, int excluded) {
      Best b = no_best();
      if (i < n2 && id != excluded && prob > 0)
        b = Best{log(prob) + (sub == draw_sub ? noise : noise64(r.addr.word(sub, uint32_t(id)))), id};
      b = warp_all(b, [](Best a, Best c2) { return best_of(a, c2); });
      return b.id == INT_MAX ? -1 : b.id;
    };
    if (!verify) {
      res.sample = draw_list(0, -1);
      ES_TRACE(r.p.workspace, r.p.rows, r.row, r.rank, 15);
      return true;
    }
    const unsigned at_draft = __ballot_sync(ALL, i < n2 && id == c.draft_id);
    const double p_draft = __shfl_sync(ALL, prob, at_draft ? __ffs(at_draft) - 1 : 0);
    const double px = at_draft ? p_draft : 0.0;
    const double qx = q_of_draft(r, c, full_q, sq);
    res.accept = uniform64(r.addr.word(1, 0)) < fmin(1.0, px / qx);
    if (res.accept) return true;
    if (!full_q) {
      res.residual = draw_list(2, c.draft_id);
      return true;
    }
    Best b = no_best();
    if (i < n2 && prob > 0) {
      const W y = r.q_value(id);
      const double q = y > W(-INFINITY) ? exp(double(y) - double(r.all.qmax)) / sq : 0.0;
      const double rr = fmax(prob - q, 0.0);
      if (rr > 0) b = Best{log(rr) + noise64(r.addr.word(2, uint32_t(id))), id};
    }
    b = warp_all(b, [](Best a, Best c2) { return best_of(a, c2); });
    res.residual = b.id == INT_MAX ? -1 : b.id;
    return true;
  }

  // Rank 0 finishes a list row: the m gathered candidates hold the kept
  // n_keep tokens first once sorted. Oracle formulas throughout (FP64).
  //
  // With open.hi > 0, the list holds only the n_keep largest tokens of a kept
  // set that may run past it (top-p without top-k), and `open` bounds the oracle's
  // top-p target, top_p * fsum(kept set). The nucleus is settled when the
  // shortest prefix reaching the target is the same for every target within
  // the bounds, or when min-p ends the kept set inside the list (its sum is
  // then exact); otherwise the call returns false with nothing written.
  // Block-uniform result.
  __device__ static bool list_finish(R& r, const RowCtx& c, int m, int n_keep, bool verify, bool full_q, double sq,
                                     RowResult& res, Interval open) {
    auto& s = r.s;
    r.sort_candidates(m);
    ES_TRACE(r.p.workspace, r.p.rows, r.row, r.rank, 10);
    if (n_keep <= 32) {
      if (threadIdx.x == 0) s.ival[3] = 0;
      __syncthreads();
      if (warp_id() == 0) {
        const bool settled = finish_small(r, c, n_keep, verify, full_q, sq, res, open);
        if (lane_id() == 0) s.ival[3] = settled;
      }
      __syncthreads();
      return s.ival[3] != 0;
    }
    const int i = threadIdx.x;
    if (!r.in_bounds(n_keep <= LIST_MAX && m <= CAP, 11)) n_keep = min(n_keep, LIST_MAX);
    const bool in = i < n_keep;
    const int id = in ? s.u.cand.id[i] : INT_MAX;
    double w = 0;
    bool ok = false;
    if (in) {
      const W v = key_value(Key(s.u.cand.key[i]));
      w = exp(r.x64(v));
      ok = w >= r.min_p && w > 0;
    }
    // min-p and positivity remove a suffix of the order.
    const int first_out = block_all(in && !ok ? i : INT_MAX, [](int a, int b) { return a < b ? a : b; }, s.red.ints);
    const int n1 = min(n_keep, first_out);
    const u128 f = i < n1 ? fx_of(w) : u128(0);
    u128 total;
    const u128 prefix = block_scan(f, s.red.fxs, &total);
    bool near;
    const double d1 = fx_round(total, uint32_t(n1), &near);
    r.count_near_tie(near);
    int n2 = n1;
    double denominator = d1;
    if (r.top_p < 1) {
      // The length of the shortest prefix whose rounded sum reaches t (0 if
      // none in the list); the first token's weight is exactly 1.
      auto first_reach = [&](double t) {
        if (t <= 1.0) return 1;
        bool nr = false;
        const bool reach = i < n1 && fx_reaches(prefix, uint32_t(i + 1), t, &nr);
        const int first = block_all(reach ? i : INT_MAX, [](int a, int b) { return a < b ? a : b; }, s.red.ints);
        return first == INT_MAX ? 0 : first + 1;
      };
      if (open.hi > 0 && n1 == n_keep) {
        const int a = first_reach(open.lo), b = first_reach(open.hi);
        if (b == 0 || a != b) return false;
        n2 = b;
      } else {
        const int f = first_reach(r.top_p * d1);
        n2 = f ? f : n1;
      }
      if (i == n2 - 1) s.fxval = prefix;
      __syncthreads();
      denominator = fx_round(s.fxval, uint32_t(n2), &near);
      r.count_near_tie(near);
      __syncthreads();
    }
    ES_TRACE(r.p.workspace, r.p.rows, r.row, r.rank, 11);
    const double prob = i < n2 ? w / denominator : 0.0;
    if (i < LIST_MAX) s.lp[i] = prob;
    __syncthreads();
    // One draw over the list: argmax log(p) + G, lowest ID on ties.
    auto draw_list = [&](uint32_t sub, int excluded) {
      Best b = no_best();
      if (i < n2 && id != excluded && prob > 0) b = Best{log(prob) + noise64(r.addr.word(sub, uint32_t(id))), id};
      b = block_all(b, [](Best a, Best c2) { return best_of(a, c2); }, s.red.bests);
      return b.id == INT_MAX ? -1 : b.id;
    };
    if (!verify) {
      res.sample = draw_list(0, -1);
      ES_TRACE(r.p.workspace, r.p.rows, r.row, r.rank, 12);
      return true;
    }
    const int at_draft = block_all(i < n2 && id == c.draft_id ? i : INT_MAX, [](int a, int b) { return a < b ? a : b; },
                                   s.red.ints);
    const double px = at_draft == INT_MAX ? 0.0 : s.lp[at_draft];
    const double qx = q_of_draft(r, c, full_q, sq);
    res.accept = uniform64(r.addr.word(1, 0)) < fmin(1.0, px / qx);
    if (res.accept) return true;
    if (!full_q) {
      res.residual = draw_list(2, c.draft_id);
      return true;
    }
    Best b = no_best();
    if (i < n2 && prob > 0) {
      const W y = r.q_value(id);
      const double q = y > W(-INFINITY) ? exp(double(y) - double(r.all.qmax)) / sq : 0.0;
      const double rr = fmax(prob - q, 0.0);
      if (rr > 0) b = Best{log(rr) + noise64(r.addr.word(2, uint32_t(id))), id};
    }
    b = block_all(b, [](Best a, Best c2) { return best_of(a, c2); }, s.red.bests);
    res.residual = b.id == INT_MAX ? -1 : b.id;
    return true;
  }

  // The warp-level list path (es_fast.cuh) for a top-k of n_keep <=
  // FAST_KEEP tokens: the window from the tile-maximum bins merged with the
  // statistics, the gather by every warp over its share of the rank's tiles
  // into rank 0's candidate buffer, one exchange, and rank 0's warp finish
  // (or its block finish when more than FAST_CAND candidates arrived).
  // Returns true when the row is finished on rank 0 (no rank reads another's
  // memory afterwards); false, the same on every rank, when it does not
  // apply (no window in WIN_BINS bins, or more than CAP candidates).
  __device__ static bool fast_list(R& r, const RowCtx& c, int n_keep, bool verify, RowResult& res, const Params& p) {
    auto& s = r.s;
    if (warp_id() == 0) {
      const int j = window_warp(s.win, n_keep);
      if (lane_id() == 0) s.ival[0] = j;
    }
    __syncthreads();
    const int j = s.ival[0];
    ES_TRACE(p.workspace, p.rows, r.row, r.rank, 4);
    if (j < 0) return false;
    const int bin = r.top_bin - j;
    // Token IDs are global: a per-phase shard's columns start at p.col0
    // (such calls take this path only without a mask).
    const SliceRef<T> src =
        r.resident ? SliceRef<T>{r.slice, 1, r.has_mask ? reinterpret_cast<const int32_t*>(r.mask_s) : nullptr, 1,
                                 r.hi - r.lo, p.col0 + r.lo}
                   : SliceRef<T>{r.tbase + int64_t(r.lo) * p.t_s1, p.t_s1,
                                 r.has_mask ? p.mask + int64_t(r.row) * p.m_s0 + int64_t(r.lo >> 5) * p.m_s1 : nullptr,
                                 p.m_s1, r.hi - r.lo, p.col0 + r.lo};
    int mine;
    {
      const int nt = r.tile_count();
      if (!r.in_bounds(nt <= (r.p.slice_words * 32 + 31) / 32, 9)) return false;
      const int per = (nt + WARPS - 1) / WARPS;
      const int t0 = min(nt, warp_id() * per), t1 = min(nt, t0 + per);
      mine = gather_warp<T, W>(src, r.tmax, t0, t1, bin, r.peer(s.u.cand.key, 0), r.peer(s.u.cand.id, 0),
                               r.peer(&s.n_cand, 0), CAP);
    }
    mine = block_all(lane_id() == 0 ? mine : 0, [](int x, int y) { return x + y; }, s.red.ints);
    if (int(threadIdx.x) < r.ranks) r.peer(s.pushed, threadIdx.x)[r.rank] = mine;
    ES_TRACE(p.workspace, p.rows, r.row, r.rank, 14);
    r.exchange();
    ES_TRACE(p.workspace, p.rows, r.row, r.rank, 5);
    int m = 0;
    for (int rr = 0; rr < r.ranks; ++rr) m += s.pushed[rr];
    if (r.phases) {
      if (r.rank != 0) return true;  // rank 0 finishes the row
      m = phase_candidates(r, m, n_keep);
      if (m == -2) return true;  // a peer never published: the row is marked invalid
      if (m < 0) return false;   // too many candidates: rank 0 finishes the row in FP64
    } else {
      if (m > CAP) return false;  // the block path's radix selection decides
      if (r.rank != 0) return true;
    }
    if (!r.in_bounds(n_keep <= LIST_MAX && m >= 0 && m <= CAP, 10)) return false;
    if (m <= FAST_CAND && n_keep <= FAST_KEEP) {
      if (warp_id() == 0) {
        const ListIn in{s.u.cand.key, s.u.cand.id, m, n_keep, double(r.maxv), r.temperature, r.min_p, r.top_p,
                        r.addr, verify ? 1 : 0, c.draft_id, &diagnostics(p.workspace, p.rows)->near_ties};
        const ListOut o = finish_warp<W>(in);
        res.sample = o.sample;
        res.accept = o.accept;
        res.residual = o.residual;
      }
      ES_TRACE(p.workspace, p.rows, r.row, r.rank, 12);
    } else {
      list_finish(r, c, m, n_keep, verify, false, 0.0, res, Interval{0, 0});
    }
    return true;
  }

  // Per-phase sharded calls, rank 0 after its cluster's gather of m window
  // candidates: sends this GPU's best into its slot on every GPU, then
  // assembles every GPU's from its own buffer, in GPU order, in the
  // candidate buffer. The kept set is the first n_keep of the row's order,
  // and each of those is among the first n_keep of its own GPU's candidates,
  // so a GPU sends all m when m <= n_keep, else its first n_keep after a
  // warp sort (m <= FAST_CAND); more candidates are an overflow. Returns the
  // number assembled; -1 when a GPU overflowed (the row is then finished in
  // FP64, the same decision on every GPU); -2 when a GPU's words never arrived.
  __device__ static int phase_candidates(R& r, int m, int n_keep) {
    static_assert(FAST_CAND <= PHASE_SEND, "a sorted candidate list fits a slot");
    auto& s = r.s;
    const Params& p = r.p;
    const int n = p.sh.count;
    const uint32_t tag = r.phase_tag();
    const int send = m > FAST_CAND ? -1 : min(m, n_keep);
    if (warp_id() == 0) {
      uint64_t key[2];
      int32_t id[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int e = lane_id() + 32 * h;
        key[h] = send >= 0 && e < m ? s.u.cand.key[e] : 0;
        id[h] = send >= 0 && e < m ? s.u.cand.id[e] : INT_MAX;
      }
      if (send >= 0 && send < m) warp_sort<64, sizeof(W) == 8>(key, id);
      for (int to = 0; to < n; ++to) {
        uint64_t* slot = r.phase_slot(to, p.sh.rank) + PHASE_COUNT_WORD;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int e = lane_id() + 32 * h;
          if (e < send) {
            st_tagged_sys(slot + 1 + 3 * e, uint32_t(key[h]), tag);
            st_tagged_sys(slot + 2 + 3 * e, uint32_t(key[h] >> 32), tag);
            st_tagged_sys(slot + 3 + 3 * e, uint32_t(id[h]), tag);
          }
        }
        if (lane_id() == 0) st_tagged_sys(slot, send < 0 ? PHASE_OVERFLOW : uint32_t(send), tag);
      }
    }
    __syncthreads();  // warp 0 is done with the candidate buffer
    ES_TRACE(p.workspace, p.rows, r.row, r.rank, 19);
    bool ok = true;
    if (int(threadIdx.x) < n) {
      uint32_t c = 0;
      ok = r.phase_read(threadIdx.x, PHASE_COUNT_WORD, c);
      s.peer_n[threadIdx.x] = c;
    }
    if (__syncthreads_or(!ok)) return -2;
    ES_TRACE(p.workspace, p.rows, r.row, r.rank, 20);
    for (int g = 0; g < n; ++g)  // the same on every thread
      if (s.peer_n[g] == PHASE_OVERFLOW || !r.in_bounds(s.peer_n[g] <= uint32_t(PHASE_SEND), 12)) return -1;
    int off = 0;
    for (int g = 0; g < n; ++g) {
      const int c = int(s.peer_n[g]);
      for (int i = threadIdx.x; i < 3 * c && ok; i += THREADS) {
        const int e = i / 3, w = i - 3 * e;
        uint32_t d = 0;
        ok = r.phase_read(g, PHASE_COUNT_WORD + 1 + i, d);
        if (w == 2) s.u.cand.id[off + e] = int32_t(d);
        else reinterpret_cast<uint32_t*>(&s.u.cand.key[off + e])[w] = d;
      }
      off += c;
    }
    if (__syncthreads_or(!ok)) return -2;
    ES_TRACE(p.workspace, p.rows, r.row, r.rank, 21);
    return off;  // <= MAX_SHARDS * PHASE_SEND <= CAP
  }

  // Per-phase sharded calls: the whole row in FP64 (es_reference.cuh) by
  // rank 0 alone, reading every GPU's shard, for rows the exchange cannot
  // finish. The same on every GPU.
  __device__ static RowResult phase_fp64(R& r, const RowCtx& c) {
    const Params& p = r.p;
    static_assert(sizeof(RefShared) <= sizeof(decltype(r.s.u)), "the FP64 path's shared state fits the candidate buffer");
    RefShared& rs = *reinterpret_cast<RefShared*>(&r.s.u);
    double* w = reinterpret_cast<double*>(p.sh.scratch) + int64_t(r.row) * p.vocab * 2;
    uint64_t* keys = reinterpret_cast<uint64_t*>(w + p.vocab);
    const int row = r.row;
    // It reads every GPU's shard: each GPU's ready flag (a system-scope
    // release once its shard is written) first, bounded.
    if (threadIdx.x == 0) {
      int ok = 1;
      for (int g = 0; g < p.sh.count && ok; ++g)
        for (uint32_t spins = 0; ld_acquire_sys(p.sh.ready[g]) < p.sh.epoch;)
          if (++spins >= (1u << 20)) {
            ok = 0;
            break;
          }
      r.s.ival[2] = ok;
      if (!ok) {
        atomicAdd(&diagnostics(p.workspace, p.rows)->wait_timeouts, 1u);
        r.s.timeout = 1;
      }
    }
    __syncthreads();
    if (r.s.ival[2] == 0) return RowResult{ES_INVALID_INPUT, ES_INVALID_INPUT, 0, -1, -1, {0, 0, 0}};
    fence_acq_rel_sys();
    return reference_row<THREADS>(
        p, row, c,
        [&](int t) {
          const int g = t / p.sh.cols;
          return double(widen(static_cast<const T*>(p.sh.target[g])[int64_t(row) * p.t_s0 + int64_t(t - g * p.sh.cols) * p.t_s1]));
        },
        [&](int t) {
          return p.mask == nullptr ||
                 ((uint32_t(p.mask[int64_t(row) * p.m_s0 + int64_t(t >> 5) * p.m_s1]) >> (t & 31)) & 1u);
        },
        [&](int t) {
          const int g = t / p.sh.cols;
          return double(widen(static_cast<const T*>(p.sh.draft[g])[int64_t(row) * p.q_s0 + int64_t(t - g * p.sh.cols) * p.q_s1]));
        },
        w, keys, rs);
  }

  // Returns true when rank 0 finishes the row alone (a list row): the other
  // ranks may then exit, since no rank touches another's memory afterwards.
  __device__ __forceinline__ static bool positive(R& r, const RowCtx& c, bool verify, bool full_q, double sq, RowResult& res,
                                  const Params& p) {
    const int valid = r.all.valid;
    const int64_t k = c.top_k;
    const int n_keep = (k > 0 && k < valid) ? int(k) : valid;
    const int list_max = p.exact_draws ? 0 : min(p.list_max, LIST_MAX);
    // A list row: the kept set is at most list_max tokens. Otherwise top-p
    // without top-k: on real logits the nucleus is a handful of the largest
    // tokens, so lists of the largest 32, then list_max, tokens are tried
    // against bounds on the kept set's total, and the exact full-row
    // selection below decides when neither list settles the boundary.
    const bool list_row = n_keep <= list_max;
    const bool top_p_list = !list_row && n_keep == valid && r.top_p < 1 && list_max > 0;
    if (list_row && n_keep < valid && n_keep <= FAST_KEEP && p.fast && !full_q && r.top_bin >= 0 &&
        fast_list(r, c, n_keep, verify, res, p))
      return true;
    Interval target{0, 0};
    if (top_p_list) {
      const Interval total = r.approx_mass([](Key, int) { return true; }, false);
      target = Interval{r.top_p * total.lo, r.top_p * total.hi};  // rounding is monotone
    }
    int tried = 0;
    for (int attempt = 0; attempt < (list_row ? 1 : top_p_list ? 2 : 0); ++attempt) {
      int m, len = n_keep;
      Interval open{0, 0};
      if (list_row) {
        if (n_keep < valid) {
          m = r.gather_near(n_keep);
          ES_TRACE(p.workspace, p.rows, r.row, r.rank, 5);
          if (m < 0) {
            const Cut<Key> cut = r.select_nth(n_keep, [](Key, int, W) { return true; });
            m = r.gather_all([&](W v, int t) { return cut.keeps(order_key(v), t); });
          }
        } else {
          m = r.gather_all([](W, int) { return true; });
        }
      } else {
        const int want = min(attempt == 0 ? 32 : list_max, valid);
        if (want <= tried) break;
        m = r.gather_near(want);
        if (m < 0) break;  // the same on every rank
        len = min(m, list_max);
        if (len < valid) open = target;
      }
      bool settled = false;
      if (r.rank == 0) settled = list_finish(r, c, m, len, verify, full_q, sq, res, open);
      if (list_row) return true;
      if (r.broadcast_verdict(settled)) return true;
      tried = len;
    }
    Cut<Key> cut_k{0, 0, 0}, cut_p{0, 0, 0};
    if (k > 0 && k < valid) cut_k = r.select_nth(int(k), [](Key, int, W) { return true; });
    ES_TRACE(p.workspace, p.rows, r.row, r.rank, 4);
    double sp = 0;
    bool sp_known = false;
    if (r.top_p < 1) {
      cut_p = r.top_p_cut(cut_k, &sp);
      sp_known = true;
    }
    ES_TRACE(p.workspace, p.rows, r.row, r.rank, 5);
    auto kept = [cut_k, cut_p](Key key, int t) { return cut_k.keeps(key, t) && cut_p.keeps(key, t); };
    const bool cuts = cut_k.on || cut_p.on;
    if (!verify) {
      res.sample = r.draw(0, -1, kept, cuts, p.exact_draws != 0);
      ES_TRACE(p.workspace, p.rows, r.row, r.rank, 12);
      return false;
    }
    const int x = c.draft_id;
    double wx = 0;  // the draft token's weight, if kept
    if (r.valid_global(x)) {
      const W v = r.value_global(x);
      if (kept(order_key(v), x)) {
        const double w = exp(r.x64(v));
        if (w >= r.min_p && w > 0) wx = w;
      }
    }
    const double qx = q_of_draft(r, c, full_q, sq);
    const double u = uniform64(r.addr.word(1, 0));
    // The oracle's test u < min(1, (wx / sp) / qx) falls as sp grows (every
    // step rounds monotonically), so bounds on sp usually settle it without
    // the exact sum, which one-hot residual draws do not need either.
    int accept = wx == 0 ? 0 : -1;
    if (accept < 0 && !sp_known && !p.exact_draws) {
      const Interval m = r.approx_mass(kept, cuts);
      if (u < fmin(1.0, (wx / m.hi) / qx)) accept = 1;
      else if (m.lo > 0 && !(u < fmin(1.0, (wx / m.lo) / qx))) accept = 0;
    }
    if (!sp_known && (accept < 0 || (accept == 0 && full_q))) sp = r.exact_mass(kept);
    if (accept < 0) accept = u < fmin(1.0, (wx / sp) / qx);
    res.accept = accept != 0;
    if (res.accept) return false;
    res.residual = full_q ? r.draw_residual_q(kept, sp, sq) : r.draw(2, x, kept, cuts, p.exact_draws != 0);
    return false;
  }

  // positive() for kernels compiled without the list paths (calls with
  // list_max = 0): the cuts, the ratio test and the draws over the full row,
  // with the group-screened draw.
  __device__ __forceinline__ static bool positive_rows(R& r, const RowCtx& c, bool verify, bool full_q, double sq,
                                                       RowResult& res, const Params& p) {
    const int valid = r.all.valid;
    const int64_t k = c.top_k;
    const int n_keep = (k > 0 && k < valid) ? int(k) : valid;
    Cut<Key> cut_k{0, 0, 0}, cut_p{0, 0, 0};
    if (k > 0 && k < valid) cut_k = r.select_nth(int(k), [](Key, int, W) { return true; });
    ES_TRACE(p.workspace, p.rows, r.row, r.rank, 4);
    double sp = 0;
    bool sp_known = false;
    if (r.top_p < 1) {
      cut_p = r.top_p_cut(cut_k, &sp);
      sp_known = true;
    }
    ES_TRACE(p.workspace, p.rows, r.row, r.rank, 5);
    auto kept = [cut_k, cut_p](Key key, int t) { return cut_k.keeps(key, t) && cut_p.keeps(key, t); };
    const bool cuts = cut_k.on || cut_p.on;
    if (!verify) {
      res.sample = r.draw_groups(0, -1, kept, cuts, p.exact_draws != 0);
      ES_TRACE(p.workspace, p.rows, r.row, r.rank, 12);
      return false;
    }
    const int x = c.draft_id;
    double wx = 0;  // the draft token's weight, if kept
    if (r.valid_global(x)) {
      const W v = r.value_global(x);
      if (kept(order_key(v), x)) {
        const double w = exp(r.x64(v));
        if (w >= r.min_p && w > 0) wx = w;
      }
    }
    const double qx = q_of_draft(r, c, full_q, sq);
    const double u = uniform64(r.addr.word(1, 0));
    // The oracle's test u < min(1, (wx / sp) / qx) falls as sp grows (every
    // step rounds monotonically), so bounds on sp usually settle it without
    // the exact sum, which one-hot residual draws do not need either.
    int accept = wx == 0 ? 0 : -1;
    if (accept < 0 && !sp_known && !p.exact_draws) {
      const Interval m = r.approx_mass(kept, cuts);
      if (u < fmin(1.0, (wx / m.hi) / qx)) accept = 1;
      else if (m.lo > 0 && !(u < fmin(1.0, (wx / m.lo) / qx))) accept = 0;
    }
    if (!sp_known && (accept < 0 || (accept == 0 && full_q))) sp = r.exact_mass(kept);
    if (accept < 0) accept = u < fmin(1.0, (wx / sp) / qx);
    res.accept = accept != 0;
    if (res.accept) return false;
    res.residual = full_q ? r.draw_residual_q(kept, sp, sq) : r.draw_groups(2, x, kept, cuts, p.exact_draws != 0);
    return false;
  }
};

// The warm-up warp (es_fast.cuh): the warp-level list steps once on dummy
// data in the block's FP64 list arrays, which no list uses before the first
// cluster exchange, and that exchange cannot complete before this warp has
// exited. Writes nothing else.
template <int DT> __device__ void warm_up(Smem<typename Types<DT>::W>& s) {
  using T = typename Types<DT>::T;
  using W = typename Types<DT>::W;
  struct Dry {
    T row[64];
    W tmax[2];
    uint32_t counts[WIN_BINS];
    uint64_t key[FAST_CAND];
    int32_t id[FAST_CAND];
    int counter, sink;
  };
  static_assert(sizeof(Dry) <= sizeof(s.lw) + sizeof(s.lp), "the dry run fits the list arrays");
  Dry& d = *reinterpret_cast<Dry*>(s.lw);
  const int lane = lane_id();
  // Two tiles of a falling row, 16 down to 8.125 in steps of 1/8.
  for (int h = 0; h < 2; ++h) {
    d.row[lane + 32 * h] = T(16.f - 0.125f * float(lane + 32 * h));
  }
  if (lane < 2) d.tmax[lane] = W(16.f - 4.f * float(lane));
  for (int b = lane; b < WIN_BINS; b += 32) d.counts[b] = b < 16 ? 1u : 0u;
  if (lane == 0) d.counter = 0;
  __syncwarp();
  const int j = window_warp(d.counts, 2);
  const SliceRef<T> src{d.row, 1, nullptr, 0, 64, 0};
  const int bin = abs_bin(W(16)) - max(j, 0) - 8;
  const int m = gather_warp<T, W>(src, d.tmax, 0, 2, bin, d.key, d.id, &d.counter, FAST_CAND);
  __syncwarp();
  ListIn in{d.key, d.id, min(m, FAST_CAND), 20, 16.0, 0.6, 0.01, 0.95, Address{1u, 2u, 3u, 4u}, 0, -1, nullptr};
  const int sink = finish_warp<W>(in).sample;
  in.verify = 1;
  in.draft_id = d.id[3];
  const ListOut o = finish_warp<W>(in);
  if (lane == 0) d.sink = sink + o.accept + o.residual;
}

// MIN_BLOCKS: resident CTAs per SM the register allocation must allow (3 for
// large streamed batches, else 2). Blocks have THREADS row threads, plus a
// warm-up warp with WARM (p.warm). LISTS: the list paths are compiled in
// (calls with list_max > 0); without them the kernel is smaller and its
// full-row draws screen whole groups first.
template <int DT, int MIN_BLOCKS, bool WARM, bool LISTS>
__global__ void __launch_bounds__(THREADS + (WARM ? 32 : 0), MIN_BLOCKS) rows_kernel(const __grid_constant__ Params p) {
  static_assert(LISTS || !WARM, "the warm-up warp runs the list path");
  using K = RowKernel<DT>;
  using R = typename K::R;
  using T = typename K::T;
  using W = typename K::W;
  extern __shared__ __align__(128) uint8_t raw[];
  Smem<W>& s = *reinterpret_cast<Smem<W>*>(raw);
  const bool stream = p.stream_rows != 0;
  uint32_t* mask_s = reinterpret_cast<uint32_t*>(raw + smem_head<DT>());
  W* tmax = reinterpret_cast<W*>(raw + smem_tmax<DT>(p.slice_words, stream));
  T* slice = reinterpret_cast<T*>(raw + smem_slice<DT>(p.slice_words, stream));
  R r(p, s, mask_s, tmax, slice);
  ES_TRACE(p.workspace, p.rows, r.row, r.rank, 0);
  // A per-phase sharded call's end-of-call flag kernel follows on the
  // stream as a programmatic dependent: it may be scheduled now, and waits
  // on the device for this grid's completion.
  if (r.phases) allow_dependent_grid();

  // 1. Start copying this rank's slice (and mask words) before waiting for
  //    the preparation kernel: they are inputs, which it never writes.
  //    Resident rows copy the whole slice; streamed rows fill the TMA ring.
  bool lost = false;  // a bounded wait gave up: the row is not trusted
  for (int i = threadIdx.x; i < ABS_BINS && int(threadIdx.x) < THREADS; i += THREADS) r.hist_abs[i] = 0;
  if (threadIdx.x == 0) {
    s.n_cand = 0;  // rank 0's candidate counter, before any peer can push (the first cluster exchange)
    mbar_init(&s.bar, 1);
    for (int i = 0; i < MAX_RING_STAGES; ++i) mbar_init(&s.ring_bar[i], 1);
    mbar_init_fence();
    s.timeout = 0;
    if (r.sharded) {
      // A vocabulary-sharded call: only rows of this GPU's requests, and
      // only once every GPU has written its shard (offsets are an input:
      // malformed ones are caught by the preparation kernel).
      const int req = request_of(p, r.row);
      s.ctx.skip = req < p.sh.req_begin || req >= p.sh.req_end;
      if (!s.ctx.skip)
        for (int g = 0; g < p.sh.count; ++g)
          for (uint32_t spins = 0; ld_acquire_sys(p.sh.ready[g]) < p.sh.epoch;)
            if (++spins >= PEER_WAIT_LIMIT) {
              s.timeout = 1;
              break;
            }
    }
  }
  __syncthreads();
  if (WARM && warp_id() >= WARPS) {  // the warm-up warp
    warm_up<DT>(s);
    return;
  }
  if (r.sharded) {
    if (s.ctx.skip) return;  // the same on every rank of the cluster
    lost = s.timeout != 0;
  }
  const int n = r.hi - r.lo;
  if (stream) {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(&s.bar, 0);
      if (p.vector_load)
        for (int c = 0; c < min(p.stream_rows, r.ring_chunks()); ++c) r.ring_issue(c, c);
    }
  } else if (p.vector_load) {
    const uint32_t bytes = uint32_t(n) * uint32_t(sizeof(T)), bulk = bytes & ~15u;
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(&s.bar, bulk);
      r.bulk_columns(slice, r.lo, int(bulk / sizeof(T)), &s.bar);
    }
    for (int i = int(bulk / sizeof(T)) + threadIdx.x; i < n; i += THREADS) slice[i] = *r.target_at(r.lo + i);
  } else {
    if (threadIdx.x == 0) mbar_arrive_expect_tx(&s.bar, 0);
    for (int i = threadIdx.x; i < n; i += THREADS) slice[i] = *r.target_at(r.lo + i);
  }
  if (!stream && p.mask != nullptr)
    for (int w = threadIdx.x; w < (n + 31) / 32; w += THREADS)
      mask_s[w] = uint32_t(p.mask[int64_t(r.row) * p.m_s0 + int64_t(r.lo / 32 + w) * p.m_s1]);

  // 2. The copy (resident rows). The preparation kernel's outputs are not
  //    needed before the statistics, so it runs alongside them.
  for (uint32_t spins = 0; !mbar_try_wait(&s.bar, 0);)
    if (++spins >= WAIT_LIMIT) {
      lost = true;
      break;
    }
  lost = sync_rows_or(lost);
  ES_TRACE(p.workspace, p.rows, r.row, r.rank, 2);
  if (lost && threadIdx.x == 0) atomicAdd(&diagnostics(p.workspace, p.rows)->wait_timeouts, 1u);

  // 3. Validation and the row maximum.
  r.stats_pass(lost);
  ES_TRACE(p.workspace, p.rows, r.row, r.rank, 3);

  // 4. The preparation kernel's statuses and counters; the row's request and
  //    parameters (the same on every rank), gathered by it and loaded by
  //    the statistics pass before its exchange.
  ES_TRACE(p.workspace, p.rows, r.row, r.rank, 1);
  if (s.ctx.skip) {  // the same decision on every rank; every copy has landed
    r.cluster.sync();  // no rank leaves while a peer may still read its statistics slot
    return;
  }
  const RowCtx c = s.ctx;
  const bool draft_row = r.row + 1 < c.end, full_q = draft_row && c.kind == 1;
  const bool verify = draft_row && p.mode == ES_RATIO;
  r.temperature = c.temperature;
  r.top_p = c.top_p;
  r.min_p = c.min_p;
  r.addr = Address{c.stream, c.position, uint32_t(c.seed), uint32_t(c.seed >> 32)};
  if (r.phases) {
    // A per-phase sharded call: the row's statistics over every GPU, then
    // the list path with the candidates exchanged, or FP64 over the whole row.
    RowResult res{ES_OK, ES_OK, 0, -1, -1, {0, 0, 0}};
    bool done = !r.phase_stats();  // a peer that never published leaves the row invalid
    if (!done) {
      const int valid = r.all.valid;
      const int n_keep = (c.top_k > 0 && c.top_k < valid) ? int(c.top_k) : valid;
      const bool listed = !r.all.bad && valid > 0 && c.temperature > 0 && !full_q && !p.exact_draws &&
                          !r.has_mask && p.fast && n_keep < valid && n_keep <= min(p.list_max, LIST_MAX) &&
                          r.top_bin >= 0;
      if (listed) {
        const double inv = 1.0 / c.temperature;
        r.slow_x = !(inv < 1e30 && inv > 1e-30);
        r.inv_t = r.slow_x ? 0.f : float(inv);
        r.ln_mp = c.min_p > 0 ? float(log(c.min_p)) : -INFINITY;
        r.mp_tol = c.min_p > 0 ? 1e-6f * (1.f + fabsf(r.ln_mp)) : 0.f;
        done = K::fast_list(r, c, n_keep, verify, res, p);
      }
    }
    if (r.rank != 0) return;  // rank 0 alone from here; no rank reads another's shared memory any more
    if (!done) res = K::phase_fp64(r, c);
    ES_TRACE(p.workspace, p.rows, r.row, r.rank, 22);
    if (threadIdx.x == 0) {
      if (s.timeout != 0) {
        res.target_status = ES_INVALID_INPUT;
        res.status = ES_INVALID_INPUT;
      }
      row_results(p.workspace)[r.row] = res;
      __threadfence();
      const uint32_t arrived = atomicAdd(&arrivals(p.workspace, p.rows)[c.begin], 1u) + 1;
      if (arrived == uint32_t(c.end - c.begin)) {
        __threadfence();
        finish_request(p, c.req, c.begin, c.end);
      }
    }
    return;
  }
  if (full_q) r.q_stats_pass();  // the same on every rank
  RowResult res{ES_OK, ES_OK, 0, -1, -1, {0, 0, 0}};
  res.target_status = r.all.bad ? ES_INVALID_INPUT : r.all.valid == 0 ? ES_NO_VALID_TOKEN : ES_OK;
  res.status = res.target_status;
  double sq = 0;
  if (res.status == ES_OK && full_q) {
    if (r.all.qbad) res.status = ES_INVALID_INPUT;
    else if (r.all.qvalid == 0) res.status = ES_NO_VALID_TOKEN;
    else {
      sq = r.q_mass();
      const W y = r.q_value(c.draft_id);
      const double wq = y > W(-INFINITY) ? exp(double(y) - double(r.all.qmax)) : 0.0;
      if (!(wq / sq > 0)) res.status = ES_DRAFT_ZERO_PROB;
    }
  }

  // 5. The kept set, the ratio test and the draws.
  bool solo = false;
  if (res.status == ES_OK) {
    if (c.temperature == 0) {
      K::greedy(r, c, verify, full_q, sq, res);
    } else {
      const double inv = 1.0 / c.temperature;
      r.slow_x = !(inv < 1e30 && inv > 1e-30);
      r.inv_t = r.slow_x ? 0.f : float(inv);
      r.ln_mp = c.min_p > 0 ? float(log(c.min_p)) : -INFINITY;
      r.mp_tol = c.min_p > 0 ? 1e-6f * (1.f + fabsf(r.ln_mp)) : 0.f;
      if constexpr (LISTS) solo = K::positive(r, c, verify, full_q, sq, res, p);
      else solo = K::positive_rows(r, c, verify, full_q, sq, res, p);
    }
  }

  // 6. Publish; the request's last row to finish commits it.
  ES_TRACE(p.workspace, p.rows, r.row, r.rank, 6);
  if (!solo) r.cluster.sync();  // no rank reads another's shared memory after this point
  ES_TRACE(p.workspace, p.rows, r.row, r.rank, 7);
  if (r.rank == 0 && threadIdx.x == 0) {
    if (s.timeout != 0) {  // a copy of a later pass never arrived on some rank: the row is not trusted
      res.target_status = ES_INVALID_INPUT;
      res.status = ES_INVALID_INPUT;
    }
    row_results(p.workspace)[r.row] = res;
    __threadfence();
    const uint32_t done = atomicAdd(&arrivals(p.workspace, p.rows)[c.begin], 1u) + 1;
    if (done == uint32_t(c.end - c.begin)) {
      __threadfence();
      finish_request(p, c.req, c.begin, c.end);
    }
  }
}

// Launch of the row kernel: a (C, rows) grid of C-block clusters, with
// programmatic stream serialization after the preparation kernel.
// One kernel family's launch: LISTS picks the kernels compiled with the
// list paths (calls with list_max > 0) or without them.
template <int DT, bool LISTS> cudaError_t launch_family(const Params& p, int cluster, cudaStream_t stream) {
  const size_t smem = smem_bytes<DT>(p.slice_words, p.stream_rows);
  void (*kernel)(Params);
  if constexpr (LISTS)
    kernel = p.min_blocks == 3 ? (p.warm ? rows_kernel<DT, 3, true, true> : rows_kernel<DT, 3, false, true>)
                               : (p.warm ? rows_kernel<DT, 2, true, true> : rows_kernel<DT, 2, false, true>);
  else
    kernel = p.min_blocks == 3 ? rows_kernel<DT, 3, false, false> : rows_kernel<DT, 2, false, false>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  if (cluster > 8) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(unsigned(cluster), unsigned(p.rows), 1);
  config.blockDim = dim3(p.warm ? THREADS + 32 : THREADS, 1, 1);
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = unsigned(cluster);
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attrs;
  config.numAttrs = 2;
  return cudaLaunchKernelEx(&config, kernel, p);
}

// Calls without lists launch kernels compiled in translation units of their
// own (es_rows_full_*.cu): the compiler's inlining and register allocation
// depend on everything a translation unit holds, and apart the list kernels
// compile as they do alone.
template <int DT> cudaError_t launch_rows_full(const Params& p, int cluster, cudaStream_t stream);
template <> cudaError_t launch_rows_full<ES_F32>(const Params&, int, cudaStream_t);
template <> cudaError_t launch_rows_full<ES_F64>(const Params&, int, cudaStream_t);
template <> cudaError_t launch_rows_full<ES_F16>(const Params&, int, cudaStream_t);
template <> cudaError_t launch_rows_full<ES_BF16>(const Params&, int, cudaStream_t);

template <int DT> cudaError_t launch_rows(const Params& p, int cluster, cudaStream_t stream) {
  if (p.list_max == 0) return launch_rows_full<DT>(p, cluster, stream);
  return launch_family<DT, true>(p, cluster, stream);
}

// Launch of the independent FP64 kernel (dispatch="reference"): one block per row.
template <int DT> cudaError_t launch_reference(const Params& p, cudaStream_t stream) {
  reference_rows<DT><<<unsigned(p.rows), REF_THREADS, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace es
