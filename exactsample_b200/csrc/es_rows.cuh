// The row kernel: one thread-block cluster per target row.
//
// Each of the cluster's C blocks ("ranks") owns a contiguous slice of the
// row (a multiple of 32 tokens, so slices align with mask words and with the
// Philox groups of four). Small batches copy the slice once from HBM into
// shared memory with TMA bulk copies, and every pass reads it there; larger
// batches stream it through a ring of TMA stages, once for the statistics
// and again for each later whole-row pass (mostly from L2). The ranks
// combine partial results through distributed shared memory after a cluster
// barrier. Each rank merges the C partial results itself, in rank order, so
// every rank holds bitwise the same row-level values and takes the same
// branches; no result depends on C, on the batch, or on timing.
//
// What a row computes follows the oracle (python/exactsample/reference.py,
// distribution() and verify_reference()):
//   validation and maximum          reference row_stats (csrc/verify/fused.cuh:409-519)
//   top-k candidates near the max   row_hist / row_gather (fused.cuh:686-798)
//   exact top-k cut                 buffer_select / select_next (fused.cuh:962-1184)
//   FP64 list finish                fused_rows<LIST> (fused.cuh:1250-1444)
//   full-row kept set and draws     fused_rows<FULL> (fused.cuh:1446-1785)
//   ratio / coupled verification    fused.cuh:1396-1443, 1606-1621; verify.cu:169-217
// Every decision is exact:
//   * the kept set (mask, min-p, top-k, top-p): top-k by integer radix
//     selection on order-preserving keys with token-ID tie breaking; min-p per
//     token (FP32 with a margin, FP64 near the threshold); top-p by a radix
//     selection weighted by FP64 weights summed exactly in 128-bit fixed
//     point, i.e. the oracle's correctly rounded math.fsum;
//   * normalizers and the ratio test: FP64 on exact sums, as in the oracle,
//     or bounds on a sum where every value within them gives the same
//     decision (a top-p boundary, a ratio test): FP32 sums with an error
//     bound, the exact sum only when the bounds leave the decision open;
//   * draws over lists (at most 256 tokens): the oracle's FP64 log(p) + G;
//     over larger kept sets: a certified FP32 argmax of x + G with an FP64
//     rescore of every token that could still win.
#pragma once
#include "es_fast.cuh"
#include "es_prepare.cuh"

namespace es {

template <int DT> struct Types;
template <> struct Types<ES_F32> { using T = float; using W = float; using Key = uint32_t; };
template <> struct Types<ES_F64> { using T = double; using W = double; using Key = uint64_t; };
template <> struct Types<ES_F16> { using T = __half; using W = float; using Key = uint32_t; };
template <> struct Types<ES_BF16> { using T = __nv_bfloat16; using W = float; using Key = uint32_t; };


// An exact cut of the order (value desc, token ID asc): keeps the tokens at or
// before (key, id). `on == 0` keeps everything.
template <class Key> struct Cut {
  int on;
  Key key;
  int id;
  __device__ __forceinline__ bool keeps(Key k, int t) const { return !on || k > key || (k == key && t <= id); }
};

// |x32 - x| <= X_ERR |x| for x = (v - max) / T (three FP32 roundings, or one
// FP64 -> FP32 conversion).
constexpr float X_ERR = 2.0e-7f;
// |s32 - (x + G)| <= SCORE_ERR (1 + |x32| + |G32|) for s32 = x32 + noise32:
// X_ERR |x| + NOISE_ERR (1 + |G|) + one rounding of the sum, with margin.
constexpr float SCORE_ERR = 1.5e-6f;
// Tokens are pruned only this far below the best lower bound so far, so a
// pruned bound rarely blocks the certificate of a different winner.
constexpr float PRUNE_MARGIN = 1e-3f;
// NOISE_MAX + SCORE_ERR (1 + NOISE_MAX): the noise part of the largest score
// bound a token with x <= 0 can have.
constexpr float LIVE_OFFSET = NOISE_MAX + SCORE_ERR * (1.f + NOISE_MAX);
// A float at least ln 2.
constexpr float LN2_UP = 0.69314725f;
// Distance windows (logits below the maximum) tried for list candidates.
constexpr int WINDOWS = 8;
__device__ __forceinline__ float window_width(int i) { return 0.25f * float(1 << i); }  // 0.25 .. 32

// exp((v - max) / T) >= min_p and > 0 in FP64, for the rare token whose
// FP32 value is too close to a threshold (out of line: keeps the loops lean).
static __device__ __noinline__ bool weight_kept_fp64(double v, double maxv, double temperature, double min_p) {
  const double w = exp((v - maxv) / temperature);
  return w >= min_p && w > 0;
}

template <class W> struct Stats {
  W vmax, qmax;  // largest valid target value; largest proposal value (full q)
  int32_t valid, bad, qvalid, qbad;
  int32_t top_bin;  // abs_bin(vmax), -1 without a valid value
};

// A rank's share of an approximate kept-set mass (approx_mass): FP32 weights
// summed in FP64, split by whether min-p certainly keeps the token.
struct MassPart {
  double kept;   // weights of tokens min-p certainly keeps
  double unsure; // weights of tokens too close to the min-p threshold to tell
  double err;    // bound on the error of the two sums
  uint32_t n;    // tokens in either
};
// Bounds on a sum: lo <= exact <= hi.
struct Interval {
  double lo, hi;
};
// |__expf(x32) - exp(x)| <= MASS_ERR (1 + |x|) __expf(x32): X_ERR |x| from
// x32, and __expf's documented bound of (2 + 1.173 |x|) ulp (CUDA C++
// Programming Guide, intrinsic functions), with a factor of about three to
// spare.
constexpr double MASS_ERR = 1.0e-6;
// Candidate tiles (32 tokens) a rank scans for list candidates before it
// falls back to a full pass.
constexpr int TILE_CAP = 256;

template <class W> struct Smem {
  uint64_t bar;
  uint64_t ring_bar[MAX_RING_STAGES];
  int32_t timeout;
  RowCtx ctx;
  // Published to the other ranks, double-buffered by exchange parity.
  Stats<W> stats[2];
  uint32_t hist[2][RADIX];
  int32_t wcount[2][WINDOWS];
  u128 fx[2];
  uint32_t fxn[2];
  Pick pick[2];
  Best best[2];
  MassPart mass_part[2];
  int32_t slot[2];
  // Block scratch.
  union {
    Pick picks[WARPS];
    Best bests[WARPS];
    u128 fxs[WARPS];
    int32_t ints[WARPS];
    uint32_t uints[WARPS];
    int32_t win[WARPS][WINDOWS];
    Stats<W> stats[WARPS];
    MassPart masses[WARPS];
  } red;
  // Peers' published slots, copied here by a few threads after an exchange.
  union {
    Stats<W> stats[16];
    Pick picks[16];
    Best bests[16];
    u128 fx[16];
    MassPart masses[16];
    int32_t ints[16 * WINDOWS + 16];
  } peers;
  uint32_t peer_n[16];
  uint32_t win[WIN_BINS];  // tile maxima of the whole row in the WIN_BINS absolute bins from the row's top bin down
  // The statistics exchange's inbox: every rank stores its statistics and
  // tile-maximum bins (from its own top bin down) into every rank's slot
  // before the exchange, so that afterwards each rank reads only its own
  // shared memory. (Per-phase sharded calls reuse in_win afterwards.)
  Stats<W> in_stats[16];
  alignas(16) uint16_t in_win[16][WIN_BINS];
  int32_t pushed[16];  // per-rank counts each rank writes into every rank's copy
  int32_t verdict;     // rank 0's decision on a top-p list, written into every rank's copy
  int32_t tiles[TILE_CAP];
  int32_t n_tiles;
  int32_t ival[4];
  u128 fxval;
  double dval;
  float floor_score;
  int32_t n_cand;
  // Rank 0's candidate buffer (list rows) or the weighted-selection buckets (top-p rows).
  union {
    struct {
      uint64_t key[CAP];
      int32_t id[CAP];
    } cand;
    u128 mass[2][RADIX];
  } u;
  // Rank 0's FP64 list: weights and probabilities in list order. The
  // warm-up warp uses them as scratch (it exits before the first cluster
  // exchange, long before any list).
  double lw[LIST_MAX];
  double lp[LIST_MAX];
};

static_assert(sizeof(decltype(Smem<float>::u)) >= ABS_BINS * sizeof(uint32_t), "the tile histogram fits the candidate buffer");
static_assert(sizeof(decltype(Smem<double>::u)) >= ABS_BINS * sizeof(uint32_t), "the tile histogram fits the candidate buffer");

// Adds (v, 1) to bucket b of mass/count, aggregated over the warp's lanes that
// share a bucket (one atomic per distinct bucket). Called by the whole warp;
// lanes with b < 0 contribute nothing.
__device__ __forceinline__ void warp_bucket_add(u128* mass, uint32_t* count, int b, u128 v) {
  unsigned todo = __ballot_sync(0xffffffffu, b >= 0);
  while (todo) {
    const int leader = __ffs(todo) - 1;
    const int bb = __shfl_sync(0xffffffffu, b, leader);
    const unsigned same = __ballot_sync(0xffffffffu, b == bb);
    u128 part = b == bb ? v : u128(0);
    if (mass) part = warp_all(part, [](u128 a, u128 c) { return a + c; });
    if (lane_id() == leader) {
      if (mass) {
        unsigned long long* m = reinterpret_cast<unsigned long long*>(&mass[bb]);
        const unsigned long long lo = uint64_t(part), hi = uint64_t(part >> 64);
        const unsigned long long old = atomicAdd(m, lo);
        const unsigned long long carry = old + lo < old ? 1ull : 0ull;
        if (hi + carry) atomicAdd(m + 1, hi + carry);
      }
      atomicAdd(&count[bb], uint32_t(__popc(same)));
    }
    todo &= ~same;
  }
}

template <int DT> struct Row {
  using T = typename Types<DT>::T;
  using W = typename Types<DT>::W;
  using Key = typename Types<DT>::Key;
  static constexpr int KEY_BITS = int(sizeof(Key) * 8);

  const Params& p;
  Smem<W>& s;
  uint32_t* mask_s;  // this rank's mask words (resident rows)
  uint32_t* hist_abs;  // statistics pass: tile maxima per absolute bin (ABS_BINS, aliasing the candidate buffer)
  W* tmax;           // per 32-token tile of the slice: the largest valid value (-inf if none)
  T* slice;          // this rank's logits (resident rows) or the TMA ring (streamed rows)
  const T* tbase;    // the row in global memory (not sharded)
  bool resident, vec, sharded;
  bool phases;  // a per-phase sharded call: this GPU's columns only, partial results exchanged with the peers
  bool dense;  // after the statistics: no mask and every token of the row valid
  cg::cluster_group cluster;
  int rank, ranks, row, lo, hi, groups;
  int xc;  // exchanges so far (the same on every rank)
  int ring_seq;  // streamed rows: chunks the TMA ring has carried so far (fixes each stage's phase)
  int argmax_;  // the greedy token once argmax_id() has found it, else -1

  // Row-level values, identical on every rank after the statistics merge.
  Stats<W> all;
  W maxv;
  int top_bin;  // the row maximum's absolute bin (-1: no valid token)
  double temperature, top_p, min_p;
  float inv_t, ln_mp, mp_tol;
  bool slow_x, has_mask;
  Address addr;

  __device__ Row(const Params& p_, Smem<W>& s_, uint32_t* m, W* tm, T* sl)
      : p(p_), s(s_), mask_s(m), hist_abs(reinterpret_cast<uint32_t*>(&s_.u)), tmax(tm), slice(sl),
        cluster(cg::this_cluster()) {
    rank = int(cluster.block_rank());
    ranks = int(cluster.num_blocks());
    row = blockIdx.y;
    lo = min(p.width, rank * p.slice_words * 32);
    hi = min(p.width, lo + p.slice_words * 32);
    groups = (hi - lo + 3) / 4;
    xc = 0;
    ring_seq = 0;
    argmax_ = -1;
    has_mask = p.mask != nullptr;
    resident = !p.stream_rows;
    vec = p.vector_load != 0;
    sharded = pulls_columns(p);
    phases = p.sh.count > 1 && p.sh.phases;
    dense = false;
    tbase = static_cast<const T*>(p.target) + int64_t(row) * p.t_s0;
  }

  // ---- global memory ----
  // Column t of the row's target and proposal logits: in the caller's
  // tensors, or in shard t / cols of a vocabulary-sharded call (a peer GPU's
  // buffer for most columns).
  __device__ __forceinline__ const T* target_at(int t) const {
    if (!sharded) return tbase + int64_t(t) * p.t_s1;
    const int g = t / p.sh.cols;
    return static_cast<const T*>(p.sh.target[g]) + int64_t(row) * p.t_s0 + int64_t(t - g * p.sh.cols) * p.t_s1;
  }
  __device__ __forceinline__ const T* draft_at(int t) const {
    if (!sharded) return static_cast<const T*>(p.draft) + int64_t(row) * p.q_s0 + int64_t(t) * p.q_s1;
    const int g = t / p.sh.cols;
    return static_cast<const T*>(p.sh.draft[g]) + int64_t(row) * p.q_s0 + int64_t(t - g * p.sh.cols) * p.q_s1;
  }
  // TMA bulk copies of columns [c0, c0 + n) of the target row into dst
  // (16-byte aligned, n * sizeof(T) a multiple of 16), in pieces of at most
  // BULK_CHUNK bytes that never cross a shard boundary (shard widths are
  // multiples of 16 columns), all completing on `bar`.
  __device__ void bulk_columns(void* dst, int c0, int n, uint64_t* bar) const {
    uint8_t* d = static_cast<uint8_t*>(dst);
    while (n > 0) {
      int piece = min(n, int(BULK_CHUNK / sizeof(T)));
      if (sharded) piece = min(piece, (c0 / p.sh.cols + 1) * p.sh.cols - c0);
      bulk_load(d, target_at(c0), uint32_t(piece) * uint32_t(sizeof(T)), bar);
      d += size_t(piece) * sizeof(T);
      c0 += piece;
      n -= piece;
    }
  }

  // ---- slice access ----
  // Mask bits of local group g (tokens allowed and inside the slice).
  __device__ __forceinline__ unsigned group_bits(int g) const {
    const int t = 4 * g;
    unsigned bits = 0xfu;
    if (has_mask) {
      const uint32_t word = resident ? mask_s[t >> 5]
                                     : uint32_t(__ldg(p.mask + int64_t(row) * p.m_s0 + int64_t((lo + t) >> 5) * p.m_s1));
      bits = (word >> (t & 31)) & 0xfu;
    }
    const int left = hi - lo - t;
    if (left < 4) bits &= (1u << max(left, 0)) - 1u;
    return bits;
  }
  // The four values of local group g: shared memory for resident rows,
  // global memory (L2) otherwise; -inf past the slice.
  __device__ __forceinline__ void values(int g, W v[4]) const {
    if (resident) {
      load4(slice + 4 * g, v);
    } else if (vec && 4 * g + 4 <= hi - lo) {
      load4_global(target_at(lo + 4 * g), v);  // four columns never straddle a shard boundary
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = 4 * g + j;
        v[j] = t < hi - lo ? widen(*target_at(lo + t)) : W(-INFINITY);
      }
    }
  }
  // Values of local group g and the bits of its valid tokens (allowed, inside
  // the slice, above -inf).
  __device__ __forceinline__ unsigned group(int g, W v[4]) const {
    values(g, v);
    unsigned bits = group_bits(g);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (!(v[j] > W(-INFINITY))) bits &= ~(1u << j);
    return bits;
  }
  // A single token anywhere in the row, from global memory.
  __device__ __forceinline__ W value_global(int t) const {
    return widen(*target_at(t));
  }
  __device__ __forceinline__ bool allowed_global(int t) const {
    return !has_mask || ((uint32_t(p.mask[int64_t(row) * p.m_s0 + int64_t(t >> 5) * p.m_s1]) >> (t & 31)) & 1u);
  }
  __device__ __forceinline__ bool valid_global(int t) const {
    return allowed_global(t) && value_global(t) > W(-INFINITY);
  }
  __device__ __forceinline__ W q_value(int t) const {
    return widen(*draft_at(t));
  }

  // ---- cluster exchange ----
  // Publish into slot parity(), exchange(), then read slot parity() ^ 1 of
  // every rank. A slot is rewritten two exchanges later, after every rank has
  // passed the exchange that follows its reads.
  __device__ __forceinline__ int parity() const { return xc & 1; }
  __device__ __forceinline__ void exchange() {
    cluster.sync();
    ++xc;
  }
  template <class X> __device__ __forceinline__ X* peer(X* local, int r) { return cluster.map_shared_rank(local, r); }

  // ---- temperature-scaled values ----
  __device__ __forceinline__ double x64(W v) const { return (double(v) - double(maxv)) / temperature; }
  __device__ __forceinline__ float x32(W v) const {
    if constexpr (sizeof(W) == 8) {
      return __double2float_rn(x64(v));
    } else {
      if (slow_x) return __double2float_rn(x64(v));
      return __fmul_rn(__fsub_rn(v, maxv), inv_t);
    }
  }
  // w = exp(x64) >= min_p and w > 0, decided exactly: FP32 settles tokens
  // clear of both thresholds, FP64 the rest.
  __device__ __forceinline__ bool weight_kept(W v, float x) const {
    const float tol = __fadd_rn(__fmul_rn(X_ERR, fabsf(x)), mp_tol);
    const float gap = __fsub_rn(x, ln_mp);
    if (x > -744.f && gap > tol) return true;
    if (x < -746.f || gap < -tol) return false;
    return weight_kept_fp64(double(v), double(maxv), temperature, min_p);
  }
  __device__ __forceinline__ bool exact_weight_kept(W v) const {
    return weight_kept_fp64(double(v), double(maxv), temperature, min_p);
  }

  __device__ __forceinline__ bool in_bounds(bool cond, int site) const {
    return ES_IN_BOUNDS(p.workspace, p.rows, cond, uint32_t(site));
  }

  __device__ void count_fallback() {
    if (rank == 0 && threadIdx.x == 0) atomicAdd(fallback_count(p.workspace), 1u);
  }
  __device__ void count_near_tie(bool near) {
    if (near && rank == 0 && threadIdx.x == 0) atomicAdd(&diagnostics(p.workspace, p.rows)->near_ties, 1u);
  }

  // ---- the statistics pass ----
  __device__ static Stats<W> merge_stats(Stats<W> a, Stats<W> b) {
    Stats<W> m;
    m.vmax = a.vmax > b.vmax ? a.vmax : b.vmax;
    m.qmax = a.qmax > b.qmax ? a.qmax : b.qmax;
    m.valid = a.valid + b.valid;
    m.bad = a.bad | b.bad;
    m.qvalid = a.qvalid + b.qvalid;
    m.qbad = a.qbad | b.qbad;
    m.top_bin = a.top_bin > b.top_bin ? a.top_bin : b.top_bin;
    return m;
  }
  __device__ Stats<W> block_stats(Stats<W> v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      Stats<W> y;
      y.vmax = shfl_xor(v.vmax, o); y.qmax = shfl_xor(v.qmax, o);
      y.valid = shfl_xor(v.valid, o); y.bad = shfl_xor(v.bad, o); y.qvalid = shfl_xor(v.qvalid, o);
      y.qbad = shfl_xor(v.qbad, o);
      y.top_bin = shfl_xor(v.top_bin, o);
      v = merge_stats(v, y);
    }
    if (lane_id() == 0) s.red.stats[warp_id()] = v;
    sync_rows();
    Stats<W> m = s.red.stats[0];
    for (int w = 1; w < WARPS; ++w) m = merge_stats(m, s.red.stats[w]);
    sync_rows();
    return m;
  }
  // Statistics accumulated over groups.
  struct Acc {
    W best;
    int valid, bad;
  };
  // Groups [g_begin, g_end) of the slice (g_begin a multiple of 8; every
  // tile either wholly inside or the slice's last): NaN / +inf anywhere
  // (even masked), the valid count, the maximum, and each 32-token tile's
  // maximum. The 8 lanes of a tile combine its maximum by shuffles.
  //
  // A whole unmasked group takes the short path: the sum of its four values
  // scaled by 1/4 is NaN or +inf exactly when one of them is (four finite
  // quarters cannot overflow, and -inf + +inf is NaN), and -inf exactly when
  // one is -inf otherwise; -inf values are counted only then.
  template <class Load> __device__ __forceinline__ void stats_groups(int g_begin, int g_end, Load load, Acc& a) {
    for (int base = g_begin + warp_id() * 32; base < g_end; base += THREADS) {
      const int g = base + lane_id();
      W tile = W(-INFINITY);
      if (g < g_end) {
        W v[4];
        load(g, v);
        if (!has_mask && 4 * g + 4 <= hi - lo) {
          const W q = (v[0] * W(0.25) + v[1] * W(0.25)) + (v[2] * W(0.25) + v[3] * W(0.25));
          a.bad |= !(q < W(INFINITY));
          int n = 4;
          if (q == W(-INFINITY))
            n = int(v[0] > W(-INFINITY)) + int(v[1] > W(-INFINITY)) + int(v[2] > W(-INFINITY)) +
                int(v[3] > W(-INFINITY));
          a.valid += n;
          const W m01 = v[0] > v[1] ? v[0] : v[1], m23 = v[2] > v[3] ? v[2] : v[3];
          tile = m01 > m23 ? m01 : m23;
        } else {
          const unsigned bits = group_bits(g);
          const int inside = hi - lo - 4 * g;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (j < inside) a.bad |= !(v[j] < W(INFINITY)) & (v[j] != W(-INFINITY));  // NaN or +inf
            const bool ok = ((bits >> j) & 1u) && v[j] > W(-INFINITY);
            a.valid += ok;
            if (ok && v[j] > tile) tile = v[j];
          }
        }
        if (tile > a.best) a.best = tile;
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        const W other = shfl_xor(tile, o);
        tile = other > tile ? other : tile;
      }
      if ((lane_id() & 7) == 0 && g < g_end && in_bounds(unsigned(g >> 3) < unsigned(tile_count()), 1))
        tmax[g >> 3] = tile;
    }
  }
  // Tiles (32 tokens) of this rank's slice; the last may be partial.
  __device__ __forceinline__ int tile_count() const { return (groups + 7) / 8; }
  // Local token i of the slice (0 <= i < hi - lo): its value and whether the
  // mask allows it.
  __device__ __forceinline__ W value_local(int i) const {
    if (resident && !in_bounds(unsigned(i) < unsigned(p.slice_words * 32), 7)) return W(-INFINITY);
    return resident ? widen(slice[i]) : widen(*target_at(lo + i));
  }
  __device__ __forceinline__ bool allowed_local(int i) const {
    if (!has_mask) return true;
    const uint32_t word = resident ? mask_s[i >> 5]
                                   : uint32_t(p.mask[int64_t(row) * p.m_s0 + int64_t((lo >> 5) + (i >> 5)) * p.m_s1]);
    return (word >> (i & 31)) & 1u;
  }
  // The lowest-ID valid token of this rank's slice whose value is `target`
  // (INT_MAX if none). Only the first tile whose maximum reaches `target`
  // is read, so `target` must be at least every valid value of the slice
  // that precedes it (the row or slice maximum). Block-uniform.
  __device__ int first_at_value(W target) {
    int first_tile = INT_MAX;
    for (int t = threadIdx.x; t < tile_count(); t += THREADS)
      if (tmax[t] >= target) {
        first_tile = t;  // a thread's tiles ascend: its first hit is its lowest
        break;
      }
    first_tile = block_all(first_tile, [](int x, int y) { return x < y ? x : y; }, s.red.ints);
    int found = INT_MAX;
    if (first_tile != INT_MAX && warp_id() == 0) {
      const int i = 32 * first_tile + lane_id();
      const bool hit = i < hi - lo && allowed_local(i) && value_local(i) == target;
      const unsigned b = __ballot_sync(0xffffffffu, hit);
      if (b) found = lo + 32 * first_tile + __ffs(b) - 1;
    }
    return block_all(found, [](int x, int y) { return x < y ? x : y; }, s.red.ints);
  }
  // The row's greedy token: the lowest ID whose value is the row maximum,
  // over the cluster (found on first use, then kept). Every thread of every
  // rank calls it at the same point.
  __device__ int argmax_id() {
    if (argmax_ < 0) argmax_ = cluster_min(first_at_value(maxv));
    return argmax_;
  }
  // Bytes of the slice the TMA ring carries (whole 16-byte units), in chunks.
  __device__ __forceinline__ uint32_t ring_bytes() const { return (uint32_t(hi - lo) * uint32_t(sizeof(T))) & ~15u; }
  __device__ __forceinline__ int ring_chunks() const { return int((ring_bytes() + RING_CHUNK - 1) / RING_CHUNK); }
  // Thread 0 starts the TMA copy of chunk c into the ring stage of the
  // ring's seq-th use.
  __device__ __forceinline__ void ring_issue(int c, int seq) {
    const uint32_t off = uint32_t(c) * RING_CHUNK, len = min(RING_CHUNK, ring_bytes() - off);
    const int stage = seq % p.stream_rows;
    uint64_t* bar = &s.ring_bar[stage];
    mbar_arrive_expect_tx(bar, len);
    bulk_columns(reinterpret_cast<uint8_t*>(slice) + stage * RING_CHUNK, lo + int(off / sizeof(T)),
                 int(len / sizeof(T)), bar);
  }
  // ---- tile histogram ----
  // Adds tiles [t0, t1)'s maxima to the absolute histogram: every warp over
  // its share, one atomic per distinct bin per warp step.
  __device__ void hist_tiles(int t0, int t1) {
    for (int base = t0 + int(threadIdx.x) - lane_id(); base < t1; base += THREADS) {
      const int t = base + lane_id();
      const W m = t < t1 ? tmax[t] : W(-INFINITY);
      const int b = m > W(-INFINITY) ? abs_bin(m) : -1;
      const unsigned same = __match_any_sync(0xffffffffu, b);
      if (b >= 0 && lane_id() == __ffs(same) - 1 && in_bounds(b < ABS_BINS, 4))
        atomicAdd(&hist_abs[b], uint32_t(__popc(same)));
    }
  }
  // ---- per-phase sharded calls ----
  // GPU g's slot of this row in GPU `to`'s exchange buffer.
  __device__ __forceinline__ uint64_t* phase_slot(int to, int g) const {
    return reinterpret_cast<PhaseRow*>(p.sh.exchange[to])[row].slot[g];
  }
  // The call's tag: never 0, so a zeroed buffer matches no call.
  __device__ __forceinline__ uint32_t phase_tag() const { return uint32_t(p.sh.epoch % 0xffffffffull) + 1u; }
  // Word w of GPU g's slot in this GPU's buffer, once it carries the call's
  // tag (bounded). A word that never arrives counts a timeout and marks the
  // row on rank 0; returns false.
  __device__ bool phase_read(int g, int w, uint32_t& datum) {
    if (ld_tagged_sys(phase_slot(p.sh.rank, g) + w, phase_tag(), datum, 1u << 20)) return true;
    atomicAdd(&diagnostics(p.workspace, p.rows)->wait_timeouts, 1u);
    atomicOr(peer(&s.timeout, 0), 1);
    return false;
  }
  // After the statistics merge: rank 0 stores this GPU's row statistics and
  // window bins into its slot on every GPU; then every rank reads every
  // GPU's from its own buffer and merges them in GPU order, so that all
  // ranks of all GPUs hold the whole row's values (as the cluster merge
  // makes them over ranks). False if a GPU's words never arrived.
  __device__ bool phase_stats() {
    const int n = p.sh.count;
    const uint32_t tag = phase_tag();
    if (rank == 0) {
      const uint64_t vbits = uint64_t(__double_as_longlong(double(all.vmax)));
      for (int i = threadIdx.x; i < n * PHASE_STAT_WORDS; i += THREADS) {
        const int to = i / PHASE_STAT_WORDS, w = i - to * PHASE_STAT_WORDS;
        uint32_t d;
        if (w == 0) d = uint32_t(vbits);
        else if (w == 1) d = uint32_t(vbits >> 32);
        else if (w == 2) d = uint32_t(all.valid);
        else if (w == 3) d = uint32_t(all.bad != 0) | (uint32_t(all.top_bin + 1) << 1);
        else d = min(s.win[2 * (w - 4)], 65535u) | (min(s.win[2 * (w - 4) + 1], 65535u) << 16);
        st_tagged_sys(phase_slot(to, p.sh.rank) + w, d, tag);
      }
    }
    ES_TRACE(p.workspace, p.rows, row, rank, 16);
    // Every GPU's words, into the cluster-window inbox (free since the
    // cluster exchange: no rank writes it again in this call).
    static_assert(sizeof(s.in_win) >= MAX_SHARDS * PHASE_STAT_WORDS * sizeof(uint32_t), "the words fit the inbox");
    uint32_t* words = reinterpret_cast<uint32_t*>(&s.in_win[0][0]);
    bool ok = true;
    for (int i = threadIdx.x; i < n * PHASE_STAT_WORDS; i += THREADS) {
      const int g = i / PHASE_STAT_WORDS;
      uint32_t d = 0;
      if (ok) ok = phase_read(g, i - g * PHASE_STAT_WORDS, d);
      words[i] = d;
    }
    if (__syncthreads_or(!ok)) return false;
    ES_TRACE(p.workspace, p.rows, row, rank, 17);
    if (threadIdx.x == 0) {
      Stats<W> m{W(-INFINITY), all.qmax, 0, 0, all.qvalid, all.qbad, -1};
      for (int g = 0; g < n; ++g) {
        const uint32_t* q = words + g * PHASE_STAT_WORDS;
        const W v = W(__longlong_as_double(int64_t((uint64_t(q[1]) << 32) | q[0])));
        const int top = int(q[3] >> 1) - 1;
        m.vmax = v > m.vmax ? v : m.vmax;
        m.valid += int(q[2]);
        m.bad |= int(q[3] & 1u);
        m.top_bin = max(m.top_bin, top);
        s.peer_n[g] = uint32_t(top);
      }
      s.in_stats[0] = m;
    }
    __syncthreads();
    all = s.in_stats[0];
    maxv = all.vmax;
    top_bin = all.top_bin;
    dense = !has_mask && all.valid == p.vocab;
    if (int(threadIdx.x) < PHASE_BINS) {
      uint32_t c = 0;
      for (int g = 0; g < n; ++g) {
        const int top = int(s.peer_n[g]), b = int(threadIdx.x) - (top_bin - top);  // GPU g's bin index
        if (top >= 0 && b >= 0) c += (words[g * PHASE_STAT_WORDS + 4 + b / 2] >> (16 * (b & 1))) & 0xffffu;
      }
      s.win[threadIdx.x] = c;
    }
    __syncthreads();
    ES_TRACE(p.workspace, p.rows, row, rank, 18);
    return true;
  }

  // The statistics pass over the whole slice: from shared memory (resident),
  // through the TMA ring (streamed, 16-byte aligned rows), or from global
  // memory; then the cluster merge. Returns false if a copy never arrived.
  __device__ bool stats_pass(bool timed_out) {
    Acc a{W(-INFINITY), 0, 0};
    bool lost = timed_out;
    if (resident) {
      stats_groups(0, groups, [&](int g, W v[4]) {
        if (in_bounds(4 * g + 4 <= p.slice_words * 32, 2)) load4(slice + 4 * g, v);
      }, a);
    } else if (vec) {
      constexpr int GPC = int(RING_CHUNK / (4 * sizeof(T)));  // groups per chunk
      const int ring_groups = int(ring_bytes() / (4 * sizeof(T))) & ~7;  // whole tiles
      const int chunks = ring_chunks(), stages = p.stream_rows;
      for (int c = 0; c < chunks; ++c) {
        uint32_t spins = 0;
        while (!mbar_try_wait(&s.ring_bar[c % stages], uint32_t(c / stages) & 1u))
          if (++spins >= (1u << 22)) {
            lost = true;
            break;
          }
        const T* stage = slice + (c % stages) * (RING_CHUNK / sizeof(T)) - int64_t(c) * GPC * 4;
        stats_groups(c * GPC, min((c + 1) * GPC, ring_groups), [&](int g, W v[4]) {
          if (in_bounds(g >= c * GPC && g < (c + 1) * GPC && c % stages < MAX_RING_STAGES, 3)) load4(stage + 4 * g, v);
        }, a);
        sync_rows();  // every row thread is done with this stage
        if (threadIdx.x == 0 && c + stages < chunks) ring_issue(c + stages, c + stages);
      }
      ring_seq = chunks;
      stats_groups(ring_groups, groups, [&](int g, W v[4]) { values(g, v); }, a);  // the last partial tile
    } else {
      stats_groups(0, groups, [&](int g, W v[4]) { values(g, v); }, a);
    }
    lost = sync_rows_or(lost);
    hist_tiles(0, tile_count());  // block_stats below syncs before the histogram is read
    if (lost) a.bad = 1;  // a slice copy never arrived: the row is not trusted
    const int own_top = a.best > W(-INFINITY) ? abs_bin(a.best) : -1;
    const Stats<W> merged = block_stats(Stats<W>{a.best, W(-INFINITY), a.valid, a.bad, 0, 0, own_top});
    // Store the statistics and the WIN_BINS tile-maximum bins from this
    // rank's top bin down into every rank's inbox (the histogram is
    // complete: block_stats synced); the exchange orders the stores.
    if (int(threadIdx.x) < ranks && in_bounds(ranks <= 16 && rank < ranks, 5))
      *peer(&s.in_stats[rank], threadIdx.x) = merged;
    if (int(threadIdx.x) < WIN_BINS) {
      const int b = merged.top_bin - int(threadIdx.x);
      const uint16_t n = uint16_t(merged.top_bin >= 0 && b >= 0 ? min(hist_abs[b], 65535u) : 0u);
      for (int r = 0; r < ranks; ++r) peer(s.in_win[rank], r)[threadIdx.x] = n;
    }
    // The preparation kernel's outputs: its grid is long done by now, so the
    // context load overlaps the exchange.
    wait_for_prerequisite_grid();
    if (threadIdx.x == 0) {
      if (*malformed_flag(p.workspace) != 0) s.ctx.skip = 1;
      else s.ctx = row_contexts(p.workspace, p.rows)[row];
    }
    ES_TRACE(p.workspace, p.rows, row, rank, 8);
    exchange();
    ES_TRACE(p.workspace, p.rows, row, rank, 9);
    all = s.in_stats[0];
    for (int r = 1; r < ranks; ++r) all = merge_stats(all, s.in_stats[r]);
    maxv = all.vmax;
    top_bin = all.top_bin;
    dense = !has_mask && all.valid == p.vocab;
    // The row's tile maxima in the WIN_BINS bins from its top bin down: rank
    // r sent the bins from its own top bin (at most the row's) down.
    if (p.fast && int(threadIdx.x) < WIN_BINS) {
      uint32_t n = 0;
      for (int r = 0; r < ranks; ++r) {
        const int shift = top_bin - s.in_stats[r].top_bin;  // >= 0
        if (s.in_stats[r].top_bin >= 0 && int(threadIdx.x) >= shift &&
            in_bounds(int(threadIdx.x) - shift < WIN_BINS, 6))
          n += s.in_win[r][threadIdx.x - shift];
      }
      s.win[threadIdx.x] = n;
    }
    __syncthreads();
    return !lost;
  }

  // A later pass over the slice: f(g, v, bits) for every group g, with v its
  // four values and bits its valid tokens (allowed, inside the slice, above
  // -inf). All lanes of a warp call f together (past the slice with bits 0),
  // so f may use warp collectives. Resident rows read shared memory;
  // streamed rows go through the TMA ring again, which keeps 16 KB stages in
  // flight where plain loads would keep a few hundred bytes per warp. A copy
  // that never arrives (a bounded wait) marks the row on rank 0.
  template <class F> __device__ void slice_pass(F f) {
    constexpr int GPC = int(RING_CHUNK / (4 * sizeof(T)));  // groups per chunk
    const bool ring = !resident && vec;
    const int ring_groups = ring ? int(ring_bytes() / (4 * sizeof(T))) & ~7 : 0;
    const int chunks = ring ? ring_chunks() : 0, stages = p.stream_rows;
    if (threadIdx.x == 0)
      for (int c = 0; c < min(stages, chunks); ++c) ring_issue(c, ring_seq + c);
    bool lost = false;
    // Segments: the ring's chunks, then the rest of the slice (all of it for
    // resident rows) from shared or global memory. One call site for f.
    for (int c = 0; c <= chunks; ++c) {
      const int seq = ring_seq + c;
      int g0 = ring_groups, g1 = groups;
      const T* src = resident ? slice : nullptr;
      if (c < chunks) {
        for (uint32_t spins = 0; !lost && !mbar_try_wait(&s.ring_bar[seq % stages], uint32_t(seq / stages) & 1u);)
          if (++spins >= (1u << 22)) lost = true;
        src = slice + (seq % stages) * (RING_CHUNK / sizeof(T)) - int64_t(c) * GPC * 4;
        g0 = c * GPC;
        g1 = min(g0 + GPC, ring_groups);
      }
      auto load = [&](int g, W* v) {
        if (src == nullptr) return group(g, v);
        load4(src + 4 * g, v);
        unsigned bits = group_bits(g);
        if (!dense)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (!(v[j] > W(-INFINITY))) bits &= ~(1u << j);
        return bits;
      };
      for (int base = g0 + warp_id() * 32; base < g1; base += THREADS) {
        const int g = base + lane_id();
        W v[4] = {W(-INFINITY), W(-INFINITY), W(-INFINITY), W(-INFINITY)};
        unsigned bits = 0;
        if (g < g1) bits = load(g, v);
        f(g, v, bits);
      }
      if (c < chunks) {
        lost = __syncthreads_or(lost);  // every thread is done with this stage
        if (threadIdx.x == 0 && c + stages < chunks) ring_issue(c + stages, seq + stages);
      }
    }
    ring_seq += chunks;
    if (lost && threadIdx.x == 0) {
      atomicAdd(&diagnostics(p.workspace, p.rows)->wait_timeouts, 1u);
      atomicOr(peer(&s.timeout, 0), 1);
    }
  }

  // The proposal row's checks (NaN / +inf, valid count) and maximum, for a
  // full-q draft row, merged over the cluster into all.qmax / qvalid / qbad.
  __device__ void q_stats_pass() {
    W qmax = W(-INFINITY);
    int qvalid = 0, qbad = 0;
    for (int t = lo + int(threadIdx.x); t < hi; t += THREADS) {
      const W y = q_value(t);
      qbad |= isnan(y) | (y == W(INFINITY));
      qvalid += y > W(-INFINITY);
      qmax = y > qmax ? y : qmax;
    }
    const Stats<W> merged = block_stats(Stats<W>{W(-INFINITY), qmax, 0, 0, qvalid, qbad});
    if (threadIdx.x == 0) s.stats[parity()] = merged;
    exchange();
    if (int(threadIdx.x) < ranks) s.peers.stats[threadIdx.x] = *peer(&s.stats[parity() ^ 1], threadIdx.x);
    __syncthreads();
    Stats<W> q = s.peers.stats[0];
    for (int r = 1; r < ranks; ++r) q = merge_stats(q, s.peers.stats[r]);
    all.qmax = q.qmax;
    all.qvalid = q.qvalid;
    all.qbad = q.qbad;
    __syncthreads();
  }

  // ---- cluster-wide reductions ----
  __device__ u128 cluster_sum(u128 local, uint32_t n_local, uint32_t* n_total) {
    const u128 bsum = block_all(local, [](u128 a, u128 b) { return a + b; }, s.red.fxs);
    const uint32_t bn = block_all(n_local, [](uint32_t a, uint32_t b) { return a + b; }, s.red.uints);
    if (threadIdx.x == 0) {
      s.fx[parity()] = bsum;
      s.fxn[parity()] = bn;
    }
    exchange();
    if (int(threadIdx.x) < ranks) {
      s.peers.fx[threadIdx.x] = *peer(&s.fx[parity() ^ 1], threadIdx.x);
      s.peer_n[threadIdx.x] = *peer(&s.fxn[parity() ^ 1], threadIdx.x);
    }
    __syncthreads();
    u128 total = 0;
    uint32_t n = 0;
    for (int r = 0; r < ranks; ++r) {
      total += s.peers.fx[r];
      n += s.peer_n[r];
    }
    *n_total = n;
    __syncthreads();
    return total;
  }
  __device__ int cluster_min(int local) {
    const int b = block_all(local, [](int a, int c) { return a < c ? a : c; }, s.red.ints);
    if (threadIdx.x == 0) s.slot[parity()] = b;
    exchange();
    if (int(threadIdx.x) < ranks) s.peers.ints[threadIdx.x] = *peer(&s.slot[parity() ^ 1], threadIdx.x);
    __syncthreads();
    int m = INT_MAX;
    for (int r = 0; r < ranks; ++r) m = min(m, s.peers.ints[r]);
    __syncthreads();
    return m;
  }

  // The FP64 argmax over the cluster (lowest ID on ties); -1 if empty.
  __device__ int cluster_best(Best b) {
    b = block_all(b, [](Best a, Best c) { return best_of(a, c); }, s.red.bests);
    if (threadIdx.x == 0) s.best[parity()] = b;
    exchange();
    if (int(threadIdx.x) < ranks) s.peers.bests[threadIdx.x] = *peer(&s.best[parity() ^ 1], threadIdx.x);
    __syncthreads();
    Best winner = no_best();
    for (int r = 0; r < ranks; ++r) winner = best_of(winner, s.peers.bests[r]);
    __syncthreads();
    return winner.id == INT_MAX ? -1 : winner.id;
  }

  // ---- radix selection (integer, exact) ----
  // The n-th (1-based) valid token in (value desc, ID asc) order among those
  // `admit` accepts (1 <= n <= their count): 8-bit digits of the order key
  // from the top, one shared-memory pass and one cluster exchange of 256
  // counts per level, then the n-th lowest ID among tokens with that key.
  template <class Admit> __device__ Cut<Key> select_nth(int n, Admit admit) {
    Key prefix = 0, known = 0;
    int need = n, digit = 0;
    for (int shift = KEY_BITS - 8; shift >= 0; shift -= 8) {
      uint32_t* h = s.hist[parity()];
      for (int i = threadIdx.x; i < RADIX; i += THREADS) h[i] = 0;
      __syncthreads();
      slice_pass([&](int g, const W* v, unsigned bits) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          int d = -1;
          if ((bits >> j) & 1u) {
            const Key k = order_key(v[j]);
            if ((k & known) == prefix && admit(k, lo + 4 * g + j, v[j])) d = int((k >> shift) & 255);
          }
          warp_bucket_add(nullptr, h, d, 0);
        }
      });
      exchange();
      // Thread i owns digit 255 - i: merged counts, scanned from the top.
      if (threadIdx.x == 0) { s.ival[0] = 0; s.ival[1] = 0; }
      int cnt = 0;
      for (int r = 0; r < ranks; ++r) cnt += int(peer(s.hist[parity() ^ 1], r)[255 - threadIdx.x]);
      int total;
      const int cum = block_scan(cnt, s.red.ints, &total);
      if (cum >= need && cum - cnt < need) {
        s.ival[0] = 255 - int(threadIdx.x);
        s.ival[1] = cum - cnt;
      }
      __syncthreads();
      digit = s.ival[0] & 255;
      need -= s.ival[1];
      prefix |= Key(digit) << shift;
      known |= Key(255) << shift;
      __syncthreads();
    }
    // Ties at the key: ranks own contiguous ID ranges, so the last level's
    // per-rank counts of the digit locate the need-th lowest ID.
    int before = 0, owner = -1;
    for (int r = 0; r < ranks && owner < 0; ++r) {
      const int c = int(peer(s.hist[parity() ^ 1], r)[digit]);
      if (before + c >= need) owner = r;
      else before += c;
    }
    int id = INT_MAX;
    if (owner == rank)
      id = nth_local(need - before, [&](W v, int t, Key k) { return k == prefix && admit(k, t, v); });
    id = cluster_min(owner == rank ? id : INT_MAX);
    return Cut<Key>{1, prefix, id};
  }

  // The n-th (1-based) valid token of this rank's slice in ID order that
  // `match` accepts; INT_MAX if there are fewer. Block-uniform.
  template <class Match> __device__ int nth_local(int n, Match match) {
    const int per = (groups + THREADS - 1) / THREADS;  // thread i takes groups [i*per, (i+1)*per)
    const int g0 = threadIdx.x * per, g1 = min(groups, g0 + per);
    int c = 0;
    for (int g = g0; g < g1; ++g) {
      W v[4];
      const unsigned bits = group(g, v);
      for (int j = 0; j < 4; ++j) c += ((bits >> j) & 1u) && match(v[j], lo + 4 * g + j, order_key(v[j]));
    }
    int total;
    const int incl = block_scan(c, s.red.ints, &total);
    int found = INT_MAX;
    if (incl >= n && incl - c < n) {
      int k = incl - c;
      for (int g = g0; g < g1 && found == INT_MAX; ++g) {
        W v[4];
        const unsigned bits = group(g, v);
        for (int j = 0; j < 4; ++j)
          if (((bits >> j) & 1u) && match(v[j], lo + 4 * g + j, order_key(v[j])) && ++k == n) {
            found = lo + 4 * g + j;
            break;
          }
      }
    }
    return block_all(found, [](int a, int b) { return a < b ? a : b; }, s.red.ints);
  }

  // ---- list candidates ----
  // Appends this rank's valid tokens that `take` accepts to rank 0's
  // candidate buffer from `offset` on (there are at most CAP in all), then
  // exchanges.
  template <class Take> __device__ void gather(int offset, Take take) {
    if (threadIdx.x == 0) s.n_cand = 0;
    __syncthreads();
    uint64_t* keys = peer(s.u.cand.key, 0);
    int32_t* ids = peer(s.u.cand.id, 0);
    for (int g = threadIdx.x; g < groups; g += THREADS) {
      W v[4];
      const unsigned bits = group(g, v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = lo + 4 * g + j;
        if (!((bits >> j) & 1u) || !take(v[j], t)) continue;
        const int at_ = offset + atomicAdd(&s.n_cand, 1);
        if (at_ < CAP) {
          keys[at_] = uint64_t(order_key(v[j]));
          ids[at_] = t;
        }
      }
    }
    exchange();
  }
  // Counts this rank's valid tokens that `take` accepts, exchanges, and
  // gathers them to rank 0 if they fit; returns the total (> CAP: nothing
  // was gathered).
  template <class Take> __device__ int gather_all(Take take) {
    int c = 0;
    for (int g = threadIdx.x; g < groups; g += THREADS) {
      W v[4];
      const unsigned bits = group(g, v);
      for (int j = 0; j < 4; ++j) c += ((bits >> j) & 1u) && take(v[j], lo + 4 * g + j);
    }
    c = block_all(c, [](int a, int b) { return a + b; }, s.red.ints);
    if (threadIdx.x == 0) s.slot[parity()] = c;
    exchange();
    if (int(threadIdx.x) < ranks) s.peers.ints[threadIdx.x] = *peer(&s.slot[parity() ^ 1], threadIdx.x);
    __syncthreads();
    int total = 0, offset = 0;
    for (int r = 0; r < ranks; ++r) {
      const int cr = s.peers.ints[r];
      total += cr;
      if (r < rank) offset += cr;
    }
    __syncthreads();
    if (total <= CAP) gather(offset, take);
    return total;
  }
  // Distance below the row maximum in 0.5-logit bins (DIST_BINS: 64 or more).
  __device__ __forceinline__ int dist_bin(W v) const {
    const float d = float(maxv - v);  // monotone in v
    return d < float(DIST_BINS / 2) ? int(d * 2.f) : DIST_BINS;
  }
  // The top-n valid tokens (and every token tied with the n-th) gathered to
  // rank 0. The ranks histogram their 32-token tiles by the distance of each
  // tile's maximum below the row's (shared-memory atomics); the first bin b
  // where the cumulative tile count reaches n bounds the n-th token (every
  // such tile has a token within bin b), so every valid token with bin <= b
  // is gathered, from those tiles only: they are listed, then read by one
  // warp each (one token per lane). Slots in rank 0's buffer come from an
  // atomic counter there, one per warp and tile; each rank pushes its count
  // to every rank before the closing exchange. Returns the count, or -1 if
  // no bin below 64 logits qualifies or the tokens do not fit the buffer
  // (the caller then radix-selects).
  __device__ int gather_near(int n) {
    uint32_t* h = s.hist[parity()];
    for (int i = threadIdx.x; i < RADIX; i += THREADS) h[i] = 0;
    if (threadIdx.x == 0) {
      s.n_cand = 0;
      s.n_tiles = 0;
    }
    __syncthreads();
    const int nt = tile_count();
    for (int t = threadIdx.x; t < nt; t += THREADS) {
      const W m = tmax[t];
      if (!(m > W(-INFINITY))) continue;  // no valid token in the tile
      const int b = dist_bin(m);
      if (b < DIST_BINS) atomicAdd(&h[b], 1u);
    }
    exchange();
    int cnt = 0;
    if (int(threadIdx.x) < DIST_BINS)
      for (int rr = 0; rr < ranks; ++rr) cnt += int(peer(s.hist[parity() ^ 1], rr)[threadIdx.x]);
    int total;
    const int cum = block_scan(cnt, s.red.ints, &total);
    if (threadIdx.x == 0) s.ival[0] = -1;
    __syncthreads();
    if (int(threadIdx.x) < DIST_BINS && cum >= n && cum - cnt < n) s.ival[0] = threadIdx.x;
    __syncthreads();
    const int window = s.ival[0];
    ES_TRACE(p.workspace, p.rows, row, rank, 4);
    if (window < 0) return -1;  // the same on every rank
    // List this rank's tiles within the window.
    for (int t = threadIdx.x; t < nt; t += THREADS) {
      const W m = tmax[t];
      if (m > W(-INFINITY) && dist_bin(m) <= window) {
        const int at_ = atomicAdd(&s.n_tiles, 1);
        if (at_ < TILE_CAP) s.tiles[at_] = t;
      }
    }
    __syncthreads();
    ES_TRACE(p.workspace, p.rows, row, rank, 13);
    const int listed = s.n_tiles;
    int* counter = peer(&s.n_cand, 0);
    uint64_t* keys = peer(s.u.cand.key, 0);
    int32_t* ids = peer(s.u.cand.id, 0);
    int mine = 0;  // tokens this warp gathered (the same in every lane)
    // Token lane of tile t: its value, -inf if it is past the slice or masked.
    auto load_tile = [&](int t) {
      const int i = 32 * t + lane_id();
      return i < hi - lo && allowed_local(i) ? value_local(i) : W(-INFINITY);
    };
    // Tiles' tokens within the window, appended by the whole warp
    // (warp-uniform call; t[b] < 0 marks no tile): one atomic on rank 0's
    // counter reserves the slots of all of them.
    auto take_tiles = [&](const int* t, const W* v, int count) {
      unsigned hits[4];
      int total = 0;
      for (int b = 0; b < count; ++b) {
        const bool hit = t[b] >= 0 && v[b] > W(-INFINITY) && dist_bin(v[b]) <= window;
        hits[b] = __ballot_sync(0xffffffffu, hit);
        total += __popc(hits[b]);
      }
      if (total == 0) return;
      int base = 0;
      if (lane_id() == 0) base = atomicAdd(counter, total);
      base = __shfl_sync(0xffffffffu, base, 0);
      for (int b = 0; b < count; ++b) {
        if ((hits[b] >> lane_id()) & 1u) {
          const int at_ = base + __popc(hits[b] & ((1u << lane_id()) - 1u));
          if (at_ < CAP) {
            keys[at_] = uint64_t(order_key(v[b]));
            ids[at_] = lo + 32 * t[b] + lane_id();
          }
        }
        base += __popc(hits[b]);
      }
      mine += total;
    };
    if (listed <= TILE_CAP) {
      // A warp's listed tiles in batches: all of a batch's loads (L2 for
      // streamed rows) are in flight before the first is used.
      constexpr int BATCH = 4;
      for (int k0 = warp_id(); k0 < listed; k0 += WARPS * BATCH) {
        W v[BATCH];
        int t[BATCH];
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
          const int k = k0 + b * WARPS;
          t[b] = k < listed ? s.tiles[k] : -1;
          v[b] = t[b] >= 0 ? load_tile(t[b]) : W(-INFINITY);
        }
        take_tiles(t, v, BATCH);
      }
    } else {  // too many tiles to list: every warp walks the tile maxima
      for (int t = warp_id(); t < nt; t += WARPS) {
        const W m = tmax[t];
        if (m > W(-INFINITY) && dist_bin(m) <= window) {
          const W v = load_tile(t);
          take_tiles(&t, &v, 1);
        }
      }
    }
    ES_TRACE(p.workspace, p.rows, row, rank, 14);
    mine = block_all(lane_id() == 0 ? mine : 0, [](int x, int y) { return x + y; }, s.red.ints);
    if (int(threadIdx.x) < ranks) peer(s.pushed, threadIdx.x)[rank] = mine;
    exchange();
    int gathered = 0;
    for (int rr = 0; rr < ranks; ++rr) gathered += s.pushed[rr];
    return gathered <= CAP ? gathered : -1;
  }

  // Sorts rank 0's m candidates into (key desc, ID asc) order (bitonic):
  // up to 32 within warp 0's registers, more in shared memory.
  __device__ void sort_candidates(int m) {
    if (!in_bounds(m <= CAP, 8)) m = CAP;
    if (m <= 32) {
      if (warp_id() == 0) {
        const int i = lane_id();
        uint64_t key = i < m ? s.u.cand.key[i] : 0;  // empty lanes sort last
        int32_t id = i < m ? s.u.cand.id[i] : INT_MAX;
#pragma unroll
        for (int k = 2; k <= 32; k <<= 1)
#pragma unroll
          for (int j = k >> 1; j > 0; j >>= 1) {
            const uint64_t other_key = __shfl_xor_sync(0xffffffffu, key, j);
            const int32_t other_id = __shfl_xor_sync(0xffffffffu, id, j);
            const bool mine_first = key > other_key || (key == other_key && id < other_id);
            const bool keep_first = ((i & j) == 0) == ((i & k) == 0);
            if (mine_first != keep_first) {
              key = other_key;
              id = other_id;
            }
          }
        s.u.cand.key[i] = key;
        s.u.cand.id[i] = id;
      }
      __syncthreads();
      return;
    }
    if (m <= LIST_MAX) {
      // Rank sort: each candidate's position is the number of candidates
      // before it in the order ((key, ID) pairs are distinct), then one scatter.
      const int i = threadIdx.x;
      uint64_t key = 0;
      int32_t id = INT_MAX;
      int rank_i = 0;
      if (i < m) {
        key = s.u.cand.key[i];
        id = s.u.cand.id[i];
        for (int j = 0; j < m; ++j) {
          const uint64_t kj = s.u.cand.key[j];
          rank_i += kj > key || (kj == key && s.u.cand.id[j] < id);
        }
      }
      __syncthreads();
      if (i < m) {
        s.u.cand.key[rank_i] = key;
        s.u.cand.id[rank_i] = id;
      }
      __syncthreads();
      return;
    }
    int size = 1;
    while (size < m) size <<= 1;
    uint64_t* key = s.u.cand.key;
    int32_t* id = s.u.cand.id;
    for (int i = m + threadIdx.x; i < size; i += THREADS) {
      key[i] = 0;
      id[i] = INT_MAX;
    }
    __syncthreads();
    for (int k = 2; k <= size; k <<= 1)
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = threadIdx.x; i < size; i += THREADS) {
          const int l = i ^ j;
          if (l <= i) continue;
          const bool desc = (i & k) == 0;
          const bool i_first = key[i] > key[l] || (key[i] == key[l] && id[i] < id[l]);
          if (i_first != desc) {
            const uint64_t tk = key[i]; key[i] = key[l]; key[l] = tk;
            const int32_t ti = id[i]; id[i] = id[l]; id[l] = ti;
          }
        }
        __syncthreads();
      }
  }

  // ---- exact sums ----
  // Sum of exact FP64 weights over this row's valid tokens that `kept`
  // accepts (with the exact min-p test), over the cluster.
  template <class Kept> __device__ double exact_mass(Kept kept) {
    u128 acc = 0;
    uint32_t n = 0;
    slice_pass([&](int g, const W* v, unsigned bits) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (!((bits >> j) & 1u) || !kept(order_key(v[j]), lo + 4 * g + j)) continue;
        const double w = exp(x64(v[j]));
        if (!(w >= min_p && w > 0)) continue;
        acc += fx_of(w);
        ++n;
      }
    });
    uint32_t total_n;
    const u128 total = cluster_sum(acc, n, &total_n);
    bool near;
    const double r = fx_round(total, total_n, &near);
    count_near_tie(near);
    return r;
  }
  // The proposal's normalizer: the exact sum of exp(y - max y) over the q row.
  __device__ double q_mass() {
    u128 acc = 0;
    uint32_t n = 0;
    for (int t = lo + int(threadIdx.x); t < hi; t += THREADS) {
      const W y = q_value(t);
      if (!(y > W(-INFINITY))) continue;
      const double w = exp(double(y) - double(all.qmax));
      if (!(w > 0)) continue;
      acc += fx_of(w);
      ++n;
    }
    uint32_t total_n;
    const u128 total = cluster_sum(acc, n, &total_n);
    bool near;
    const double r = fx_round(total, total_n, &near);
    count_near_tie(near);
    return r;
  }

  // ---- approximate sums ----
  // Bounds on the exact sum of the FP64 weights exp(x) of the valid tokens
  // `kept` accepts whose weight min-p keeps, i.e. on the oracle's fsum of
  // that set before its rounding, from FP32 weights e = __expf(x32), each
  // within MASS_ERR (1 + |x|) e of exact. A thread sums e and e |x| in FP32
  // over at most eight groups (32 additions, each rounding by at most 2^-24
  // of the partial sum, all terms being positive) before adding the partial
  // sums into FP64. Tokens too close to the min-p threshold count only in
  // the upper bound, as does 2^-120 for every counted token (an FP64 weight
  // that the FP32 exponential flushes to zero). One exchange.
  template <class Kept> __device__ Interval approx_mass(Kept kept, bool cuts) {
    float s32 = 0.f, u32 = 0.f, ex32 = 0.f;  // weights kept, unsure; sum of e |x|
    double s64 = 0, u64 = 0, ex64 = 0;
    uint32_t n = 0;
    int fold = 0;
    const bool min_p_on = min_p > 0;
    slice_pass([&](int g, const W* v, unsigned bits) {
      if (!bits) return;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (!((bits >> j) & 1u)) continue;
        if (cuts && !kept(order_key(v[j]), lo + 4 * g + j)) continue;
        const float x = x32(v[j]);
        if (!(x >= -746.f)) continue;  // exp(x) is 0 in FP64
        bool sure = x > -744.f;
        if (min_p_on) {
          const float tol = __fadd_rn(__fmul_rn(X_ERR, fabsf(x)), mp_tol);
          const float gap = __fsub_rn(x, ln_mp);
          if (gap < -tol) continue;  // min-p certainly drops it
          sure = sure && gap > tol;
        }
        const float e = __expf(x);
        ex32 = __fmaf_rn(e, -x, ex32);
        if (sure) s32 = __fadd_rn(s32, e);
        else u32 = __fadd_rn(u32, e);
        ++n;
      }
      if (++fold == 8) {
        s64 += double(s32);
        u64 += double(u32);
        ex64 += double(ex32);
        s32 = u32 = ex32 = 0.f;
        fold = 0;
      }
    });
    s64 += double(s32);
    u64 += double(u32);
    ex64 += double(ex32);
    // This thread's error bound: the weights' own, and the FP32 additions'.
    const double total = s64 + u64;
    const double err = MASS_ERR * (total + ex64) * (1.0 + 0x1p-19) + 0x1p-19 * total + double(n) * 0x1p-120;
    MassPart m{s64, u64, err, n};
    auto merge = [](MassPart a, MassPart b) {
      return MassPart{a.kept + b.kept, a.unsure + b.unsure, a.err + b.err, a.n + b.n};
    };
#pragma unroll
    for (int o = 16; o; o >>= 1)
      m = merge(m, MassPart{shfl_xor(m.kept, o), shfl_xor(m.unsure, o), shfl_xor(m.err, o), shfl_xor(m.n, o)});
    if (lane_id() == 0) s.red.masses[warp_id()] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      MassPart b = s.red.masses[0];
      for (int w = 1; w < WARPS; ++w) b = merge(b, s.red.masses[w]);
      s.mass_part[parity()] = b;
    }
    exchange();
    if (int(threadIdx.x) < ranks) s.peers.masses[threadIdx.x] = *peer(&s.mass_part[parity() ^ 1], threadIdx.x);
    __syncthreads();
    MassPart t = s.peers.masses[0];
    for (int r = 1; r < ranks; ++r) t = merge(t, s.peers.masses[r]);
    __syncthreads();
    // FP64 additions of at most a few thousand partial sums: below 1e-12.
    const double all = t.kept + t.unsure;
    const double lo_ = t.kept - 1e-12 * t.kept - t.err;
    const double hi_ = all + 1e-12 * all + t.err;
    // The bounds' own FP64 roundings.
    return Interval{lo_ * (1.0 - 0x1p-40), hi_ * (1.0 + 0x1p-40)};
  }

  // Rank 0 tells every rank a block-uniform decision (written into each
  // rank's copy before the exchange, so no rank reads rank 0 afterwards).
  __device__ bool broadcast_verdict(bool v) {
    if (rank == 0 && int(threadIdx.x) < ranks) *peer(&s.verdict, threadIdx.x) = v ? 1 : 0;
    exchange();
    return s.verdict != 0;
  }

  // ---- top-p over a full row ----
  // The shortest prefix of the kept set K (valid, cut_k, min-p) in (value
  // desc, ID asc) order whose correctly rounded sum reaches top_p * fsum(K):
  // a radix selection over the order key whose buckets carry exact weight
  // sums, then the tie position inside the selected key. Returns the cut and
  // the prefix's rounded sum (the normalizer).
  __device__ Cut<Key> top_p_cut(Cut<Key> cut_k, double* normalizer) {
    Key prefix = 0, known = 0;
    u128 above = 0;
    uint32_t above_n = 0;
    double target = 0;
    int digit = 0, last_count = 0;
    for (int shift = KEY_BITS - 8; shift >= 0; shift -= 8) {
      u128* mass = s.u.mass[parity()];
      uint32_t* count = s.hist[parity()];
      for (int i = threadIdx.x; i < RADIX; i += THREADS) {
        mass[i] = 0;
        count[i] = 0;
      }
      __syncthreads();
      slice_pass([&](int g, const W* v, unsigned bits) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          int d = -1;
          u128 f = 0;
          if ((bits >> j) & 1u) {
            const Key k = order_key(v[j]);
            const int t = lo + 4 * g + j;
            if ((k & known) == prefix && cut_k.keeps(k, t)) {
              const double w = exp(x64(v[j]));
              if (w >= min_p && w > 0) {
                d = int((k >> shift) & 255);
                f = fx_of(w);
              }
            }
          }
          warp_bucket_add(mass, count, d, f);
        }
      });
      ES_TRACE(p.workspace, p.rows, row, rank, shift == KEY_BITS - 8 ? 10 : 11);
      exchange();
      // Thread i owns digit 255 - i: merged mass and count, scanned from the top.
      u128 m = 0;
      uint32_t c = 0;
      for (int r = 0; r < ranks; ++r) {
        m += peer(s.u.mass[parity() ^ 1], r)[255 - threadIdx.x];
        c += peer(s.hist[parity() ^ 1], r)[255 - threadIdx.x];
      }
      u128 m_total;
      uint32_t c_total;
      const u128 m_cum = block_scan(m, s.red.fxs, &m_total);
      const uint32_t c_cum = block_scan(c, s.red.uints, &c_total);
      if (shift == KEY_BITS - 8) {
        bool near;
        const double total = fx_round(m_total, c_total, &near);
        count_near_tie(near);
        target = top_p * total;
        if (target <= 1.0) {
          // The first kept token (the maximum, weight exactly 1) reaches it.
          *normalizer = 1.0;
          return Cut<Key>{1, order_key(maxv), argmax_id()};
        }
      }
      bool near = false;
      const bool reach = c > 0 && fx_reaches(above + m_cum, above_n + c_cum, target, &near);
      int first = block_all(reach ? int(threadIdx.x) : INT_MAX, [](int a, int b) { return a < b ? a : b; },
                            s.red.ints);
      if (first == INT_MAX)  // only if rounding slack hid the crossing: the last non-empty digit
        first = block_all(c > 0 ? int(threadIdx.x) : 0, [](int a, int b) { return a > b ? a : b; }, s.red.ints);
      count_near_tie(block_all(int(int(threadIdx.x) == first && near), [](int a, int b) { return a | b; }, s.red.ints) != 0);
      if (int(threadIdx.x) == first) {
        s.fxval = m_cum - m;
        s.ival[0] = 255 - first;
        s.ival[1] = int(c_cum - c);
        s.ival[2] = int(c);
      }
      __syncthreads();
      above += s.fxval;
      above_n += uint32_t(s.ival[1]);
      digit = s.ival[0];
      last_count = s.ival[2];
      prefix |= Key(digit) << shift;
      known |= Key(255) << shift;
      __syncthreads();
    }
    // The selected key's tokens are tied, with one weight w*: the boundary is
    // the j-th of them in ID order, j the smallest with fl(above + j w*) >= target.
    const W v_star = key_value(prefix);
    const u128 w_star = fx_of(exp(x64(v_star)));
    int lo_j = 1, hi_j = last_count;
    bool near = false;
    while (lo_j < hi_j) {
      const int mid = (lo_j + hi_j) / 2;
      bool nr;
      if (fx_reaches(above + w_star * u128(mid), above_n + mid, target, &nr)) hi_j = mid;
      else lo_j = mid + 1;
    }
    const int j = max(lo_j, 1);
    *normalizer = fx_round(above + w_star * u128(j), above_n + j, &near);
    count_near_tie(near);
    int before = 0, owner = -1;
    for (int r = 0; r < ranks && owner < 0; ++r) {
      const int c = int(peer(s.hist[parity() ^ 1], r)[digit]);
      if (before + c >= j) owner = r;
      else before += c;
    }
    int id = INT_MAX;
    if (owner == rank)
      id = nth_local(j - before, [&](W v, int t, Key k) {
        return k == prefix && cut_k.keeps(k, t) && exact_weight_kept(v);
      });
    id = cluster_min(owner == rank ? id : INT_MAX);
    return Cut<Key>{1, prefix, id};
  }

  // ---- draws ----
  // Certified FP32 argmax of x + G over the valid tokens that `kept` accepts
  // (and min-p keeps), except `excluded`; an FP64 rescore of every token
  // whose bound reaches the FP32 winner's lower bound when the certificate
  // fails (or of every token, with exact_only). Returns -1 if none is kept.
  // `cuts`: `kept` rejects tokens (a top-k or top-p cut is on), so it is
  // applied before the Philox words are made.
  template <class Kept> __device__ int draw(uint32_t sub, int excluded, Kept kept, bool cuts, bool exact_only) {
    // A kept token's score bounds the winner's from below: the maximum
    // (x = 0), unless it is excluded.
    const int greedy = argmax_id();
    if (threadIdx.x == 0) {
      float floor = -INFINITY;
      const int t = greedy != excluded ? greedy : INT_MAX;
      if (t != INT_MAX && valid_global(t)) {
        const W v = value_global(t);
        const float x = x32(v);
        if (kept(order_key(v), t) && weight_kept(v, x)) {
          const float g = noise32(addr.word(sub, uint32_t(t)));
          const float sc = __fadd_rn(x, g);
          floor = __fsub_rn(sc, 1.01f * SCORE_ERR * (1.f + fabsf(x) + fabsf(g)));
        }
      }
      s.floor_score = floor;
    }
    __syncthreads();
    const float floor = exact_only ? -INFINITY : s.floor_score;
    Pick best = no_pick();
    float skipped = -INFINITY;
    if (!exact_only) {
      // Screens, from cheap to exact, against bar = the best lower bound so
      // far (or the floor) less PRUNE_MARGIN. A token screened out has an
      // upper bound below the bar, so `skipped` takes the bar itself: below
      // the winner's lower bound by the margin, it never blocks the
      // certificate. The screens' own FP32 roundings (about 1e-5) are
      // covered by slacks of 1e-3 and 1e-4.
      //
      slice_pass([&](int g, const W* v, unsigned bits) {
        if (!bits) return;
        const float bar = fmaxf(floor, best.lo) - PRUNE_MARGIN;
        // 1. Value: x + NOISE_MAX + SCORE_ERR (1 + |x| + NOISE_MAX) < bar,
        //    i.e. (x <= 0) x < (bar - LIVE_OFFSET) / (1 - SCORE_ERR).
        const float x_live = __fsub_rn(__fmul_rn(__fsub_rn(bar, LIVE_OFFSET), 1.f + 2.f * SCORE_ERR), 1e-3f);
        float xs[4];
        unsigned live = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          xs[j] = x32(v[j]);
          if (((bits >> j) & 1u) && xs[j] >= x_live && (!cuts || kept(order_key(v[j]), lo + 4 * g + j)))
            live |= 1u << j;
        }
        if (live != bits) skipped = fmaxf(skipped, bar);
        if (!live) return;
        const Words r = addr.group(sub, uint32_t((lo >> 2) + g));
        // 2. Noise, integers only: G(w) <= (clz(~w) + 1) ln 2, since
        //    -log(u) >= 1 - u >= 2^-(clz(~w) + 1); first for the group (its
        //    largest live x with its largest bound), then per token.
        auto cheap_ub = [](float x, int l) {
          const float gn = __fmul_rn(float(l + 1), LN2_UP);
          return __fadd_rn(__fadd_rn(__fmul_rn(x, 1.f - SCORE_ERR), __fmul_rn(gn, 1.f + SCORE_ERR)), SCORE_ERR + 1e-4f);
        };
        int lz[4], lmax = 0;
        float xmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          lz[j] = __clz(~r.w[j]);
          if ((live >> j) & 1u) {
            lmax = max(lmax, lz[j]);
            xmax = fmaxf(xmax, xs[j]);
          }
        }
        if (cheap_ub(xmax, lmax) < bar) {
          skipped = fmaxf(skipped, bar);
          return;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (!((live >> j) & 1u)) continue;
          const float x = xs[j];
          if (cheap_ub(x, lz[j]) < bar) {
            skipped = fmaxf(skipped, bar);
            continue;
          }
          // 3. The rare token that might still win: exact membership, a
          //    tighter noise bound, then the certified FP32 score.
          const int t = lo + 4 * g + j;
          if (t == excluded || (!cuts && !kept(order_key(v[j]), t)) || !weight_kept(v[j], x)) continue;
          const float gu = noise_upper(r.w[j]);
          const float ub = x + gu + SCORE_ERR * (1.f + fabsf(x) + fabsf(gu));
          if (ub < fmaxf(floor, best.lo) - PRUNE_MARGIN) {
            skipped = fmaxf(skipped, ub);
            continue;
          }
          const float G = noise32(r.w[j]);
          const float sc = __fadd_rn(x, G);
          const float err = SCORE_ERR * (1.f + fabsf(x) + fabsf(G));
          best = pick_of(best, Pick{sc, sc - err, sc + err, -INFINITY, t});
        }
      });
    }
    ES_TRACE(p.workspace, p.rows, row, rank, 13);
    best.others = fmaxf(best.others, skipped);
    best = block_all(best, [](Pick a, Pick b) { return pick_of(a, b); }, s.red.picks);
    if (threadIdx.x == 0) s.pick[parity()] = best;
    exchange();
    if (int(threadIdx.x) < ranks) s.peers.picks[threadIdx.x] = *peer(&s.pick[parity() ^ 1], threadIdx.x);
    __syncthreads();
    Pick top = no_pick();
    for (int r = 0; r < ranks; ++r) top = pick_of(top, s.peers.picks[r]);
    __syncthreads();
    if (!exact_only) {
      if (top.id == INT_MAX) return -1;
      if (top.lo > top.others) return top.id;
      count_fallback();
    }
    ES_TRACE(p.workspace, p.rows, row, rank, 14);
    // FP64: every kept token whose upper bound reaches the threshold.
    const float threshold = exact_only ? -INFINITY : top.lo;
    Best b = no_best();
    for (int g = threadIdx.x; g < groups; g += THREADS) {
      W v[4];
      const unsigned bits = group(g, v);
      unsigned live = 0;
      float xs[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = lo + 4 * g + j;
        xs[j] = 0.f;
        if (!((bits >> j) & 1u) || t == excluded) continue;
        const float x = x32(v[j]);
        if (!kept(order_key(v[j]), t) || !weight_kept(v[j], x)) continue;
        xs[j] = x;
        if (exact_only || x + NOISE_MAX + SCORE_ERR * (1.f + fabsf(x) + NOISE_MAX) >= threshold) live |= 1u << j;
      }
      if (!live) continue;
      const Words r = addr.group(sub, uint32_t((lo >> 2) + g));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (!((live >> j) & 1u)) continue;
        if (!exact_only) {
          const float gu = noise_upper(r.w[j]);
          if (xs[j] + gu + SCORE_ERR * (1.f + fabsf(xs[j]) + fabsf(gu)) < threshold) continue;
        }
        b = best_of(b, Best{x64(v[j]) + noise64(r.w[j]), lo + 4 * g + j});
      }
    }
    return cluster_best(b);
  }

  // The residual draw max(p - q, 0) of a full-q draft row over the kept set,
  // in FP64 exactly as the oracle forms it: p = w / Sp, q = wq / Sq.
  // draw() for kernels compiled without the list paths: every group of four
  // tokens is screened whole before its tokens are, and the Philox words come
  // from the row's precomputed rounds. Same result as draw().
  template <class Kept> __device__ int draw_groups(uint32_t sub, int excluded, Kept kept, bool cuts, bool exact_only) {
    // A kept token's score bounds the winner's from below: the maximum
    // (x = 0), unless it is excluded.
    const int greedy = argmax_id();
    if (threadIdx.x == 0) {
      float floor = -INFINITY;
      const int t = greedy != excluded ? greedy : INT_MAX;
      if (t != INT_MAX && valid_global(t)) {
        const W v = value_global(t);
        const float x = x32(v);
        if (kept(order_key(v), t) && weight_kept(v, x)) {
          const float g = noise32(addr.word(sub, uint32_t(t)));
          const float sc = __fadd_rn(x, g);
          floor = __fsub_rn(sc, 1.01f * SCORE_ERR * (1.f + fabsf(x) + fabsf(g)));
        }
      }
      s.floor_score = floor;
    }
    __syncthreads();
    const float floor = exact_only ? -INFINITY : s.floor_score;
    Pick best = no_pick();
    float skipped = -INFINITY;
    if (!exact_only) {
      // Screens, from cheap to exact, against bar = the best lower bound so
      // far (or the floor) less PRUNE_MARGIN. A token screened out has an
      // upper bound below the bar, so `skipped` takes the bar itself: below
      // the winner's lower bound by the margin, it never blocks the
      // certificate. The screens' own FP32 roundings (about 1e-5) are
      // covered by slacks of 1e-3 and 1e-4.
      //
      // `bar` follows best.lo (it only rises); x_live is the value screen's
      // threshold for it: x + NOISE_MAX + SCORE_ERR (1 + |x| + NOISE_MAX) < bar,
      // i.e. (x <= 0) x < (bar - LIVE_OFFSET) / (1 - SCORE_ERR).
      float bar = 0.f, x_live = 0.f;
      auto raise_bar = [&]() {
        bar = fmaxf(floor, best.lo) - PRUNE_MARGIN;
        x_live = __fsub_rn(__fmul_rn(__fsub_rn(bar, LIVE_OFFSET), 1.f + 2.f * SCORE_ERR), 1e-3f);
      };
      raise_bar();
      // Noise, integers only: G(w) <= (clz(~w) + 1) ln 2, since
      // -log(u) >= 1 - u >= 2^-(clz(~w) + 1); the bound rises with x and with
      // the word.
      auto cheap_ub = [](float x, int l) {
        const float gn = __fmul_rn(float(l + 1), LN2_UP);
        return __fadd_rn(__fadd_rn(__fmul_rn(x, 1.f - SCORE_ERR), __fmul_rn(gn, 1.f + SCORE_ERR)), SCORE_ERR + 1e-4f);
      };
      const PhiloxRow ph = addr.row(sub);
      slice_pass([&](int g, const W* v, unsigned bits) {
        if (!bits) return;
        float xs[4];
        unsigned live = 0;
        Words r;
        if (!cuts) {
          // Every valid token is a candidate: the group is screened whole,
          // with one x (x32 is monotone, so the largest valid value has the
          // largest x) and one noise bound (the largest of the four words
          // has the largest).
          W vm = W(-INFINITY);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if ((bits >> j) & 1u) vm = v[j] > vm ? v[j] : vm;
          const float xg = x32(vm);
          if (xg < x_live) {
            skipped = fmaxf(skipped, bar);
            return;
          }
          r = ph.group(uint32_t((lo >> 2) + g));
          const uint32_t wm = max(max(r.w[0], r.w[1]), max(r.w[2], r.w[3]));
          if (cheap_ub(xg, __clz(~wm)) < bar) {
            skipped = fmaxf(skipped, bar);
            return;
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            xs[j] = x32(v[j]);
            if (((bits >> j) & 1u) && xs[j] >= x_live) live |= 1u << j;
          }
        } else {
          // A cut rejects most tokens: membership first, so that the
          // rejected ones need no Philox words.
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            xs[j] = x32(v[j]);
            if (((bits >> j) & 1u) && xs[j] >= x_live && kept(order_key(v[j]), lo + 4 * g + j)) live |= 1u << j;
          }
          if (live != bits) skipped = fmaxf(skipped, bar);
          if (!live) return;
          r = ph.group(uint32_t((lo >> 2) + g));
          int lmax = 0;
          float xmax = -INFINITY;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if ((live >> j) & 1u) {
              lmax = max(lmax, int(__clz(~r.w[j])));
              xmax = fmaxf(xmax, xs[j]);
            }
          if (cheap_ub(xmax, lmax) < bar) {
            skipped = fmaxf(skipped, bar);
            return;
          }
        }
        if (live != bits) skipped = fmaxf(skipped, bar);
        // The per-token screens of the live tokens.
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (!((live >> j) & 1u)) continue;
          const float x = xs[j];
          if (cheap_ub(x, __clz(~r.w[j])) < bar) {
            skipped = fmaxf(skipped, bar);
            continue;
          }
          // The rare token that might still win: exact membership, a
          // tighter noise bound, then the certified FP32 score.
          const int t = lo + 4 * g + j;
          if (t == excluded || (!cuts && !kept(order_key(v[j]), t)) || !weight_kept(v[j], x)) continue;
          const float gu = noise_upper(r.w[j]);
          const float ub = x + gu + SCORE_ERR * (1.f + fabsf(x) + fabsf(gu));
          if (ub < bar) {
            skipped = fmaxf(skipped, ub);
            continue;
          }
          const float G = noise32(r.w[j]);
          const float sc = __fadd_rn(x, G);
          const float err = SCORE_ERR * (1.f + fabsf(x) + fabsf(G));
          best = pick_of(best, Pick{sc, sc - err, sc + err, -INFINITY, t});
          raise_bar();
        }
      });
    }
    ES_TRACE(p.workspace, p.rows, row, rank, 13);
    best.others = fmaxf(best.others, skipped);
    best = block_all(best, [](Pick a, Pick b) { return pick_of(a, b); }, s.red.picks);
    if (threadIdx.x == 0) s.pick[parity()] = best;
    exchange();
    if (int(threadIdx.x) < ranks) s.peers.picks[threadIdx.x] = *peer(&s.pick[parity() ^ 1], threadIdx.x);
    __syncthreads();
    Pick top = no_pick();
    for (int r = 0; r < ranks; ++r) top = pick_of(top, s.peers.picks[r]);
    __syncthreads();
    if (!exact_only) {
      if (top.id == INT_MAX) return -1;
      if (top.lo > top.others) return top.id;
      count_fallback();
    }
    ES_TRACE(p.workspace, p.rows, row, rank, 14);
    // FP64: every kept token whose upper bound reaches the threshold.
    const float threshold = exact_only ? -INFINITY : top.lo;
    Best b = no_best();
    for (int g = threadIdx.x; g < groups; g += THREADS) {
      W v[4];
      const unsigned bits = group(g, v);
      unsigned live = 0;
      float xs[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = lo + 4 * g + j;
        xs[j] = 0.f;
        if (!((bits >> j) & 1u) || t == excluded) continue;
        const float x = x32(v[j]);
        if (!kept(order_key(v[j]), t) || !weight_kept(v[j], x)) continue;
        xs[j] = x;
        if (exact_only || x + NOISE_MAX + SCORE_ERR * (1.f + fabsf(x) + NOISE_MAX) >= threshold) live |= 1u << j;
      }
      if (!live) continue;
      const Words r = addr.group(sub, uint32_t((lo >> 2) + g));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (!((live >> j) & 1u)) continue;
        if (!exact_only) {
          const float gu = noise_upper(r.w[j]);
          if (xs[j] + gu + SCORE_ERR * (1.f + fabsf(xs[j]) + fabsf(gu)) < threshold) continue;
        }
        b = best_of(b, Best{x64(v[j]) + noise64(r.w[j]), lo + 4 * g + j});
      }
    }
    return cluster_best(b);
  }

  // The residual draw max(p - q, 0) of a full-q draft row over the kept set,
  // in FP64 exactly as the oracle forms it: p = w / Sp, q = wq / Sq.
  template <class Kept> __device__ int draw_residual_q(Kept kept, double sp, double sq) {
    Best b = no_best();
    for (int g = threadIdx.x; g < groups; g += THREADS) {
      W v[4];
      const unsigned bits = group(g, v);
      bool any = false;
      double r4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        r4[j] = 0;
        const int t = lo + 4 * g + j;
        if (!((bits >> j) & 1u) || !kept(order_key(v[j]), t)) continue;
        const double w = exp(x64(v[j]));
        if (!(w >= min_p && w > 0)) continue;
        const W y = q_value(t);
        const double q = y > W(-INFINITY) ? exp(double(y) - double(all.qmax)) / sq : 0.0;
        r4[j] = fmax(w / sp - q, 0.0);
        any |= r4[j] > 0;
      }
      if (!any) continue;
      const Words r = addr.group(2, uint32_t((lo >> 2) + g));
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (r4[j] > 0) b = best_of(b, Best{log(r4[j]) + noise64(r.w[j]), lo + 4 * g + j});
    }
    return cluster_best(b);
  }
};

}  // namespace es
