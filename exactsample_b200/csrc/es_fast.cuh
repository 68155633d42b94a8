// Warp-level steps of the common list row: a top-k of at most FAST_KEEP
// tokens whose candidates fit one warp (FAST_CAND). They are the same steps
// as the block-level list path in es_rows.cuh / es_kernel.cuh (window of
// tile maxima, gather of the window's tokens, sort, FP64 finish), written so
// that one warp runs each of them without block barriers.
//
// Why warp-level and out of line: on a B200 the first execution of this
// code on an SM waits on instruction fetch for most of its time (the sort
// and FP64 finish of a C2a row take about 12 us cold against 3.4 us warm, by
// %globaltimer traces), and every row reaches it at the same moment, right
// after its statistics pass. The row kernel therefore launches one extra
// warp per block that calls these same functions (__noinline__: one copy of
// the code) on dummy data in shared memory while the row streams; by the
// time the row needs them their instructions are cached. Dry calls write
// only the dummy buffers they are given.
//
// Exactness is that of the block path: the window is a bound on the n-th
// largest valid value, the gather takes every valid token at or above the
// window's lower edge (ties at the n-th value included), the order is
// (value desc, ID asc), and the finish uses the oracle's FP64 formulas with
// fixed-point sums (python/exactsample/reference.py:55-104 distribution(),
// :125-176 sampling and the ratio test; reference fused_rows<LIST>,
// csrc/verify/fused.cuh:1250-1444).
#pragma once
#include "es_layout.cuh"

namespace es {

__device__ __forceinline__ float widen(float v) { return v; }
__device__ __forceinline__ double widen(double v) { return v; }
__device__ __forceinline__ float widen(__half v) { return __half2float(v); }
__device__ __forceinline__ float widen(__nv_bfloat16 v) { return __bfloat162float(v); }

// Four consecutive values of a shared-memory slice.
__device__ __forceinline__ void load4(const float* s, float v[4]) {
  const float4 x = *reinterpret_cast<const float4*>(s);
  v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
}
__device__ __forceinline__ void load4(const double* s, double v[4]) {
  const double2 x = reinterpret_cast<const double2*>(s)[0], y = reinterpret_cast<const double2*>(s)[1];
  v[0] = x.x; v[1] = x.y; v[2] = y.x; v[3] = y.y;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* s, float v[4]) {
  const uint2 x = *reinterpret_cast<const uint2*>(s);
  v[0] = __uint_as_float(x.x << 16); v[1] = __uint_as_float(x.x & 0xffff0000u);
  v[2] = __uint_as_float(x.y << 16); v[3] = __uint_as_float(x.y & 0xffff0000u);
}
__device__ __forceinline__ void load4(const __half* s, float v[4]) {
  const uint2 x = *reinterpret_cast<const uint2*>(s);
  v[0] = __half2float(__ushort_as_half(uint16_t(x.x))); v[1] = __half2float(__ushort_as_half(uint16_t(x.x >> 16)));
  v[2] = __half2float(__ushort_as_half(uint16_t(x.y))); v[3] = __half2float(__ushort_as_half(uint16_t(x.y >> 16)));
}

// Four consecutive values from global memory (16-byte aligned rows).
__device__ __forceinline__ void load4_global(const float* g, float v[4]) {
  const float4 x = __ldg(reinterpret_cast<const float4*>(g));
  v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
}
__device__ __forceinline__ void load4_global(const double* g, double v[4]) {
  const double2 x = __ldg(reinterpret_cast<const double2*>(g)), y = __ldg(reinterpret_cast<const double2*>(g) + 1);
  v[0] = x.x; v[1] = x.y; v[2] = y.x; v[3] = y.y;
}
template <class H> __device__ __forceinline__ void load4_global(const H* g, float v[4]) {
  const uint2 x = __ldg(reinterpret_cast<const uint2*>(g));
  load4(reinterpret_cast<const H*>(&x), v);
}

template <class W> struct KeyOf;
template <> struct KeyOf<float> { using type = uint32_t; };
template <> struct KeyOf<double> { using type = uint64_t; };

// Tile maxima are histogrammed during the statistics pass in absolute bins
// of 0.5 logit, bin(v) = floor(2 v) + ABS_ZERO clamped to [0, ABS_BINS):
// every rank bins alike without knowing the row maximum, so the histogram
// travels with the statistics in one cluster exchange. Values beyond +-256
// share the end bins (still monotone, so still a valid bound).
constexpr int ABS_BINS = 1024;
constexpr int ABS_ZERO = 512;
constexpr int WIN_BINS = 128;  // bins a rank publishes, from its own top bin down
constexpr int FAST_CAND = 64;  // candidates the warp sort takes (two per lane)
constexpr int FAST_KEEP = 32;  // kept tokens the warp finish takes (one per lane)
static_assert(WIN_BINS == PHASE_BINS, "a per-phase record carries one cluster window");

__device__ __forceinline__ int abs_bin(float v) {
  const float b = fminf(fmaxf(floorf(__fmul_rn(v, 2.f)), -float(ABS_ZERO)), float(ABS_BINS - ABS_ZERO - 1));
  return int(b) + ABS_ZERO;  // NaN lands in bin 0 (fmaxf returns the other operand)
}
__device__ __forceinline__ int abs_bin(double v) {
  const double b = fmin(fmax(floor(v * 2.0), -double(ABS_ZERO)), double(ABS_BINS - ABS_ZERO - 1));
  return int(b) + ABS_ZERO;
}

// The correctly rounded (nearest, ties to even) double of s units of
// 2^-FX_SHIFT, by normalising the 128-bit sum and letting the hardware round
// its top 64 bits with a sticky bit for everything below them; the scale
// is an exact power of two.
__device__ __forceinline__ double fx_round_rn(u128 s) {
  if (s == 0) return 0.0;
  const uint64_t hi = uint64_t(s >> 64), lo = uint64_t(s);
  const int lz = hi ? __clzll(hi) : 64 + __clzll(lo);
  const u128 t = s << lz;
  const uint64_t top = uint64_t(t >> 64) | (uint64_t(t) != 0 ? 1ull : 0ull);
  const double d = __ull2double_rn(top);
  // s = t * 2^-lz and t ~ top * 2^64, so s * 2^-FX_SHIFT ~ top * 2^(64 - lz - FX_SHIFT),
  // with 64 - lz - FX_SHIFT in [-163, -36]: a normal power of two.
  const int e = 64 - lz - FX_SHIFT;
  return d * __longlong_as_double(int64_t(e + 1023) << 52);
}

// The window: counts[j] is the number of tiles whose maximum lies in bin
// top - j (j < WIN_BINS). Returns the smallest j at which the cumulative
// count from the top reaches n (the window's lowest bin is top - j), or -1.
static __device__ __noinline__ int window_warp(const uint32_t* counts, int n) {
  constexpr unsigned ALL = 0xffffffffu;
  static_assert(WIN_BINS == 4 * 32, "four bins per lane");
  const int lane = lane_id();
  uint32_t c[4], sum = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    c[k] = counts[4 * lane + k];
    sum += c[k];
  }
  uint32_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(ALL, incl, o);
    if (lane >= o) incl += y;
  }
  unsigned found = UINT_MAX;
  if (incl >= uint32_t(n) && incl - sum < uint32_t(n)) {
    uint32_t cum = incl - sum;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      cum += c[k];
      if (cum >= uint32_t(n) && found == UINT_MAX) found = unsigned(4 * lane + k);
    }
  }
  found = __reduce_min_sync(ALL, found);
  return found == UINT_MAX ? -1 : int(found);
}

// Where a rank's slice lives: element i of the slice at values[i * vstride]
// (shared memory for resident rows, global memory otherwise), mask word w
// at mask[w * mstride] (NULL: no mask), n tokens, global ID of element 0 lo.
template <class T> struct SliceRef {
  const T* values;
  int64_t vstride;
  const int32_t* mask;
  int64_t mstride;
  int n, lo;
};

// Appends every valid token of tiles [t0, t1) whose absolute bin is at least
// `bin` to (keys, ids) from slots reserved on *counter (one atomic per batch
// of tiles; slots at or past cap are counted but not written). Only tiles
// whose maximum reaches the bin are read: the warp lists them first (from
// the tile maxima in shared memory), then loads BATCH of them at a time, all
// in flight together. Returns the number of tokens this warp appended (the
// same in every lane).
template <class T, class W>
__device__ __noinline__ int gather_warp(const SliceRef<T>& src, const W* tmax, int t0, int t1, int bin,
                                        uint64_t* keys, int32_t* ids, int* counter, int cap) {
  constexpr unsigned ALL = 0xffffffffu;
  constexpr int BATCH = 8;
  const int lane = lane_id();
  int mine = 0;
  int base = t0;
  unsigned pending = 0;  // hit tiles of the 32 from `base` not yet read
  while (true) {
    // The next BATCH listed tiles (warp-uniform).
    int tt[BATCH];
    int n = 0;
    while (n < BATCH) {
      if (!pending) {
        if (base >= t1) break;
        const int t = base + lane;
        bool hit = false;
        if (t < t1) {
          const W m = tmax[t];
          hit = m > W(-INFINITY) && abs_bin(m) >= bin;
        }
        pending = __ballot_sync(ALL, hit);
        if (!pending) {
          base += 32;
          continue;
        }
      }
      tt[n++] = base + __ffs(pending) - 1;
      pending &= pending - 1;
      if (!pending) base += 32;
    }
    if (n == 0) break;
    W v[BATCH];
#pragma unroll
    for (int b = 0; b < BATCH; ++b) {
      v[b] = W(-INFINITY);
      if (b < n) {
        const int i = 32 * tt[b] + lane;
        if (i < src.n) {
          const bool allowed =
              src.mask == nullptr || ((uint32_t(src.mask[int64_t(i >> 5) * src.mstride]) >> (i & 31)) & 1u);
          if (allowed) v[b] = widen(src.values[int64_t(i) * src.vstride]);
        }
      }
    }
    unsigned take[BATCH];
    int total = 0;
#pragma unroll
    for (int b = 0; b < BATCH; ++b) {
      take[b] = __ballot_sync(ALL, b < n && v[b] > W(-INFINITY) && abs_bin(v[b]) >= bin);
      total += __popc(take[b]);
    }
    if (total == 0) continue;
    int slot = 0;
    if (lane == 0) slot = atomicAdd(counter, total);
    slot = __shfl_sync(ALL, slot, 0);
#pragma unroll
    for (int b = 0; b < BATCH; ++b) {
      if ((take[b] >> lane) & 1u) {
        const int at_ = slot + __popc(take[b] & ((1u << lane) - 1u));
        if (at_ < cap) {
          keys[at_] = uint64_t(order_key(v[b]));
          ids[at_] = src.lo + 32 * tt[b] + lane;
        }
      }
      slot += __popc(take[b]);
    }
    mine += total;
  }
  return mine;
}

// One list row's finish by one warp.
struct ListIn {
  const uint64_t* key;  // m candidates (order keys and token IDs), any order
  const int32_t* id;
  int m;                // <= FAST_CAND
  int n_keep;           // <= FAST_KEEP: the first n_keep in (key desc, ID asc) order are kept
  double maxv, temperature, min_p, top_p;
  Address addr;
  int verify;           // ratio test of draft_id (one-hot draft), residual on rejection
  int draft_id;
  uint32_t* near_ties;  // diagnostics counter (NULL: not counted)
};
struct ListOut {
  int32_t sample, accept, residual;
};

// (key desc, ID asc): whether (ka, ia) comes first.
__device__ __forceinline__ bool precedes(uint64_t ka, int32_t ia, uint64_t kb, int32_t ib) {
  return ka > kb || (ka == kb && ia < ib);
}

// Bitonic sort into (key desc, ID asc) order of N = 32 or 64 entries held
// N / 32 per lane (entry e = lane + 32 h), fully unrolled. For 32-bit keys
// the pair is one 64-bit composite, key above (2^32 - 1 - ID), so one
// comparison orders it; 64-bit keys compare the pair. Empty entries are
// (0, INT_MAX) and sort last.
template <int N, bool WIDE> __device__ __forceinline__ void warp_sort(uint64_t key[2], int32_t id[2]) {
  constexpr unsigned ALL = 0xffffffffu;
  constexpr int H = N / 32;
  const int lane = lane_id();
  uint64_t c[2];
  if constexpr (!WIDE) {
#pragma unroll
    for (int h = 0; h < H; ++h) c[h] = (key[h] << 32) | uint64_t(0xffffffffu - uint32_t(id[h]));
  }
#pragma unroll
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j == 32) {  // k == 64: entries lane and lane + 32, the whole sequence descending
        if constexpr (!WIDE) {
          if (c[1] > c[0]) {
            const uint64_t t = c[0]; c[0] = c[1]; c[1] = t;
          }
        } else if (precedes(key[1], id[1], key[0], id[0])) {
          const uint64_t tk = key[0]; key[0] = key[1]; key[1] = tk;
          const int32_t ti = id[0]; id[0] = id[1]; id[1] = ti;
        }
        continue;
      }
#pragma unroll
      for (int h = 0; h < H; ++h) {
        const int e = lane + 32 * h;
        const bool first_here = ((e & j) == 0) == ((e & k) == 0);  // this entry takes the earlier of the pair
        if constexpr (!WIDE) {
          const uint64_t o = __shfl_xor_sync(ALL, c[h], j);
          c[h] = first_here ? (o > c[h] ? o : c[h]) : (o > c[h] ? c[h] : o);
        } else {
          const uint64_t ok = __shfl_xor_sync(ALL, key[h], j);
          const int32_t oi = __shfl_xor_sync(ALL, id[h], j);
          if (precedes(key[h], id[h], ok, oi) != first_here) {
            key[h] = ok;
            id[h] = oi;
          }
        }
      }
    }
  }
  if constexpr (!WIDE) {
#pragma unroll
    for (int h = 0; h < H; ++h) {
      key[h] = c[h] >> 32;
      id[h] = int32_t(0xffffffffu - uint32_t(c[h]));
    }
  }
}

// Argmax of score over the lanes with `in` (lowest ID on equal scores, as
// best_of), by reductions over the score's order key; -1 if no lane is in.
__device__ __forceinline__ int warp_argmax(double score, int32_t id, bool in) {
  constexpr unsigned ALL = 0xffffffffu;
  if (!__ballot_sync(ALL, in)) return -1;
  const uint64_t k = in ? order_key(score) : 0;
  const uint32_t khi = uint32_t(k >> 32);
  const uint32_t mhi = __reduce_max_sync(ALL, khi);
  const uint32_t mlo = __reduce_max_sync(ALL, khi == mhi ? uint32_t(k) : 0u);
  const bool top = in && khi == mhi && uint32_t(k) == mlo;
  return int(__reduce_min_sync(ALL, top ? uint32_t(id) : UINT_MAX));
}

// Sorts the candidates, keeps the first n_keep, applies min-p and top-p with
// exact sums, and draws (or runs the ratio test and the residual draw) with
// the oracle's FP64 formulas. Every lane returns the same result.
template <class W> __device__ __noinline__ ListOut finish_warp(const ListIn& in) {
  using Key = typename KeyOf<W>::type;
  constexpr unsigned ALL = 0xffffffffu;
  const int i = lane_id();
  uint64_t key[2];
  int32_t id[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int e = i + 32 * h;
    key[h] = e < in.m ? in.key[e] : 0;
    id[h] = e < in.m ? in.id[e] : INT_MAX;
  }
  constexpr bool WIDE = sizeof(W) == 8;
  if (in.m > 32) warp_sort<64, WIDE>(key, id);
  else warp_sort<32, WIDE>(key, id);
  // Lane i holds the i-th token of the order; the first n_keep are kept.
  const bool kept = i < in.n_keep;
  const int tok = kept ? id[0] : INT_MAX;
  // The noise of this row's one draw over the list (substream 2 for a ratio
  // test's residual, else 0) does not depend on the weights.
  const uint32_t sub = in.verify ? 2u : 0u;
  const double noise = kept ? noise64(in.addr.word(sub, uint32_t(tok))) : 0.0;
  double w = 0;
  bool ok = false;
  if (kept) {
    w = exp((double(key_value(Key(key[0]))) - in.maxv) / in.temperature);
    ok = w >= in.min_p && w > 0;
  }
  // min-p and positivity remove a suffix of the order.
  const unsigned out = __ballot_sync(ALL, kept && !ok);
  const int n1 = out ? min(in.n_keep, __ffs(out) - 1) : in.n_keep;
  // Inclusive prefix sums of the exact weights; lane i's prefix holds i + 1 terms.
  u128 prefix = i < n1 ? fx_of(w) : u128(0);
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t lo = __shfl_up_sync(ALL, uint64_t(prefix), o);
    const uint64_t hi = __shfl_up_sync(ALL, uint64_t(prefix >> 64), o);
    if (i >= o) prefix += (u128(hi) << 64) | lo;
  }
  // Every lane rounds its own prefix; the true prefix lies within
  // [prefix, prefix + i + 1) units, so a rounding that differs at the two
  // ends is a near tie (counted, as by the block path).
  const double rounded = i < n1 ? fx_round_rn(prefix) : 0.0;
  const bool near = i < n1 && fx_round_rn(prefix + u128(uint32_t(i + 1))) != rounded;
  const double total = __shfl_sync(ALL, rounded, n1 - 1);
  bool near_used = __shfl_sync(ALL, near, n1 - 1);
  int n2 = n1;
  double denominator = total;
  if (in.top_p < 1) {
    // The shortest prefix whose rounded sum reaches top_p * total (the
    // first token's weight is exactly 1), as fx_reaches decides it.
    const double target = in.top_p * total;
    if (target <= 1.0) {
      n2 = 1;
    } else {
      const unsigned hits = __ballot_sync(ALL, i < n1 && rounded >= target);
      n2 = hits ? __ffs(hits) : n1;
    }
    denominator = __shfl_sync(ALL, rounded, n2 - 1);
    near_used |= __shfl_sync(ALL, near, n2 - 1);
  }
  if (near_used && i == 0 && in.near_ties != nullptr) atomicAdd(in.near_ties, 1u);
  const double prob = i < n2 ? w / denominator : 0.0;
  ListOut r{-1, 0, -1};
  if (!in.verify) {
    r.sample = warp_argmax(prob > 0 ? log(prob) + noise : 0.0, tok, i < n2 && prob > 0);
    return r;
  }
  // Ratio test against a one-hot draft: u < min(1, p(draft) / 1).
  const unsigned at_draft = __ballot_sync(ALL, i < n2 && tok == in.draft_id);
  const double p_draft = __shfl_sync(ALL, prob, at_draft ? __ffs(at_draft) - 1 : 0);
  const double px = at_draft ? p_draft : 0.0;
  r.accept = uniform64(in.addr.word(1, 0)) < fmin(1.0, px);
  if (r.accept) return r;
  // The residual max(p - q, 0) of a one-hot draft: p without the draft token.
  const bool live = i < n2 && tok != in.draft_id && prob > 0;
  r.residual = warp_argmax(live ? log(prob) + noise : 0.0, tok, live);
  return r;
}

}  // namespace es
