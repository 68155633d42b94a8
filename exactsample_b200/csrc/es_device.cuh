// Device building blocks of the B200 row kernels: the counter-based RNG, the
// Gumbel noise in FP32 (with certified bounds) and FP64, order-preserving
// keys, exact fixed-point sums, certified argmax records, and the sm_100
// primitives (TMA bulk copies with mbarriers, cluster shared memory,
// programmatic dependent launch).
//
// Everything here is compiled with --fmad=false: the FP32 error bounds below
// assume every multiply and add rounds separately.
#pragma once
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "exactsample_b200.h"

namespace es {
namespace cg = cooperative_groups;
typedef unsigned __int128 u128;

constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

// ---------------------------------------------------------------------------
// Philox4x32-10 (Random123), the v1 address of the reference's RNG contract
// (include/exactsample/philox.h:14-34, docs/rng.md): key = (seed lo, seed hi),
// counter = (stream, position, substream, token / 4), lane = token % 4.
struct Words { uint32_t w[4]; };

__device__ __forceinline__ Words philox(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                        uint32_t k1) {
#pragma unroll
  for (int round = 0; round < 10; ++round) {
    const uint32_t lo0 = c0 * 0xD2511F53u, hi0 = __umulhi(c0, 0xD2511F53u);
    const uint32_t lo1 = c2 * 0xCD9E8D57u, hi1 = __umulhi(c2, 0xCD9E8D57u);
    c0 = hi1 ^ c1 ^ k0;
    c1 = lo1;
    c2 = hi0 ^ c3 ^ k1;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return Words{{c0, c1, c2, c3}};
}

// The words of every group of one row and substream. Only the counter's
// last word (the group) varies, and it enters round 1 by one XOR into the
// third word; round 2's first product does not depend on it. So round 1 and
// half of round 2 are computed once: with a2 = round 1's third word before
// the XOR, b0 = the XOR terms of round 2's first word, b2 and b3 = round 2's
// third and fourth words, and (k0, k1) = round 3's key, a group's words are
// round 2's remaining product and 8 full rounds (the same 10-round
// Philox4x32 as philox()).
constexpr uint32_t PHILOX_M0 = 0xD2511F53u, PHILOX_M1 = 0xCD9E8D57u;
constexpr uint32_t PHILOX_W0 = 0x9E3779B9u, PHILOX_W1 = 0xBB67AE85u;
struct PhiloxRow {
  uint32_t a2, b0, b2, b3, k0, k1;
  __device__ __forceinline__ Words group(uint32_t g) const {
    const uint32_t x = a2 ^ g;
    uint32_t c0 = __umulhi(x, PHILOX_M1) ^ b0, c1 = x * PHILOX_M1, c2 = b2, c3 = b3, key0 = k0, key1 = k1;
#pragma unroll
    for (int round = 2; round < 10; ++round) {
      const uint32_t lo0 = c0 * PHILOX_M0, hi0 = __umulhi(c0, PHILOX_M0);
      const uint32_t lo1 = c2 * PHILOX_M1, hi1 = __umulhi(c2, PHILOX_M1);
      c0 = hi1 ^ c1 ^ key0;
      c1 = lo1;
      c2 = hi0 ^ c3 ^ key1;
      c3 = lo0;
      key0 += PHILOX_W0;
      key1 += PHILOX_W1;
    }
    return Words{{c0, c1, c2, c3}};
  }
};

// One request row's RNG address without the substream and token.
struct Address {
  uint32_t stream, position, k0, k1;
  __device__ __forceinline__ Words group(uint32_t substream, uint32_t group) const {
    return philox(stream, position, substream, group, k0, k1);
  }
  __device__ __forceinline__ uint32_t word(uint32_t substream, uint32_t token) const {
    return group(substream, token >> 2).w[token & 3];
  }
  // Counter (stream, position, substream, g) for every group g: rounds 1
  // and 2 as far as they do not depend on g (PhiloxRow).
  __device__ __forceinline__ PhiloxRow row(uint32_t substream) const {
    const uint32_t a0 = __umulhi(substream, PHILOX_M1) ^ position ^ k0;  // round 1's first word
    const uint32_t a1 = substream * PHILOX_M1;                            // its second
    const uint32_t a3 = stream * PHILOX_M0;                               // its fourth
    const uint32_t k0b = k0 + PHILOX_W0, k1b = k1 + PHILOX_W1;            // round 2's key
    PhiloxRow r;
    r.a2 = __umulhi(stream, PHILOX_M0) ^ k1;
    r.b0 = a1 ^ k0b;
    r.b2 = __umulhi(a0, PHILOX_M0) ^ a3 ^ k1b;
    r.b3 = a0 * PHILOX_M0;
    r.k0 = k0b + PHILOX_W0;
    r.k1 = k1b + PHILOX_W1;
    return r;
  }
};

// u = (w + 0.5) / 2^32 in FP64, exact (docs/rng.md).
__device__ __forceinline__ double uniform64(uint32_t w) { return (double(w) + 0.5) * 0x1p-32; }

// The oracle's noise in FP64: -log(-log(u)) (reference rng.py:64-65).
__device__ __forceinline__ double noise64(uint32_t w) { return -log(-log(uniform64(w))); }

// FP32 noise G(w) = -log(-log u). -log(u) is formed from u below 1/2 and from
// log1p(-(1 - u)) above, with 1 - u = (~w + 0.5) / 2^32 exact in the word,
// so the large-noise tail keeps its resolution. Bound (checked for all 2^32
// words by tests/test_noise_bounds.py on the GPU):
//   |noise32(w) - G(w)| <= NOISE_ERR * (1 + |G(w)|).
constexpr float NOISE_ERR = 1.0e-6f;
// Every G(w) is at most NOISE_MAX (the largest is 22.8739, at w = 2^32 - 1).
constexpr float NOISE_MAX = 22.875f;

__device__ __forceinline__ float noise32(uint32_t w) {
  float e;
  if (w < 0x80000000u) {
    const float u = __fmul_rn(__fadd_rn(__uint2float_rn(w), 0.5f), 0x1p-32f);
    e = -logf(u);
  } else {
    const float t = __fmul_rn(__fadd_rn(__uint2float_rn(~w), 0.5f), 0x1p-32f);
    e = -log1pf(-t);
  }
  return -logf(e);
}

// A cheap upper bound on G(w), two fast logarithms: -log(u) is bounded below
// by a shaved fast-log value (u < 1/2) or by 1 - u (u >= 1/2).
__device__ __forceinline__ float noise_upper(uint32_t w) {
  float e;
  if (w < 0x80000000u) {
    const float u = __fmul_rn(__fadd_rn(__uint2float_rn(w), 0.5f), 0x1p-32f);
    e = __fmul_rn(-__logf(u), 1.f - 4e-6f);
  } else {
    e = __fmul_rn(__fmul_rn(__fadd_rn(__uint2float_rn(~w), 0.5f), 0x1p-32f), 1.f - 4e-6f);
  }
  const float g = -__logf(e);
  return __fadd_rn(g, __fmul_rn(4e-6f, __fadd_rn(1.f, fabsf(g))));
}

// ---------------------------------------------------------------------------
// Order-preserving unsigned keys: key(a) > key(b) iff a > b; -0 and +0 share
// a key, as they compare equal in the oracle's sort.
__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t b = __float_as_uint(v == 0.f ? 0.f : v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ uint64_t order_key(double v) {
  const uint64_t b = uint64_t(__double_as_longlong(v == 0. ? 0. : v));
  return (b >> 63) ? ~b : (b | (1ull << 63));
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
__device__ __forceinline__ double key_value(uint64_t k) {
  return __longlong_as_double(int64_t((k >> 63) ? (k & ~(1ull << 63)) : ~k));
}

// ---------------------------------------------------------------------------
// Exact sums. A weight w in [0, 2^27) becomes floor(w * 2^FX_SHIFT), a
// 128-bit integer; sums of those are exact, associative and commutative, so a
// total does not depend on how the row is split. Each term is truncated by
// less than one unit (2^-100), so the true sum of n terms lies in
// [S, S + n) units: far inside half an ulp of any sum >= 1 (every kept set
// contains its maximum, whose weight is exactly 1).
constexpr int FX_SHIFT = 100;

__device__ __forceinline__ u128 fx_of(double w) {
  const uint64_t bits = uint64_t(__double_as_longlong(w));
  const int exponent = int((bits >> 52) & 0x7ff);
  if (exponent == 0 || w <= 0) return 0;  // zero, or far below one unit
  const uint64_t mantissa = (bits & ((1ull << 52) - 1)) | (1ull << 52);
  const int shift = exponent - 1075 + FX_SHIFT;
  if (shift >= 0) return u128(mantissa) << shift;
  if (shift > -53) return u128(mantissa >> (-shift));
  return 0;
}

// The double nearest to S units (ties to even); *near_tie reports that the
// true sum, within [S, S + n), may round the other way.
__device__ inline double fx_round(u128 s, uint32_t n, bool* near_tie) {
  *near_tie = false;
  if (s == 0) return 0.0;
  const uint64_t hi = uint64_t(s >> 64), lo = uint64_t(s);
  const int top = hi ? 127 - __clzll(hi) : 63 - __clzll(lo);  // highest set bit
  if (top < 53) return double(uint64_t(s)) * 0x1p-100;         // exact
  const int drop = top - 52;
  const u128 one = 1;
  const u128 rest = s & ((one << drop) - 1), half = one << (drop - 1);
  uint64_t m = uint64_t(s >> drop);
  const bool up = rest > half || (rest == half && (m & 1));
  // The tie point is at `half`; the true remainder lies in [rest, rest + n).
  if ((rest <= half && half < rest + n) || rest + n > (one << drop)) *near_tie = true;
  int e = drop - FX_SHIFT;
  if (up) {
    ++m;
    if (m >> 53) { m >>= 1; ++e; }
  }
  return ldexp(double(m), e);
}

// Whether the correctly rounded true sum (within [S, S + n) units) is >= t,
// for t > 1 (a sum's rounding reaches t iff it passes the midpoint between t
// and its predecessor; an exact midpoint rounds to t when t's mantissa is even).
__device__ inline bool fx_reaches(u128 s, uint32_t n, double t, bool* near_tie) {
  *near_tie = false;
  const uint64_t bits = uint64_t(__double_as_longlong(t));
  const double below = __longlong_as_double(int64_t(bits - 1));
  const u128 mid = (fx_of(t) + fx_of(below)) >> 1;
  const bool even = (bits & 1) == 0;
  if (mid >= s && mid < s + n) *near_tie = mid != s || !even;
  return s > mid || (s == mid && even);
}

// ---------------------------------------------------------------------------
// Certified argmax. mid is the FP32 score, [lo, hi] bounds the exact one;
// others bounds every exact score except the winner's. The winner is certain
// when lo > others. The merge keeps the larger mid (lower ID on ties), so it
// is associative and commutative: the result never depends on the order or
// grouping of a reduction.
struct Pick {
  float mid, lo, hi, others;
  int id;
};
__device__ __forceinline__ Pick no_pick() { return {-INFINITY, -INFINITY, -INFINITY, -INFINITY, INT_MAX}; }
__device__ __forceinline__ Pick pick_of(Pick a, Pick b) {
  const bool b_wins = b.mid > a.mid || (b.mid == a.mid && b.id < a.id);
  Pick w = b_wins ? b : a;
  const Pick l = b_wins ? a : b;
  w.others = fmaxf(fmaxf(a.others, b.others), l.hi);
  return w;
}
// Exact (FP64) argmax with the lowest ID winning ties.
struct Best {
  double v;
  int id;
};
__device__ __forceinline__ Best no_best() { return {-INFINITY, INT_MAX}; }
__device__ __forceinline__ Best best_of(Best a, Best b) {
  return (b.v > a.v || (b.v == a.v && b.id < a.id)) ? b : a;
}

// ---------------------------------------------------------------------------
// Warp and block reductions (fixed order, every lane receives the result).
template <class T> __device__ __forceinline__ T shfl_xor(T v, int o) { return __shfl_xor_sync(0xffffffffu, v, o); }
__device__ __forceinline__ u128 shfl_xor(u128 v, int o) {
  const uint64_t lo = __shfl_xor_sync(0xffffffffu, uint64_t(v), o);
  const uint64_t hi = __shfl_xor_sync(0xffffffffu, uint64_t(v >> 64), o);
  return (u128(hi) << 64) | lo;
}
__device__ __forceinline__ Pick shfl_xor(Pick p, int o) {
  return {shfl_xor(p.mid, o), shfl_xor(p.lo, o), shfl_xor(p.hi, o), shfl_xor(p.others, o), shfl_xor(p.id, o)};
}
__device__ __forceinline__ Best shfl_xor(Best b, int o) { return {shfl_xor(b.v, o), shfl_xor(b.id, o)}; }

template <class T, class Op> __device__ __forceinline__ T warp_all(T v, Op op) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = op(v, shfl_xor(v, o));
  return v;
}
// Block-wide reduction; `scratch` holds WARPS values. Ends with a barrier so
// that scratch can be reused at once.
template <class T, class Op> __device__ __forceinline__ T block_all(T v, Op op, T* scratch) {
  v = warp_all(v, op);
  if (lane_id() == 0) scratch[warp_id()] = v;
  __syncthreads();
  T r = scratch[0];
#pragma unroll
  for (int w = 1; w < WARPS; ++w) r = op(r, scratch[w]);
  __syncthreads();
  return r;
}
// Barrier 1 over the block's first THREADS threads only (the row's warps):
// an extra warp outside them (the row kernel's warm-up warp) never holds
// them up. The _or form also ORs a predicate over those threads.
__device__ __forceinline__ void sync_rows() { asm volatile("bar.sync 1, %0;" ::"n"(THREADS) : "memory"); }
__device__ __forceinline__ bool sync_rows_or(bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred a, b;\n\t"
      "setp.ne.u32 a, %1, 0;\n\t"
      "bar.red.or.pred b, 1, %2, a;\n\t"
      "selp.u32 %0, 1, 0, b;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(p)), "n"(THREADS)
      : "memory");
  return r != 0;
}
// Inclusive prefix sum over the block in thread order; *total gets the sum.
template <class T> __device__ __forceinline__ T block_scan(T v, T* scratch, T* total) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y;
    if constexpr (sizeof(T) == 16) {
      const uint64_t lo = __shfl_up_sync(0xffffffffu, uint64_t(v), o);
      const uint64_t hi = __shfl_up_sync(0xffffffffu, uint64_t(v >> 64), o);
      y = (T(hi) << 64) | lo;
    } else {
      y = __shfl_up_sync(0xffffffffu, v, o);
    }
    if (lane_id() >= o) v += y;
  }
  if (lane_id() == 31) scratch[warp_id()] = v;
  __syncthreads();
  T before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < WARPS; ++w) {
    if (w < warp_id()) before += scratch[w];
    all += scratch[w];
  }
  __syncthreads();
  *total = all;
  return before + v;
}

// ---------------------------------------------------------------------------
// sm_90+/sm_100 primitives.
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return uint32_t(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// Global -> this CTA's own shared memory bulk copy (TMA, one destination). dst, src
// and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
// Flags shared between GPUs (vocabulary-sharded calls): a system-scope
// release store and acquire load of a 64-bit word in global memory (a peer
// GPU's memory for the loads).
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// System-scope loads of words a peer GPU publishes (after the acquire of
// its flag and fence_acq_rel_sys), never served from a stale L1 line.
__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint16_t ld_relaxed_sys(const uint16_t* p) {
  uint16_t v;
  asm volatile("ld.relaxed.sys.global.u16 %0, [%1];" : "=h"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
// Tagged words of the per-phase exchange: the datum in the low half, the
// call's tag in the high half, one aligned 64-bit store or load (single-copy
// atomic), so that the tag vouches for the datum beside it.
__device__ __forceinline__ void st_tagged_sys(uint64_t* p, uint32_t datum, uint32_t tag) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"((uint64_t(tag) << 32) | datum) : "memory");
}
// Polls the word until it carries `tag` (at most `limit` loads); false if it never did.
__device__ __forceinline__ bool ld_tagged_sys(const uint64_t* p, uint32_t tag, uint32_t& datum, uint32_t limit) {
  for (uint32_t spins = 0;;) {
    const uint64_t v = ld_relaxed_sys(p);
    if (uint32_t(v >> 32) == tag) {
      datum = uint32_t(v);
      return true;
    }
    if (++spins >= limit) return false;
  }
}
// Programmatic dependent launch: the row kernel starts its loads while the
// preparation kernel runs, and waits for it before reading what it wrote.
__device__ __forceinline__ void wait_for_prerequisite_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependent_grid() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace es
