// dispatch="reference": an independent, simple FP64 kernel, one block per
// target row, for cross-checking the fused row kernel in a debug run. It
// shares with the fused path only the preparation kernel (metadata checks),
// the per-request commit (finish_request), the RNG (Philox, noise64) and the
// exact fixed-point sums; everything a row decides is computed here again,
// in the oracle's order (python/exactsample/reference.py:55-104
// distribution(), :125-176 draws and the ratio test), with plain passes over
// the row:
//   1. validity (NaN / +inf anywhere), the valid count, maximum and argmax;
//   2. FP64 weights exp((v - max) / T) with min-p, stored with each token's
//      order key in the row's scratch;
//   3. top-k by radix selection on the order keys, ties by token ID;
//   4. the total as a correctly rounded fixed-point sum;
//   5. top-p: the largest key whose suffix mass (rounded) reaches
//      top_p * total, by binary search over the 64-bit key space (one pass
//      per step), then the tied tokens in ID order;
//   6. FP64 draws: argmax of log(p) + G over every kept token (lowest ID on
//      ties), the ratio test u < min(1, p / q) and the residual draw.
// It replaces the reference's reference_rows (csrc/verify/verify.cu:59-164),
// which runs one thread per request with a heap sort of the whole row.
//
// Scratch: 16 bytes per token per row (FP64 weight, 64-bit order key) past
// the call's records, inside the reference-sized workspace (20 * vocab bytes
// per row, api.h workspace_size with reference=true).
#pragma once
#include "es_rows.cuh"

namespace es {

constexpr int REF_THREADS = 512;
constexpr int REF_WARPS = REF_THREADS / 32;

__host__ __device__ constexpr uint64_t reference_scratch_offset(int64_t rows) {
  return (workspace_needed(rows) + 15) / 16 * 16;
}
__host__ __device__ constexpr uint64_t reference_scratch_bytes(int64_t rows, int64_t vocab) {
  return uint64_t(rows) * uint64_t(vocab) * 16;
}

struct RefShared {
  uint32_t hist[256];
  u128 fx[REF_WARPS];
  uint32_t n[REF_WARPS];
  double d[REF_WARPS];
  int32_t i[REF_WARPS];
  int32_t flag[REF_WARPS];
  uint64_t key;
  int32_t value;
};

// Block reductions over NT threads (every thread receives the result).
template <int NT, class T, class Op> __device__ T ref_reduce(T v, Op op, T* scratch) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = op(v, shfl_xor(v, o));
  if (lane_id() == 0) scratch[warp_id()] = v;
  __syncthreads();
  T r = scratch[0];
  for (int w = 1; w < NT / 32; ++w) r = op(r, scratch[w]);
  __syncthreads();
  return r;
}
template <int NT> __device__ inline u128 ref_sum(u128 v, RefShared& sh) {
  return ref_reduce<NT>(v, [](u128 a, u128 b) { return a + b; }, sh.fx);
}
template <int NT> __device__ inline uint32_t ref_count(uint32_t v, RefShared& sh) {
  return ref_reduce<NT>(v, [](uint32_t a, uint32_t b) { return a + b; }, sh.n);
}

// The n-th largest 64-bit key (1-based) among the tokens `in` accepts, by
// 8-bit radix selection from the top; *above gets how many accepted keys
// are larger.
template <int NT, class In>
__device__ uint64_t ref_select_key(int vocab, const uint64_t* keys, In in, uint32_t n, uint32_t* above, RefShared& sh) {
  uint64_t prefix = 0, known = 0;
  uint32_t need = n, larger = 0;
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int b = threadIdx.x; b < 256; b += NT) sh.hist[b] = 0;
    __syncthreads();
    for (int t = threadIdx.x; t < vocab; t += NT)
      if (in(t) && (keys[t] & known) == prefix) atomicAdd(&sh.hist[(keys[t] >> shift) & 255], 1u);
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t cum = 0;
      int digit = 0;
      for (int b = 255; b >= 0; --b) {
        if (cum + sh.hist[b] >= need) {
          digit = b;
          break;
        }
        cum += sh.hist[b];
      }
      sh.value = digit;
      sh.n[0] = cum;
    }
    __syncthreads();
    const int digit = sh.value;
    need -= sh.n[0];
    larger += sh.n[0];
    prefix |= uint64_t(digit) << shift;
    known |= uint64_t(255) << shift;
    __syncthreads();
  }
  *above = larger;
  return prefix;
}

// The n-th smallest token ID (1-based) among the tokens `in` accepts.
template <int NT, class In> __device__ int ref_select_id(int vocab, In in, uint32_t n, RefShared& sh) {
  uint32_t prefix = 0, known = 0, need = n;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = threadIdx.x; b < 256; b += NT) sh.hist[b] = 0;
    __syncthreads();
    for (int t = threadIdx.x; t < vocab; t += NT)
      if (in(t) && (uint32_t(t) & known) == prefix) atomicAdd(&sh.hist[(uint32_t(t) >> shift) & 255], 1u);
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t cum = 0;
      int digit = 255;
      for (int b = 0; b < 256; ++b) {
        if (cum + sh.hist[b] >= need) {
          digit = b;
          break;
        }
        cum += sh.hist[b];
      }
      sh.value = digit;
      sh.n[0] = cum;
    }
    __syncthreads();
    need -= sh.n[0];
    prefix |= uint32_t(sh.value) << shift;
    known |= 255u << shift;
    __syncthreads();
  }
  return int(prefix);
}

// argmax over tokens of score(t) (skip: -inf), lowest ID on ties; -1 if none.
template <int NT, class Score> __device__ int ref_argmax(int vocab, Score score, RefShared& sh) {
  double best = -INFINITY;
  int id = INT_MAX;
  for (int t = threadIdx.x; t < vocab; t += NT) {
    const double s = score(t);
    if (s > best) {  // ascending t: a later equal score keeps the lower ID
      best = s;
      id = t;
    }
  }
  const Best b = ref_reduce<NT>(Best{best, id}, [](Best a, Best c) { return best_of(a, c); },
                                reinterpret_cast<Best*>(sh.fx));
  return b.v > -INFINITY ? b.id : -1;
}

// One row by one block of NT threads: returns the row's result. value(t)
// and allowed(t) give target token t of the whole row, qvalue(t) the
// proposal's (full-q draft rows); w and keys are the row's scratch (vocab
// doubles and 64-bit keys).
template <int NT, class Value, class Allowed, class QValue>
__device__ __noinline__ RowResult reference_row(const Params& p, int row, const RowCtx& c, Value value, Allowed allowed,
                                   QValue qvalue, double* w, uint64_t* keys, RefShared& sh) {
  const int vocab = p.vocab;
  const bool draft_row = row + 1 < c.end, full_q = draft_row && c.kind == 1;
  const bool verify = draft_row && p.mode == ES_RATIO;
  const Address addr{c.stream, c.position, uint32_t(c.seed), uint32_t(c.seed >> 32)};
  RowResult res{ES_OK, ES_OK, 0, -1, -1, {0, 0, 0}};
  // 1. Validity, maximum and argmax of the target row (and of q for full-q rows).
  int bad = 0;
  uint32_t valid = 0;
  Best top = no_best();
  for (int t = threadIdx.x; t < vocab; t += NT) {
    const double v = value(t);
    bad |= isnan(v) || v == INFINITY;
    if (v > -INFINITY && allowed(t)) {
      ++valid;
      top = best_of(top, Best{v, t});
    }
  }
  bad = ref_reduce<NT>(bad, [](int a, int b) { return a | b; }, sh.i);
  valid = ref_count<NT>(valid, sh);
  top = ref_reduce<NT>(top, [](Best a, Best b) { return best_of(a, b); }, reinterpret_cast<Best*>(sh.fx));
  res.target_status = bad ? ES_INVALID_INPUT : valid == 0 ? ES_NO_VALID_TOKEN : ES_OK;
  res.status = res.target_status;
  double qmax = -INFINITY, sq = 0;
  if (res.status == ES_OK && full_q) {
    int qbad = 0;
    uint32_t qvalid = 0;
    double m = -INFINITY;
    for (int t = threadIdx.x; t < vocab; t += NT) {
      const double v = qvalue(t);
      qbad |= isnan(v) || v == INFINITY;
      qvalid += v > -INFINITY;
      m = fmax(m, v);
    }
    qbad = ref_reduce<NT>(qbad, [](int a, int b) { return a | b; }, sh.i);
    qvalid = ref_count<NT>(qvalid, sh);
    qmax = ref_reduce<NT>(m, [](double a, double b) { return fmax(a, b); }, sh.d);
    if (qbad) {
      res.status = ES_INVALID_INPUT;
    } else if (qvalid == 0) {
      res.status = ES_NO_VALID_TOKEN;
    } else {
      u128 f = 0;
      uint32_t n = 0;
      for (int t = threadIdx.x; t < vocab; t += NT) {
        const double v = qvalue(t);
        const double e = v > -INFINITY ? exp(v - qmax) : 0.0;
        if (e > 0) {
          f += fx_of(e);
          ++n;
        }
      }
      bool near;
      sq = fx_round(ref_sum<NT>(f, sh), ref_count<NT>(n, sh), &near);
      const double vd = qvalue(c.draft_id);
      const double wq = vd > -INFINITY ? exp(vd - qmax) : 0.0;
      if (!(wq / sq > 0)) res.status = ES_DRAFT_ZERO_PROB;
    }
  }
  auto q_of = [&](int t) {
    if (!full_q) return 1.0;
    const double v = qvalue(t);
    return v > -INFINITY ? exp(v - qmax) / sq : 0.0;
  };

  if (res.status == ES_OK && c.temperature == 0) {
    // A point mass at the greedy token.
    const int g = top.id;
    res.sample = g;
    if (verify) {
      res.accept = c.draft_id == g;
      if (!res.accept) res.residual = (!full_q || 1.0 - q_of(g) > 0) ? g : -1;
    }
  } else if (res.status == ES_OK) {
    // 2. Weights with min-p; order keys.
    const double maxv = top.v;
    uint32_t kept = 0;
    for (int t = threadIdx.x; t < vocab; t += NT) {
      const double v = value(t);
      double e = 0;
      if (v > -INFINITY && allowed(t)) {
        e = exp((v - maxv) / c.temperature);
        if (!(e >= c.min_p && e > 0)) e = 0;
      }
      w[t] = e;
      keys[t] = order_key(v);
      kept += e > 0;
    }
    __syncthreads();
    kept = ref_count<NT>(kept, sh);
    // 3. Top-k: keep the first k in (value desc, ID asc) order.
    if (c.top_k > 0 && uint32_t(c.top_k) < kept) {
      uint32_t above = 0;
      const uint64_t kth = ref_select_key<NT>(vocab, keys, [&](int t) { return w[t] > 0; }, uint32_t(c.top_k), &above, sh);
      const int last = ref_select_id<NT>(vocab, [&](int t) { return w[t] > 0 && keys[t] == kth; },
                                     uint32_t(c.top_k) - above, sh);
      for (int t = threadIdx.x; t < vocab; t += NT)
        if (w[t] > 0 && (keys[t] < kth || (keys[t] == kth && t > last))) w[t] = 0;
      __syncthreads();
    }
    // 4. The total, correctly rounded.
    auto suffix = [&](uint64_t from, uint32_t* count) {  // kept weights with key >= from
      u128 f = 0;
      uint32_t n = 0;
      for (int t = threadIdx.x; t < vocab; t += NT)
        if (w[t] > 0 && keys[t] >= from) {
          f += fx_of(w[t]);
          ++n;
        }
      *count = ref_count<NT>(n, sh);
      return ref_sum<NT>(f, sh);
    };
    uint32_t n_all;
    const u128 all = suffix(0, &n_all);
    bool near;
    double den = fx_round(all, n_all, &near);
    // 5. Top-p: the shortest prefix whose rounded sum reaches top_p * total.
    uint64_t cut_key = 0;
    int cut_id = INT_MAX;
    if (c.top_p < 1) {
      const double target = c.top_p * den;
      // The largest key K whose suffix {key >= K} reaches the target.
      uint64_t lo = 0, hi = ~0ull;
      while (lo < hi) {
        const uint64_t mid = lo + (hi - lo) / 2 + 1;
        uint32_t n;
        const u128 s = suffix(mid, &n);
        if (fx_round(s, n, &near) >= target) lo = mid;
        else hi = mid - 1;
      }
      cut_key = lo;
      uint32_t n_above;
      const u128 above = lo == ~0ull ? u128(0) : suffix(lo + 1, &n_above);
      if (lo == ~0ull) n_above = 0;
      // The tied tokens at cut_key share one weight: the j-th in ID order ends the prefix.
      uint32_t n_tied;
      suffix(lo, &n_tied);
      n_tied -= n_above;
      double wstar = 0;
      for (int t = threadIdx.x; t < vocab; t += NT)
        if (w[t] > 0 && keys[t] == lo) wstar = w[t];
      wstar = ref_reduce<NT>(wstar, [](double a, double b) { return fmax(a, b); }, sh.d);
      uint32_t j = 1;
      while (j < n_tied && fx_round(above + fx_of(wstar) * u128(j), n_above + j, &near) < target) ++j;
      den = fx_round(above + fx_of(wstar) * u128(j), n_above + j, &near);
      cut_id = ref_select_id<NT>(vocab, [&](int t) { return w[t] > 0 && keys[t] == lo; }, j, sh);
    }
    auto prob = [&](int t) {
      if (!(w[t] > 0) || keys[t] < cut_key || (keys[t] == cut_key && t > cut_id)) return 0.0;
      return w[t] / den;
    };
    // 6. Draws.
    auto word = [&](uint32_t sub, int t) { return addr.word(sub, uint32_t(t)); };
    if (!verify) {
      res.sample = ref_argmax<NT>(vocab, [&](int t) {
        const double q = prob(t);
        return q > 0 ? log(q) + noise64(word(0, t)) : -INFINITY;
      }, sh);
    } else {
      const double px = prob(c.draft_id), qx = q_of(c.draft_id);
      res.accept = uniform64(word(1, 0)) < fmin(1.0, px / qx);
      if (!res.accept)
        res.residual = ref_argmax<NT>(vocab, [&](int t) {
          const double r = full_q ? fmax(prob(t) - q_of(t), 0.0) : (t == c.draft_id ? 0.0 : prob(t));
          return r > 0 ? log(r) + noise64(word(2, t)) : -INFINITY;
        }, sh);
    }
  }
  return res;
}

template <int DT>
__global__ void __launch_bounds__(REF_THREADS) reference_rows(const __grid_constant__ Params p) {
  using T = typename Types<DT>::T;
  __shared__ RefShared sh;
  static_assert(sizeof(RefShared::fx) >= REF_WARPS * sizeof(Best), "argmax scratch");
  const int row = blockIdx.x, vocab = p.vocab;
  if (*malformed_flag(p.workspace) != 0) return;  // every request already failed
  const RowCtx c = row_contexts(p.workspace, p.rows)[row];
  if (c.skip) return;  // the request failed its metadata checks
  double* w = reinterpret_cast<double*>(p.workspace + reference_scratch_offset(p.rows)) + int64_t(row) * vocab * 2;
  uint64_t* keys = reinterpret_cast<uint64_t*>(w + vocab);
  const T* x = static_cast<const T*>(p.target) + int64_t(row) * p.t_s0;
  const T* y = static_cast<const T*>(p.draft) + int64_t(row) * p.q_s0;
  const RowResult res = reference_row<REF_THREADS>(
      p, row, c, [&](int t) { return double(widen(x[int64_t(t) * p.t_s1])); },
      [&](int t) {
        return p.mask == nullptr || ((uint32_t(p.mask[int64_t(row) * p.m_s0 + int64_t(t >> 5) * p.m_s1]) >> (t & 31)) & 1u);
      },
      [&](int t) { return double(widen(y[int64_t(t) * p.q_s1])); }, w, keys, sh);
  // The request's last row to finish commits it.
  if (threadIdx.x == 0) {
    row_results(p.workspace)[row] = res;
    __threadfence();
    const uint32_t done = atomicAdd(&arrivals(p.workspace, p.rows)[c.begin], 1u) + 1;
    if (done == uint32_t(c.end - c.begin)) {
      __threadfence();
      finish_request(p, c.req, c.begin, c.end);
    }
  }
}

}  // namespace es
