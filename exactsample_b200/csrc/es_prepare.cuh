// Batch preparation (offsets and per-request metadata checks, output reset)
// and the per-request finish that commits accepted drafts and the final
// token. Semantics follow the reference's initialize / metadata_status /
// finalize (csrc/verify/verify.cu:6-56 and :169-217) and the oracle's
// verify_reference (python/exactsample/reference.py:177-254).
#pragma once
#include "es_layout.cuh"

namespace es {

#ifdef ES_CHECKS
static __device__ __noinline__ void check_failed(uint8_t* ws, int64_t rows, uint32_t site) {
  Diagnostics* d = diagnostics(ws, rows);
  atomicAdd(&d->check_failures, 1u);
  atomicCAS(&d->first_site, 0u, site);
}
#endif

// Whether cu_rows is malformed: cu[0] != 0, cu[R] != rows, or a pair out of
// order or out of range. The whole block computes it.
__device__ inline bool offsets_malformed(const Params& p) {
  __shared__ int bad;
  if (threadIdx.x == 0) bad = at(p.cu_rows, p.cu_s, 0) != 0 || at(p.cu_rows, p.cu_s, p.requests) != p.rows;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < p.requests; i += blockDim.x) {
    const int64_t x = at(p.cu_rows, p.cu_s, i), y = at(p.cu_rows, p.cu_s, i + 1);
    if (x < 0 || y > p.rows || x > y) atomicExch(&bad, 1);
  }
  __syncthreads();
  return bad != 0;
}

// INVALID_INPUT for request metadata the contract rejects before any row is
// read (reference verify.cu:6-27; oracle reference.py:178-196 and the
// parameter checks of distribution(), reference.py:43-52).
__device__ inline int32_t metadata_status(const Params& p, int64_t req) {
  const int64_t begin = at(p.cu_rows, p.cu_s, req), end = at(p.cu_rows, p.cu_s, req + 1);
  if (begin < 0 || end > p.rows || end <= begin || end - begin > int64_t(p.max_draft) + 1) return ES_INVALID_INPUT;
  const double t = at(p.temperature, p.temp_s, req), tp = at(p.top_p, p.topp_s, req), mp = at(p.min_p, p.minp_s, req);
  const int64_t k = at(p.top_k, p.topk_s, req), kind = at(p.draft_kind, p.kind_s, req);
  if (!isfinite(t) || t < 0 || !isfinite(tp) || tp <= 0 || tp > 1 || !isfinite(mp) || mp < 0 || mp > 1 || k < 0 ||
      k > p.vocab || kind < 0 || kind > 1)
    return ES_INVALID_INPUT;
  if ((p.mode == ES_COUPLED && kind == 1) || (kind == 1 && end - begin > 1 && p.draft == nullptr))
    return ES_INVALID_INPUT;
  const int64_t stream = at(p.streams, p.stream_s, req);
  if (stream < 0 || stream > int64_t(UINT32_MAX)) return ES_INVALID_INPUT;
  for (int64_t row = begin; row < end; ++row) {
    const int64_t pos = at(p.positions, p.pos_s, row);
    if (pos < 0 || pos > int64_t(UINT32_MAX)) return ES_INVALID_INPUT;
    if (row + 1 < end) {
      const int64_t id = p.draft_ids[req * p.d_s0 + (row - begin) * p.d_s1];
      if (id < 0 || id >= p.vocab) return ES_INVALID_INPUT;
    }
  }
  return ES_OK;
}

// Commits one request from its rows' results (run by one thread, after every
// row of the request has published its RowResult).
//   * the first row whose target failed gives the status; failing that, the
//     first row whose proposal failed (oracle: targets are validated first);
//   * ratio mode accepts draft i iff the row's test passed; coupled mode iff
//     the row's substream-0 draw equals the draft;
//   * the first rejection emits the residual (ratio) or the draw (coupled);
//     with no rejection the bonus row's draw follows the D accepted drafts;
//   * a rejection without residual mass is INVALID_INPUT (contract: an
//     impossible zero-residual rejection is an error, not an EOS).
__device__ inline void finish_request(const Params& p, int64_t req, int begin, int end) {
  const RowResult* results = row_results(p.workspace);
  // The outcome: a failed status, or `accepted` drafts followed by `last`.
  int32_t failed = ES_OK;
  for (int pass = 0; pass < 2 && failed == ES_OK; ++pass)
    for (int row = begin; row < end; ++row) {
      const int32_t s = pass == 0 ? __ldcg(&results[row].target_status) : __ldcg(&results[row].status);
      if (s != ES_OK) {
        failed = s;
        break;
      }
    }
  const int drafts = end - begin - 1;
  int accepted = drafts;
  int64_t last = -1;
  if (failed == ES_OK) {
    for (int i = 0; i < drafts; ++i) {
      const int row = begin + i;
      const int64_t draft = p.draft_ids[req * p.d_s0 + int64_t(i) * p.d_s1];
      const int32_t sample = __ldcg(&results[row].sample);
      const bool accept = p.mode == ES_COUPLED ? sample == draft : __ldcg(&results[row].accept) != 0;
      if (!accept) {
        accepted = i;
        last = p.mode == ES_COUPLED ? sample : __ldcg(&results[row].residual);
        if (last < 0) failed = ES_INVALID_INPUT;
        break;
      }
    }
    if (accepted == drafts) last = __ldcg(&results[end - 1].sample);
  }
  for (int set = 0; set < output_sets(p); ++set) {
    const Outputs o = output_set(p, set);
    if (failed != ES_OK) {
      o.status[req * p.st_s] = failed;
      continue;
    }
    int64_t* tokens = o.tokens + req * p.tok_s0;
    for (int j = 0; j < accepted; ++j) tokens[j * p.tok_s1] = p.draft_ids[req * p.d_s0 + int64_t(j) * p.d_s1];
    tokens[accepted * p.tok_s1] = last;
    o.accepted[req * p.acc_s] = accepted;
  }
}

}  // namespace es
