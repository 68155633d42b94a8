// The C ABI (include/exactsample_b200.h): argument validation, workspace
// sizing, cluster sizing and the launch sequence of one call.
//
// The checks and their messages follow the reference's torch binding
// (csrc/bindings.cpp:50-119), so a caller sees the same errors whether it
// comes through the torch op or calls this library directly.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <numeric>
#include <string>

#include "es_kernel.cuh"

namespace es {
// One block validates cu_rows for very large batches (the preparation
// kernel's blocks then read the flag instead of re-checking every offset).
__global__ void __launch_bounds__(1024) check_offsets(const __grid_constant__ Params p) {
  const bool bad = offsets_malformed(p);
  if (threadIdx.x == 0) *malformed_flag(p.workspace) = bad;
}

// One thread per request: outputs reset to the failed state (tokens -1,
// accepted 0), metadata status, path, and the request's arrival counter.
__global__ void __launch_bounds__(128) prepare(const __grid_constant__ Params p) {
  if (blockIdx.x == 0) ES_TRACE(p.workspace, p.rows, 0, 15, 0);  // development builds: when preparation starts
  allow_dependent_grid();  // the row kernel may launch now and start loading logits
  // A vocabulary-sharded call: the stream's earlier work (this GPU's shard)
  // is done, so tell the peers.
  if (p.sh.count > 1 && blockIdx.x == 0 && threadIdx.x == 0)
    st_release_sys(const_cast<uint64_t*>(p.sh.ready[p.sh.rank]), p.sh.epoch);
  bool bad;
  if (p.offsets_inline) {
    bad = offsets_malformed(p);
  } else {
    bad = *malformed_flag(p.workspace) != 0;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (p.offsets_inline) *malformed_flag(p.workspace) = bad;
    *fallback_count(p.workspace) = 0;
  }
  if (p.rows > 0 && blockIdx.x == 0) {
    uint32_t* d = reinterpret_cast<uint32_t*>(diagnostics(p.workspace, p.rows));
    for (int i = threadIdx.x; i < int(sizeof(Diagnostics) / 4); i += blockDim.x) d[i] = 0;
  }
  const int64_t req = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (req >= p.requests) return;
  // A vocabulary-sharded call resets only this GPU's requests, in every
  // GPU's output buffers; their owners write the others.
  const bool owned = p.sh.count <= 1 || (req >= p.sh.req_begin && req < p.sh.req_end);
  const int32_t status = bad ? ES_INVALID_INPUT : metadata_status(p, req);
  if (owned)
    for (int set = 0; set < output_sets(p); ++set) {
      const Outputs o = output_set(p, set);
      for (int64_t i = 0; i <= p.max_draft; ++i) o.tokens[req * p.tok_s0 + i * p.tok_s1] = -1;
      o.accepted[req * p.acc_s] = 0;
      o.path[req * p.path_s] = p.exact_draws ? ES_PATH_REFERENCE : ES_PATH_FUSED;
      o.status[req * p.st_s] = status;
    }
  if (bad) return;  // rows cannot be attributed; the row kernel reads the flag
  const int64_t begin = at(p.cu_rows, p.cu_s, req), end = at(p.cu_rows, p.cu_s, req + 1);
  if (begin < 0 || end > p.rows || begin >= end) return;
  RowCtx c{};
  c.req = int32_t(req);
  c.begin = int32_t(begin);
  c.end = int32_t(end);
  c.skip = status != ES_OK || !owned;
  if (!c.skip) {
    arrivals(p.workspace, p.rows)[begin] = 0;
    c.kind = int32_t(at(p.draft_kind, p.kind_s, req));
    c.top_k = int32_t(at(p.top_k, p.topk_s, req));
    c.temperature = at(p.temperature, p.temp_s, req);
    c.top_p = at(p.top_p, p.topp_s, req);
    c.min_p = at(p.min_p, p.minp_s, req);
    c.seed = uint64_t(at(p.seeds, p.seed_s, req));
    c.stream = uint32_t(at(p.streams, p.stream_s, req));
  }
  RowCtx* out = row_contexts(p.workspace, p.rows);
  for (int64_t row = begin; row < end; ++row) {
    if (!c.skip) {
      c.position = uint32_t(at(p.positions, p.pos_s, row));
      c.draft_id = row + 1 < end ? int32_t(p.draft_ids[req * p.d_s0 + (row - begin) * p.d_s1]) : -1;
    }
    out[row] = c;
  }
  if (blockIdx.x == 0) ES_TRACE(p.workspace, p.rows, 0, 15, 1);  // development builds: block 0 done
}

// Vocabulary-sharded calls: a GPU's "shard written" and "outputs done" flags.
// One thread stores `epoch` with system-scope release once the stream's
// earlier work is done; one thread waits (bounded) until every listed flag
// has reached `epoch`, counting a give-up in *timeouts.
__global__ void signal_flag(uint64_t* flag, uint64_t epoch) {
  __threadfence_system();
  st_release_sys(flag, epoch);
}
struct FlagSet {
  const uint64_t* flag[MAX_SHARDS];
  int32_t count;
  int32_t rank;  // finish_flags: this GPU's slot in every GPU's array
  uint64_t epoch;
  uint32_t* timeouts;
};
__device__ void wait_all(const FlagSet& f) {
  for (int g = 0; g < f.count; ++g)
    for (uint32_t spins = 0; ld_acquire_sys(f.flag[g]) < f.epoch;)
      if (++spins >= (1u << 20)) {
        if (f.timeouts != nullptr) atomicAdd(f.timeouts, 1u);
        break;
      }
  __threadfence_system();
}
__global__ void wait_flags(const __grid_constant__ FlagSet f) { wait_all(f); }
// The end of a sharded call on one GPU, one thread per GPU g: this GPU's tag
// into its slot of GPU g's array (a remote system-scope release), then GPU
// g's tag from this GPU's own array (local polls). Launched as a programmatic
// dependent of the row kernel, so it first waits for every earlier grid on
// the stream to complete.
__global__ void finish_flags(uint64_t* mine, const __grid_constant__ FlagSet f) {
  wait_for_prerequisite_grid();
  const int g = threadIdx.x;
  if (g >= f.count) return;
  __threadfence_system();
  st_release_sys(const_cast<uint64_t*>(f.flag[g]) + f.rank, f.epoch);
  for (uint32_t spins = 0; ld_acquire_sys(mine + g) < f.epoch;)
    if (++spins >= (1u << 20)) {
      if (f.timeouts != nullptr) atomicAdd(f.timeouts, 1u);
      break;
    }
  __threadfence_system();
}

template <int DT> cudaError_t launch_rows(const Params& p, int cluster, cudaStream_t stream);
template <int DT> cudaError_t launch_reference(const Params& p, cudaStream_t stream);
extern template cudaError_t launch_reference<ES_F32>(const Params&, cudaStream_t);
extern template cudaError_t launch_reference<ES_F64>(const Params&, cudaStream_t);
extern template cudaError_t launch_reference<ES_F16>(const Params&, cudaStream_t);
extern template cudaError_t launch_reference<ES_BF16>(const Params&, cudaStream_t);
extern template cudaError_t launch_rows<ES_F32>(const Params&, int, cudaStream_t);
extern template cudaError_t launch_rows<ES_F64>(const Params&, int, cudaStream_t);
extern template cudaError_t launch_rows<ES_F16>(const Params&, int, cudaStream_t);
extern template cudaError_t launch_rows<ES_BF16>(const Params&, int, cudaStream_t);
}  // namespace es

namespace {
using es::Params;

thread_local std::string g_error;

int fail(int code, const std::string& message) {
  g_error = message;
  return code;
}

size_t element_size(int32_t dtype) {
  switch (dtype) {
    case ES_F32: case ES_I32: return 4;
    case ES_F64: case ES_I64: return 8;
    case ES_F16: case ES_BF16: return 2;
    case ES_U8: return 1;
    default: return 0;
  }
}
int64_t numel(const es_tensor& t) {
  int64_t n = 1;
  for (int d = 0; d < t.ndim; ++d) n *= t.size[d];
  return n;
}
// [first byte, one past the last byte] of a strided view.
bool extent(const es_tensor& t, uintptr_t* begin, uintptr_t* end) {
  if (numel(t) == 0) return false;
  const size_t e = element_size(t.dtype);
  uintptr_t span = e;
  for (int d = 0; d < t.ndim; ++d) span += uintptr_t(t.size[d] - 1) * uintptr_t(t.stride[d]) * e;
  *begin = reinterpret_cast<uintptr_t>(t.data);
  *end = *begin + span;
  return true;
}
// Address intervals prove disjointness (bindings.cpp:25-37).
bool disjoint(const es_tensor& a, const es_tensor& b) {
  uintptr_t a0, a1, b0, b1;
  if (!extent(a, &a0, &a1) || !extent(b, &b0, &b1)) return true;
  return a1 <= b0 || b1 <= a0;
}
// A view whose elements never share an address (bindings.cpp:38-44).
bool no_internal_overlap(const es_tensor& t) {
  if (numel(t) <= 1) return true;
  for (int d = 0; d < t.ndim; ++d)
    if (t.size[d] > 1 && t.stride[d] == 0) return false;
  if (t.ndim == 1 || t.size[0] <= 1 || t.size[1] <= 1) return true;
  const int64_t divisor = std::gcd(t.stride[0], t.stride[1]);
  return t.size[0] <= t.stride[1] / divisor || t.size[1] <= t.stride[0] / divisor;
}
bool check(const es_tensor& t, int32_t dtype, int ndim, const char* name) {
  if (t.dtype != dtype || t.ndim != ndim || (t.data == nullptr && numel(t) != 0)) {
    g_error = std::string(name) + " has wrong device, dtype or rank";
    return false;
  }
  for (int d = 0; d < ndim; ++d)
    if (t.stride[d] < 0 || t.size[d] < 0) {
      g_error = std::string(name) + " has a negative stride";
      return false;
    }
  return true;
}
bool is_logit_dtype(int32_t d) { return d == ES_F32 || d == ES_F64 || d == ES_F16 || d == ES_BF16; }

// Ranks per row and the row mode.
//   * Resident rows: each rank keeps its slice (about RESIDENT_BYTES) in
//     shared memory, so later passes never touch HBM; chosen when every
//     row's cluster fits on the GPU at once (small batches), with as many
//     ranks per row as that allows (up to 16) to spread a row over SMs.
//   * Streamed rows: each rank streams its slice through a TMA ring and later
//     passes re-read global memory (L2); about three ranks per SM in all (one
//     rank per row from 444 rows on), since one rank streams a row at well
//     under an SM's share of HBM bandwidth.
constexpr size_t RESIDENT_BYTES = 80 * 1024;
constexpr int SM_COUNT = 148, RESIDENT_SLOTS = 2 * SM_COUNT, STREAM_SLOTS = 3 * SM_COUNT;
constexpr size_t MAX_SMEM = 227 * 1024;

template <int DT> size_t smem_for(int sw, int stages) { return es::smem_bytes<DT>(sw, stages); }
size_t smem_for_dtype(int dtype, int sw, int stages) {
  switch (dtype) {
    case ES_F32: return smem_for<ES_F32>(sw, stages);
    case ES_F64: return smem_for<ES_F64>(sw, stages);
    case ES_F16: return smem_for<ES_F16>(sw, stages);
    default: return smem_for<ES_BF16>(sw, stages);
  }
}

int choose_cluster(int64_t rows, int64_t vocab, int dtype, bool full_rows, int* slice_words, size_t* smem,
                   int* stream, int* min_blocks) {
  const int64_t words = (vocab + 31) / 32;
  const size_t row_bytes = size_t(vocab) * element_size(dtype);
  const int resident_min = int(std::max<size_t>(1, (row_bytes + RESIDENT_BYTES - 1) / RESIDENT_BYTES));
  int c;
  bool streamed;
  if (resident_min <= 16 && rows * resident_min <= RESIDENT_SLOTS) {
    streamed = false;
    c = int(std::min<int64_t>(16, std::max<int64_t>(resident_min, RESIDENT_SLOTS / std::max<int64_t>(rows, 1))));
    if (vocab < 4096) c = resident_min;  // tiny rows: one rank
  } else {
    streamed = true;
    c = int(std::min<int64_t>(16, std::max<int64_t>(1, STREAM_SLOTS / std::max<int64_t>(rows, 1))));
    // Rows finished by whole-row passes (no lists: list_max 0, or FP64-only
    // draws) do several passes after the statistics: one rank per row leaves
    // each row's passes to 8 warps, so take two even at the price of a
    // second wave (320 rows at T = 1: 491 -> 384 us on a B200).
    if (full_rows) c = std::max(c, 2);
  }
  // EXACTSAMPLE_CLUSTER=n asks for n ranks per row (1..16), e.g. to show that
  // results do not depend on the split; EXACTSAMPLE_STREAM=0/1 forces the row
  // mode. Shared-memory limits may raise the rank count.
  if (const char* forced = std::getenv("EXACTSAMPLE_CLUSTER")) {
    const int n = std::atoi(forced);
    if (n >= 1 && n <= 16) c = n;
  }
  if (const char* forced = std::getenv("EXACTSAMPLE_STREAM")) {
    if (forced[0] == '0') streamed = false;
    if (forced[0] == '1') streamed = true;
  }
  // The TMA ring: four 16 KB stages while every rank has a place on the GPU
  // with two per SM. Beyond that three ranks share an SM: the kernel is
  // compiled for three blocks per SM (80 registers) and the ring has two
  // stages (a third measured no faster). EXACTSAMPLE_RING=2..4 forces the
  // depth.
  const bool three = streamed && rows * c > RESIDENT_SLOTS;
  for (;; ++c) {
    if (c > 16) return -1;
    const int sw = int((words + c - 1) / c);
    const int used = int((words + sw - 1) / sw);  // no empty ranks
    int stages = 0;
    if (streamed) {
      stages = es::MAX_RING_STAGES;
      if (three) stages = 2;
      if (const char* forced = std::getenv("EXACTSAMPLE_RING")) {
        const int n = std::atoi(forced);
        if (n >= 2 && n <= es::MAX_RING_STAGES) stages = n;
      }
    }
    const size_t bytes = smem_for_dtype(dtype, sw, stages);
    if (bytes <= MAX_SMEM) {
      *slice_words = sw;
      *smem = bytes;
      *stream = stages;
      *min_blocks = three ? 3 : 2;
      return used;
    }
  }
}

int device_check() {
  static thread_local int checked_device = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(ES_ERR_DEVICE, "no CUDA device is available");
  if (dev == checked_device) return ES_SUCCESS;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10)
    return fail(ES_ERR_DEVICE, "exactsample_b200 requires an sm_100 (B200) GPU");
  checked_device = dev;
  return ES_SUCCESS;
}

// `own_scratch`: 0 when the caller provides the workspace (sized by the
// reference's formula); otherwise the bytes of the library's static scratch
// that a->workspace describes (es_verify_static), checked against what this
// call's kernels actually use.
// `sh`: a vocabulary-sharded call's shard table (NULL otherwise); its
// target_logits (and draft_logits) are this GPU's shard.
int verify_impl(const es_args* a, cudaStream_t stream, cudaEvent_t before, cudaEvent_t after,
                uint64_t own_scratch = 0, const es_shards* sh = nullptr) {
  g_error.clear();
  if (a == nullptr) return fail(ES_ERR_ARGUMENT, "null arguments");
  const es_tensor& logits = a->target_logits;
  if (logits.ndim != 2 || (logits.data == nullptr && numel(logits) != 0))
    return fail(ES_ERR_ARGUMENT, "target_logits must be a 2D CUDA tensor");
  if (!is_logit_dtype(logits.dtype))
    return fail(ES_ERR_ARGUMENT, "exactsample logits require float16/bfloat16/float32/float64");
  if (logits.stride[0] < 0 || logits.stride[1] < 0) return fail(ES_ERR_ARGUMENT, "target_logits has a negative stride");
  if (!check(a->cu_rows, ES_I64, 1, "cu_rows")) return ES_ERR_ARGUMENT;
  if (a->cu_rows.size[0] < 1) return fail(ES_ERR_ARGUMENT, "cu_rows must contain an endpoint");
  const int64_t requests = a->cu_rows.size[0] - 1, rows = logits.size[0];
  int64_t vocab = logits.size[1];
  if (sh != nullptr) {
    if (!(sh->count >= 2 && sh->count <= es::MAX_SHARDS && sh->rank >= 0 && sh->rank < sh->count))
      return fail(ES_ERR_ARGUMENT, "shards: count must be in [2, 8] and rank in [0, count)");
    if (!(sh->cols > 0 && sh->cols % 16 == 0 && sh->vocab > (sh->count - 1) * sh->cols &&
          sh->vocab <= sh->count * sh->cols && sh->vocab <= INT32_MAX))
      return fail(ES_ERR_ARGUMENT, "shards: cols must be a positive multiple of 16 with (count - 1) * cols < vocab <= count * cols");
    const int64_t width = std::min<int64_t>(sh->cols, sh->vocab - int64_t(sh->rank) * sh->cols);
    if (logits.size[1] != width) return fail(ES_ERR_ARGUMENT, "shards: target_logits must be this GPU's shard [rows, its columns]");
    if (!(sh->req_begin >= 0 && sh->req_begin <= sh->req_end && sh->req_end <= requests))
      return fail(ES_ERR_ARGUMENT, "shards: the request range must lie in [0, requests]");
    if (sh->phases && !(sh->req_begin == 0 && sh->req_end == requests))
      return fail(ES_ERR_ARGUMENT, "shards: a per-phase call finishes every request on every GPU");
    vocab = sh->vocab;
  }
  if (requests == 0 && rows != 0) return fail(ES_ERR_ARGUMENT, "an empty request batch cannot contain target rows");
  if (!(vocab > 0 && vocab <= INT32_MAX && rows <= INT32_MAX && requests <= INT32_MAX))
    return fail(ES_ERR_ARGUMENT, "exactsample dimensions exceed int32 kernel indexing");
  if (rows > 65535) return fail(ES_ERR_ARGUMENT, "exactsample supports at most 65535 target rows per call");
  if (!(a->max_draft >= 0 && a->max_draft < INT32_MAX)) return fail(ES_ERR_ARGUMENT, "invalid max_draft");
  if (!(a->mode >= 0 && a->mode <= 1 && a->dispatch >= 0 && a->dispatch <= 2))
    return fail(ES_ERR_ARGUMENT, "invalid mode/dispatch");
  if (!(a->list_max >= 0 && a->list_max <= 256)) return fail(ES_ERR_ARGUMENT, "list_max must be in [0, 256]");
  if (!check(a->draft_ids, ES_I64, 2, "draft_ids")) return ES_ERR_ARGUMENT;
  if (!(a->draft_ids.size[0] == requests && a->draft_ids.size[1] >= a->max_draft))
    return fail(ES_ERR_ARGUMENT, "draft_ids capacity mismatch");
  const es_tensor* fp[3] = {&a->temperature, &a->top_p, &a->min_p};
  for (const es_tensor* t : fp) {
    if (!check(*t, ES_F64, 1, "floating request parameter")) return ES_ERR_ARGUMENT;
    if (t->size[0] != requests) return fail(ES_ERR_ARGUMENT, "request parameter length mismatch");
  }
  const es_tensor* ip[4] = {&a->top_k, &a->draft_kind, &a->seeds, &a->stream_ids};
  for (const es_tensor* t : ip) {
    if (!check(*t, ES_I64, 1, "integer request parameter")) return ES_ERR_ARGUMENT;
    if (t->size[0] != requests) return fail(ES_ERR_ARGUMENT, "request parameter length mismatch");
  }
  if (!check(a->positions, ES_I64, 1, "positions")) return ES_ERR_ARGUMENT;
  if (a->positions.size[0] != rows) return fail(ES_ERR_ARGUMENT, "positions must be per target row");
  const bool has_draft = a->draft_logits.ndim != 0, has_mask = a->mask.ndim != 0;
  if (has_draft) {
    const es_tensor& q = a->draft_logits;
    if (q.ndim != 2 || q.size[0] != rows || q.size[1] != logits.size[1] || q.stride[0] < 0 || q.stride[1] < 0 ||
        (q.data == nullptr && numel(q) != 0))
      return fail(ES_ERR_ARGUMENT, "draft_logits shape/device mismatch");
    if (q.dtype != logits.dtype) return fail(ES_ERR_ARGUMENT, "draft_logits must have the target_logits dtype");
  }
  if (has_mask) {
    if (!check(a->mask, ES_I32, 2, "mask")) return ES_ERR_ARGUMENT;
    if (!(a->mask.size[0] == rows && a->mask.size[1] == (vocab + 31) / 32))
      return fail(ES_ERR_ARGUMENT, "mask shape mismatch");
  }
  const es_tensor& ws = a->workspace;
  if (!check(ws, ES_U8, 1, "workspace")) return ES_ERR_ARGUMENT;
  if (!(ws.stride[0] == 1 || ws.size[0] <= 1)) return fail(ES_ERR_ARGUMENT, "workspace must be contiguous");
  if (uint64_t(rows) > uint64_t(INT64_MAX - 8) / (sizeof(es::RowResult) + uint64_t(vocab) * 20))
    return fail(ES_ERR_ARGUMENT, "workspace size overflow");
  if (own_scratch == 0) {
    uint64_t need = 0;
    es_workspace_bytes(rows, vocab, a->dispatch == ES_REFERENCE, &need);
    if (uint64_t(ws.size[0]) < need)
      return fail(ES_ERR_CAPACITY, a->dispatch == ES_REFERENCE
                                       ? "workspace capacity exceeded (the reference path needs a plan made with reference=True)"
                                       : "workspace capacity exceeded");
  } else if (es::workspace_needed(rows) > own_scratch) {
    return fail(ES_ERR_CAPACITY, "target rows exceed the static scratch of es_verify_static");
  }
  if (reinterpret_cast<uintptr_t>(ws.data) % 8 != 0) return fail(ES_ERR_ALIGNMENT, "workspace alignment must be 8 bytes");
  if (!check(a->tokens, ES_I64, 2, "tokens")) return ES_ERR_ARGUMENT;
  if (!(a->tokens.size[0] >= requests && a->tokens.size[1] >= a->max_draft + 1))
    return fail(ES_ERR_CAPACITY, "tokens capacity exceeded");
  const es_tensor* small[3] = {&a->accepted_len, &a->status, &a->path_used};
  for (const es_tensor* t : small) {
    if (!check(*t, ES_I32, 1, "output")) return ES_ERR_ARGUMENT;
    if (t->size[0] < requests) return fail(ES_ERR_CAPACITY, "output capacity exceeded");
  }
  const es_tensor* inputs[13] = {&logits, &a->cu_rows, &a->draft_ids, &a->temperature, &a->top_k, &a->top_p,
                                 &a->min_p, &a->draft_kind, &a->seeds, &a->stream_ids, &a->positions,
                                 has_draft ? &a->draft_logits : nullptr, has_mask ? &a->mask : nullptr};
  const es_tensor* outputs[5] = {&ws, &a->tokens, &a->accepted_len, &a->status, &a->path_used};
  for (int i = 0; i < 5; ++i) {
    if (!no_internal_overlap(*outputs[i])) return fail(ES_ERR_ALIAS, "output has overlapping strides");
    for (const es_tensor* in : inputs)
      if (in != nullptr && !disjoint(*outputs[i], *in))
        return fail(ES_ERR_ALIAS, "exactsample input/output aliasing is forbidden");
    for (int j = 0; j < i; ++j)
      if (!disjoint(*outputs[i], *outputs[j])) return fail(ES_ERR_ALIAS, "exactsample outputs alias");
  }
  if (sh != nullptr) {
    // Every GPU's buffers, laid out as this GPU's.
    for (int g = 0; g < sh->count; ++g)
      if (sh->target[g] == nullptr || sh->ready[g] == nullptr || sh->tokens[g] == nullptr ||
          sh->accepted[g] == nullptr || sh->status[g] == nullptr || sh->path[g] == nullptr ||
          (has_draft && sh->draft[g] == nullptr))
        return fail(ES_ERR_ARGUMENT, "shards: every GPU needs its shard, flag and output buffers");
    if (sh->target[sh->rank] != logits.data || (has_draft && sh->draft[sh->rank] != a->draft_logits.data) ||
        sh->tokens[sh->rank] != a->tokens.data || sh->accepted[sh->rank] != a->accepted_len.data ||
        sh->status[sh->rank] != a->status.data || sh->path[sh->rank] != a->path_used.data)
      return fail(ES_ERR_ARGUMENT, "shards: this GPU's entries must be the call's own tensors");
    const size_t e = element_size(logits.dtype);
    bool aligned = logits.stride[1] == 1 && (uint64_t(logits.stride[0]) * e) % 16 == 0;
    for (int g = 0; g < sh->count; ++g) {
      aligned &= reinterpret_cast<uintptr_t>(sh->target[g]) % 16 == 0;
      if (has_draft) aligned &= reinterpret_cast<uintptr_t>(sh->draft[g]) % 16 == 0;
    }
    if (has_draft) aligned &= a->draft_logits.stride[1] == 1 && a->draft_logits.stride[0] == logits.stride[0];
    if (!aligned) return fail(ES_ERR_ALIGNMENT, "shards: shard buffers must be contiguous rows on 16-byte boundaries");
    if (sh->phases) {
      for (int g = 0; g < sh->count; ++g)
        if (sh->exchange[g] == nullptr || reinterpret_cast<uintptr_t>(sh->exchange[g]) % 16 != 0)
          return fail(ES_ERR_ARGUMENT, "shards: a per-phase call needs every GPU's exchange buffer (16-byte aligned)");
      if (sh->scratch == nullptr || reinterpret_cast<uintptr_t>(sh->scratch) % 16 != 0)
        return fail(ES_ERR_ARGUMENT, "shards: a per-phase call needs this GPU's scratch (16-byte aligned)");
    }
  }
  if (requests == 0) return ES_SUCCESS;
  const int dev = device_check();
  if (dev != ES_SUCCESS) return dev;

  Params p{};
  p.target = logits.data; p.t_s0 = logits.stride[0]; p.t_s1 = logits.stride[1];
  if (has_draft) { p.draft = a->draft_logits.data; p.q_s0 = a->draft_logits.stride[0]; p.q_s1 = a->draft_logits.stride[1]; }
  p.cu_rows = static_cast<const int64_t*>(a->cu_rows.data); p.cu_s = a->cu_rows.stride[0];
  p.draft_ids = static_cast<const int64_t*>(a->draft_ids.data);
  p.d_s0 = a->draft_ids.stride[0]; p.d_s1 = a->draft_ids.stride[1];
  p.temperature = static_cast<const double*>(a->temperature.data); p.temp_s = a->temperature.stride[0];
  p.top_k = static_cast<const int64_t*>(a->top_k.data); p.topk_s = a->top_k.stride[0];
  p.top_p = static_cast<const double*>(a->top_p.data); p.topp_s = a->top_p.stride[0];
  p.min_p = static_cast<const double*>(a->min_p.data); p.minp_s = a->min_p.stride[0];
  p.draft_kind = static_cast<const int64_t*>(a->draft_kind.data); p.kind_s = a->draft_kind.stride[0];
  p.seeds = static_cast<const int64_t*>(a->seeds.data); p.seed_s = a->seeds.stride[0];
  p.streams = static_cast<const int64_t*>(a->stream_ids.data); p.stream_s = a->stream_ids.stride[0];
  p.positions = static_cast<const int64_t*>(a->positions.data); p.pos_s = a->positions.stride[0];
  if (has_mask) { p.mask = static_cast<const int32_t*>(a->mask.data); p.m_s0 = a->mask.stride[0]; p.m_s1 = a->mask.stride[1]; }
  p.workspace = static_cast<uint8_t*>(ws.data);
  p.tokens = static_cast<int64_t*>(a->tokens.data); p.tok_s0 = a->tokens.stride[0]; p.tok_s1 = a->tokens.stride[1];
  p.accepted = static_cast<int32_t*>(a->accepted_len.data); p.acc_s = a->accepted_len.stride[0];
  p.status = static_cast<int32_t*>(a->status.data); p.st_s = a->status.stride[0];
  p.path = static_cast<int32_t*>(a->path_used.data); p.path_s = a->path_used.stride[0];
  p.rows = int32_t(rows); p.requests = int32_t(requests); p.vocab = int32_t(vocab);
  p.max_draft = int32_t(a->max_draft); p.mode = int32_t(a->mode); p.dispatch = int32_t(a->dispatch);
  p.exact_draws = a->dispatch == ES_REFERENCE;
  p.list_max = p.exact_draws ? 0 : int32_t(a->list_max);
  p.offsets_inline = requests <= 8192;
  p.fast = !p.exact_draws && p.list_max > 0 && (sh == nullptr || sh->phases);
  p.col0 = 0;
  p.width = int32_t(vocab);
  if (sh != nullptr && sh->phases) {
    p.col0 = int32_t(int64_t(sh->rank) * sh->cols);
    p.width = int32_t(logits.size[1]);
  }
  p.warm = p.fast;
  if (const char* forced = std::getenv("EXACTSAMPLE_FAST")) {  // 0: the block-level list path only; 1: no warm-up warp
    if (forced[0] == '0') p.fast = p.warm = 0;
    if (forced[0] == '1') p.warm = 0;
  }
  if (sh != nullptr) {
    es::Shards& t = p.sh;
    t.count = sh->count;
    t.rank = sh->rank;
    t.cols = int32_t(sh->cols);
    t.req_begin = int32_t(sh->req_begin);
    t.req_end = int32_t(sh->req_end);
    t.epoch = sh->epoch;
    t.phases = sh->phases != 0;
    t.scratch = static_cast<uint8_t*>(sh->scratch);
    for (int g = 0; g < sh->count; ++g) {
      t.target[g] = sh->target[g];
      t.draft[g] = has_draft ? sh->draft[g] : nullptr;
      t.tokens[g] = static_cast<int64_t*>(sh->tokens[g]);
      t.accepted[g] = static_cast<int32_t*>(sh->accepted[g]);
      t.status[g] = static_cast<int32_t*>(sh->status[g]);
      t.path[g] = static_cast<int32_t*>(sh->path[g]);
      t.ready[g] = sh->ready[g];
      t.exchange[g] = static_cast<uint8_t*>(sh->exchange[g]);
    }
  }

  int cluster = 1;
  size_t smem = 0;
  if (rows > 0) {
    // A column-pulling sharded call finishes about rows / count of the rows
    // on this GPU; a per-phase one every row over this GPU's columns.
    const bool pulls = sh != nullptr && !sh->phases;
    const int64_t busy = pulls ? (rows + sh->count - 1) / sh->count : rows;
    const bool full_rows = p.exact_draws || a->list_max == 0;
    cluster = choose_cluster(busy, p.width, logits.dtype, full_rows, &p.slice_words, &smem, &p.stream_rows,
                             &p.min_blocks);
    if (cluster < 0) return fail(ES_ERR_UNSUPPORTED, "vocabulary too large for one 16-block cluster's shared memory");
    // The warm-up warp pays off where rows are split over ranks (one rank
    // per row leaves the chain after the statistics a smaller share) and
    // streamed: its dry run (about 20 us of cold instruction fetch) hides
    // behind a stream of 20 us or more, but would hold back the first
    // cluster exchange of resident rows, whose statistics take a few us.
    if (cluster < 2 || p.stream_rows == 0) p.warm = 0;
    const size_t e = element_size(logits.dtype);
    p.vector_load = logits.stride[1] == 1 && reinterpret_cast<uintptr_t>(logits.data) % 16 == 0 &&
                    (uint64_t(logits.stride[0]) * e) % 16 == 0;  // always so for shards (checked above)
  }
  cudaGetLastError();  // clear a stale error so the checks below report this call's launches
  if (!p.offsets_inline) es::check_offsets<<<1, 1024, 0, stream>>>(p);
  es::prepare<<<unsigned((requests + 127) / 128), 128, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  // dispatch="reference": the independent FP64 kernel (es_reference.cuh),
  // whose per-row scratch a reference-sized workspace always holds; a
  // smaller scratch (es_verify_static) takes the fused kernel's FP64-only draws.
  const uint64_t ws_bytes = own_scratch ? own_scratch : uint64_t(ws.size[0]);
  const bool reference_kernel = p.exact_draws && sh == nullptr &&
                                ws_bytes >= es::reference_scratch_offset(rows) + es::reference_scratch_bytes(rows, vocab);
  if (e == cudaSuccess && rows > 0 && reference_kernel) {
    if (before != nullptr) cudaEventRecord(before, stream);
    switch (logits.dtype) {
      case ES_F32: e = es::launch_reference<ES_F32>(p, stream); break;
      case ES_F64: e = es::launch_reference<ES_F64>(p, stream); break;
      case ES_F16: e = es::launch_reference<ES_F16>(p, stream); break;
      default: e = es::launch_reference<ES_BF16>(p, stream); break;
    }
    if (after != nullptr) cudaEventRecord(after, stream);
  } else if (e == cudaSuccess && rows > 0) {
    if (before != nullptr) cudaEventRecord(before, stream);
    switch (logits.dtype) {
      case ES_F32: e = es::launch_rows<ES_F32>(p, cluster, stream); break;
      case ES_F64: e = es::launch_rows<ES_F64>(p, cluster, stream); break;
      case ES_F16: e = es::launch_rows<ES_F16>(p, cluster, stream); break;
      default: e = es::launch_rows<ES_BF16>(p, cluster, stream); break;
    }
    if (after != nullptr) cudaEventRecord(after, stream);
  }
  if (e != cudaSuccess) return fail(ES_ERR_LAUNCH, std::string("exactsample kernel launch failed: ") + cudaGetErrorString(e));
  return ES_SUCCESS;
}

// ---- es_verify_static: scratch owned by the library ----
// One scratch area per device, in static device memory, for callers that
// cannot allocate device memory. It holds the per-call records that a
// caller-provided workspace would (flags, counters, one result, arrival
// counter and context record per target row): about 116 bytes per row, so
// 512 KiB covers ES_STATIC_MAX_ROWS rows.
constexpr uint64_t STATIC_SCRATCH_BYTES = 512 * 1024;
constexpr int MAX_DEVICES = 64;
static_assert(es::workspace_needed(ES_STATIC_MAX_ROWS) <= STATIC_SCRATCH_BYTES,
              "the static scratch holds the records of ES_STATIC_MAX_ROWS rows");
}  // namespace

static __device__ __align__(256) uint8_t es_static_scratch[STATIC_SCRATCH_BYTES];

namespace {
std::mutex g_scratch_mutex;
void* g_scratch[MAX_DEVICES] = {};

// The current device's scratch address, looked up on the first call made with
// that device current (this also loads the library's module on the device).
int static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(ES_ERR_DEVICE, "no CUDA device is available");
  if (dev < 0 || dev >= MAX_DEVICES) return fail(ES_ERR_DEVICE, "device ordinal beyond es_verify_static's table");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, es_static_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(ES_ERR_DEVICE, std::string("es_verify_static could not find its scratch on this device: ") +
                                     cudaGetErrorString(e));
    g_scratch[dev] = p;
  }
  *out = g_scratch[dev];
  return ES_SUCCESS;
}
}  // namespace

extern "C" {

int es_workspace_bytes(int64_t rows, int64_t vocab, int32_t reference, uint64_t* bytes) {
  if (rows < 0 || vocab < 1 || bytes == nullptr) return fail(ES_ERR_ARGUMENT, "invalid workspace shape");
  const uint64_t scratch = reference ? uint64_t(vocab) * 20 : 0;
  *bytes = 8 + uint64_t(rows) * (32 + (scratch > 12288 ? scratch : 12288));
  return ES_SUCCESS;
}

int es_verify(const es_args* args, void* stream) {
  return verify_impl(args, static_cast<cudaStream_t>(stream), nullptr, nullptr);
}

int es_verify_timed(const es_args* args, void* stream, void* before, void* after) {
  return verify_impl(args, static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(before),
                     static_cast<cudaEvent_t>(after));
}

int es_verify_static(const es_args* args, void* stream) {
  g_error.clear();
  if (args == nullptr) return fail(ES_ERR_ARGUMENT, "null arguments");
#ifdef ES_TRACE_PHASES
  // Phase traces are written past the per-row records, where only a
  // reference-sized workspace has room.
  return fail(ES_ERR_UNSUPPORTED, "es_verify_static is not available in a phase-tracing build");
#endif
  if (args->workspace.ndim != 0 || args->workspace.data != nullptr)
    return fail(ES_ERR_ARGUMENT, "es_verify_static uses its own scratch: leave workspace empty (zeroed)");
  if (args->target_logits.ndim == 2 && args->target_logits.size[0] > ES_STATIC_MAX_ROWS)
    return fail(ES_ERR_CAPACITY, "es_verify_static handles at most " + std::to_string(ES_STATIC_MAX_ROWS) +
                                     " target rows per call (got " + std::to_string(args->target_logits.size[0]) +
                                     "); use es_verify with a workspace for more");
  void* scratch = nullptr;
  if (const int rc = static_scratch(&scratch); rc != ES_SUCCESS) return rc;
  es_args a = *args;
  a.workspace.data = scratch;
  a.workspace.size[0] = int64_t(STATIC_SCRATCH_BYTES);
  a.workspace.stride[0] = 1;
  a.workspace.dtype = ES_U8;
  a.workspace.ndim = 1;
  return verify_impl(&a, static_cast<cudaStream_t>(stream), nullptr, nullptr, STATIC_SCRATCH_BYTES);
}

int es_verify_sharded(const es_args* args, const es_shards* shards, void* stream) {
  if (shards == nullptr) {
    g_error = "null shards";
    return ES_ERR_ARGUMENT;
  }
  return verify_impl(args, static_cast<cudaStream_t>(stream), nullptr, nullptr, 0, shards);
}

int es_shard_exchange_bytes(int64_t rows, uint64_t* bytes) {
  g_error.clear();
  if (rows < 0 || bytes == nullptr) return fail(ES_ERR_ARGUMENT, "invalid exchange shape");
  *bytes = uint64_t(rows) * sizeof(es::PhaseRow);
  return ES_SUCCESS;
}

int es_shard_signal(uint64_t* flag, uint64_t epoch, void* stream) {
  g_error.clear();
  if (flag == nullptr) return fail(ES_ERR_ARGUMENT, "null flag");
  if (const int dev = device_check(); dev != ES_SUCCESS) return dev;
  cudaGetLastError();
  es::signal_flag<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(flag, epoch);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ES_SUCCESS : fail(ES_ERR_LAUNCH, std::string("flag launch failed: ") + cudaGetErrorString(e));
}

int es_shard_wait(const uint64_t* const* flags, int32_t count, uint64_t epoch, uint32_t* timeouts, void* stream) {
  g_error.clear();
  if (flags == nullptr || count < 1 || count > es::MAX_SHARDS) return fail(ES_ERR_ARGUMENT, "flags: 1 to 8 flags");
  es::FlagSet f{};
  for (int g = 0; g < count; ++g) {
    if (flags[g] == nullptr) return fail(ES_ERR_ARGUMENT, "null flag");
    f.flag[g] = flags[g];
  }
  f.count = count;
  f.epoch = epoch;
  f.timeouts = timeouts;
  if (const int dev = device_check(); dev != ES_SUCCESS) return dev;
  cudaGetLastError();
  es::wait_flags<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(f);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ES_SUCCESS : fail(ES_ERR_LAUNCH, std::string("wait launch failed: ") + cudaGetErrorString(e));
}

int es_shard_finish(uint64_t* done, const uint64_t* const* flags, int32_t count, uint64_t epoch, uint32_t* timeouts,
                    void* stream) {
  g_error.clear();
  if (done == nullptr || flags == nullptr || count < 1 || count > es::MAX_SHARDS)
    return fail(ES_ERR_ARGUMENT, "flags: this GPU's slot array and 1 to 8 slot arrays");
  es::FlagSet f{};
  f.rank = -1;
  for (int g = 0; g < count; ++g) {
    if (flags[g] == nullptr) return fail(ES_ERR_ARGUMENT, "null flag");
    f.flag[g] = flags[g];
    if (flags[g] == done) f.rank = g;
  }
  if (f.rank < 0) return fail(ES_ERR_ARGUMENT, "this GPU's slot array must be one of the slot arrays");
  f.count = count;
  f.epoch = epoch;
  f.timeouts = timeouts;
  if (const int dev = device_check(); dev != ES_SUCCESS) return dev;
  cudaGetLastError();
  cudaLaunchConfig_t config{};
  config.gridDim = dim3(1);
  config.blockDim = dim3(32);
  config.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&config, es::finish_flags, done, f);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? ES_SUCCESS : fail(ES_ERR_LAUNCH, std::string("finish launch failed: ") + cudaGetErrorString(e));
}

int es_ipc_alloc(uint64_t bytes, void** ptr, void* handle) {
  g_error.clear();
  if (ptr == nullptr || handle == nullptr || bytes == 0) return fail(ES_ERR_ARGUMENT, "invalid allocation request");
  if (const int dev = device_check(); dev != ES_SUCCESS) return dev;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p != nullptr) cudaFree(p);
    return fail(ES_ERR_DEVICE, std::string("shared allocation failed: ") + cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return ES_SUCCESS;
}

int es_ipc_open(const void* handle, void** ptr) {
  g_error.clear();
  if (ptr == nullptr || handle == nullptr) return fail(ES_ERR_ARGUMENT, "invalid handle");
  if (const int dev = device_check(); dev != ES_SUCCESS) return dev;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? ES_SUCCESS : fail(ES_ERR_DEVICE, std::string("opening a peer's allocation failed: ") + cudaGetErrorString(e));
}

int es_ipc_close(void* ptr) {
  g_error.clear();
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? ES_SUCCESS : fail(ES_ERR_DEVICE, cudaGetErrorString(e));
}

int es_ipc_free(void* ptr) {
  g_error.clear();
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? ES_SUCCESS : fail(ES_ERR_DEVICE, cudaGetErrorString(e));
}

const char* es_last_error(void) { return g_error.c_str(); }

int es_abi_version(void) { return ES_ABI_VERSION; }

}  // extern "C"
