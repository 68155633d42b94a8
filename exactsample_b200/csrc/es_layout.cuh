// Kernel arguments, workspace layout and per-row records shared by the
// preparation kernel, the row kernel and the host launcher.
#pragma once
#include "es_device.cuh"

namespace es {

constexpr int LIST_MAX = 256;   // largest kept set finished as an FP64 list (the plan's list_max caps it)
static_assert(THREADS >= LIST_MAX, "one thread per list entry");
constexpr int CAP = 512;        // candidate buffer of a list row (cluster rank 0's shared memory)
static_assert(CAP >= LIST_MAX, "a list's kept tokens fit the candidate buffer");
constexpr int DIST_BINS = 128;  // distance-below-maximum bins of 0.5 logit, plus one "far" bin
constexpr int RADIX = 256;      // digits per radix-select level
#ifndef ES_RING_CHUNK
#define ES_RING_CHUNK 16384
#endif
#ifndef ES_RING_STAGES
#define ES_RING_STAGES 4
#endif
constexpr int MAX_RING_STAGES = ES_RING_STAGES;     // streamed rows: deepest TMA ring
constexpr uint32_t RING_CHUNK = ES_RING_CHUNK;      // bytes per ring stage
static_assert(RING_CHUNK % 1024 == 0 && RING_CHUNK <= 16384, "a ring stage holds whole 32-token tiles of any dtype");
constexpr uint32_t BULK_CHUNK = 16384; // bytes per TMA bulk copy

// Vocabulary-sharded calls: the row's columns live on `count` GPUs, shard g
// holding columns [g * cols, min(vocab, (g + 1) * cols)) in a buffer every
// GPU can read (the same layout on each: the target strides of Params). This
// GPU finishes requests [req_begin, req_end) and writes their outputs into
// every GPU's output buffers. count <= 1: not sharded.
constexpr int MAX_SHARDS = 8;
struct Shards {
  int32_t count, rank, cols;
  int32_t req_begin, req_end;
  int32_t pad;
  uint64_t epoch;                   // this call's number, the same on every GPU
  const void* target[MAX_SHARDS];
  const void* draft[MAX_SHARDS];
  int64_t* tokens[MAX_SHARDS];
  int32_t* accepted[MAX_SHARDS];
  int32_t* status[MAX_SHARDS];
  int32_t* path[MAX_SHARDS];
  const uint64_t* ready[MAX_SHARDS];  // each GPU's "shard written" flag (>= epoch once written)
  int32_t phases;                   // per-phase mode: every GPU streams only its shard (see PhaseRow)
  int32_t pad2;
  uint8_t* exchange[MAX_SHARDS];    // per-phase mode: each GPU's PhaseRow inboxes
  uint8_t* scratch;                 // per-phase mode: this GPU's FP64 scratch, 16 bytes per token per row
};

// One row's inbox in a GPU's exchange buffer (per-phase sharded calls): a
// slot per GPU, which that GPU fills with remote stores, so that every
// reader polls its own memory. A slot holds the GPU's row statistics and its
// tile-maximum bins (from its own top bin down), then its best window
// candidates (global token IDs). Every entry is one 64-bit word: a 32-bit
// datum below the call's 32-bit tag (the epoch, never 0), stored and loaded
// whole, so a reader that sees its call's tag in a word also sees that
// word's datum, with no fence and no separate flag.
constexpr int PHASE_BINS = 128;
constexpr int PHASE_SEND = 64;  // candidates a GPU sends for a row, at most (its first in the order)
constexpr int PHASE_STAT_WORDS = 4 + PHASE_BINS / 2;  // max (low, high), valid, bad | (top bin + 1) << 1, bins in pairs
constexpr int PHASE_COUNT_WORD = PHASE_STAT_WORDS;    // candidates sent, or PHASE_OVERFLOW
constexpr int PHASE_SLOT_WORDS = PHASE_COUNT_WORD + 1 + 3 * PHASE_SEND;  // then key low, key high, ID each
constexpr uint32_t PHASE_OVERFLOW = 0xffffffffu;
struct alignas(16) PhaseRow {
  uint64_t slot[MAX_SHARDS][PHASE_SLOT_WORDS];
};
static_assert(sizeof(PhaseRow) % 16 == 0, "PhaseRow keeps 16-byte alignment");
static_assert(MAX_SHARDS * PHASE_SEND <= CAP, "every GPU's candidates fit the candidate buffer");

// Kernel arguments (filled by es_verify from es_args); strides in elements.
struct Params {
  const void* target;
  int64_t t_s0, t_s1;
  const void* draft;
  int64_t q_s0, q_s1;
  const int64_t* cu_rows;
  int64_t cu_s;
  const int64_t* draft_ids;
  int64_t d_s0, d_s1;
  const double* temperature;
  int64_t temp_s;
  const int64_t* top_k;
  int64_t topk_s;
  const double* top_p;
  int64_t topp_s;
  const double* min_p;
  int64_t minp_s;
  const int64_t* draft_kind;
  int64_t kind_s;
  const int64_t* seeds;
  int64_t seed_s;
  const int64_t* streams;
  int64_t stream_s;
  const int64_t* positions;
  int64_t pos_s;
  const int32_t* mask;
  int64_t m_s0, m_s1;
  uint8_t* workspace;
  int64_t* tokens;
  int64_t tok_s0, tok_s1;
  int32_t* accepted;
  int64_t acc_s;
  int32_t* status;
  int64_t st_s;
  int32_t* path;
  int64_t path_s;
  int32_t rows, requests, vocab, max_draft;
  int32_t mode, dispatch, list_max;
  int32_t slice_words;     // 32-token mask words per cluster rank
  int32_t vector_load;     // rows contiguous and 16-byte aligned: TMA bulk loads
  int32_t offsets_inline;  // the preparation kernel validates cu_rows itself
  int32_t exact_draws;     // dispatch="reference": every draw scored in FP64, no lists
  int32_t stream_rows;     // 0: rows stay in shared memory; else the depth (2..4) of the TMA ring they stream through
  int32_t min_blocks;      // blocks per SM the row kernel's registers must allow (2, or 3 for large streamed batches)
  int32_t fast;            // list rows of at most FAST_KEEP kept tokens may take the warp-level path (es_fast.cuh)
  int32_t col0, width;     // this call's columns: [col0, col0 + width) of the vocab (col0 > 0 only for a per-phase shard)
  int32_t warm;            // the row kernel has a warm-up warp past its THREADS row threads
  Shards sh;
};

// One GPU's output buffers (the caller's, or shard g's in a sharded call).
struct Outputs {
  int64_t* tokens;
  int32_t *accepted, *status, *path;
};
__device__ __forceinline__ bool pulls_columns(const Params& p) { return p.sh.count > 1 && !p.sh.phases; }
__device__ __forceinline__ int output_sets(const Params& p) { return pulls_columns(p) ? p.sh.count : 1; }
__device__ __forceinline__ Outputs output_set(const Params& p, int i) {
  if (pulls_columns(p)) return Outputs{p.sh.tokens[i], p.sh.accepted[i], p.sh.status[i], p.sh.path[i]};
  return Outputs{p.tokens, p.accepted, p.status, p.path};
}

// Per-row outcome, written by the row's cluster rank 0 and read by whichever
// row of the request finishes last.
struct RowResult {
  int32_t target_status;  // status of the target distribution
  int32_t status;         // target status, else the proposal's
  int32_t accept;         // ratio mode: the draft was accepted
  int32_t sample;         // substream-0 draw (bonus rows, coupled mode)
  int32_t residual;       // substream-2 draw after a rejection (-1: no residual mass)
  int32_t pad[3];
};
static_assert(sizeof(RowResult) == 32, "RowResult is 32 bytes");

// A row's request and parameters, gathered by the preparation kernel so the
// row kernel fetches them with one round trip.
struct alignas(16) RowCtx {
  int32_t req, begin, end, draft_id, kind, skip;  // skip: the request failed its metadata checks
  uint32_t stream, position;
  int32_t top_k, pad0;
  double temperature, top_p, min_p;
  uint64_t seed;
  uint64_t pad1;
};
static_assert(sizeof(RowCtx) == 80, "RowCtx is 80 bytes");

// Counters kept after the per-row arrays (reset by the preparation kernel).
struct Diagnostics {
  uint32_t near_ties;       // exact sums whose rounding sat within the fixed-point slack of a tie
  uint32_t wait_timeouts;   // bounded waits that gave up
  uint32_t check_failures;  // checked builds (-DES_CHECKS): bounds checks that failed (their access skipped)
  uint32_t first_site;      // checked builds: the site number of the first failed check
  uint32_t pad[12];
};
static_assert(sizeof(Diagnostics) == 64, "Diagnostics is 64 bytes");

// Workspace (bytes): [0] malformed-offsets flag, [4] FP64 recomputation count,
// [8] RowResult[rows], then one arrival counter per row (used at each
// request's first row), then Diagnostics, then RowCtx[rows] (at the next
// 16-byte aligned address: the workspace itself need only be 8-byte aligned).
// Always within the reference's 8 + rows * (32 + 12288) bytes.
__host__ __device__ inline int32_t* malformed_flag(uint8_t* ws) { return reinterpret_cast<int32_t*>(ws); }
__host__ __device__ inline uint32_t* fallback_count(uint8_t* ws) { return reinterpret_cast<uint32_t*>(ws + 4); }
__host__ __device__ inline RowResult* row_results(uint8_t* ws) { return reinterpret_cast<RowResult*>(ws + 8); }
__host__ __device__ inline uint32_t* arrivals(uint8_t* ws, int64_t rows) {
  return reinterpret_cast<uint32_t*>(ws + 8 + rows * sizeof(RowResult));
}
__host__ __device__ inline Diagnostics* diagnostics(uint8_t* ws, int64_t rows) {
  return reinterpret_cast<Diagnostics*>(ws + 8 + rows * (sizeof(RowResult) + 4));
}
__host__ __device__ inline RowCtx* row_contexts(uint8_t* ws, int64_t rows) {
  const uintptr_t at = reinterpret_cast<uintptr_t>(ws) + 8 + rows * (sizeof(RowResult) + 4) + sizeof(Diagnostics);
  return reinterpret_cast<RowCtx*>((at + 15) & ~uintptr_t(15));
}

// Bytes used, whatever the workspace's alignment: at most 8 + 116 * rows + 79,
// far below the 8 + 12320 * rows provided.
__host__ __device__ constexpr uint64_t workspace_needed(int64_t rows) {
  if (rows == 0) return 8;
  return 8 + uint64_t(rows) * (sizeof(RowResult) + 4) + sizeof(Diagnostics) + 15 + uint64_t(rows) * sizeof(RowCtx);
}

template <class T> __device__ __forceinline__ T at(const T* p, int64_t stride, int64_t i) { return p[i * stride]; }

// Bounds checks of checked builds (-DES_CHECKS), the stand-in for a memory
// checker where none may run: ES_IN_BOUNDS(ws, rows, cond, site) is cond;
// a false cond adds one to the workspace's check_failures, records the first
// failing site, and the caller skips the access. Nothing traps. In other
// builds the macro is `true` and costs nothing.
#ifdef ES_CHECKS
static __device__ __noinline__ void check_failed(uint8_t* ws, int64_t rows, uint32_t site);
#define ES_IN_BOUNDS(ws, rows, cond, site) ((cond) ? true : (es::check_failed((ws), (rows), (site)), false))
#else
#define ES_IN_BOUNDS(ws, rows, cond, site) true
#endif

// Phase timestamps for development builds (-DES_TRACE_PHASES): rank r of row
// `row` stores %globaltimer at phase k in the workspace past every record
// this file lays out (the reference-sized workspace has room for them).
#ifdef ES_TRACE_PHASES
__device__ __forceinline__ void trace_phase(uint8_t* ws, int64_t rows, int row, int rank, int k) {
  if (threadIdx.x != 0) return;
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  reinterpret_cast<uint64_t*>(ws + 8 + rows * 1024)[(int64_t(row) * 16 + rank) * 32 + k] = t;
}
#define ES_TRACE(ws, rows, row, rank, k) trace_phase(ws, rows, row, rank, k)
#else
#define ES_TRACE(ws, rows, row, rank, k) ((void)0)
#endif

}  // namespace es
