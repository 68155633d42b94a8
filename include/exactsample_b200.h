/*
 * exactsample_b200: C ABI of the B200 (sm_100a) sampling and speculative-
 * verification kernels.
 *
 * This header replaces the reference's C++ ABI
 *   include/exactsample/api.h:7-44   (Status, Path, DType, Matrix, Vector,
 *                                     RowResult, Arguments, workspace_size,
 *                                     exactsample::launch)
 * and the argument checks of its torch binding
 *   csrc/bindings.cpp:45-136          (verify_out: dtype, rank, capacity,
 *                                     alignment and aliasing checks)
 * with plain C: every tensor is a pointer plus sizes and strides (in
 * elements), and every error is a negative return code with a message.
 *
 * Semantics are those of the exactsample decoding contract v1.0
 * (docs/contract.md, docs/rng.md of the reference): per-request statuses,
 * tokens -1 on failure, Philox4x32-10 at (seed, stream, position, substream,
 * token / 4).
 *
 * Ownership and threading: every buffer is caller-owned device memory on the
 * current CUDA device; es_verify only enqueues kernels on `stream` and never
 * allocates or synchronizes. One call at a time may use a given workspace
 * (calls on one stream are ordered; overlapping calls on different streams
 * that share a workspace race).
 */
#ifndef EXACTSAMPLE_B200_H
#define EXACTSAMPLE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ES_ABI_VERSION 1

/* Per-request status (api.h:7, docs/contract.md "Shapes and failure boundaries"). */
enum es_status { ES_OK = 0, ES_NO_VALID_TOKEN = 1, ES_INVALID_INPUT = 2, ES_DRAFT_ZERO_PROB = 3 };
/* path_used values (api.h:8). */
enum es_path { ES_PATH_REFERENCE = 0, ES_PATH_FUSED = 1 };
/* Element types (api.h:9 for the logits; the rest name the other tensors). */
enum es_dtype { ES_F32 = 0, ES_F64 = 1, ES_F16 = 2, ES_BF16 = 3, ES_I32 = 4, ES_I64 = 5, ES_U8 = 6 };
/* Verification mode and dispatch (api.h:32; cuda.py:149-150). */
enum es_mode { ES_RATIO = 0, ES_COUPLED = 1 };
enum es_dispatch { ES_AUTO = 0, ES_REFERENCE = 1, ES_FUSED = 2 };

/* Return codes. Structural problems are reported before anything is
 * enqueued; per-request numerical problems are statuses, not errors. */
enum es_error {
  ES_SUCCESS = 0,
  ES_ERR_ARGUMENT = -1,    /* a tensor has the wrong dtype, rank, shape or a negative stride */
  ES_ERR_CAPACITY = -2,    /* workspace or output too small */
  ES_ERR_ALIGNMENT = -3,   /* workspace not 8-byte aligned */
  ES_ERR_ALIAS = -4,       /* an output overlaps an input or another output */
  ES_ERR_UNSUPPORTED = -5, /* a shape this build does not handle (e.g. vocab too large for one cluster) */
  ES_ERR_LAUNCH = -6,      /* a CUDA launch failed (message has cudaGetErrorString) */
  ES_ERR_DEVICE = -7       /* the current device is not an sm_100 GPU */
};

/* A strided view of at most two dimensions; sizes and strides in elements.
 * A 1-D tensor uses size[0] / stride[0]. A zeroed descriptor (ndim == 0)
 * marks an absent optional tensor (draft_logits, mask); data may be NULL
 * only for a tensor with no elements. */
typedef struct es_tensor {
  void* data;
  int64_t size[2];
  int64_t stride[2];
  int32_t dtype; /* enum es_dtype */
  int32_t ndim;
} es_tensor;

/* The arguments of one call (api.h:20-35 Arguments; bindings.cpp:139-146
 * schema of exactsample::verify_out, in the same order). */
typedef struct es_args {
  es_tensor target_logits; /* f32/f64/f16/bf16 [rows, vocab] */
  es_tensor cu_rows;       /* i64 [requests + 1] */
  es_tensor draft_ids;     /* i64 [requests, >= max_draft] */
  es_tensor draft_logits;  /* optional, target dtype and shape */
  es_tensor temperature;   /* f64 [requests] */
  es_tensor top_k;         /* i64 [requests], 0 disables */
  es_tensor top_p;         /* f64 [requests] */
  es_tensor min_p;         /* f64 [requests] */
  es_tensor draft_kind;    /* i64 [requests], 0 one-hot, 1 full */
  es_tensor seeds;         /* i64 [requests], uint64 bits */
  es_tensor stream_ids;    /* i64 [requests], [0, 2^32) */
  es_tensor positions;     /* i64 [rows], [0, 2^32) */
  es_tensor mask;          /* optional i32 [rows, ceil(vocab / 32)] */
  es_tensor workspace;     /* u8 [>= es_workspace_bytes], contiguous, 8-byte aligned */
  es_tensor tokens;        /* out i64 [>= requests, >= max_draft + 1] */
  es_tensor accepted_len;  /* out i32 [>= requests] */
  es_tensor status;        /* out i32 [>= requests] */
  es_tensor path_used;     /* out i32 [>= requests] */
  int64_t mode;            /* enum es_mode */
  int64_t dispatch;        /* enum es_dispatch */
  int64_t max_draft;
  int64_t list_max;        /* [0, 256]: largest kept set processed as an FP64 list; 0 skips lists */
} es_args;

/* Workspace bytes for `rows` target rows (api.h:39-43 workspace_size, and
 * cuda.py:89): 8 + rows * (32 + max(12288, 20 * vocab if reference)). */
int es_workspace_bytes(int64_t rows, int64_t vocab, int32_t reference, uint64_t* bytes);

/* Validates the arguments and enqueues the call on `stream` (a
 * cudaStream_t; NULL is the legacy default stream). Replaces
 * exactsample::launch (api.h:44, csrc/verify/verify.cu:220-228) together
 * with the checks of bindings.cpp:50-119. */
int es_verify(const es_args* args, void* stream);

/* The same call, with `before` and `after` (cudaEvent_t, either may be NULL)
 * recorded on `stream` immediately around the row kernel. Measurement only:
 * it exists so that benchmarks can time the dominant kernel by itself. */
int es_verify_timed(const es_args* args, void* stream, void* before, void* after);

/* es_verify without a caller-provided workspace. No counterpart in the
 * reference, whose launch always takes the caller's workspace.
 *
 * For callers that cannot allocate device memory: for example a sampler
 * plugin inside a serving engine that reserves all of the GPU's memory up
 * front and hands its plugins no scratch buffer, or a C host that has no
 * device allocator of its own. The call allocates nothing (no cudaMalloc or
 * cudaFree, no allocating library routine): its scratch is a fixed area of
 * static device memory in this library, one per device, of 512 KiB, enough
 * for ES_STATIC_MAX_ROWS target rows. A call with more rows returns
 * ES_ERR_CAPACITY before anything is enqueued. `args->workspace` must be left
 * empty (zeroed); every other field means what it means for es_verify.
 *
 * The first call on a device does the set-up: it looks up that device's
 * scratch address (cudaGetSymbolAddress, with the device current), which also
 * loads the library's kernels there. Make that first call before any stream
 * capture. The address is kept for the life of the process, so resetting the
 * device (cudaDeviceReset) after that first call is not supported.
 *
 * The scratch needs no clearing between calls: each call's first kernel
 * writes every flag, counter and per-row record that its later kernels read.
 * But it is one area per device, shared by every call on that device: calls
 * queued on one stream are ordered, while calls that overlap on different
 * streams race on the scratch and give wrong results. Serialize them. */
#define ES_STATIC_MAX_ROWS 4096
int es_verify_static(const es_args* args, void* stream);

/* ---- Vocabulary-sharded calls (no counterpart in the reference) ----
 *
 * N GPUs (2..8, one process each) hold contiguous shards of the vocabulary of
 * every row: shard g holds columns [g * cols, min(vocab, (g + 1) * cols)),
 * cols a multiple of 16, in a buffer every GPU can read (es_ipc_alloc on its
 * owner, es_ipc_open on the others). All other inputs are replicated. Each
 * GPU finishes the requests [req_begin, req_end), streaming their full rows
 * (its own shard from HBM, the others' over NVLink with TMA bulk copies), and
 * writes their outputs into every GPU's output buffers, which must therefore
 * be registered buffers too. Results are identical to an unsharded call.
 *
 * One call on each GPU, all with the same arguments and epoch (a call
 * number, increasing from 1), in this order on the GPU's stream, after this
 * GPU's shard is written:
 *   es_verify_sharded(args, shards)        raises this GPU's ready flag, and
 *                                          waits for every GPU's before
 *                                          reading a shard;
 *   es_shard_finish(slots[rank], slots, count, epoch)
 *                                          stores this GPU's tag into its
 *                                          slot of every GPU's slot array
 *                                          and waits for every GPU's tag in
 *                                          its own: afterwards every GPU's
 *                                          outputs are complete and no GPU
 *                                          reads this GPU's shard or buffers.
 *                                          slots[g] is GPU g's array of
 *                                          `count` 64-bit words (zeroed when
 *                                          allocated), readable and writable
 *                                          by every GPU.
 * es_shard_signal and es_shard_wait raise one flag and wait for a set of
 * flags (es_shard_signal on the ready flag is the first step of
 * es_verify_sharded), for a caller that runs several shards on one GPU and
 * must issue every shard's signal before any shard's wait: a done flag per
 * shard takes the place of the slot arrays there.
 * Every wait is bounded (about a second): a wait that gives up marks the
 * affected rows INVALID_INPUT (es_verify_sharded) or adds one to *timeouts
 * (es_shard_wait). */
#define ES_MAX_SHARDS 8
typedef struct es_shards {
  int32_t count;          /* GPUs holding shards, 2..ES_MAX_SHARDS */
  int32_t rank;           /* this GPU's shard */
  int64_t cols;           /* columns per shard (the last holds the rest) */
  int64_t vocab;          /* columns of the whole row */
  int64_t req_begin;      /* requests this GPU finishes: [req_begin, req_end) */
  int64_t req_end;
  uint64_t epoch;         /* this call's number, the same on every GPU */
  const void* target[ES_MAX_SHARDS];  /* every GPU's target shard buffer; [rank] is args->target_logits */
  const void* draft[ES_MAX_SHARDS];   /* every GPU's draft shard buffer (full-q drafts), else NULL */
  void* tokens[ES_MAX_SHARDS];        /* every GPU's outputs, laid out as args' outputs */
  void* accepted[ES_MAX_SHARDS];
  void* status[ES_MAX_SHARDS];
  void* path[ES_MAX_SHARDS];
  const uint64_t* ready[ES_MAX_SHARDS];  /* every GPU's "shard written" flag */
  /* Per-phase mode (phases != 0): every GPU reads only its own shard and
   * finishes every request into its own outputs; the GPUs exchange per-row
   * partial results (statistics and tile-maximum bins, then each GPU's best
   * window candidates): each GPU stores its own into every GPU's exchange
   * buffer (es_shard_exchange_bytes bytes, zeroed when allocated, writable
   * by every GPU) and reads the others' from its own. Rows the exchange
   * cannot finish (no window, more than 64 candidates on a GPU that must cut
   * them, or a request outside the top-k list path: greedy, full-q drafts,
   * masks, lists over 256) are finished by the independent FP64 path
   * reading the whole row from every shard, with `scratch` (rows * vocab *
   * 16 bytes of this GPU's memory). req_begin and req_end must cover every
   * request, and target/draft/ready/tokens/... keep their meaning (only this
   * GPU's output pointers are written). */
  int32_t phases;
  int32_t pad;
  void* exchange[ES_MAX_SHARDS];
  void* scratch;
} es_shards;

/* Bytes of one GPU's exchange buffer for a per-phase sharded call of up to
 * `rows` target rows. No counterpart in the reference. */
int es_shard_exchange_bytes(int64_t rows, uint64_t* bytes);

/* es_verify for one GPU of a sharded call: args->target_logits (and
 * draft_logits) are this GPU's shard [rows, its columns]; draft_ids, mask
 * and the rest describe the whole rows (vocab = shards->vocab). */
int es_verify_sharded(const es_args* args, const es_shards* shards, void* stream);
/* Stores `epoch` into `flag` (this GPU's ready or done flag) once the
 * stream's earlier work is done. */
int es_shard_signal(uint64_t* flag, uint64_t epoch, void* stream);
/* Waits on the stream until every flags[i] (i < count) has reached `epoch`. */
int es_shard_wait(const uint64_t* const* flags, int32_t count, uint64_t epoch, uint32_t* timeouts, void* stream);
/* This GPU's tag into slot `rank` of every GPU's slot array (rank: the
 * index of `done`, this GPU's array, in `flags`, every GPU's), then a wait
 * for every GPU's tag in `done`; one launch, which waits on the device for
 * the stream's earlier kernels. */
int es_shard_finish(uint64_t* done, const uint64_t* const* flags, int32_t count, uint64_t epoch, uint32_t* timeouts,
                    void* stream);
/* Device memory other processes on this node can map: es_ipc_alloc returns a
 * zeroed allocation and its 64-byte handle; es_ipc_open maps a handle made
 * by another process (es_ipc_close unmaps it, es_ipc_free frees one's own). */
int es_ipc_alloc(uint64_t bytes, void** ptr, void* handle);
int es_ipc_open(const void* handle, void** ptr);
int es_ipc_close(void* ptr);
int es_ipc_free(void* ptr);

/* The message of the last error returned on this thread ("" after success). */
const char* es_last_error(void);

/* ES_ABI_VERSION of the loaded library. */
int es_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* EXACTSAMPLE_B200_H */
