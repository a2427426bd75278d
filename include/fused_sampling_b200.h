/*
 * fused_sampling_b200.h -- C ABI of the B200 (sm_100a) fused top-k / top-p token sampler.
 *
 * Hot path: [B, V] FP16/BF16 logits -> [B] int64 token ids, in one kernel launch per call.
 * Stage order and semantics are those of the reference operator (sathviknookala/llm_sampling_kernel):
 *   top-k (exactly k, ties to the lowest token id) -> FP32 softmax over the k survivors ->
 *   cumulative sum -> exclusive-prefix top-p cut (keep i iff c_{i-1} < p; p >= 1 keeps all) ->
 *   inverse-CDF draw: first i <= r with cum_i >= u * cum_r.
 *
 * Every entry point is asynchronous on the given stream, never aborts, never traps, and allocates
 * nothing: outputs (and, where stated, workspace) are caller-owned device memory.
 * Plain C types only; the stream is a cudaStream_t (NULL = legacy default stream).
 *
 * Reference interfaces each entry point replaces are cited as path:line inside the reference
 * project.
 */
#ifndef FUSED_SAMPLING_B200_H
#define FUSED_SAMPLING_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FS_API __attribute__((visibility("default")))
#else
#define FS_API
#endif

/* Binary-compatible with cudaStream_t. */
typedef struct CUstream_st* fs_stream_t;

typedef enum fs_status {
  FS_OK = 0,
  FS_EINVAL = 1,        /* invalid argument: shape, k, p, null pointer, stride           */
  FS_EUNSUPPORTED = 2,  /* valid request outside what this build implements             */
  FS_ELAUNCH = 3,       /* a CUDA launch / attribute call failed (see fs_last_error)     */
  FS_ETIMEOUT = 4,      /* a bounded device-side wait ran out (multi-GPU exchange)       */
  FS_EWORKSPACE = 5     /* workspace pointer missing or smaller than fs_*_workspace_size */
} fs_status;

typedef enum fs_dtype { FS_F16 = 0, FS_BF16 = 1 } fs_dtype;

/* Per-row status codes written to row_status (when non-NULL). A row with a non-zero status
 * gets token id -1, keep = 0 and renormed = 0; its input matches the rejections of the
 * reference's validate_logits (benchmarks/reference.py:20-26). */
enum {
  FS_ROW_OK = 0,
  FS_ROW_NAN = 1,         /* "logits contain NaN"                          */
  FS_ROW_POSINF = 2,      /* "logits contain +inf"                         */
  FS_ROW_ALL_NEGINF = 3,  /* "logits contain a row that is entirely -inf"  */
  FS_ROW_BAD_PARAM = 4,   /* per-row k < 1, or per-row p outside (0, 1]     */
  FS_ROW_TIMEOUT = 5      /* a bounded device wait of the launch ran out: no result for the row */
};

/* Source of the per-row uniform u in [0, 1), in priority order:
 *   uniforms != NULL : u = uniforms[b]                      (caller-supplied)
 *   seed_ptr != NULL : seed = *seed_ptr, offset = *offset_ptr + offset_intragraph
 *                      (graph-captured torch generator state, at::PhiloxCudaState "captured")
 *   otherwise        : seed, offset by value.
 * The generated uniform is the reference's splitmix64 contract
 * (csrc/fused_sampling.cuh:65-71) evaluated at row index (row_base + b). */
typedef struct fs_rng {
  const float* uniforms;
  uint64_t seed;
  uint64_t offset;
  const int64_t* seed_ptr;
  const int64_t* offset_ptr;
  uint64_t offset_intragraph;
  int64_t row_base;
} fs_rng;

typedef struct fs_sample_args {
  const void* logits;        /* device, rows of 16-bit floats                            */
  int32_t dtype;             /* fs_dtype                                                 */
  int64_t batch;             /* B >= 1 (<= 65535)                                        */
  int64_t vocab;             /* V >= 1 (<= 1 << 19)                                      */
  int64_t row_stride;        /* elements between row starts, >= V                        */
  int64_t id_base;           /* added to every emitted id (vocab-shard offset), else 0   */
  int64_t top_k;             /* k >= 1, clamped to V; with top_k_rows, the bound K       */
  float top_p;               /* p in (0, 1]; ignored when top_p_rows != NULL             */
  const int32_t* top_k_rows; /* optional device [B] per-row k (each clamped to K)        */
  const float* top_p_rows;   /* optional device [B] per-row p                            */
  fs_rng rng;
  int64_t* out_ids;          /* device [B] sampled ids (required by fs_sample)           */
  int64_t* topk_ids;         /* optional device [B, K]: top-K ids, value desc, id asc    */
  uint8_t* keep;             /* optional device [B, K]: nucleus mask                     */
  float* renormed;           /* optional device [B, K]: p_i / Z_p inside the nucleus     */
  int32_t* row_status;       /* optional device [B]: FS_ROW_*                            */
  int32_t splits;            /* 0 = auto; else CTAs per row (1..16, rounded up to 2^n)    */
  int32_t stop_phase;        /* 0 = full pipeline; 1..FS_NUM_PHASES ablation stop point  */
  int32_t path;              /* FS_PATH_* (AUTO = 0 picks)                               */
  void* workspace;           /* device scratch for the streaming and wide paths (below)  */
  uint64_t workspace_bytes;  /* its size; >= fs_workspace_size(args)                     */
  float temperature;         /* softmax temperature T > 0; 0 or 1 = none (see below)     */
  uint32_t input_flags;      /* FS_INPUT_* bits (0: none)                                */
} fs_sample_args;

/* input_flags. FS_INPUT_READY: the logits are complete when the call is enqueued -- nothing still
 * running on the GPU writes them (e.g. host memory the CPU filled before the call, or a buffer
 * written by a kernel that has finished). The cluster path then issues its reads of the logits
 * before it waits for the stream's previous kernel (programmatic dependent launch), so that for
 * logits in pinned host memory the transfer over PCIe overlaps the previous call. Without the
 * flag the reads follow that wait, which is what a producer that lets its dependents start early
 * requires. No counterpart in the reference (its operators take device tensors only). */
#define FS_INPUT_READY 1u

/* Pointers marked "device" above may be any address the kernels can dereference on the current
 * device: device memory, or pinned host memory mapped into the device's address space (memory
 * from cudaHostAlloc / cudaMallocHost under unified addressing; pass the address that
 * cudaPointerGetAttributes reports as devicePointer). Logits in pinned host memory are then read
 * in place over PCIe and the outputs written there, with no copy-engine transfer; the caller keeps
 * those buffers alive and unmodified until the stream has passed the call. The workspace, the
 * per-row k / p / uniform arrays and the generator pointers stay in device memory. */

/* Temperature. The selected candidates' logits are divided by T in IEEE fp32 before the softmax,
 * which is what sampling fp32 logits / T gives (the convention of a temperature warper applied to
 * fp32 logits ahead of the top-k / top-p warpers). The selection itself is unchanged: fp32
 * division by T > 0 is strictly increasing on 16-bit float inputs, so the top-k set and its order
 * (value desc, id asc) are those of the raw logits. A row whose largest scaled logit overflows to
 * +inf gets FS_ROW_POSINF, as an infinite logit would. T < 0, NaN or inf: FS_EINVAL. */

/* Execution paths. CLUSTER: one launch, one thread-block cluster per row, no workspace (the
 * latency path). STREAM: two launches - independent CTAs per row slice write candidate lists to
 * the workspace, one warp per row merges them (the throughput path for large batches, k <= 256).
 * WIDE: any top_k up to V (top-p only when top_k >= V); nothing is sorted: a per-key count
 * histogram of each row (workspace: 256 KiB per row, cleared by the call) and exact fixed-point
 * probability masses per key locate the cut and the draw (a memset and four launches). It
 * produces token ids and row status only (no topk_ids / keep / renormed); AUTO takes it when
 * top_k exceeds the 8192-candidate buffer of the other paths.
 * AUTO picks by batch size and k. All paths compute the same ids. */
enum { FS_PATH_AUTO = 0, FS_PATH_CLUSTER = 1, FS_PATH_STREAM = 2, FS_PATH_WIDE = 3 };

#define FS_NUM_PHASES 7

/* Bytes of device workspace the call described by args needs (0 when its path needs none).
 * The workspace holds per-call scratch only (candidate lists, key histograms): no state persists
 * between calls, and it needs no initialisation. Calls that may run concurrently need separate
 * workspaces. */
FS_API uint64_t fs_workspace_size(const fs_sample_args* args);

/* Fused top-k + top-p + sample, [B, V] -> [B].
 * Replaces: sample_fused / stages_fused / run_fused  (csrc/fused_sampling.cu:426-458,503-513)
 * and the pybind entries sample_fused, stages_fused (csrc/bindings.cpp:20,22). */
FS_API fs_status fs_sample(const fs_sample_args* args, fs_stream_t stream);

/* fs_sample without a caller workspace (no counterpart in the reference). For callers that
 * cannot allocate device memory at call time. The scratch of the streaming and wide paths is one
 * static device array of FS_STATIC_SCRATCH_BYTES per device; a call that needs more returns
 * FS_EWORKSPACE. args->workspace is ignored. The first call on a device (and the first after a
 * cudaDeviceReset, which loads the module again) looks the array up (cudaGetSymbolAddress): make
 * it before any stream capture. Nothing is allocated or freed per call (the wide path clears its
 * part of the array on the stream). Calls that overlap in time (other streams, other host
 * threads) share the array and race: serialise them. */
#define FS_STATIC_SCRATCH_BYTES (16ull << 20)
FS_API fs_status fs_sample_noalloc(const fs_sample_args* args, fs_stream_t stream);

/* Top-K candidate ids only ([B, K] into args->topk_ids; out_ids may be NULL).
 * Replaces: topk_fused (csrc/fused_sampling.cu:460-473, csrc/bindings.cpp:21). */
FS_API fs_status fs_topk(const fs_sample_args* args, fs_stream_t stream);

/* Ablation: run the pipeline up to phase args->stop_phase (1..FS_NUM_PHASES) and write a
 * phase-dependent int64 per row into out_ids. Phase FS_NUM_PHASES is the production path.
 * Replaces: probe_phase (csrc/fused_sampling.cu:475-501, csrc/bindings.cpp:23). */
FS_API fs_status fs_probe_phase(const fs_sample_args* args, fs_stream_t stream);

/* ---- vocab-sharded tensor parallelism (no counterpart in the reference) -------------------
 * Packed candidate = (order_key << 32) | (0xFFFFFFFF - global_id), where order_key is the
 * 16-bit order-preserving key of the logit (-0 folded onto +0). Larger packed value = larger
 * logit, lower id on ties. Each row of a candidate block holds K packed candidates sorted
 * descending, followed by one status word (FS_ROW_* of the shard row). Padding is 0. */

/* Local half: top-K candidates of a [B, V_shard] shard, ids offset by args->id_base.
 * cand_out: device [B, K + 1] uint64. Uses args: logits, dtype, batch, vocab, row_stride,
 * id_base, top_k, splits. */
FS_API fs_status fs_shard_candidates(const fs_sample_args* args, uint64_t* cand_out, fs_stream_t stream);

/* Merge half: exact top-k over `parts` candidate blocks laid out [parts, B, K + 1] (the
 * all-gather of every shard's cand_out), then the softmax / top-p / draw tail. Every rank
 * that runs it with the same rng produces the same ids. Uses args: dtype, batch, top_k (K),
 * top_p, top_k_rows, top_p_rows, rng, out_ids, topk_ids, keep, renormed, row_status. */
FS_API fs_status fs_merge_sample(const fs_sample_args* args, const uint64_t* cand, int32_t parts,
                          fs_stream_t stream);

/* Exchange and merge without a collective library (no counterpart in the reference; the
 * peer-to-peer form of the all-gather + fs_merge_sample pair): every rank pushes its [B, K + 1] candidate
 * block (from fs_shard_candidates) into every rank's receive buffer over NVLink and raises one
 * flag per (row, source rank) there, then waits for its own flags and merges. All ranks call it
 * with the same epoch (1, 2, 3, ... per call), or each with its own epoch_counter (below).
 * Buffers, set up once per process group:
 *   recv  : device [2][world][max_batch][K + 1] uint64, flags: device [2][world][max_batch]
 *           uint32 (zeroed before the first call),
 *   peer_recv / peer_flags: device arrays of `world` pointers to every rank's recv / flags
 *           (this rank's own included), mapped with fs_ipc_open.
 * A flag that does not arrive within wait_polls polls (0 = the default, about a second) marks
 * the row FS_ROW_TIMEOUT (id -1); the exchange is then out of step between the ranks: tear the
 * buffers down and set them up again before the next call. Uses args: dtype, batch, top_k (K),
 * top_p, rng, out_ids, row_status.
 * epoch_counter (optional): device memory of 2 uint32 on this rank's GPU, zeroed before the first
 * call. When set, `epoch` is ignored: each call reads its epoch from the counter and the launch
 * advances it (1, 2, ..., 2^32 - 1, then 2, 3, ...), so nothing changes between calls on the host
 * and the launch can be captured in a CUDA graph and replayed. */
typedef struct fs_tp_peers {
  int32_t world;
  int32_t rank;
  int64_t max_batch;
  uint32_t epoch;
  int64_t wait_polls;
  uint64_t* recv;
  uint32_t* flags;
  uint64_t* const* peer_recv;
  uint32_t* const* peer_flags;
  uint32_t* epoch_counter;
} fs_tp_peers;
FS_API fs_status fs_tp_merge_sample(const fs_sample_args* args, const uint64_t* local_cand,
                                    const fs_tp_peers* tp, fs_stream_t stream);

/* CUDA IPC plumbing for the buffers above, used once at set-up: fs_ipc_alloc allocates a zeroed
 * device buffer on the current device (its own allocation, so its address is the base an IPC
 * handle describes), fs_ipc_handle exports it (FS_IPC_HANDLE_BYTES bytes), a peer process maps
 * it with fs_ipc_open and unmaps it with fs_ipc_close; fs_ipc_free releases it. */
#define FS_IPC_HANDLE_BYTES 64
FS_API fs_status fs_ipc_alloc(uint64_t bytes, void** dev_ptr_out);
FS_API fs_status fs_ipc_free(void* dev_ptr);
FS_API fs_status fs_ipc_handle(const void* dev_ptr, void* handle_out);
FS_API fs_status fs_ipc_open(const void* handle, void** dev_ptr_out);
FS_API fs_status fs_ipc_close(void* dev_ptr);

/* ---- floor probes (measurement brackets) ---------------------------------------------------
 * Replace: probe_noop / probe_scan_rowblock / probe_scan_split (csrc/probes.cu:86-125). */
FS_API fs_status fs_probe_noop(int64_t* out, int64_t batch, fs_stream_t stream);
/* argmax per row (lowest id on ties), one CTA per row. */
FS_API fs_status fs_probe_scan_rowblock(const void* logits, int32_t dtype, int64_t batch, int64_t vocab,
                                 int64_t row_stride, int64_t* out, fs_stream_t stream);
/* argmax per row with `splits` CTAs per row, merged through a thread-block cluster. */
FS_API fs_status fs_probe_scan_split(const void* logits, int32_t dtype, int64_t batch, int64_t vocab,
                              int64_t row_stride, int32_t splits, int64_t* out,
                              fs_stream_t stream);

/* ---- introspection ------------------------------------------------------------------------
 * Replaces: kernel_attrs (csrc/fused_sampling.cu:515-540, csrc/bindings.cpp:24). */
typedef struct fs_kernel_attr {
  char name[64];
  int32_t param;          /* kernel variant parameter (uint4 chunks per thread, or 0)   */
  int32_t block;          /* threads per CTA                                            */
  int32_t regs;           /* registers per thread                                       */
  int32_t local_bytes;    /* local (spill) memory per thread                            */
  int32_t static_smem;    /* static shared memory per CTA                               */
  int32_t blocks_per_sm;  /* theoretical resident CTAs per SM at the typical smem size  */
} fs_kernel_attr;

/* Fills up to `cap` rows, returns the number of kernels described (may exceed cap), or -1. */
FS_API int32_t fs_kernel_attrs(fs_kernel_attr* rows, int32_t cap);

/* Human-readable message of the last error raised on the calling host thread. */
FS_API const char* fs_last_error(void);

/* Plan of a call (automatic path), for logging and tests: CTAs per row, 16-byte chunks per
 * thread, threads per CTA, survivor capacity, maxima per thread / lanes per maximum, path,
 * workspace. */
typedef struct fs_plan_info {
  int32_t splits;
  int32_t chunks;
  int32_t threads;
  int32_t capacity;
  int32_t maxima_per_thread;
  int32_t lanes_per_max;
  int32_t smem_bytes;
  int32_t path;              /* FS_PATH_CLUSTER, FS_PATH_STREAM or FS_PATH_WIDE */
  uint64_t workspace_bytes;  /* 0 unless the path is FS_PATH_STREAM */
} fs_plan_info;
FS_API fs_status fs_plan(int64_t batch, int64_t vocab, int64_t top_k, int32_t splits, fs_plan_info* out);

/* Library version string. */
FS_API const char* fs_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FUSED_SAMPLING_B200_H */
