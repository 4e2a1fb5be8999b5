/*
 * mlora_b200.h — C ABI of the B200 (sm_100a) multi-LoRA hot path.
 *
 * Plain pointers and sizes only; every device pointer is a CUDA device
 * address, every `stream` is a cudaStream_t (NULL = legacy default stream).
 * No entry point allocates device memory or synchronises the host, so every
 * one of them may be captured into a CUDA graph.
 *
 * Each entry point replaces one operator of the reference project
 * (Rick0037/multi_lora); the citation is given as file:line within that
 * project. Return value: MLORA_OK or a negative MLORA_ERR_* code; the message
 * of the last failure on the calling thread is in mlora_last_error().
 */
#ifndef MLORA_B200_H_
#define MLORA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types (torch.bfloat16 / torch.float16 / torch.float32) */
#define MLORA_BF16 0
#define MLORA_F16 1
#define MLORA_F32 2

/* return codes */
#define MLORA_OK 0
#define MLORA_ERR_INVALID_ARGUMENT (-1)
#define MLORA_ERR_UNSUPPORTED_DTYPE (-2)
#define MLORA_ERR_CUDA (-3)

/* bits a kernel sets in the optional device status word (uint32) when the
 * routing metadata would take it out of bounds; the access is skipped. */
#define MLORA_STATUS_SLOT_RANGE 0x1u    /* weight_indices[i] outside [0, num_slots) */
#define MLORA_STATUS_RANK_RANGE 0x2u    /* lora_ranks[s] outside [0, max_rank] (clamped) */
#define MLORA_STATUS_INDPTR 0x4u        /* seg_indptr decreasing or past the row count */
#define MLORA_STATUS_SCATTER_RANGE 0x8u /* scatter descriptor outside its buffers */
#define MLORA_STATUS_TIMEOUT 0x10u      /* a bounded wait for an async copy gave up */

/*
 * Segment routing of one step; mirrors KernelInputMetaData
 * (multi_lora/batch_info.py:26-42). All arrays are device int32 except
 * `scalings`, which has element type `scalings_dtype` (the reference stores
 * it in the model dtype, batch_info.py:164-165). Segment i covers token rows
 * [seg_indptr[i], seg_indptr[i+1]) and uses adapter slot weight_indices[i];
 * slot s has rank lora_ranks[s] (0 = base model, no LoRA) and scaling
 * scalings[s]. seg_lens is accepted for interface parity and not read: the
 * boundaries come from seg_indptr, as in backend/torch_backend.py:38-41.
 */
typedef struct mlora_kernel_input_metadata {
  int32_t bs;                     /* number of segments */
  int32_t max_len;                /* longest segment (host int, as in the reference) */
  int32_t num_slots;              /* K: slots in the pool (length of lora_ranks/scalings) */
  int32_t scalings_dtype;         /* MLORA_BF16 / MLORA_F16 / MLORA_F32 */
  const int32_t* seg_lens;        /* [>= bs] (may be NULL) */
  const int32_t* seg_indptr;      /* [>= bs + 1] */
  const int32_t* weight_indices;  /* [>= bs] */
  const int32_t* lora_ranks;      /* [num_slots] */
  const void* scalings;           /* [num_slots] */
} mlora_kernel_input_metadata_t;

/*
 * Shrink (LoRA A stage): output[t, n] = dtype(sum_k x[t, k] * weights[slot, n, k])
 * for every token t of a segment routed to `slot` and n < min(max_rank,
 * lora_ranks[slot] * stack_num); fp32 accumulation. Other columns and rank-0
 * segments are not written.
 *   x        [rows, in_dim] of `dtype`, row stride x_row_stride (elements)
 *   weights  [num_slots, max_rank, in_dim] of `dtype`, contiguous
 *   output   [rows, >= max_rank], row stride output_row_stride, element type
 *            `output_dtype` (= dtype, or MLORA_F32 for unrounded partial sums
 *            that a tensor-parallel all-reduce completes)
 *   status   optional device uint32 (see MLORA_STATUS_*), may be NULL
 * Replaces sgemm_lora_a_fwd, multi_lora/kernels/sgemm_lora_a.py:186-274
 * (called from backend/triton_backend.py:34-45).
 */
int mlora_sgemm_lora_a_fwd(const void* x, int64_t rows, int64_t in_dim, int64_t x_row_stride,
                           const void* weights, int64_t max_rank,
                           const mlora_kernel_input_metadata_t* meta,
                           void* output, int64_t output_row_stride, int32_t output_dtype,
                           int32_t dtype, int32_t stack_num, uint32_t* status, void* stream);

/*
 * Expand (LoRA B stage), fused scaling and residual add, in place:
 *   y[t, o] = dtype( dtype(scalings[slot] * sum_{k<rank} mid[t, k] * weights[slot, o, k]) + y[t, o] )
 *   mid      [rows, >= max_rank] of `mid_dtype` (dtype, or MLORA_F32 partial
 *            sums, which are rounded to dtype on read)
 *   weights  [num_slots, out_dim, max_rank] of `dtype`, contiguous
 *   y        [rows, out_dim] of `dtype`, row stride y_row_stride (a strided
 *            slice of a wider output is allowed, multi_lora/layers.py:82-83)
 * Replaces sgemm_lora_b_fwd with base_output given, multi_lora/kernels/
 * sgemm_lora_b.py:156-236 (backend/triton_backend.py:47-61).
 */
int mlora_sgemm_lora_b_fwd(const void* mid, int64_t rows, int64_t mid_row_stride, int32_t mid_dtype,
                           const void* weights, int64_t out_dim, int64_t max_rank,
                           const mlora_kernel_input_metadata_t* meta,
                           void* y, int64_t y_row_stride,
                           int32_t dtype, uint32_t* status, void* stream);

/*
 * apply_lora: shrink into `mid`, then expand into y (both launches on
 * `stream`). Replaces LoRABackend.apply_lora, multi_lora/backend/base.py:60-89.
 */
int mlora_apply_lora(const void* x, int64_t rows, int64_t in_dim, int64_t x_row_stride,
                     const void* a_stack, const void* b_stack, int64_t out_dim, int64_t max_rank,
                     const mlora_kernel_input_metadata_t* meta,
                     void* mid, int64_t mid_row_stride,
                     void* y, int64_t y_row_stride,
                     int32_t dtype, uint32_t* status, void* stream);

/*
 * apply_lora over n (1..4) projections that share x and the routing, e.g.
 * q/k/v of one attention block or gate/up of one MLP: projection i uses
 * a_stacks[i] [num_slots, max_rank, in_dim], b_stacks[i]
 * [num_slots, out_dims[i], max_rank] and updates ys[i] (row stride
 * y_row_strides[i]) in place, exactly as n separate mlora_apply_lora calls
 * would. For short segments all n run in one launch. `mid` ([rows, >=
 * max_rank], may be NULL when the fused path applies) is scratch for the
 * two-launch path; its contents afterwards are unspecified.
 * Batches the reference's per-projection LinearWithLoRA.add_delta calls
 * (multi_lora/layers.py:76-88) the way QKVProjGroup batches the base GEMM
 * (layers.py:91-125); the reference's kernels reserve a stack_num parameter
 * for it (kernels/sgemm_lora_a.py:51).
 */
int mlora_apply_lora_group(const void* x, int64_t rows, int64_t in_dim, int64_t x_row_stride, int32_t n,
                           const void* const* a_stacks, const void* const* b_stacks, const int64_t* out_dims,
                           void* const* ys, const int64_t* y_row_strides, int64_t max_rank,
                           const mlora_kernel_input_metadata_t* meta, void* mid, int64_t mid_row_stride,
                           int32_t dtype, uint32_t* status, void* stream);

/*
 * Same result as mlora_apply_lora_group (two launches per projection: shrink,
 * then expand), for callers that cannot allocate device memory: the
 * intermediate mid lives in a 1 MiB device array owned by the library, so the
 * caller passes only inputs and outputs and the call allocates nothing (no
 * cudaMalloc, cudaFree or allocating library routine). Use it where a host
 * gives this library no allocator, or where cudaMalloc's device
 * synchronisation is not acceptable.
 * Limit: rows * max_rank * element size <= 1 MiB (e.g. 32768 rows at bf16 and
 * max_rank 16); larger calls return MLORA_ERR_INVALID_ARGUMENT.
 * Every GPU that loads the library holds the 1 MiB until the process exits.
 * The first call on a device looks up the array's device address (with that
 * device current) and caches it with the current context; a call in another
 * context on that device (after cudaDeviceReset, or a non-primary context
 * made current through the driver API) looks it up again. Make the first call
 * in a context before any stream capture. All calls
 * on a device share the array: calls that overlap on the GPU race and give
 * wrong results. Nothing in it needs to start at zero.
 * This entry point has no counterpart in the reference project.
 */
int mlora_apply_lora_group_noalloc(const void* x, int64_t rows, int64_t in_dim, int64_t x_row_stride, int32_t n,
                                   const void* const* a_stacks, const void* const* b_stacks, const int64_t* out_dims,
                                   void* const* ys, const int64_t* y_row_strides, int64_t max_rank,
                                   const mlora_kernel_input_metadata_t* meta, int32_t dtype, uint32_t* status,
                                   void* stream);

/*
 * RMSNorm: y[r, :] = dtype( x_f32 * rsqrt(mean(x_f32^2) + eps) * w_f32 ).
 * Row r of x starts at (r / inner) * stride_outer + (r % inner) * stride_inner
 * (elements); y is [rows, hidden] with row stride y_row_stride. w has
 * element type w_dtype. Replaces rmsnorm_fwd, multi_lora/kernels/
 * rmsnorm.py:48-92 (kernel :18-45).
 */
int mlora_rmsnorm_fwd(const void* x, int64_t rows, int64_t hidden, int64_t stride_outer,
                      int64_t stride_inner, int64_t inner, const void* w, int32_t w_dtype,
                      void* y, int64_t y_row_stride, float eps, int32_t dtype, void* stream);

/*
 * Residual add fused with RMSNorm, for the add that precedes a decoder
 * layer's norm (hidden = residual + hidden; residual = hidden; norm(hidden)):
 *   residual[r, :] = dtype(residual[r, :] + x[r, :])                 (in place)
 *   y[r, :]        = dtype(res_f32 * rsqrt(mean(res_f32^2) + eps) * w_f32)
 * with res_f32 the rounded sum just written. Bit-identical to an add in
 * `dtype` followed by mlora_rmsnorm_fwd, in one pass over the row. Rows of x,
 * residual and y are dense with the given row strides (elements). Replaces
 * the separate residual add + rmsnorm_fwd pair the reference plans to fuse
 * (OPTIMIZATION_TODO.md:125-142, task T22; kernels/rmsnorm.py:48-92).
 */
int mlora_fused_add_rmsnorm_fwd(const void* x, int64_t x_row_stride, void* residual, int64_t residual_row_stride,
                                int64_t rows, int64_t hidden, const void* w, int32_t w_dtype, void* y,
                                int64_t y_row_stride, float eps, int32_t dtype, void* stream);

/*
 * One block of a staged adapter bank and where it goes in the slot stacks.
 * Source: `rows` x `cols` dense elements at `src_offset` within a stage row.
 * Destination: element [row, col] of slot s lands at
 *   dst + (s * slot_stride + row * dst_row_stride + col) * element_size.
 * An A block [rank, in] is (rows=rank, cols=in, dst_row_stride=in) and a B
 * block [out, rank] is (rows=out, cols=rank, dst_row_stride=max_rank), as in
 * the offset tables of multi_lora/pool.py:60-94.
 */
typedef struct mlora_scatter_rect {
  int64_t src_offset;
  int64_t dst;            /* device address of the destination stack's element 0 */
  int64_t slot_stride;    /* elements between slots */
  int64_t rows;
  int64_t cols;
  int64_t dst_row_stride; /* elements between destination rows */
} mlora_scatter_rect_t;

/*
 * Slot load scatter: for every adapter i < h (stage row i, slot slots[i]) and
 * every rectangle, copy the block from the stage into its slot. `stage` is
 * [h, stage_row_elems] of `dtype`; `slots` is a device int64 [h]; `rects` a
 * device array of n_rects descriptors; max_rect_elems bounds rows*cols over
 * the rectangles (it sizes the grid). A rectangle whose source lies outside
 * the stage row sets MLORA_STATUS_SCATTER_RANGE and is skipped. The launch
 * does not overlap the kernels that follow it on `stream`.
 * Replaces scatter_stage, multi_lora/kernels/scatter_bank.py:68-93
 * (kernel :18-65), called from pool.py:231-232.
 */
int mlora_scatter_stage(const void* stage, int64_t stage_row_elems, int32_t h, const int64_t* slots,
                        const mlora_scatter_rect_t* rects, int32_t n_rects, int64_t max_rect_elems,
                        int32_t dtype, uint32_t* status, void* stream);

/*
 * Tensor-parallel row-parallel projections without a separate all-reduce.
 *
 * A row-parallel projection (o, down) shards x and A on the input dim; each
 * rank's shrink gives a partial [rows, rank] that must be summed over the
 * ranks before the expand (the baseline: an NCCL all-reduce of fp32
 * partials). Here the shrink stores each partial value straight into every
 * rank's receive buffer over NVLink (plain peer stores), as one 8-byte word
 * holding the fp32 value and the call's tag; the expand polls the words it
 * needs until they carry this call's tag (bounded; on timeout
 * MLORA_STATUS_TIMEOUT is set and the item is skipped), sums the ranks'
 * partials in rank order, rounds to `dtype` and adds this rank's output
 * columns. The tag comes from a counter in each rank's buffer that the expand
 * advances (calls completed), so the calls may be captured in a CUDA graph;
 * every rank must issue the same calls in the same order.
 *
 * Each rank owns one buffer of mlora_peer_exchange_bytes() bytes, made by
 * mlora_peer_buffer_create (zeroed; its IPC handle is sent to the other ranks,
 * which map it with mlora_peer_buffer_open). No call here allocates except
 * mlora_peer_buffer_create. No counterpart in the reference, which has no
 * tensor parallelism; it takes the place of the NCCL all-reduce of the
 * row-parallel shrink partials (multi_lora_b200/tensor_parallel.py).
 */
#define MLORA_MAX_PEERS 8
#define MLORA_IPC_HANDLE_BYTES 64

typedef struct mlora_peer_exchange {
  int32_t tp;        /* ranks in the group, 1..MLORA_MAX_PEERS */
  int32_t rank;      /* this rank */
  int32_t max_rows;  /* rows (tokens) a call may have */
  int32_t max_rank;  /* max_rank of the slot stacks */
  void* buffers[MLORA_MAX_PEERS]; /* rank q's exchange buffer as mapped in this process (buffers[rank]: own) */
} mlora_peer_exchange_t;

/* Bytes of one rank's exchange buffer: tagged partial words
 * [2][tp][max_rows][max_rank] of 8 bytes (two halves alternate between
 * calls) and two uint32 counters. */
size_t mlora_peer_exchange_bytes(int32_t tp, int32_t max_rows, int32_t max_rank);

/* cudaMalloc + zero a buffer on the current device, and its IPC handle
 * (MLORA_IPC_HANDLE_BYTES bytes written to ipc_handle). Synchronises the device. */
int mlora_peer_buffer_create(size_t bytes, void** buffer, void* ipc_handle);
/* Map another process's buffer from its IPC handle (peer access enabled). */
int mlora_peer_buffer_open(const void* ipc_handle, void** buffer);
/* Unmap a buffer opened with mlora_peer_buffer_open. */
int mlora_peer_buffer_close(void* buffer);
/* Free a buffer made by mlora_peer_buffer_create. */
int mlora_peer_buffer_destroy(void* buffer);

/*
 * One row-parallel projection on this rank: shrink of its input shard with
 * the partials exchanged as above, then the expand of its output columns.
 *   x        [rows, in_shard] (row stride x_row_stride), this rank's input columns
 *   a_shard  [num_slots, max_rank, in_shard]; b_shard [num_slots, out_cols, max_rank]
 *   y        [rows, out_cols] (row stride y_row_stride): this rank's columns of
 *            the pre-all-reduce partial output, updated in place
 * phase: 0 = shrink then expand (normal use); 1 = shrink and publish only;
 * 2 = wait and expand only. Phases 1 and 2 let one process drive several
 * ranks' exchanges on ONE GPU (every rank's phase 1 before any rank's phase 2),
 * so that no kernel ever waits for a kernel queued after it.
 * Kernels: decode batches (rows < 256, meta->max_len <= 16) run one fused
 * launch (shrink, exchange, expand) when its grid fits in one wave, other
 * shapes the streaming shrink/expand pair; mlora_last_apply_path() returns 1
 * or 3 accordingly and mlora_set_apply_path() can force either.
 * Shape range: bf16/f16, in_shard % 16 == 0, max_rank % 8 == 0 and <= 64,
 * out_cols % 8 == 0, 16-byte aligned operands; otherwise
 * MLORA_ERR_INVALID_ARGUMENT (use the NCCL path).
 */
int mlora_row_parallel_apply_p2p(const void* x, int64_t rows, int64_t in_shard, int64_t x_row_stride,
                                 const void* a_shard, const void* b_shard, int64_t out_cols, int64_t max_rank,
                                 const mlora_kernel_input_metadata_t* meta, void* y, int64_t y_row_stride,
                                 const mlora_peer_exchange_t* xchg, int32_t phase, int32_t dtype, uint32_t* status,
                                 void* stream);

/* Programmatic dependent launch (on by default; env MLORA_PDL=0 turns it off). */
void mlora_set_pdl(int enable);
int mlora_get_pdl(void);

/* Message of the last failed call on this thread ("" if none). */
const char* mlora_last_error(void);

/* ABI version: major * 10000 + minor * 100 + patch. */
int mlora_version(void);

/* Diagnostics: which path the last mlora_apply_lora on this thread took
 * (1 = one fused launch, 2 = shrink + expand launches, 3 = the streaming
 * shrink/expand kernel pair, 4 = the tensor-core (tcgen05) shrink/expand pair
 * for long segments, 0 = none yet). mlora_sgemm_lora_a_fwd / _b_fwd set it
 * too: 3 when they ran the streaming kernel (segments of at most 64 rows,
 * bf16/f16, aligned operands), 2 for the general kernel. */
int mlora_last_apply_path(void);

/* Tuning and tests: force the path mlora_apply_lora / mlora_apply_lora_group
 * try first (0 = automatic, 1 = fused, 2 = shrink + expand, 3 = streaming
 * pair, 4 = tensor-core pair). A shape the forced path cannot take falls
 * through tensor-core -> stream -> fused -> shrink + expand. Process-wide; the
 * environment variable MLORA_APPLY_PATH (fused | split | stream | tc) sets the
 * initial value. No reference counterpart. */
void mlora_set_apply_path(int path);
int mlora_get_apply_path(void);

#ifdef __cplusplus
}
#endif

#endif /* MLORA_B200_H_ */
