// Internal launch interface between the C-ABI layer (capi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/mlora_b200.h"

namespace mlora {

struct ShrinkArgs {
  const void* x;          // [S, in] rows at x_stride elements
  int64_t x_stride;
  const void* w;          // A stack: A[s, n, k] = w[s*w_slot_stride + n*w_row_stride + k]
  int64_t w_slot_stride;
  int64_t w_row_stride;
  void* out;              // mid [S, >= max_rank] rows at out_stride elements
  int64_t out_stride;
  const int32_t* seg_indptr;      // [bs + 1]
  const int32_t* weight_indices;  // [bs]
  const int32_t* lora_ranks;      // [num_slots]
  int bs, S, in_dim, max_rank, num_slots, stack_num;
  uint32_t* status;  // optional device status word
  int vec_ok;        // 128-bit loads legal for x and A
};

struct ExpandArgs {
  const void* mid;        // [S, >= max_rank] rows at mid_stride elements
  int64_t mid_stride;
  const void* w;          // B stack: B[s, o, k] = w[s*w_slot_stride + o*w_row_stride + k]
  int64_t w_slot_stride;
  int64_t w_row_stride;
  void* y;                // [S, out] rows at y_stride elements, updated in place
  int64_t y_stride;
  const int32_t* seg_indptr;
  const int32_t* weight_indices;
  const int32_t* lora_ranks;
  const void* scalings;   // [num_slots] of scalings_dtype
  int scalings_dtype;
  int bs, S, out_dim, max_rank, num_slots;
  uint32_t* status;
  int vec_ok;    // 128-bit loads legal for B
  int y_vec_ok;  // paired stores legal for y
};

struct RmsNormArgs {
  const void* x;          // row r at (r / inner) * stride_outer + (r % inner) * stride_inner
  int64_t stride_outer;
  int64_t stride_inner;
  int64_t inner;
  const void* w;          // [hidden] of w_dtype
  int w_dtype;
  void* y;                // [rows, hidden] rows at y_stride elements
  int64_t y_stride;
  int64_t rows;
  int hidden;
  float eps;
  int vec_ok;
  int w_vec;              // w 16-byte aligned: its chunks load as vectors
  // fused add (optional): row r of x is first replaced by T(x[r] + add[r]),
  // written to res + r * res_stride, and that rounded sum is normalised
  const void* add;        // nullptr: plain RMSNorm
  int64_t add_stride;
  void* res;
  int64_t res_stride;
};

// Tensor-parallel exchange of row-parallel shrink partials over peer memory
// (buffers of mlora_peer_exchange_t, include/mlora_b200.h). tp == 0: off.
// A partial value travels in one 8-byte word: the fp32 bits in the low half,
// the call's tag (epoch + 1) in the high half, written and read as one
// single-copy-atomic 8-byte access, so the reader needs no separate flag.
constexpr int kMaxPeers = 8;
struct PeerXchg {
  unsigned long long* recv[kMaxPeers];  // rank q's words [2][tp][rows][R], mapped in this process
  uint32_t* ctr;                        // this rank's counters: [0] epoch (calls completed), [1] CTAs of the call's last kernel that finished
  int tp, rank, rows;
};
// One projection of a fused apply_lora launch; up to kMaxFusedModules
// projections that share x and the routing go in one launch (e.g. q/k/v).
constexpr int kMaxFusedModules = 4;
struct FusedModule {
  const void* a;          // A stack [K, R, in], contiguous
  const void* b;          // B stack [K, out, R], contiguous
  void* y;                // [S, out] at y_stride, updated in place
  void* mid;              // optional [S, >= R] at mid_stride (shrink output, as the API returns it)
  int64_t y_stride;
  int64_t mid_stride;
  int out_dim;
  int ob;                 // output columns per cluster CTA (multiple of 8), set by the launcher
  int y_tma;              // y rows may be staged with bulk copies (alignment holds)
};

struct FusedArgs {
  const void* x;          // [S, in] rows at x_stride elements
  int64_t x_stride;
  FusedModule mod[kMaxFusedModules];
  int n_mod;
  const int32_t* seg_indptr;
  const int32_t* weight_indices;
  const int32_t* lora_ranks;
  const void* scalings;
  int scalings_dtype;
  int bs, S, in_dim, R, num_slots;
  int ks;                 // input columns per cluster CTA (multiple of 8), set by the launcher
  int ob_max;             // largest module ob (sizes the shared-memory B and y tiles)
  uint32_t* status;
  // tp > 0 (one projection): row-parallel exchange. The cluster's partial of
  // mid goes to every rank's buffer and mid is the sum of all ranks' partials.
  // phase 0: both in one launch; 1: publish only; 2: wait and expand only.
  PeerXchg xchg;
  int phase;
};

cudaError_t launch_apply_fused(FusedArgs a, int dtype, cudaStream_t st, bool pdl);

// Streaming apply (persistent shrink + expand kernels, csrc/apply_stream.cu).
constexpr int kMaxStreamModules = 4;

struct StreamModule {
  const void* a;          // A stack [K, R, in], contiguous
  const void* b;          // B stack [K, out, R], contiguous
  void* y;                // [S, out] at y_stride, updated in place
  int64_t y_stride;
  int out_dim;
};
struct StreamArgs {
  const void* x;          // [S, in] rows at x_stride elements
  int64_t x_stride;
  StreamModule mod[kMaxStreamModules];
  int n_mod;
  void* mid;              // [S, >= n_mod * R] at mid_stride: projection m's shrink output in columns [m*R, m*R + rank)
  int64_t mid_stride;
  const int32_t* seg_indptr;
  const int32_t* weight_indices;
  const int32_t* lora_ranks;
  const void* scalings;
  int scalings_dtype;
  int bs, S, in_dim, R, num_slots;
  uint32_t* status;
  int phase;              // 0: shrink then expand; 1: shrink only; 2: expand only
  int mid_f32;            // 1: mid holds fp32 (the shrink writes unrounded sums, the expand rounds them to T)
  PeerXchg xchg;          // tp > 0: partials go to every rank's buffer, the expand sums all ranks' (not `mid`)
};
cudaError_t launch_apply_stream(const StreamArgs& a, int dtype, cudaStream_t st, bool pdl);

// Tensor-core apply for long segments (csrc/prefill_tc.cu).
constexpr int kMaxPrefillModules = 4;
struct PrefillModule {
  const void* a;          // A stack [K, R, in], contiguous
  const void* b;          // B stack [K, out, R], contiguous
  void* y;                // [S, out] at y_stride, updated in place
  int64_t y_stride;
  int out_dim;
};
// What the C ABI hands over; the launcher turns it into tensor maps.
struct PrefillLaunch {
  const void* x;
  int64_t x_stride;
  PrefillModule mod[kMaxPrefillModules];
  int n_mod;
  void* mid;              // [S, >= n_mod * R] at mid_stride: projection m in columns [m*R, m*R + rank)
  int64_t mid_stride;
  const int32_t* seg_indptr;
  const int32_t* weight_indices;
  const int32_t* lora_ranks;
  const void* scalings;
  int scalings_dtype;
  int bs, S, in_dim, R, num_slots;
  uint32_t* status;
};
// Kernel parameter block (passed as __grid_constant__; tensor maps are 64-byte aligned).
struct PrefillArgs {
  CUtensorMap x_map;                          // x [S, in], box 64 x 128
  CUtensorMap mid_map;                        // mid [S, n_mod * R], box 64 x 128
  CUtensorMap a_map[kMaxPrefillModules];      // A [K * R, in], box 64 x R
  CUtensorMap b_map[kMaxPrefillModules];      // B [K * out, R], box 64 x 128
  CUtensorMap y_map[kMaxPrefillModules];      // y [S, out], box 64 x 128
  PrefillModule mod[kMaxPrefillModules];
  int n_mod;
  void* mid;
  int64_t mid_stride;
  const int32_t* seg_indptr;
  const int32_t* weight_indices;
  const int32_t* lora_ranks;
  const void* scalings;
  int scalings_dtype;
  int bs, S, in_dim, R, num_slots;
  int tc_stages;                              // shrink ring depth (set by the launcher)
  uint32_t* status;
};
cudaError_t launch_apply_prefill(const PrefillLaunch& l, int dtype, cudaStream_t st, bool pdl);

// Sets the message mlora_last_error() returns on this thread; returns `code`.
int report_error(int code, const char* msg);
// The apply path forced by mlora_set_apply_path / MLORA_APPLY_PATH (0:
// automatic), and the one this thread's last call ran (mlora_last_apply_path).
int forced_apply_path();
void note_apply_path(int path);
cudaError_t launch_shrink(const ShrinkArgs& a, int dtype, bool out_f32, cudaStream_t st, bool pdl);
cudaError_t launch_expand(const ExpandArgs& a, int dtype, bool mid_f32, cudaStream_t st, bool pdl);
cudaError_t launch_rmsnorm(const RmsNormArgs& a, int dtype, cudaStream_t st, bool pdl);
cudaError_t launch_scatter(const void* stage, int64_t stage_row_elems, int h, const int64_t* slots,
                           const mlora_scatter_rect_t* rects, int n_rects, int64_t max_rect_elems, int es,
                           uint32_t* status, cudaStream_t st);

// Launch with the programmatic-stream-serialisation attribute when `pdl`.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 bool pdl, Args&&... args) {
  if (grid.x == 0 || grid.y == 0 || grid.z == 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

}  // namespace mlora
