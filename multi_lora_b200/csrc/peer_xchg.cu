// Row-parallel projections with the shrink partials exchanged over peer
// memory (include/mlora_b200.h: mlora_peer_exchange_t and friends): buffer
// set-up through CUDA IPC, and the entry point that launches the fused decode
// kernel (csrc/apply_fused.cu) or the streaming shrink/expand pair
// (csrc/apply_stream.cu) in exchange mode.
#include <cstring>

#include "../../include/mlora_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace {

int xfail(int code, const char* msg) { return mlora::report_error(code, msg); }

int cuda_rc(cudaError_t e) { return e == cudaSuccess ? MLORA_OK : xfail(MLORA_ERR_CUDA, cudaGetErrorString(e)); }

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

struct XLayout {
  size_t recv, ctr, total;
  XLayout(int tp, int rows, int R) {
    recv = 0;  // [2][tp][rows][R] words of 8 bytes
    ctr = recv + (size_t)2 * tp * rows * R * sizeof(unsigned long long);
    total = (ctr + 2 * sizeof(uint32_t) + 255) / 256 * 256;
  }
};

}  // namespace

extern "C" {

size_t mlora_peer_exchange_bytes(int32_t tp, int32_t max_rows, int32_t max_rank) {
  if (tp < 1 || tp > MLORA_MAX_PEERS || max_rows < 1 || max_rank < 1) return 0;
  return XLayout(tp, max_rows, max_rank).total;
}

int mlora_peer_buffer_create(size_t bytes, void** buffer, void* ipc_handle) {
  if (bytes == 0 || buffer == nullptr || ipc_handle == nullptr)
    return xfail(MLORA_ERR_INVALID_ARGUMENT, "bytes / buffer / ipc_handle invalid");
  static_assert(sizeof(cudaIpcMemHandle_t) == MLORA_IPC_HANDLE_BYTES, "IPC handle size");
  void* p = nullptr;
  if (int rc = cuda_rc(cudaMalloc(&p, bytes))) return rc;
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    (void)cudaFree(p);
    return cuda_rc(e);
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *buffer = p;
  return MLORA_OK;
}

int mlora_peer_buffer_open(const void* ipc_handle, void** buffer) {
  if (ipc_handle == nullptr || buffer == nullptr) return xfail(MLORA_ERR_INVALID_ARGUMENT, "NULL argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return cuda_rc(cudaIpcOpenMemHandle(buffer, h, cudaIpcMemLazyEnablePeerAccess));
}

int mlora_peer_buffer_close(void* buffer) { return cuda_rc(cudaIpcCloseMemHandle(buffer)); }

int mlora_peer_buffer_destroy(void* buffer) { return cuda_rc(cudaFree(buffer)); }

int mlora_row_parallel_apply_p2p(const void* x, int64_t rows, int64_t in_shard, int64_t x_row_stride,
                                 const void* a_shard, const void* b_shard, int64_t out_cols, int64_t max_rank,
                                 const mlora_kernel_input_metadata_t* meta, void* y, int64_t y_row_stride,
                                 const mlora_peer_exchange_t* xchg, int32_t phase, int32_t dtype, uint32_t* status,
                                 void* stream) {
  if (meta == nullptr || xchg == nullptr) return xfail(MLORA_ERR_INVALID_ARGUMENT, "meta / xchg is NULL");
  if (dtype != MLORA_BF16 && dtype != MLORA_F16)
    return xfail(MLORA_ERR_UNSUPPORTED_DTYPE, "the exchange path takes bf16 or f16");
  const mlora_peer_exchange_t& X = *xchg;
  if (X.tp < 1 || X.tp > MLORA_MAX_PEERS || X.rank < 0 || X.rank >= X.tp)
    return xfail(MLORA_ERR_INVALID_ARGUMENT, "exchange tp / rank out of range");
  if (phase < 0 || phase > 2) return xfail(MLORA_ERR_INVALID_ARGUMENT, "phase must be 0, 1 or 2");
  if (rows < 0 || rows > X.max_rows) return xfail(MLORA_ERR_INVALID_ARGUMENT, "rows exceed the exchange's max_rows");
  if (max_rank != X.max_rank) return xfail(MLORA_ERR_INVALID_ARGUMENT, "max_rank differs from the exchange's");
  if (meta->bs < 0 || meta->num_slots <= 0 || meta->num_slots > 65535 || meta->lora_ranks == nullptr ||
      (meta->bs > 0 && (meta->seg_indptr == nullptr || meta->weight_indices == nullptr)) || meta->scalings == nullptr)
    return xfail(MLORA_ERR_INVALID_ARGUMENT, "metadata invalid");
  for (int q = 0; q < X.tp; ++q)
    if (X.buffers[q] == nullptr || !aligned16(X.buffers[q]))
      return xfail(MLORA_ERR_INVALID_ARGUMENT, "an exchange buffer is NULL or misaligned");
  if (!(in_shard > 0 && in_shard % 16 == 0 && max_rank > 0 && max_rank % 8 == 0 && max_rank <= 64 && out_cols > 0 &&
        out_cols % 8 == 0 && x_row_stride >= in_shard && x_row_stride % 8 == 0 && y_row_stride >= out_cols &&
        y_row_stride % 8 == 0 && aligned16(x) && aligned16(a_shard) && aligned16(b_shard) && aligned16(y)))
    return xfail(MLORA_ERR_INVALID_ARGUMENT, "shape outside the exchange path (use the NCCL path)");
  if (meta->bs == 0 || rows == 0) return MLORA_OK;

  const XLayout L(X.tp, X.max_rows, X.max_rank);
  mlora::PeerXchg xc{};
  xc.tp = X.tp;
  xc.rank = X.rank;
  xc.rows = X.max_rows;
  for (int q = 0; q < X.tp; ++q)
    xc.recv[q] = reinterpret_cast<unsigned long long*>(static_cast<unsigned char*>(X.buffers[q]) + L.recv);
  xc.ctr = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(X.buffers[X.rank]) + L.ctr);
  const bool pdl = mlora_get_pdl() != 0;

  // Decode batches: the fused kernel (one launch: shrink, exchange, expand),
  // as mlora_apply_lora picks it; it declines shapes whose grid does not fit
  // in one wave. Otherwise the streaming pair.
  const int forced = mlora::forced_apply_path();
  const bool fused_pref = forced == 1 || (forced == 0 && rows < 256 && meta->max_len <= 16 &&
                                          rows <= 64LL * meta->num_slots);
  if (fused_pref) {
    mlora::FusedArgs f{};
    f.x = x;
    f.x_stride = x_row_stride;
    f.n_mod = 1;
    f.mod[0].a = a_shard;
    f.mod[0].b = b_shard;
    f.mod[0].y = y;
    f.mod[0].y_stride = y_row_stride;
    f.mod[0].mid = nullptr;
    f.mod[0].mid_stride = max_rank;
    f.mod[0].out_dim = (int)out_cols;
    f.seg_indptr = meta->seg_indptr;
    f.weight_indices = meta->weight_indices;
    f.lora_ranks = meta->lora_ranks;
    f.scalings = meta->scalings;
    f.scalings_dtype = meta->scalings_dtype;
    f.bs = meta->bs;
    f.S = (int)rows;
    f.in_dim = (int)in_shard;
    f.R = (int)max_rank;
    f.num_slots = meta->num_slots;
    f.status = status;
    f.xchg = xc;
    f.phase = phase;
    const cudaError_t e = mlora::launch_apply_fused(f, dtype, (cudaStream_t)stream, pdl);
    if (e == cudaSuccess) {
      mlora::note_apply_path(1);
      return MLORA_OK;
    }
    if (e != cudaErrorNotSupported) return cuda_rc(e);
  }

  mlora::StreamArgs sa{};
  sa.x = x;
  sa.x_stride = x_row_stride;
  sa.n_mod = 1;
  sa.mod[0].a = a_shard;
  sa.mod[0].b = b_shard;
  sa.mod[0].y = y;
  sa.mod[0].y_stride = y_row_stride;
  sa.mod[0].out_dim = (int)out_cols;
  sa.mid = nullptr;
  sa.mid_stride = max_rank;
  sa.mid_f32 = 1;
  sa.phase = phase;
  sa.seg_indptr = meta->seg_indptr;
  sa.weight_indices = meta->weight_indices;
  sa.lora_ranks = meta->lora_ranks;
  sa.scalings = meta->scalings;
  sa.scalings_dtype = meta->scalings_dtype;
  sa.bs = meta->bs;
  sa.S = (int)rows;
  sa.in_dim = (int)in_shard;
  sa.R = (int)max_rank;
  sa.num_slots = meta->num_slots;
  sa.status = status;
  sa.xchg = xc;
  const cudaError_t e = mlora::launch_apply_stream(sa, dtype, (cudaStream_t)stream, pdl);
  if (e == cudaErrorNotSupported) return xfail(MLORA_ERR_INVALID_ARGUMENT, "shape outside the exchange path");
  if (e == cudaSuccess) mlora::note_apply_path(3);
  return cuda_rc(e);
}

}  // extern "C"
