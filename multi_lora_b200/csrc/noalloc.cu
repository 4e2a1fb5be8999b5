// mlora_apply_lora_group_noalloc: the two-launch (shrink, then expand)
// apply_lora over a group of projections, with its intermediate `mid` in a
// library-owned device array instead of a caller-provided buffer.
//
// Who needs it: callers that cannot allocate device memory for the
// intermediate — for example a plugin host that hands this library only its
// inputs and outputs and no allocator, or a serving loop that must not call
// cudaMalloc because cudaMalloc synchronises the device. This entry point
// calls no cudaMalloc, cudaFree or allocating library routine.
//
// The array below is the scratch: every GPU that loads the library holds
// kNoAllocScratchBytes of it until the process exits. All calls on a device
// share it and it keeps the last call's contents; nothing in it needs to start
// at zero, because within a call the shrink writes every mid element the
// expand then reads (rank-0 segments and columns past a slot's rank are
// neither written nor read). Calls that overlap on the GPU (different streams
// without ordering between them) race on the array and give wrong results.
//
// Back-to-back calls on one stream are safe under programmatic dependent
// launch because every shrink kernel writes mid only after its
// griddepcontrol.wait (segment_gemv.cu, apply_stream.cu): it cannot start
// writing while the previous expand still reads the array. A shrink kernel
// that moved its mid writes ahead of that wait would break this entry point.
#include <mutex>

#include "../../include/mlora_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;  // 1 MiB per device

__device__ __align__(256) unsigned char g_noalloc_mid[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
// per device ordinal: the context the address was looked up in, and the address
void* g_noalloc_ctx[kMaxDevices] = {nullptr};
void* g_noalloc_ptr[kMaxDevices] = {nullptr};

// failures are reported through mlora_last_error(), like every entry point
int noalloc_fail(int code, const char* msg) { return mlora::report_error(code, msg); }

// The current driver context (CUcontext as void*), or nullptr if it cannot be read.
void* current_context() {
  using GetCtx = int (*)(void**);  // CUresult cuCtxGetCurrent(CUcontext*)
  static GetCtx fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      (void)cudaGetLastError();
      return static_cast<GetCtx>(nullptr);
    }
    return reinterpret_cast<GetCtx>(f);
  }();
  void* ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != 0) return nullptr;
  return ctx;
}

// Device address of the scratch array in the current context. The host-side
// name g_noalloc_mid is not a device address; cudaGetSymbolAddress gives the
// address in the context that is current, so it is looked up with the device
// current on the first call there and cached per device ordinal together
// with the context it belongs to. A new context on that ordinal (after
// cudaDeviceReset, or a non-primary context made current through the driver
// API) loads the module again at another address: the lookup is then repeated.
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return noalloc_fail(MLORA_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return noalloc_fail(MLORA_ERR_INVALID_ARGUMENT, "device ordinal out of range");
  void* ctx = current_context();
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr || ctx == nullptr || ctx != g_noalloc_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_mid);
    if (e != cudaSuccess || p == nullptr) {
      return noalloc_fail(MLORA_ERR_CUDA, e != cudaSuccess ? cudaGetErrorString(e) : "no scratch address");
    }
    g_noalloc_ptr[dev] = p;
    g_noalloc_ctx[dev] = ctx;  // nullptr (unreadable context): looked up again on every call
  }
  *out = g_noalloc_ptr[dev];
  return MLORA_OK;
}

int elem_bytes(int32_t dt) { return dt == MLORA_F32 ? 4 : (dt == MLORA_BF16 || dt == MLORA_F16) ? 2 : 0; }

}  // namespace

extern "C" {

int mlora_apply_lora_group_noalloc(const void* x, int64_t rows, int64_t in_dim, int64_t x_row_stride, int32_t n,
                                   const void* const* a_stacks, const void* const* b_stacks, const int64_t* out_dims,
                                   void* const* ys, const int64_t* y_row_strides, int64_t max_rank,
                                   const mlora_kernel_input_metadata_t* meta, int32_t dtype, uint32_t* status,
                                   void* stream) {
  const int es = elem_bytes(dtype);
  if (es == 0) return noalloc_fail(MLORA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype");
  if (rows < 0 || rows > INT32_MAX || max_rank <= 0 || max_rank > 65535)
    return noalloc_fail(MLORA_ERR_INVALID_ARGUMENT, "rows or max_rank out of range");
  // rows < 2^31 and max_rank * es < 2^18: the product cannot wrap in 64 bits
  if ((uint64_t)rows * (uint64_t)max_rank * (uint64_t)es > kNoAllocScratchBytes)
    return noalloc_fail(MLORA_ERR_INVALID_ARGUMENT,
                        "rows * max_rank * element size exceeds the 1 MiB no-alloc scratch "
                        "(use mlora_apply_lora_group with a caller buffer)");
  if (n < 1 || n > 4) return noalloc_fail(MLORA_ERR_INVALID_ARGUMENT, "projection count outside [1, 4]");
  if (a_stacks == nullptr || b_stacks == nullptr || out_dims == nullptr || ys == nullptr || y_row_strides == nullptr)
    return noalloc_fail(MLORA_ERR_INVALID_ARGUMENT, "projection arrays are NULL");
  void* mid = nullptr;
  if (int rc = scratch_for_current_device(&mid)) return rc;
  // shrink then expand for each projection, through the scratch mid (row stride max_rank)
  for (int i = 0; i < n; ++i) {
    int rc = mlora_sgemm_lora_a_fwd(x, rows, in_dim, x_row_stride, a_stacks[i], max_rank, meta, mid, max_rank, dtype,
                                    dtype, 1, status, stream);
    if (rc != MLORA_OK) return rc;
    rc = mlora_sgemm_lora_b_fwd(mid, rows, max_rank, dtype, b_stacks[i], out_dims[i], max_rank, meta, ys[i],
                                y_row_strides[i], dtype, status, stream);
    if (rc != MLORA_OK) return rc;
  }
  return MLORA_OK;
}

}  // extern "C"
