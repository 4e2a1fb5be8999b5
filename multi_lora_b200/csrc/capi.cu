// C-ABI entry points (include/mlora_b200.h): argument validation, layout
// checks that pick the vectorised or scalar kernel, and launch.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "../../include/mlora_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace {

thread_local char g_err[512] = {0};
thread_local int g_last_apply_path = 0;  // 1 fused, 2 shrink + expand, 3 streaming pair, 4 tensor-core pair
int g_pdl = -1;  // -1: not read from the environment yet

// apply_lora path choice: 0 = automatic; MLORA_APPLY_PATH=fused|split|stream|tc
// forces one (tuning and tests; a forced path the shape does not fit falls
// through to the next one: tc -> stream -> fused -> split).
int g_apply_path = -1;  // -1: not read from the environment yet
int apply_path_override() {
  if (g_apply_path < 0) {
    const char* e = getenv("MLORA_APPLY_PATH");
    g_apply_path = e == nullptr ? 0 : strcmp(e, "fused") == 0 ? 1 : strcmp(e, "split") == 0 ? 2
                 : strcmp(e, "stream") == 0 ? 3 : strcmp(e, "tc") == 0 ? 4 : 0;
  }
  return g_apply_path;
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MLORA_OK;
  return fail(MLORA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool pdl_on() {
  if (g_pdl < 0) {
    const char* v = getenv("MLORA_PDL");
    g_pdl = (v != nullptr && v[0] == '0') ? 0 : 1;
  }
  return g_pdl != 0;
}

int elem_size(int32_t dt) {
  switch (dt) {
    case MLORA_BF16:
    case MLORA_F16: return 2;
    case MLORA_F32: return 4;
  }
  return 0;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_meta(const mlora_kernel_input_metadata_t* m, int64_t rows) {
  if (m == nullptr) return fail(MLORA_ERR_INVALID_ARGUMENT, "kernel_input_metadata is NULL");
  if (m->bs < 0) return fail(MLORA_ERR_INVALID_ARGUMENT, "bs must be >= 0 (got %d)", m->bs);
  if (m->num_slots <= 0) return fail(MLORA_ERR_INVALID_ARGUMENT, "num_slots must be > 0 (got %d)", m->num_slots);
  if (m->num_slots > 65535) return fail(MLORA_ERR_INVALID_ARGUMENT, "num_slots %d > 65535", m->num_slots);
  if (m->bs > 0 && (m->seg_indptr == nullptr || m->weight_indices == nullptr))
    return fail(MLORA_ERR_INVALID_ARGUMENT, "seg_indptr / weight_indices are NULL");
  if (m->lora_ranks == nullptr) return fail(MLORA_ERR_INVALID_ARGUMENT, "lora_ranks is NULL");
  if (rows < 0 || rows > INT32_MAX) return fail(MLORA_ERR_INVALID_ARGUMENT, "rows %lld out of range", (long long)rows);
  return MLORA_OK;
}

}  // namespace

namespace mlora {
int report_error(int code, const char* msg) { return fail(code, "%s", msg); }
int forced_apply_path() { return apply_path_override(); }
void note_apply_path(int path) { g_last_apply_path = path; }
}  // namespace mlora

extern "C" {

const char* mlora_last_error(void) { return g_err; }
int mlora_version(void) { return 100; }
int mlora_last_apply_path(void) { return g_last_apply_path; }

void mlora_set_apply_path(int path) { g_apply_path = (path >= 0 && path <= 4) ? path : 0; }

int mlora_get_apply_path(void) { return apply_path_override(); }
void mlora_set_pdl(int enable) { g_pdl = enable ? 1 : 0; }
int mlora_get_pdl(void) { return pdl_on() ? 1 : 0; }

int mlora_sgemm_lora_a_fwd(const void* x, int64_t rows, int64_t in_dim, int64_t x_row_stride,
                           const void* weights, int64_t max_rank,
                           const mlora_kernel_input_metadata_t* meta,
                           void* output, int64_t output_row_stride, int32_t output_dtype,
                           int32_t dtype, int32_t stack_num, uint32_t* status, void* stream) {
  g_err[0] = 0;
  if (int rc = check_meta(meta, rows)) return rc;
  const int es = elem_size(dtype);
  if (es == 0) return fail(MLORA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code %d", dtype);
  const bool out_f32 = output_dtype == MLORA_F32 && dtype != MLORA_F32;
  if (output_dtype != dtype && !out_f32)
    return fail(MLORA_ERR_UNSUPPORTED_DTYPE, "output dtype %d must equal dtype %d or be f32", output_dtype, dtype);
  if (in_dim <= 0 || in_dim > INT32_MAX) return fail(MLORA_ERR_INVALID_ARGUMENT, "in_dim %lld invalid", (long long)in_dim);
  if (max_rank <= 0 || max_rank > 65535 * 4)
    return fail(MLORA_ERR_INVALID_ARGUMENT, "max_rank %lld invalid", (long long)max_rank);
  if (stack_num < 1) return fail(MLORA_ERR_INVALID_ARGUMENT, "stack_num must be >= 1");
  if (x_row_stride < in_dim) return fail(MLORA_ERR_INVALID_ARGUMENT, "x_row_stride < in_dim");
  if (output_row_stride < max_rank) return fail(MLORA_ERR_INVALID_ARGUMENT, "output_row_stride < max_rank");
  if (meta->bs == 0 || rows == 0) return MLORA_OK;
  if (x == nullptr || weights == nullptr || output == nullptr)
    return fail(MLORA_ERR_INVALID_ARGUMENT, "x / weights / output is NULL");

  // Short segments (decode): the streaming shrink kernel alone (its fp32
  // output mode is the tensor-parallel shrink partial); at cfg2's 64 rows the
  // streaming pair measured 1.8x faster than the general shrink + expand.
  const int forced = apply_path_override();
  const bool stream_pref = forced == 3 || (forced != 2 && meta->max_len <= 64);
  if (stream_pref && es == 2 && stack_num == 1 && in_dim % 16 == 0 && max_rank % 8 == 0 && max_rank <= 64 &&
      aligned(x, 16) && x_row_stride % 8 == 0 && aligned(weights, 16) && rows <= INT32_MAX) {
    mlora::StreamArgs sa{};
    sa.x = x;
    sa.x_stride = x_row_stride;
    sa.n_mod = 1;
    sa.mod[0].a = weights;
    sa.mid = output;
    sa.mid_stride = output_row_stride;
    sa.mid_f32 = out_f32 ? 1 : 0;
    sa.phase = 1;
    sa.seg_indptr = meta->seg_indptr;
    sa.weight_indices = meta->weight_indices;
    sa.lora_ranks = meta->lora_ranks;
    sa.scalings = meta->scalings;
    sa.scalings_dtype = meta->scalings_dtype;
    sa.bs = meta->bs;
    sa.S = (int)rows;
    sa.in_dim = (int)in_dim;
    sa.R = (int)max_rank;
    sa.num_slots = meta->num_slots;
    sa.status = status;
    const cudaError_t e = mlora::launch_apply_stream(sa, dtype, (cudaStream_t)stream, pdl_on());
    if (e == cudaSuccess) {
      g_last_apply_path = 3;
      return MLORA_OK;
    }
    if (e != cudaErrorNotSupported) return cuda_status(e, "streaming shrink launch");
  }

  mlora::ShrinkArgs a{};
  a.x = x;
  a.x_stride = x_row_stride;
  a.w = weights;
  a.w_row_stride = in_dim;
  a.w_slot_stride = max_rank * in_dim;
  a.out = output;
  a.out_stride = output_row_stride;
  a.seg_indptr = meta->seg_indptr;
  a.weight_indices = meta->weight_indices;
  a.lora_ranks = meta->lora_ranks;
  a.bs = meta->bs;
  a.S = (int)rows;
  a.in_dim = (int)in_dim;
  a.max_rank = (int)max_rank;
  a.num_slots = meta->num_slots;
  a.stack_num = stack_num;
  a.status = status;
  const int V = 16 / es;
  a.vec_ok = (in_dim % V == 0) && (x_row_stride % V == 0) && aligned(x, 16) && aligned(weights, 16);
  g_last_apply_path = 2;
  return cuda_status(mlora::launch_shrink(a, dtype, out_f32, (cudaStream_t)stream, pdl_on()), "shrink launch");
}

int mlora_sgemm_lora_b_fwd(const void* mid, int64_t rows, int64_t mid_row_stride, int32_t mid_dtype,
                           const void* weights, int64_t out_dim, int64_t max_rank,
                           const mlora_kernel_input_metadata_t* meta,
                           void* y, int64_t y_row_stride,
                           int32_t dtype, uint32_t* status, void* stream) {
  g_err[0] = 0;
  if (int rc = check_meta(meta, rows)) return rc;
  const int es = elem_size(dtype);
  if (es == 0) return fail(MLORA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code %d", dtype);
  const bool mid_f32 = mid_dtype == MLORA_F32 && dtype != MLORA_F32;
  if (mid_dtype != dtype && !mid_f32)
    return fail(MLORA_ERR_UNSUPPORTED_DTYPE, "mid dtype %d must equal dtype %d or be f32", mid_dtype, dtype);
  if (elem_size(meta->scalings_dtype) == 0)
    return fail(MLORA_ERR_UNSUPPORTED_DTYPE, "unsupported scalings dtype %d", meta->scalings_dtype);
  if (meta->scalings == nullptr) return fail(MLORA_ERR_INVALID_ARGUMENT, "scalings is NULL");
  if (out_dim <= 0 || out_dim > INT32_MAX) return fail(MLORA_ERR_INVALID_ARGUMENT, "out_dim %lld invalid", (long long)out_dim);
  if (max_rank <= 0 || max_rank > 65535) return fail(MLORA_ERR_INVALID_ARGUMENT, "max_rank %lld invalid", (long long)max_rank);
  if (mid_row_stride < max_rank) return fail(MLORA_ERR_INVALID_ARGUMENT, "mid_row_stride < max_rank");
  if (y_row_stride < out_dim) return fail(MLORA_ERR_INVALID_ARGUMENT, "y_row_stride < out_dim");
  if (meta->bs == 0 || rows == 0) return MLORA_OK;
  if (mid == nullptr || weights == nullptr || y == nullptr)
    return fail(MLORA_ERR_INVALID_ARGUMENT, "mid / weights / y is NULL");

  // Short segments (decode): the streaming expand kernel alone. An fp32 mid (the
  // all-reduced tensor-parallel shrink partials) is rounded to the activation
  // dtype as the kernel loads it, as the reference rounds mid before the product.
  const int forced = apply_path_override();
  const bool stream_pref = forced == 3 || (forced != 2 && meta->max_len <= 64);
  const int mid_es = mid_f32 ? 4 : es;
  if (stream_pref && es == 2 && max_rank % 8 == 0 && max_rank <= 64 && out_dim % 8 == 0 && aligned(y, 16) &&
      y_row_stride % 8 == 0 && aligned(weights, 16) && aligned(mid, 16) && (mid_row_stride * mid_es) % 16 == 0 &&
      rows <= INT32_MAX) {
    mlora::StreamArgs sa{};
    sa.n_mod = 1;
    sa.mod[0].b = weights;
    sa.mod[0].y = y;
    sa.mod[0].y_stride = y_row_stride;
    sa.mod[0].out_dim = (int)out_dim;
    sa.mid = const_cast<void*>(mid);
    sa.mid_stride = mid_row_stride;
    sa.mid_f32 = mid_f32 ? 1 : 0;
    sa.phase = 2;
    sa.seg_indptr = meta->seg_indptr;
    sa.weight_indices = meta->weight_indices;
    sa.lora_ranks = meta->lora_ranks;
    sa.scalings = meta->scalings;
    sa.scalings_dtype = meta->scalings_dtype;
    sa.bs = meta->bs;
    sa.S = (int)rows;
    sa.R = (int)max_rank;
    sa.num_slots = meta->num_slots;
    sa.status = status;
    const cudaError_t e = mlora::launch_apply_stream(sa, dtype, (cudaStream_t)stream, pdl_on());
    if (e == cudaSuccess) {
      g_last_apply_path = 3;
      return MLORA_OK;
    }
    if (e != cudaErrorNotSupported) return cuda_status(e, "streaming expand launch");
  }

  mlora::ExpandArgs a{};
  a.mid = mid;
  a.mid_stride = mid_row_stride;
  a.w = weights;
  a.w_row_stride = max_rank;
  a.w_slot_stride = out_dim * max_rank;
  a.y = y;
  a.y_stride = y_row_stride;
  a.seg_indptr = meta->seg_indptr;
  a.weight_indices = meta->weight_indices;
  a.lora_ranks = meta->lora_ranks;
  a.scalings = meta->scalings;
  a.scalings_dtype = meta->scalings_dtype;
  a.bs = meta->bs;
  a.S = (int)rows;
  a.out_dim = (int)out_dim;
  a.max_rank = (int)max_rank;
  a.num_slots = meta->num_slots;
  a.status = status;
  const int V = 16 / es;
  a.vec_ok = (max_rank % V == 0) && aligned(weights, 16);
  a.y_vec_ok = (y_row_stride % 2 == 0) && aligned(y, 2 * es);
  g_last_apply_path = 2;
  return cuda_status(mlora::launch_expand(a, dtype, mid_f32, (cudaStream_t)stream, pdl_on()), "expand launch");
}

namespace {

// Shared body of mlora_apply_lora / mlora_apply_lora_group: one fused launch
// over every projection when the shape allows it, else shrink + expand per
// projection through `mid`. `mids` (optional, per projection) receive the
// shrink output on the fused path.
int apply_impl(const void* x, int64_t rows, int64_t in_dim, int64_t x_row_stride, int32_t n,
               const void* const* a_stacks, const void* const* b_stacks, const int64_t* out_dims,
               void* const* mids, void* mid, int64_t mid_row_stride, void* const* ys, const int64_t* y_row_strides,
               int64_t max_rank, const mlora_kernel_input_metadata_t* meta, int32_t dtype, uint32_t* status,
               void* stream) {
  g_err[0] = 0;
  if (int rc = check_meta(meta, rows)) return rc;
  const int es = elem_size(dtype);
  if (es == 0) return fail(MLORA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code %d", dtype);
  if (n < 1 || n > mlora::kMaxFusedModules)
    return fail(MLORA_ERR_INVALID_ARGUMENT, "projection count %d outside [1, %d]", n, mlora::kMaxFusedModules);
  if (in_dim <= 0 || in_dim > INT32_MAX) return fail(MLORA_ERR_INVALID_ARGUMENT, "in_dim %lld invalid", (long long)in_dim);
  if (max_rank <= 0 || max_rank > 65535) return fail(MLORA_ERR_INVALID_ARGUMENT, "max_rank %lld invalid", (long long)max_rank);
  if (x_row_stride < in_dim) return fail(MLORA_ERR_INVALID_ARGUMENT, "x_row_stride < in_dim");
  if (a_stacks == nullptr || b_stacks == nullptr || out_dims == nullptr || ys == nullptr || y_row_strides == nullptr)
    return fail(MLORA_ERR_INVALID_ARGUMENT, "projection arrays are NULL");
  for (int i = 0; i < n; ++i) {
    if (out_dims[i] <= 0 || out_dims[i] > INT32_MAX)
      return fail(MLORA_ERR_INVALID_ARGUMENT, "out_dim[%d] %lld invalid", i, (long long)out_dims[i]);
    if (y_row_strides[i] < out_dims[i]) return fail(MLORA_ERR_INVALID_ARGUMENT, "y_row_stride[%d] < out_dim", i);
  }
  if (meta->bs == 0 || rows == 0) return MLORA_OK;
  if (meta->scalings == nullptr) return fail(MLORA_ERR_INVALID_ARGUMENT, "scalings is NULL");
  if (elem_size(meta->scalings_dtype) == 0)
    return fail(MLORA_ERR_UNSUPPORTED_DTYPE, "unsupported scalings dtype %d", meta->scalings_dtype);
  const int forced = apply_path_override();
  // Automatic choice: the streaming pair for large decode batches (it keeps
  // one CTA per SM busy whatever the slot count; measured 2x faster than the
  // fused kernel at 512 tokens x 128 adapters), the fused kernel below that
  // (one launch, shorter dependency chain: 2.2x faster at 64 tokens x 32 adapters).
  // Long segments (prefill) go to the tensor-core kernels when the shape fits them.
  const bool tc_pref = forced == 4 || (forced == 0 && meta->max_len >= 64);
  bool tcable = tc_pref && es == 2 && (max_rank == 16 || max_rank == 32 || max_rank == 64) && in_dim % 64 == 0 && x != nullptr && aligned(x, 16) &&
                x_row_stride % 8 == 0 && mid != nullptr && aligned(mid, 16) && mid_row_stride % 8 == 0 &&
                mid_row_stride >= (int64_t)n * max_rank && (mids == nullptr || mids[0] == mid) && rows <= INT32_MAX;
  for (int i = 0; i < n && tcable; ++i)
    tcable = a_stacks[i] != nullptr && b_stacks[i] != nullptr && ys[i] != nullptr && aligned(a_stacks[i], 16) &&
             aligned(b_stacks[i], 16) && aligned(ys[i], 16) && y_row_strides[i] % 8 == 0 && out_dims[i] % 8 == 0;
  if (tcable) {
    mlora::PrefillLaunch pl{};
    pl.x = x;
    pl.x_stride = x_row_stride;
    pl.n_mod = n;
    for (int i = 0; i < n; ++i) {
      pl.mod[i].a = a_stacks[i];
      pl.mod[i].b = b_stacks[i];
      pl.mod[i].y = ys[i];
      pl.mod[i].y_stride = y_row_strides[i];
      pl.mod[i].out_dim = (int)out_dims[i];
    }
    pl.mid = mid;
    pl.mid_stride = mid_row_stride;
    pl.seg_indptr = meta->seg_indptr;
    pl.weight_indices = meta->weight_indices;
    pl.lora_ranks = meta->lora_ranks;
    pl.scalings = meta->scalings;
    pl.scalings_dtype = meta->scalings_dtype;
    pl.bs = meta->bs;
    pl.S = (int)rows;
    pl.in_dim = (int)in_dim;
    pl.R = (int)max_rank;
    pl.num_slots = meta->num_slots;
    pl.status = status;
    const cudaError_t e = mlora::launch_apply_prefill(pl, dtype, (cudaStream_t)stream, pdl_on());
    if (e == cudaSuccess) {
      g_last_apply_path = 4;
      return MLORA_OK;
    }
    if (e != cudaErrorNotSupported) return cuda_status(e, "tensor-core apply_lora launch");
  }
  const bool stream_pref = forced == 3 || forced == 4 || (forced == 0 && rows >= 256 && meta->max_len <= 64);
  bool streamable = stream_pref && es == 2 && x != nullptr && aligned(x, 16) &&
                    x_row_stride % 8 == 0 && in_dim % 16 == 0 && max_rank % 8 == 0 && max_rank <= 64 &&
                    mid != nullptr && aligned(mid, 16) && mid_row_stride % 8 == 0 &&
                    mid_row_stride >= (int64_t)n * max_rank && (mids == nullptr || mids[0] == mid);
  for (int i = 0; i < n && streamable; ++i)
    streamable = a_stacks[i] != nullptr && b_stacks[i] != nullptr && ys[i] != nullptr && aligned(a_stacks[i], 16) &&
                 aligned(b_stacks[i], 16) && aligned(ys[i], 16) && y_row_strides[i] % 8 == 0 && out_dims[i] % 8 == 0;
  if (streamable) {
    mlora::StreamArgs sa{};
    sa.x = x;
    sa.x_stride = x_row_stride;
    sa.n_mod = n;
    for (int i = 0; i < n; ++i) {
      sa.mod[i].a = a_stacks[i];
      sa.mod[i].b = b_stacks[i];
      sa.mod[i].y = ys[i];
      sa.mod[i].y_stride = y_row_strides[i];
      sa.mod[i].out_dim = (int)out_dims[i];
    }
    sa.mid = mid;
    sa.mid_stride = mid_row_stride;
    sa.seg_indptr = meta->seg_indptr;
    sa.weight_indices = meta->weight_indices;
    sa.lora_ranks = meta->lora_ranks;
    sa.scalings = meta->scalings;
    sa.scalings_dtype = meta->scalings_dtype;
    sa.bs = meta->bs;
    sa.S = (int)rows;
    sa.in_dim = (int)in_dim;
    sa.R = (int)max_rank;
    sa.num_slots = meta->num_slots;
    sa.status = status;
    const cudaError_t e = mlora::launch_apply_stream(sa, dtype, (cudaStream_t)stream, pdl_on());
    if (e == cudaSuccess) {
      g_last_apply_path = 3;
      return MLORA_OK;
    }
    if (e != cudaErrorNotSupported) return cuda_status(e, "streaming apply_lora launch");
  }
  bool fusable = forced != 2 && es == 2 && meta->max_len <= 16 && rows <= 64LL * meta->num_slots && x != nullptr &&
                 x_row_stride % 8 == 0 && aligned(x, 16);
  for (int i = 0; i < n && fusable; ++i)
    fusable = a_stacks[i] != nullptr && b_stacks[i] != nullptr && ys[i] != nullptr && aligned(a_stacks[i], 16) &&
              aligned(b_stacks[i], 16) && (mids == nullptr || mids[i] == nullptr || mid_row_stride >= max_rank);
  if (fusable) {
    mlora::FusedArgs f{};
    f.x = x;
    f.x_stride = x_row_stride;
    f.n_mod = n;
    for (int i = 0; i < n; ++i) {
      mlora::FusedModule& m = f.mod[i];
      m.a = a_stacks[i];
      m.b = b_stacks[i];
      m.y = ys[i];
      m.y_stride = y_row_strides[i];
      m.mid = mids != nullptr ? mids[i] : nullptr;
      m.mid_stride = mid_row_stride;
      m.out_dim = (int)out_dims[i];
    }
    f.seg_indptr = meta->seg_indptr;
    f.weight_indices = meta->weight_indices;
    f.lora_ranks = meta->lora_ranks;
    f.scalings = meta->scalings;
    f.scalings_dtype = meta->scalings_dtype;
    f.bs = meta->bs;
    f.S = (int)rows;
    f.in_dim = (int)in_dim;
    f.R = (int)max_rank;
    f.num_slots = meta->num_slots;
    f.status = status;
    const cudaError_t e = mlora::launch_apply_fused(f, dtype, (cudaStream_t)stream, pdl_on());
    if (e == cudaSuccess) {
      g_last_apply_path = 1;
      return MLORA_OK;
    }
    if (e != cudaErrorNotSupported) return cuda_status(e, "fused apply_lora launch");
  }
  g_last_apply_path = 2;
  if (mid == nullptr) return fail(MLORA_ERR_INVALID_ARGUMENT, "mid buffer required for this shape");
  for (int i = 0; i < n; ++i) {
    int rc = mlora_sgemm_lora_a_fwd(x, rows, in_dim, x_row_stride, a_stacks[i], max_rank, meta, mid, mid_row_stride,
                                    dtype, dtype, 1, status, stream);
    if (rc != MLORA_OK) return rc;
    rc = mlora_sgemm_lora_b_fwd(mid, rows, mid_row_stride, dtype, b_stacks[i], out_dims[i], max_rank, meta, ys[i],
                                y_row_strides[i], dtype, status, stream);
    if (rc != MLORA_OK) return rc;
  }
  g_last_apply_path = 2;  // separate shrink and expand launches, whichever kernels they took
  return MLORA_OK;
}

}  // namespace

int mlora_apply_lora(const void* x, int64_t rows, int64_t in_dim, int64_t x_row_stride,
                     const void* a_stack, const void* b_stack, int64_t out_dim, int64_t max_rank,
                     const mlora_kernel_input_metadata_t* meta,
                     void* mid, int64_t mid_row_stride,
                     void* y, int64_t y_row_stride,
                     int32_t dtype, uint32_t* status, void* stream) {
  void* const mids[1] = {mid};
  void* const ys[1] = {y};
  const int64_t y_strides[1] = {y_row_stride};
  const int64_t outs[1] = {out_dim};
  return apply_impl(x, rows, in_dim, x_row_stride, 1, &a_stack, &b_stack, outs, mids, mid, mid_row_stride, ys,
                    y_strides, max_rank, meta, dtype, status, stream);
}

int mlora_apply_lora_group(const void* x, int64_t rows, int64_t in_dim, int64_t x_row_stride, int32_t n,
                           const void* const* a_stacks, const void* const* b_stacks, const int64_t* out_dims,
                           void* const* ys, const int64_t* y_row_strides, int64_t max_rank,
                           const mlora_kernel_input_metadata_t* meta, void* mid, int64_t mid_row_stride,
                           int32_t dtype, uint32_t* status, void* stream) {
  return apply_impl(x, rows, in_dim, x_row_stride, n, a_stacks, b_stacks, out_dims, nullptr, mid, mid_row_stride, ys,
                    y_row_strides, max_rank, meta, dtype, status, stream);
}

int mlora_rmsnorm_fwd(const void* x, int64_t rows, int64_t hidden, int64_t stride_outer,
                      int64_t stride_inner, int64_t inner, const void* w, int32_t w_dtype,
                      void* y, int64_t y_row_stride, float eps, int32_t dtype, void* stream) {
  g_err[0] = 0;
  const int es = elem_size(dtype);
  if (es == 0) return fail(MLORA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code %d", dtype);
  if (elem_size(w_dtype) == 0) return fail(MLORA_ERR_UNSUPPORTED_DTYPE, "unsupported weight dtype %d", w_dtype);
  if (hidden <= 0 || hidden > INT32_MAX) return fail(MLORA_ERR_INVALID_ARGUMENT, "hidden %lld invalid", (long long)hidden);
  if (rows < 0) return fail(MLORA_ERR_INVALID_ARGUMENT, "rows < 0");
  if (inner <= 0) return fail(MLORA_ERR_INVALID_ARGUMENT, "inner must be > 0");
  if (y_row_stride < hidden) return fail(MLORA_ERR_INVALID_ARGUMENT, "y_row_stride < hidden");
  if (rows == 0) return MLORA_OK;
  if (x == nullptr || w == nullptr || y == nullptr) return fail(MLORA_ERR_INVALID_ARGUMENT, "x / w / y is NULL");
  if ((rows + 31) / 32 > 2147483647LL) return fail(MLORA_ERR_INVALID_ARGUMENT, "too many rows");

  mlora::RmsNormArgs a{};
  a.x = x;
  a.stride_outer = stride_outer;
  a.stride_inner = stride_inner;
  a.inner = inner;
  a.w = w;
  a.w_dtype = w_dtype;
  a.y = y;
  a.y_stride = y_row_stride;
  a.rows = rows;
  a.hidden = (int)hidden;
  a.eps = eps;
  const int V = 16 / es;
  a.vec_ok = (hidden % V == 0) && (stride_outer % V == 0) && (stride_inner % V == 0) && (y_row_stride % V == 0) &&
             aligned(x, 16) && aligned(y, 16);
  a.w_vec = aligned(w, 16);
  return cuda_status(mlora::launch_rmsnorm(a, dtype, (cudaStream_t)stream, pdl_on()), "rmsnorm launch");
}

int mlora_fused_add_rmsnorm_fwd(const void* x, int64_t x_row_stride, void* residual, int64_t residual_row_stride,
                                int64_t rows, int64_t hidden, const void* w, int32_t w_dtype, void* y,
                                int64_t y_row_stride, float eps, int32_t dtype, void* stream) {
  g_err[0] = 0;
  const int es = elem_size(dtype);
  if (es == 0) return fail(MLORA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code %d", dtype);
  if (elem_size(w_dtype) == 0) return fail(MLORA_ERR_UNSUPPORTED_DTYPE, "unsupported weight dtype %d", w_dtype);
  if (hidden <= 0 || hidden > INT32_MAX) return fail(MLORA_ERR_INVALID_ARGUMENT, "hidden %lld invalid", (long long)hidden);
  if (rows < 0) return fail(MLORA_ERR_INVALID_ARGUMENT, "rows < 0");
  if (x_row_stride < hidden || residual_row_stride < hidden || y_row_stride < hidden)
    return fail(MLORA_ERR_INVALID_ARGUMENT, "a row stride is smaller than hidden");
  if (rows == 0) return MLORA_OK;
  if (x == nullptr || residual == nullptr || w == nullptr || y == nullptr)
    return fail(MLORA_ERR_INVALID_ARGUMENT, "x / residual / w / y is NULL");
  mlora::RmsNormArgs a{};
  a.x = residual;  // rows read, summed with x, written back, normalised
  a.stride_outer = residual_row_stride;
  a.stride_inner = 0;
  a.inner = 1;
  a.add = x;
  a.add_stride = x_row_stride;
  a.res = residual;
  a.res_stride = residual_row_stride;
  a.w = w;
  a.w_dtype = w_dtype;
  a.y = y;
  a.y_stride = y_row_stride;
  a.rows = rows;
  a.hidden = (int)hidden;
  a.eps = eps;
  const int V = 16 / es;
  a.vec_ok = (hidden % V == 0) && (x_row_stride % V == 0) && (residual_row_stride % V == 0) &&
             (y_row_stride % V == 0) && aligned(x, 16) && aligned(residual, 16) && aligned(y, 16);
  a.w_vec = aligned(w, 16);
  return cuda_status(mlora::launch_rmsnorm(a, dtype, (cudaStream_t)stream, pdl_on()), "fused add + rmsnorm launch");
}

int mlora_scatter_stage(const void* stage, int64_t stage_row_elems, int32_t h, const int64_t* slots,
                        const mlora_scatter_rect_t* rects, int32_t n_rects, int64_t max_rect_elems,
                        int32_t dtype, uint32_t* status, void* stream) {
  g_err[0] = 0;
  const int es = elem_size(dtype);
  if (es == 0) return fail(MLORA_ERR_UNSUPPORTED_DTYPE, "unsupported dtype code %d", dtype);
  if (h < 0 || n_rects < 0 || stage_row_elems < 0 || max_rect_elems < 0)
    return fail(MLORA_ERR_INVALID_ARGUMENT, "negative size");
  if (h == 0 || n_rects == 0 || max_rect_elems == 0) return MLORA_OK;
  if (h > 65535) return fail(MLORA_ERR_INVALID_ARGUMENT, "h %d > 65535", h);
  if (stage == nullptr || slots == nullptr || rects == nullptr)
    return fail(MLORA_ERR_INVALID_ARGUMENT, "stage / slots / rects is NULL");
  const cudaError_t e = mlora::launch_scatter(stage, stage_row_elems, h, slots, rects, n_rects, max_rect_elems, es,
                                              status, (cudaStream_t)stream);
  if (e == cudaErrorInvalidValue) return fail(MLORA_ERR_INVALID_ARGUMENT, "rectangle too large for one launch");
  return cuda_status(e, "scatter launch");
}

}  // extern "C"
