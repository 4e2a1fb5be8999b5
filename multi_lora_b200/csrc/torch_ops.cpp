// torch.ops.mlora.* — a thin PyTorch binding over the C ABI (include/mlora_b200.h).
// Checks what the reference asserts (kernels/sgemm_lora_a.py:199-208,
// sgemm_lora_b.py:168-174: contiguous rank-2 x / rank-3 weights) plus dtype,
// device and metadata-length checks, then forwards device pointers and the
// current CUDA stream. No op allocates except rmsnorm (whose reference
// allocates its output, kernels/rmsnorm.py:76); rmsnorm_out writes in place.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <vector>

#include "../../include/mlora_b200.h"

namespace {

int32_t dt_code(at::ScalarType t) {
  switch (t) {
    case at::kBFloat16: return MLORA_BF16;
    case at::kHalf: return MLORA_F16;
    case at::kFloat: return MLORA_F32;
    default: TORCH_CHECK(false, "mlora: unsupported dtype ", t);
  }
  return -1;
}

void check_cuda(const at::Tensor& t, const char* name, const at::Device& dev) {
  TORCH_CHECK(t.is_cuda(), "mlora: ", name, " must be a CUDA tensor");
  TORCH_CHECK(t.device() == dev, "mlora: ", name, " is on ", t.device(), ", expected ", dev);
}

void check_i32(const at::Tensor& t, const char* name, int64_t min_len, const at::Device& dev) {
  check_cuda(t, name, dev);
  TORCH_CHECK(t.scalar_type() == at::kInt, "mlora: ", name, " must be int32 (got ", t.scalar_type(), ")");
  TORCH_CHECK(t.dim() == 1 && t.is_contiguous(), "mlora: ", name, " must be a contiguous 1-D tensor");
  TORCH_CHECK(t.numel() >= min_len, "mlora: ", name, " has ", t.numel(), " entries, needs >= ", min_len);
}

uint32_t* status_ptr(const c10::optional<at::Tensor>& status, const at::Device& dev) {
  if (!status.has_value()) return nullptr;
  const at::Tensor& s = *status;
  check_cuda(s, "status", dev);
  TORCH_CHECK(s.scalar_type() == at::kInt && s.numel() >= 1, "mlora: status must be an int32 tensor");
  return reinterpret_cast<uint32_t*>(s.data_ptr());
}

mlora_kernel_input_metadata_t make_meta(const at::Tensor& seg_lens, const at::Tensor& seg_indptr,
                                        const at::Tensor& weight_indices, const at::Tensor& lora_ranks,
                                        const at::Tensor* scalings, int64_t bs, int64_t max_len,
                                        const at::Device& dev) {
  TORCH_CHECK(bs >= 0, "mlora: bs must be >= 0");
  check_i32(seg_indptr, "seg_indptr", bs + 1, dev);
  check_i32(weight_indices, "weight_indices", bs, dev);
  check_i32(lora_ranks, "lora_ranks", 1, dev);
  if (seg_lens.defined() && seg_lens.numel() > 0) check_i32(seg_lens, "seg_lens", bs, dev);
  mlora_kernel_input_metadata_t m{};
  m.bs = (int32_t)bs;
  m.max_len = (int32_t)max_len;
  m.num_slots = (int32_t)lora_ranks.numel();
  m.seg_lens = seg_lens.defined() && seg_lens.numel() > 0 ? seg_lens.data_ptr<int32_t>() : nullptr;
  m.seg_indptr = seg_indptr.data_ptr<int32_t>();
  m.weight_indices = weight_indices.data_ptr<int32_t>();
  m.lora_ranks = lora_ranks.data_ptr<int32_t>();
  if (scalings != nullptr) {
    check_cuda(*scalings, "scalings", dev);
    TORCH_CHECK(scalings->dim() == 1 && scalings->is_contiguous(), "mlora: scalings must be contiguous 1-D");
    TORCH_CHECK(scalings->numel() >= m.num_slots, "mlora: scalings shorter than lora_ranks");
    m.scalings = scalings->data_ptr();
    m.scalings_dtype = dt_code(scalings->scalar_type());
  }
  return m;
}

void check_rc(int rc) { TORCH_CHECK(rc == MLORA_OK, "mlora: ", mlora_last_error()); }

at::Tensor sgemm_lora_a(const at::Tensor& x, const at::Tensor& weights, const at::Tensor& seg_lens,
                        const at::Tensor& seg_indptr, const at::Tensor& weight_indices,
                        const at::Tensor& lora_ranks, int64_t bs, int64_t max_len, at::Tensor output,
                        int64_t stack_num, const c10::optional<at::Tensor>& status) {
  const at::Device dev = x.device();
  check_cuda(x, "x", dev);
  check_cuda(weights, "weights", dev);
  check_cuda(output, "output", dev);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "mlora: x must be [S, in] with unit column stride");
  TORCH_CHECK(weights.dim() == 3 && weights.is_contiguous(), "mlora: weights must be contiguous [K, max_rank, in]");
  TORCH_CHECK(weights.size(2) == x.size(1), "mlora: weights in_dim ", weights.size(2), " != x in_dim ", x.size(1));
  TORCH_CHECK(weights.scalar_type() == x.scalar_type(), "mlora: weights dtype must match x");
  TORCH_CHECK(output.dim() == 2 && output.stride(1) == 1, "mlora: output must be 2-D with unit column stride");
  TORCH_CHECK(output.size(0) >= x.size(0) && output.size(1) >= weights.size(1),
              "mlora: output ", output.sizes(), " too small for [", x.size(0), ", ", weights.size(1), "]");
  TORCH_CHECK(lora_ranks.numel() == weights.size(0), "mlora: lora_ranks length != number of slots");
  const c10::cuda::CUDAGuard guard(dev);
  const auto meta = make_meta(seg_lens, seg_indptr, weight_indices, lora_ranks, nullptr, bs, max_len, dev);
  const int rc = mlora_sgemm_lora_a_fwd(
      x.data_ptr(), x.size(0), x.size(1), x.stride(0), weights.data_ptr(), weights.size(1), &meta,
      output.data_ptr(), output.stride(0), dt_code(output.scalar_type()), dt_code(x.scalar_type()),
      (int32_t)stack_num, status_ptr(status, dev), at::cuda::getCurrentCUDAStream().stream());
  check_rc(rc);
  return output;
}

at::Tensor sgemm_lora_b(const at::Tensor& x, const at::Tensor& weights, const at::Tensor& seg_lens,
                        const at::Tensor& seg_indptr, const at::Tensor& weight_indices,
                        const at::Tensor& lora_ranks, const at::Tensor& scalings, int64_t bs, int64_t max_len,
                        at::Tensor output, const c10::optional<at::Tensor>& status) {
  const at::Device dev = x.device();
  check_cuda(x, "x", dev);
  check_cuda(weights, "weights", dev);
  check_cuda(output, "output", dev);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "mlora: mid must be [S, max_rank] with unit column stride");
  TORCH_CHECK(weights.dim() == 3 && weights.is_contiguous(), "mlora: weights must be contiguous [K, out, max_rank]");
  TORCH_CHECK(x.size(1) >= weights.size(2), "mlora: mid has ", x.size(1), " columns, weights rank ", weights.size(2));
  TORCH_CHECK(output.dim() == 2 && output.stride(1) == 1, "mlora: output must be 2-D with unit column stride");
  TORCH_CHECK(output.size(1) == weights.size(1), "mlora: output width ", output.size(1), " != out_dim ", weights.size(1));
  TORCH_CHECK(output.size(0) == x.size(0), "mlora: output rows != mid rows");
  TORCH_CHECK(weights.scalar_type() == output.scalar_type(), "mlora: weights dtype must match output");
  TORCH_CHECK(lora_ranks.numel() == weights.size(0), "mlora: lora_ranks length != number of slots");
  const c10::cuda::CUDAGuard guard(dev);
  const auto meta = make_meta(seg_lens, seg_indptr, weight_indices, lora_ranks, &scalings, bs, max_len, dev);
  const int rc = mlora_sgemm_lora_b_fwd(
      x.data_ptr(), x.size(0), x.stride(0), dt_code(x.scalar_type()), weights.data_ptr(), weights.size(1),
      weights.size(2), &meta, output.data_ptr(), output.stride(0), dt_code(output.scalar_type()),
      status_ptr(status, dev), at::cuda::getCurrentCUDAStream().stream());
  check_rc(rc);
  return output;
}

// apply_lora (backend/base.py:60-89): shrink into `mid`, expand into `output`
// in place; one fused launch for short segments.
at::Tensor apply_lora(const at::Tensor& x, const at::Tensor& a_stack, const at::Tensor& b_stack,
                      const at::Tensor& seg_lens, const at::Tensor& seg_indptr, const at::Tensor& weight_indices,
                      const at::Tensor& lora_ranks, const at::Tensor& scalings, int64_t bs, int64_t max_len,
                      at::Tensor mid, at::Tensor output, const c10::optional<at::Tensor>& status) {
  const at::Device dev = x.device();
  check_cuda(x, "x", dev);
  check_cuda(a_stack, "a_stack", dev);
  check_cuda(b_stack, "b_stack", dev);
  check_cuda(mid, "mid", dev);
  check_cuda(output, "output", dev);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "mlora: x must be [S, in] with unit column stride");
  TORCH_CHECK(a_stack.dim() == 3 && a_stack.is_contiguous(), "mlora: a_stack must be contiguous [K, max_rank, in]");
  TORCH_CHECK(b_stack.dim() == 3 && b_stack.is_contiguous(), "mlora: b_stack must be contiguous [K, out, max_rank]");
  TORCH_CHECK(a_stack.size(2) == x.size(1), "mlora: a_stack in_dim ", a_stack.size(2), " != x in_dim ", x.size(1));
  TORCH_CHECK(a_stack.size(0) == b_stack.size(0) && a_stack.size(1) == b_stack.size(2),
              "mlora: a_stack ", a_stack.sizes(), " and b_stack ", b_stack.sizes(), " disagree");
  TORCH_CHECK(a_stack.scalar_type() == x.scalar_type() && b_stack.scalar_type() == x.scalar_type() &&
                  output.scalar_type() == x.scalar_type() && mid.scalar_type() == x.scalar_type(),
              "mlora: x, stacks, mid and output must share one dtype");
  TORCH_CHECK(mid.dim() == 2 && mid.stride(1) == 1 && mid.size(0) >= x.size(0) && mid.size(1) >= a_stack.size(1),
              "mlora: mid must be [>= S, >= max_rank] with unit column stride");
  TORCH_CHECK(output.dim() == 2 && output.stride(1) == 1 && output.size(0) == x.size(0) &&
                  output.size(1) == b_stack.size(1),
              "mlora: output must be [S, out] with unit column stride");
  TORCH_CHECK(lora_ranks.numel() == a_stack.size(0), "mlora: lora_ranks length != number of slots");
  const c10::cuda::CUDAGuard guard(dev);
  const auto meta = make_meta(seg_lens, seg_indptr, weight_indices, lora_ranks, &scalings, bs, max_len, dev);
  const int rc = mlora_apply_lora(x.data_ptr(), x.size(0), x.size(1), x.stride(0), a_stack.data_ptr(),
                                  b_stack.data_ptr(), b_stack.size(1), a_stack.size(1), &meta, mid.data_ptr(),
                                  mid.stride(0), output.data_ptr(), output.stride(0), dt_code(x.scalar_type()),
                                  status_ptr(status, dev), at::cuda::getCurrentCUDAStream().stream());
  check_rc(rc);
  return output;
}

// apply_lora over projections sharing x and the routing (q/k/v, gate/up).
void apply_lora_group(const at::Tensor& x, at::TensorList a_stacks, at::TensorList b_stacks,
                      const at::Tensor& seg_lens, const at::Tensor& seg_indptr, const at::Tensor& weight_indices,
                      const at::Tensor& lora_ranks, const at::Tensor& scalings, int64_t bs, int64_t max_len,
                      at::TensorList outputs, const c10::optional<at::Tensor>& mid,
                      const c10::optional<at::Tensor>& status) {
  const at::Device dev = x.device();
  check_cuda(x, "x", dev);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "mlora: x must be [S, in] with unit column stride");
  const int64_t n = (int64_t)a_stacks.size();
  TORCH_CHECK(n >= 1 && n <= 4 && (int64_t)b_stacks.size() == n && (int64_t)outputs.size() == n,
              "mlora: 1..4 projections with one a_stack, b_stack and output each");
  std::vector<const void*> a(n), b(n);
  std::vector<void*> y(n);
  std::vector<int64_t> outs(n), ystr(n);
  const int64_t R = a_stacks[0].size(1);
  for (int64_t i = 0; i < n; ++i) {
    check_cuda(a_stacks[i], "a_stack", dev);
    check_cuda(b_stacks[i], "b_stack", dev);
    check_cuda(outputs[i], "output", dev);
    TORCH_CHECK(a_stacks[i].dim() == 3 && a_stacks[i].is_contiguous() && a_stacks[i].size(2) == x.size(1) &&
                    a_stacks[i].size(1) == R && a_stacks[i].size(0) == lora_ranks.numel(),
                "mlora: a_stack ", i, " must be contiguous [K, max_rank, in]");
    TORCH_CHECK(b_stacks[i].dim() == 3 && b_stacks[i].is_contiguous() && b_stacks[i].size(2) == R &&
                    b_stacks[i].size(0) == lora_ranks.numel(),
                "mlora: b_stack ", i, " must be contiguous [K, out, max_rank]");
    TORCH_CHECK(outputs[i].dim() == 2 && outputs[i].stride(1) == 1 && outputs[i].size(0) == x.size(0) &&
                    outputs[i].size(1) == b_stacks[i].size(1),
                "mlora: output ", i, " must be [S, out] with unit column stride");
    TORCH_CHECK(a_stacks[i].scalar_type() == x.scalar_type() && b_stacks[i].scalar_type() == x.scalar_type() &&
                    outputs[i].scalar_type() == x.scalar_type(),
                "mlora: x, stacks and outputs must share one dtype");
    a[i] = a_stacks[i].data_ptr();
    b[i] = b_stacks[i].data_ptr();
    y[i] = outputs[i].data_ptr();
    outs[i] = b_stacks[i].size(1);
    ystr[i] = outputs[i].stride(0);
  }
  void* mid_ptr = nullptr;
  int64_t mid_stride = R;
  if (mid.has_value()) {
    check_cuda(*mid, "mid", dev);
    TORCH_CHECK(mid->dim() == 2 && mid->stride(1) == 1 && mid->size(0) >= x.size(0) && mid->size(1) >= R &&
                    mid->scalar_type() == x.scalar_type(),
                "mlora: mid must be [>= S, >= max_rank] like x");
    mid_ptr = mid->data_ptr();
    mid_stride = mid->stride(0);
  }
  const c10::cuda::CUDAGuard guard(dev);
  const auto meta = make_meta(seg_lens, seg_indptr, weight_indices, lora_ranks, &scalings, bs, max_len, dev);
  const int rc = mlora_apply_lora_group(x.data_ptr(), x.size(0), x.size(1), x.stride(0), (int32_t)n, a.data(),
                                        b.data(), outs.data(), y.data(), ystr.data(), R, &meta, mid_ptr, mid_stride,
                                        dt_code(x.scalar_type()), status_ptr(status, dev),
                                        at::cuda::getCurrentCUDAStream().stream());
  check_rc(rc);
}

// Two-level row addressing of the reference (kernels/rmsnorm.py:59-81).
void rms_layout(const at::Tensor& x, int64_t hidden, int64_t rows, int64_t& so, int64_t& si, int64_t& inner,
                at::Tensor& src) {
  src = x;
  if (x.is_contiguous()) {
    inner = rows > 0 ? rows : 1;
    so = 0;
    si = hidden;
  } else if (x.dim() >= 2 && x[0].is_contiguous() && x.stride(-1) == 1) {
    inner = rows / x.size(0);
    so = x.stride(0);
    si = hidden;
    if (inner == 0) inner = 1;
  } else {
    src = x.contiguous();
    inner = rows > 0 ? rows : 1;
    so = 0;
    si = hidden;
  }
}

at::Tensor rmsnorm_out(const at::Tensor& x, const at::Tensor& weight, double eps, at::Tensor out) {
  const at::Device dev = x.device();
  check_cuda(x, "x", dev);
  check_cuda(weight, "weight", dev);
  check_cuda(out, "out", dev);
  const int64_t hidden = x.size(-1);
  TORCH_CHECK(weight.numel() == hidden && weight.is_contiguous(), "mlora: weight must be contiguous [hidden]");
  TORCH_CHECK(out.scalar_type() == x.scalar_type() && out.is_contiguous() && out.numel() == x.numel(),
              "mlora: out must be a contiguous tensor like x");
  const int64_t rows = hidden > 0 ? x.numel() / hidden : 0;
  if (rows == 0) return out;
  int64_t so, si, inner;
  at::Tensor src;
  rms_layout(x, hidden, rows, so, si, inner, src);
  const c10::cuda::CUDAGuard guard(dev);
  const int rc = mlora_rmsnorm_fwd(src.data_ptr(), rows, hidden, so, si, inner, weight.data_ptr(),
                                   dt_code(weight.scalar_type()), out.data_ptr(), hidden, (float)eps,
                                   dt_code(x.scalar_type()), at::cuda::getCurrentCUDAStream().stream());
  check_rc(rc);
  return out;
}

at::Tensor rmsnorm(const at::Tensor& x, const at::Tensor& weight, double eps) {
  at::Tensor out = at::empty(x.sizes(), x.options().memory_format(at::MemoryFormat::Contiguous));
  return rmsnorm_out(x, weight, eps, out);
}

// residual = T(residual + x) in place, out = rmsnorm(residual) (one kernel).
void fused_add_rmsnorm(const at::Tensor& x, at::Tensor residual, const at::Tensor& weight, double eps,
                       at::Tensor out) {
  const at::Device dev = x.device();
  check_cuda(x, "x", dev);
  check_cuda(residual, "residual", dev);
  check_cuda(weight, "weight", dev);
  check_cuda(out, "out", dev);
  const int64_t hidden = x.size(-1);
  TORCH_CHECK(weight.numel() == hidden && weight.is_contiguous(), "mlora: weight must be contiguous [hidden]");
  TORCH_CHECK(residual.sizes() == x.sizes() && out.sizes() == x.sizes(), "mlora: x, residual and out must match");
  TORCH_CHECK(residual.scalar_type() == x.scalar_type() && out.scalar_type() == x.scalar_type(),
              "mlora: x, residual and out must share a dtype");
  TORCH_CHECK(x.is_contiguous() && residual.is_contiguous() && out.is_contiguous(),
              "mlora: x, residual and out must be contiguous");
  const int64_t rows = hidden > 0 ? x.numel() / hidden : 0;
  const c10::cuda::CUDAGuard guard(dev);
  const int rc = mlora_fused_add_rmsnorm_fwd(x.data_ptr(), hidden, residual.data_ptr(), hidden, rows, hidden,
                                             weight.data_ptr(), dt_code(weight.scalar_type()), out.data_ptr(), hidden,
                                             (float)eps, dt_code(x.scalar_type()),
                                             at::cuda::getCurrentCUDAStream().stream());
  check_rc(rc);
}

// Slot-load scatter (scatter_bank.py:68-93 of the reference): every block of
// the h staged banks into its slot. `rects` is a CUDA int64 [n, 6] table of
// mlora_scatter_rect_t rows (src_offset, dst address, slot_stride, rows, cols,
// dst_row_stride); the destinations are the pool's slot stacks, addressed by
// device pointer as the reference's tables do.
void scatter_stage(const at::Tensor& stage, const at::Tensor& slots, const at::Tensor& rects, int64_t max_rect_elems,
                   const c10::optional<at::Tensor>& status) {
  const at::Device dev = stage.device();
  check_cuda(stage, "stage", dev);
  check_cuda(slots, "slots", dev);
  check_cuda(rects, "rects", dev);
  TORCH_CHECK(stage.dim() == 2 && stage.is_contiguous(), "mlora: stage must be a contiguous [h, total] tensor");
  TORCH_CHECK(slots.scalar_type() == at::kLong && slots.dim() == 1 && slots.is_contiguous(),
              "mlora: slots must be a contiguous int64 [h] tensor");
  TORCH_CHECK(slots.numel() <= stage.size(0), "mlora: ", slots.numel(), " slots for ", stage.size(0), " stage rows");
  TORCH_CHECK(rects.scalar_type() == at::kLong && rects.dim() == 2 && rects.size(1) == 6 && rects.is_contiguous(),
              "mlora: rects must be a contiguous int64 [n, 6] tensor");
  TORCH_CHECK(max_rect_elems >= 0, "mlora: max_rect_elems must be >= 0");
  static_assert(sizeof(mlora_scatter_rect_t) == 6 * sizeof(int64_t), "rect layout");
  const c10::cuda::CUDAGuard guard(dev);
  const int rc = mlora_scatter_stage(stage.data_ptr(), stage.size(1), (int32_t)slots.numel(),
                                     reinterpret_cast<const int64_t*>(slots.data_ptr()),
                                     reinterpret_cast<const mlora_scatter_rect_t*>(rects.data_ptr()),
                                     (int32_t)rects.size(0), max_rect_elems, dt_code(stage.scalar_type()),
                                     status_ptr(status, dev), at::cuda::getCurrentCUDAStream().stream());
  check_rc(rc);
}

}  // namespace

TORCH_LIBRARY(mlora, m) {
  m.def(
      "sgemm_lora_a(Tensor x, Tensor weights, Tensor seg_lens, Tensor seg_indptr, Tensor weight_indices, "
      "Tensor lora_ranks, int bs, int max_len, Tensor(a!) output, int stack_num=1, Tensor(b!)? status=None) "
      "-> Tensor(a!)");
  m.def(
      "sgemm_lora_b(Tensor x, Tensor weights, Tensor seg_lens, Tensor seg_indptr, Tensor weight_indices, "
      "Tensor lora_ranks, Tensor scalings, int bs, int max_len, Tensor(a!) output, Tensor(b!)? status=None) "
      "-> Tensor(a!)");
  m.def(
      "apply_lora(Tensor x, Tensor a_stack, Tensor b_stack, Tensor seg_lens, Tensor seg_indptr, "
      "Tensor weight_indices, Tensor lora_ranks, Tensor scalings, int bs, int max_len, Tensor(a!) mid, "
      "Tensor(b!) output, Tensor(c!)? status=None) -> Tensor(b!)");
  m.def(
      "apply_lora_group(Tensor x, Tensor[] a_stacks, Tensor[] b_stacks, Tensor seg_lens, Tensor seg_indptr, "
      "Tensor weight_indices, Tensor lora_ranks, Tensor scalings, int bs, int max_len, Tensor(a!)[] outputs, "
      "Tensor(b!)? mid=None, Tensor(c!)? status=None) -> ()");
  m.def("rmsnorm(Tensor x, Tensor weight, float eps) -> Tensor");
  m.def("rmsnorm_out(Tensor x, Tensor weight, float eps, Tensor(a!) out) -> Tensor(a!)");
  m.def("fused_add_rmsnorm(Tensor x, Tensor(a!) residual, Tensor weight, float eps, Tensor(b!) out) -> ()");
  m.def("scatter_stage(Tensor stage, Tensor slots, Tensor rects, int max_rect_elems, Tensor(a!)? status=None) -> ()");
}

TORCH_LIBRARY_IMPL(mlora, CUDA, m) {
  m.impl("sgemm_lora_a", &sgemm_lora_a);
  m.impl("sgemm_lora_b", &sgemm_lora_b);
  m.impl("apply_lora", &apply_lora);
  m.impl("apply_lora_group", &apply_lora_group);
  m.impl("rmsnorm", &rmsnorm);
  m.impl("rmsnorm_out", &rmsnorm_out);
  m.impl("scatter_stage", &scatter_stage);
  m.impl("fused_add_rmsnorm", &fused_add_rmsnorm);
}
