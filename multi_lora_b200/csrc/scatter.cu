// Slot loads: staged adapter banks -> per-module slot buffers.
//
// The reference stages each adapter's pinned "bank" (all A blocks, then all B
// blocks, pool.py:23-56) into one row of a device stage by a single H2D copy,
// then scatters it into the slot stacks (kernels/scatter_bank.py:18-65):
// A[key][slot, :r, :] is contiguous, B[key][slot, :, :r] is r columns of
// [out, max_rank] rows. Here every block is a rectangle descriptor
// (source offset in the bank row, destination base address, slot stride,
// rows x cols, destination row stride), and one launch copies every
// rectangle of every adapter of the chunk with 128-bit accesses where the
// layout allows. Bytes past the rank are left as they are, like the reference.
//
// The kernel writes adapter weights, so it never triggers dependent launches
// early: a following kernel that reads the weights starts after it completes.
#include "../../include/mlora_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace mlora {

constexpr int kScatterNT = 256;
constexpr int kScatterVecPerThread = 8;  // 16-byte vectors per thread per CTA

__global__ void __launch_bounds__(kScatterNT)
scatter_stage_kernel(const uint8_t* __restrict__ stage, int64_t stage_row_bytes,
                     const int64_t* __restrict__ slots, const mlora_scatter_rect_t* __restrict__ rects,
                     int es, int64_t bytes_per_cta, uint32_t* status) {
  const mlora_scatter_rect_t r = rects[blockIdx.x];
  const int i = blockIdx.z;  // adapter within the chunk (stage row)
  const int64_t slot = slots[i];
  const int64_t row_bytes = r.cols * es;
  const int64_t total = r.rows * row_bytes;
  const int64_t lo = (int64_t)blockIdx.y * bytes_per_cta;
  if (lo >= total) return;
  const int64_t hi = min(total, lo + bytes_per_cta);
  const int64_t src0 = r.src_offset * es;
  if (r.src_offset < 0 || r.rows < 0 || r.cols < 0 || slot < 0 || src0 + total > stage_row_bytes) {
    if (threadIdx.x == 0) flag_error(status, kErrScatterRange);
    return;
  }
  const uint8_t* src = stage + (int64_t)i * stage_row_bytes + src0;
  uint8_t* dst = reinterpret_cast<uint8_t*>(r.dst) + slot * r.slot_stride * es;
  const int64_t dst_row_bytes = r.dst_row_stride * es;
  const bool vec = (row_bytes % 16 == 0) && (dst_row_bytes % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(src) % 16 == 0) && (reinterpret_cast<uintptr_t>(dst) % 16 == 0) &&
                   (lo % 16 == 0);
  if (vec) {
    for (int64_t b = lo + (int64_t)threadIdx.x * 16; b < hi; b += (int64_t)kScatterNT * 16) {
      const int64_t row = b / row_bytes, col = b - row * row_bytes;
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(src + b));
      *reinterpret_cast<uint4*>(dst + row * dst_row_bytes + col) = v;
    }
  } else if (es == 2) {
    for (int64_t b = lo + (int64_t)threadIdx.x * 2; b < hi; b += (int64_t)kScatterNT * 2) {
      const int64_t row = b / row_bytes, col = b - row * row_bytes;
      *reinterpret_cast<uint16_t*>(dst + row * dst_row_bytes + col) =
          __ldcg(reinterpret_cast<const unsigned short*>(src + b));
    }
  } else {
    for (int64_t b = lo + (int64_t)threadIdx.x * 4; b < hi; b += (int64_t)kScatterNT * 4) {
      const int64_t row = b / row_bytes, col = b - row * row_bytes;
      *reinterpret_cast<uint32_t*>(dst + row * dst_row_bytes + col) =
          __ldcg(reinterpret_cast<const unsigned int*>(src + b));
    }
  }
}

cudaError_t launch_scatter(const void* stage, int64_t stage_row_elems, int h, const int64_t* slots,
                           const mlora_scatter_rect_t* rects, int n_rects, int64_t max_rect_elems, int es,
                           uint32_t* status, cudaStream_t st) {
  const int64_t bytes_per_cta = (int64_t)kScatterNT * 16 * kScatterVecPerThread;
  const int64_t max_bytes = max_rect_elems * es;
  const int64_t ny = (max_bytes + bytes_per_cta - 1) / bytes_per_cta;
  if (ny > 65535) return cudaErrorInvalidValue;
  const dim3 grid(n_rects, (unsigned)(ny > 0 ? ny : 1), h);
  // plain launch (no programmatic serialisation): readers must see complete weights
  return launch_kernel(scatter_stage_kernel, grid, dim3(kScatterNT), 0, st, false,
                       static_cast<const uint8_t*>(stage), stage_row_elems * es, slots, rects, es, bytes_per_cta,
                       status);
}

}  // namespace mlora
