// sm_100a fifth-generation tensor core (tcgen05) and tensor-map TMA helpers.
//
// Operand tiles live in shared memory in the K-major, 128-byte-swizzled
// layout that a TMA tensor load with CU_TENSOR_MAP_SWIZZLE_128B writes: rows of
// 64 bf16/f16 (128 B), the 16-byte chunk index XOR-ed with (row % 8), tiles
// aligned to 1024 B. Accumulators live in tensor memory (TMEM), allocated per
// CTA and read back row-per-thread with tcgen05.ld.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "tma.cuh"

namespace mlora {

// ---- tensor-map TMA (no multicast) -------------------------------------------

// 2-D tiled load of box {c0.., c1..} (inner, outer coordinates in elements)
// into shared memory; completes its bytes on `bar`. c0 * element size must be a
// multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

// 2-D tiled store of a shared-memory box to global (coordinates as for
// tma_load_2d; c0 * element size a multiple of 16 bytes, c0, c1 >= 0). Part
// of the bulk group that bulk_commit() closes.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int c0, int c1, const void* src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(smem_addr(src))
               : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- UMMA descriptors ---------------------------------------------------------

// Shared-memory matrix descriptor of a K-major tile whose rows are `row_bytes`
// (32, 64 or 128) long and swizzled with the same span (SWIZZLE_32B / 64B /
// 128B: the layout a TMA load with that swizzle writes), 8-row groups packed
// (stride byte offset 8 * row_bytes). Advance by 32 B (one K=16 step) with `+ 2`.
__device__ __forceinline__ uint64_t umma_desc_kmajor(const void* tile, int row_bytes) {
  const uint64_t a = (uint64_t)((smem_addr(tile) >> 4) & 0x3FFFu);
  const uint64_t layout = row_bytes == 128 ? 2ull : row_bytes == 64 ? 4ull : 6ull;
  return a | (1ull << 16)                        // leading byte offset (unused for swizzled K-major)
         | ((uint64_t)(row_bytes / 2) << 32)     // stride byte offset: 8 rows, in 16-byte units
         | (1ull << 46)                          // descriptor version (sm_100)
         | (layout << 61);                       // layout: SWIZZLE_128B / 64B / 32B
}
__device__ __forceinline__ uint64_t umma_desc_sw128(const void* tile) { return umma_desc_kmajor(tile, 128); }

// Instruction descriptor of tcgen05.mma.kind::f16: fp32 accumulate, A and B of
// the same 16-bit type (bf16 when `bf16`), both K-major, shape M x N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(bool bf16, int M, int N) {
  return (1u << 4)                                   // D: f32
         | ((bf16 ? 1u : 0u) << 7)                   // A type
         | ((bf16 ? 1u : 0u) << 10)                  // B type
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---- tcgen05 ------------------------------------------------------------------

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `bar` when every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Whole warp: allocate `ncols` TMEM columns (power of two >= 32); the base
// address is written to shared memory at `dst`.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

// Whole warp: free an allocation.
__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Whole warp: 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Byte offset of 16-bit element (row, col) in a tile of `row_bytes`-long rows
// swizzled with the same span (16-byte chunk index XOR-ed with address bits
// 7.. of the row start; the tile base is aligned to 8 rows).
__device__ __forceinline__ uint32_t sw_offset(int row, int col, int row_bytes) {
  const int sel = row_bytes == 128 ? (row & 7) : row_bytes == 64 ? ((row >> 1) & 3) : ((row >> 2) & 1);
  return (uint32_t)row * (uint32_t)row_bytes + ((uint32_t)(((col >> 3) ^ sel) << 4)) + (uint32_t)(col & 7) * 2u;
}
__device__ __forceinline__ uint32_t sw128_offset(int row, int col) { return sw_offset(row, col, 128); }

}  // namespace mlora
