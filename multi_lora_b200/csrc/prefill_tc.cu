// apply_lora for long segments (prefill) on the fifth-generation tensor cores.
//
// Semantics are those of LoRABackend.apply_lora (backend/base.py:60-89 of the
// reference): mid = T(x @ A[slot, :rank].T) with fp32 accumulation
// (sgemm_lora_a.py:11-115, the GEMM variant), then
// y = T(T(scaling * mid @ B[slot, :, :rank].T) + y) (sgemm_lora_b.py:11-90),
// for up to four projections that share x and the routing (q/k/v, gate/up).
//
// Each segment's rows are cut into tiles of 128 tokens (the last one ragged;
// rows past the segment are computed but never stored).
//   lora_shrink_tc_kernel: one CTA per (tile, K split). TMA streams 64-column blocks of x
//     (128 x 64) and of every projection's A[slot] (R x 64) through a
//     2-stage ring in the 128-byte-swizzled K-major layout (two CTAs per SM);
//     one thread issues
//     tcgen05.mma (M = 128, N = n_proj * 64, K = 16) into a TMEM accumulator;
//     every stage is released by tcgen05.commit. The epilogue reads TMEM row
//     by row (thread = token), rounds to T once and writes mid columns < rank.
//     When there are few tiles the input dim is split over a thread-block
//     cluster (up to 8 CTAs): each CTA parks its fp32 partial tile in its own
//     shared memory and every CTA sums the partials of its share of the rows
//     over distributed shared memory, in split order (deterministic).
//   lora_expand_tc_kernel: one CTA per (tile, projection, 128-column block of
//     out). TMA brings the mid tile, B[slot, block, :] and the y tile; four
//     tcgen05.mma (K = 64) fill a 128 x 128 TMEM accumulator; the epilogue
//     fuses the scaling, the rounding and the residual add and stores the
//     segment's rows with 16-byte stores.
// Shapes: bf16/f16, max_rank 16, 32 or 64, in % 64 == 0, out % 8 == 0. Adapter weights
// are requested before griddepcontrol.wait; x, mid and y after it. Waits are
// bounded; TMEM is always freed.
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc.cuh"

namespace mlora {

constexpr int kTcThreads = 128;
constexpr int kTcTileM = 128;  // tokens per tile
constexpr int kTcBK = 64;      // K block (one 128-byte swizzle row)
constexpr int kTcBN = 128;     // expand output columns per CTA
// max_rank RT in {16, 32, 64}: rank-wide tiles (mid, B) have rows of RT * 2
// bytes, swizzled with that span (32B / 64B / 128B).

struct TcTile {
  int seg, row0, rows, slot, rank;
};

// Warp 0: tile index -> segment, first row, valid rows, slot and rank. Segments
// with rank 0, an out-of-range slot or bad bounds contribute no tiles. Returns
// false (for every lane) past the last tile.
__device__ bool tc_find_tile(const PrefillArgs& p, int tile, TcTile& out) {
  const int lane = threadIdx.x & 31;
  const bool reporter = blockIdx.x == 0 && blockIdx.y == 0;
  int base = 0;
  for (int s0 = 0; s0 < p.bs; s0 += 32) {
    const int seg = s0 + lane;
    int st = 0, en = 0, slot = -1, rank = 0;
    if (seg < p.bs) {
      slot = __ldg(p.weight_indices + seg);
      st = __ldg(p.seg_indptr + seg);
      en = __ldg(p.seg_indptr + seg + 1);
      if (slot < 0 || slot >= p.num_slots) {
        if (reporter) flag_error(p.status, kErrSlotRange);
        slot = -1;
      } else if (st < 0 || en < st || en > p.S) {
        if (reporter) flag_error(p.status, kErrIndptr);
        slot = -1;
      } else {
        rank = __ldg(p.lora_ranks + slot);
        if (rank < 0 || rank > p.R) {
          if (reporter) flag_error(p.status, kErrRankRange);
          rank = rank < 0 ? 0 : p.R;
        }
      }
    }
    const int n = (slot >= 0 && rank > 0) ? (en - st + kTcTileM - 1) / kTcTileM : 0;
    int incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const bool mine = tile >= base + incl - n && tile < base + incl;
    const unsigned hit = __ballot_sync(0xffffffffu, mine);
    if (hit != 0u) {
      const int src = __ffs(hit) - 1;
      const int k = tile - (base + __shfl_sync(0xffffffffu, incl - n, src));
      out.seg = s0 + src;
      const int s_st = __shfl_sync(0xffffffffu, st, src), s_en = __shfl_sync(0xffffffffu, en, src);
      out.row0 = s_st + k * kTcTileM;
      out.rows = min(kTcTileM, s_en - out.row0);
      out.slot = __shfl_sync(0xffffffffu, slot, src);
      out.rank = __shfl_sync(0xffffffffu, rank, src);
      return true;
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
  return false;
}

__device__ __forceinline__ const CUtensorMap* tc_map(const CUtensorMap* maps, int m) { return maps + m; }

// ---------------------------------------------------------------------------
// shrink: mid[tile rows, m*R : m*R + rank] for every projection m
// ---------------------------------------------------------------------------
template <typename T, int RT>
__global__ void __launch_bounds__(kTcThreads) lora_shrink_tc_kernel(const __grid_constant__ PrefillArgs p) {
  constexpr uint32_t X_BYTES = kTcTileM * kTcBK * 2;  // 16 KB
  constexpr uint32_t A_BYTES = RT * kTcBK * 2;        // RT rows of 128 B per projection
  extern __shared__ __align__(1024) unsigned char s_raw[];
  __shared__ __align__(8) uint64_t full[4], empty[4], done;
  __shared__ uint32_t s_tmem;
  __shared__ TcTile s_tile;
  __shared__ int s_ok;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(s_raw) + 1023) & ~uintptr_t(1023));
  // blockIdx.y = tile, blockIdx.x = K split (one thread-block cluster per tile when splits > 1)
  if (warp == 0) {
    TcTile t;
    const bool ok = tc_find_tile(p, blockIdx.y, t);
    if (lane == 0) {
      s_ok = ok;
      if (ok) s_tile = t;
    }
  }
  __syncthreads();
  if (!s_ok) {  // uniform over the cluster (same tile)
    pdl_exit_early();
    return;
  }
  const TcTile t = s_tile;
  const int nm = p.n_mod;
  const int splits = gridDim.x, split = blockIdx.x;
  const int ns = p.tc_stages;
  const uint32_t stage_bytes = X_BYTES + (uint32_t)nm * A_BYTES;
  const int N = nm * RT;  // MMA N: the projections' rank rows side by side
  const uint32_t ncols = N <= 32 ? 32u : N <= 64 ? 64u : N <= 128 ? 128u : 256u;
  if (tid == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&s_tmem, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t taddr = s_tmem;
  const int KB_all = p.in_dim / kTcBK;
  const int kb0 = split * KB_all / splits;  // this CTA's K blocks [kb0, kb0 + KB)
  const int KB = (split + 1) * KB_all / splits - kb0;
  bool ok = true;

  if (tid == 0) {  // ---- TMA producer ----
    auto issue_a = [&](int kb) {
      const int s = kb % ns;
      unsigned char* st = smem + (size_t)s * stage_bytes;
      mbar_arrive_expect_tx(&full[s], stage_bytes);
      for (int m = 0; m < nm; ++m)
        tma_load_2d(st + X_BYTES + m * A_BYTES, tc_map(p.a_map, m), (kb0 + kb) * kTcBK, t.slot * p.R, &full[s]);
    };
    auto issue_x = [&](int kb) {
      unsigned char* st = smem + (size_t)(kb % ns) * stage_bytes;
      tma_load_2d(st, &p.x_map, (kb0 + kb) * kTcBK, t.row0, &full[kb % ns]);
    };
    const int pre = min(ns, KB);
    for (int kb = 0; kb < pre; ++kb) issue_a(kb);  // adapter weights: before the wait
    pdl_wait();                                     // x comes from earlier kernels
    for (int kb = 0; kb < pre; ++kb) issue_x(kb);
    for (int kb = pre; kb < KB && ok; ++kb) {
      ok = mbar_wait(&empty[kb % ns], ((kb / ns) - 1) & 1, p.status);
      if (ok) {
        issue_a(kb);
        issue_x(kb);
      }
    }
  } else if (tid == 32) {  // ---- MMA issuer ----
    const uint32_t idesc = umma_idesc_f16(Num<T>::is_bf16, kTcTileM, N);
    for (int kb = 0; kb < KB && ok; ++kb) {
      const int s = kb % ns;
      ok = mbar_wait(&full[s], (kb / ns) & 1, p.status);
      if (!ok) break;
      tc_fence_after();
      unsigned char* st = smem + (size_t)s * stage_bytes;
      const uint64_t ad = umma_desc_sw128(st), bd = umma_desc_sw128(st + X_BYTES);
#pragma unroll
      for (int k = 0; k < kTcBK / 16; ++k) umma_f16(taddr, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
      umma_commit(&empty[s]);
    }
    umma_commit(&done);
  }
  __syncwarp();
  const bool fin = mbar_wait(&done, 0, p.status);
  tc_fence_after();

  const int r = warp * 32 + lane;
  if (splits > 1) {
    // ---- split K: fp32 partials into this CTA's shared memory (the ring is
    // idle now), then each CTA of the cluster sums the splits, in split order,
    // for its share of the rows and writes them ----
    const int PS = N + 4;  // padded row (conflict-free 16-byte stores)
    float* part = reinterpret_cast<float*>(smem);
    for (int c = 0; c < (N + 31) / 32; ++c) {
      float v[32];
      tmem_ld32(taddr + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 32), v);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (c * 32 + 4 * q < N)
          *reinterpret_cast<float4*>(part + r * PS + c * 32 + 4 * q) =
              make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
    tc_fence_before();
    cluster_arrive_release();
    cluster_wait_acquire();  // every split's partials are in place
    const int rows_per = (kTcTileM + splits - 1) / splits;
    const int ra = split * rows_per, rb = min(kTcTileM, ra + rows_per);
    const uint32_t base = smem_addr(part);
    const int groups = N / 4;
    for (int e = tid; e < (rb - ra) * groups; e += kTcThreads) {
      const int row = ra + e / groups, c4 = (e % groups) * 4;
      const uint32_t off = (uint32_t)(row * PS + c4) * 4u;
      float4 acc = ld_dsmem_v4(cluster_map(base + off, 0));
      for (int q = 1; q < splits; ++q) {
        const float4 v = ld_dsmem_v4(cluster_map(base + off, (uint32_t)q));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      if (fin && row < t.rows) {
        const int m = c4 / RT, k = c4 % RT;
        T* dst = static_cast<T*>(p.mid) + (int64_t)(t.row0 + row) * p.mid_stride + m * p.R + k;
        const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (k + i < t.rank) dst[i] = Num<T>::from_f(a4[i]);
      }
    }
    cluster_arrive_release();
    cluster_wait_acquire();  // peers are done reading this CTA's partials
    __syncthreads();
    if (warp == 1) tmem_free(taddr, ncols);
    return;
  }

  // ---- epilogue: thread = token row; round once to T; columns < rank only ----
  const bool row_ok = fin && r < t.rows;
  T* mid = static_cast<T*>(p.mid) + (int64_t)(t.row0 + r) * p.mid_stride;
  for (int c = 0; c < (N + 31) / 32; ++c) {
    float v[32];
    tmem_ld32(taddr + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 32), v);
    if (row_ok) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // 8 columns at a time; RT is a multiple of 16
        const int col = c * 32 + 8 * q;
        if (col >= N) continue;
        const int m = col / RT, k = col % RT;
        T* dst = mid + m * p.R + k;
        if (k + 8 <= t.rank) {
          uint4 u;
          u.x = Pack2<T>::pack(Num<T>::from_f(v[8 * q + 0]), Num<T>::from_f(v[8 * q + 1]));
          u.y = Pack2<T>::pack(Num<T>::from_f(v[8 * q + 2]), Num<T>::from_f(v[8 * q + 3]));
          u.z = Pack2<T>::pack(Num<T>::from_f(v[8 * q + 4]), Num<T>::from_f(v[8 * q + 5]));
          u.w = Pack2<T>::pack(Num<T>::from_f(v[8 * q + 6]), Num<T>::from_f(v[8 * q + 7]));
          *reinterpret_cast<uint4*>(dst) = u;
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (k + i < t.rank) dst[i] = Num<T>::from_f(v[8 * q + i]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_free(taddr, ncols);
}

// ---------------------------------------------------------------------------
// expand: y[tile rows, block] = T(T(scale * mid @ B^T) + y)
// ---------------------------------------------------------------------------
template <typename T, int RT>
__global__ void __launch_bounds__(kTcThreads) lora_expand_tc_kernel(const __grid_constant__ PrefillArgs p) {
  constexpr int RB = RT * 2;                          // bytes per rank-wide row (= swizzle span)
  constexpr uint32_t M_BYTES = kTcTileM * RB;         // mid tile
  constexpr uint32_t B_BYTES = kTcBN * RB;            // B block
  constexpr uint32_t Y_BYTES = kTcTileM * kTcBK * 2;  // one 64-column y box, 16 KB
  extern __shared__ __align__(1024) unsigned char s_raw[];
  __shared__ __align__(8) uint64_t bar_load, bar_mma;
  __shared__ uint32_t s_tmem;
  __shared__ TcTile s_tile;
  __shared__ int s_ok;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(s_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* s_mid = smem;
  unsigned char* s_b = smem + M_BYTES;
  unsigned char* s_y = smem + M_BYTES + B_BYTES;
  // blockIdx.x -> (projection, 128-column block)
  int m = 0, blk = blockIdx.x;
  while (m + 1 < p.n_mod && blk >= (p.mod[m].out_dim + kTcBN - 1) / kTcBN) {
    blk -= (p.mod[m].out_dim + kTcBN - 1) / kTcBN;
    ++m;
  }
  const PrefillModule& mod = p.mod[m];
  const int n0 = blk * kTcBN;
  if (warp == 0) {
    TcTile t;
    const bool ok = tc_find_tile(p, blockIdx.y, t);
    if (lane == 0) {
      s_ok = ok && n0 < mod.out_dim;
      if (ok) s_tile = t;
    }
  }
  __syncthreads();
  if (!s_ok) {
    pdl_exit_early();
    return;
  }
  const TcTile t = s_tile;
  if (tid == 0) {
    mbar_init(&bar_load, 1);
    mbar_init(&bar_mma, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&s_tmem, kTcBN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  const uint32_t taddr = s_tmem;

  if (tid == 0) {
    mbar_arrive_expect_tx(&bar_load, M_BYTES + B_BYTES + 2 * Y_BYTES);
    tma_load_2d(s_b, tc_map(p.b_map, m), 0, t.slot * mod.out_dim + n0, &bar_load);  // weights: before the wait
    pdl_wait();  // mid (shrink kernel) and y (base projection)
    tma_load_2d(s_mid, &p.mid_map, m * p.R, t.row0, &bar_load);
    tma_load_2d(s_y, tc_map(p.y_map, m), n0, t.row0, &bar_load);
    tma_load_2d(s_y + Y_BYTES, tc_map(p.y_map, m), n0 + kTcBK, t.row0, &bar_load);
  }
  bool ok = mbar_wait(&bar_load, 0, p.status);
  if (t.rank < RT) {  // columns >= rank of mid (stale) and of B (stale) contribute zero
    const int w = RT - t.rank;
    for (int e = tid; e < kTcTileM * w; e += kTcThreads) {
      const int row = e / w, col = t.rank + e % w;
      *reinterpret_cast<T*>(s_mid + sw_offset(row, col, RB)) = Num<T>::from_f(0.f);
      *reinterpret_cast<T*>(s_b + sw_offset(row, col, RB)) = Num<T>::from_f(0.f);  // kTcBN == kTcTileM rows
    }
    fence_proxy_async_smem();
  }
  __syncthreads();
  if (tid == 0 && ok) {
    tc_fence_after();
    const uint32_t idesc = umma_idesc_f16(Num<T>::is_bf16, kTcTileM, kTcBN);
    const uint64_t ad = umma_desc_kmajor(s_mid, RB), bd = umma_desc_kmajor(s_b, RB);
#pragma unroll
    for (int k = 0; k < RT / 16; ++k) umma_f16(taddr, ad + 2 * k, bd + 2 * k, idesc, k != 0);
    umma_commit(&bar_mma);
  }
  __syncwarp();
  ok = __syncthreads_and(ok) && mbar_wait(&bar_mma, 0, p.status);
  tc_fence_after();

  // ---- epilogue: thread = token row ----
  const int r = warp * 32 + lane;
  const bool row_ok = ok && r < t.rows;
  float scale;
  switch (p.scalings_dtype) {
    case kBF16: scale = __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(p.scalings) + t.slot)); break;
    case kF16: scale = __half2float(__ldg(static_cast<const __half*>(p.scalings) + t.slot)); break;
    default: scale = __ldg(static_cast<const float*>(p.scalings) + t.slot); break;
  }
  T* yrow = static_cast<T*>(mod.y) + (int64_t)(t.row0 + r) * mod.y_stride + n0;
  // A whole tile (128 rows of this segment) is written back in place into the
  // staged y boxes and stored with two TMA tensor stores; a ragged tile (its
  // last rows belong to the next segment) stores its own rows with 16-byte stores.
  const bool tma_out = t.rows == kTcTileM;
#pragma unroll 1
  for (int c = 0; c < kTcBN / 32; ++c) {
    float v[32];
    tmem_ld32(taddr + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 32), v);
    if (row_ok) {
      unsigned char* yb = s_y + (c >> 1) * Y_BYTES;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int col = (c & 1) * 32 + q * 8;  // column within the 64-column box
        if (tma_out || n0 + c * 32 + q * 8 < mod.out_dim) {
          uint4* ys = reinterpret_cast<uint4*>(yb + sw128_offset(r, col));
          const uint4 yin = *ys;
          const uint32_t in[4] = {yin.x, yin.y, yin.z, yin.w};
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {  // y = T(T(scale * acc) + y), two values per packed rounding
            const uint32_t d = pack_round2<T>(v[8 * q + 2 * i] * scale, v[8 * q + 2 * i + 1] * scale);
            o[i] = pack_round2<T>(Pack2<T>::lo(d) + Pack2<T>::lo(in[i]), Pack2<T>::hi(d) + Pack2<T>::hi(in[i]));
          }
          if (tma_out) *ys = make_uint4(o[0], o[1], o[2], o[3]);
          else *reinterpret_cast<uint4*>(yrow + c * 32 + q * 8) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
  if (tma_out) {
    fence_proxy_async_smem();  // the rows written above, to the TMA (async proxy)
    __syncthreads();
    if (tid == 0 && ok) {  // columns past out_dim are clipped by the tensor map
      tma_store_2d(tc_map(p.y_map, m), n0, t.row0, s_y);
      if (n0 + kTcBK < mod.out_dim) tma_store_2d(tc_map(p.y_map, m), n0 + kTcBK, t.row0, s_y + Y_BYTES);
      bulk_commit();
      bulk_wait_read_all();  // the boxes are read before the CTA (and its shared memory) goes away
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_free(taddr, kTcBN);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      (void)cudaGetLastError();
      return (EncodeTiled) nullptr;
    }
    return reinterpret_cast<EncodeTiled>(f);
  }();
  return fn;
}

// 2-D map over a row-major [outer, inner] matrix with rows `stride_elems` apart;
// box {box_inner, box_rows}, swizzled with the box row's span (32, 64 or 128
// bytes), zero fill out of bounds.
bool encode_2d(CUtensorMap* map, const void* base, int dtype, uint64_t inner, uint64_t outer, uint64_t stride_elems,
               uint32_t box_inner, uint32_t box_rows) {
  EncodeTiled enc = encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {stride_elems * 2};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = box_inner * 2 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : box_inner * 2 == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                      : CU_TENSOR_MAP_SWIZZLE_32B;
  return enc(map, dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
             const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

long long tc_sm_count() {
  static const int n = [] {
    int dev = 0, c = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      (void)cudaGetLastError();
      return 148;
    }
    return c;
  }();
  return n;
}

template <typename K>
bool ensure_smem_tc(K kern, int bytes) {
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return true;
}

template <typename T, int RT>
cudaError_t launch_prefill_t(PrefillArgs& a, cudaStream_t st, bool pdl) {
  const int nm = a.n_mod;
  // Shrink: two-stage rings, sized so that two CTAs share an SM (with more K
  // splits, below) -- more bytes in flight per SM than one CTA with a deeper
  // ring. The ring's shared memory also holds the fp32 partial tile of the
  // K-split reduction, so it is at least that large.
  a.tc_stages = 2;
  const int ring = a.tc_stages * (kTcTileM * kTcBK * 2 + nm * RT * kTcBK * 2);
  const int part = kTcTileM * (nm * RT + 4) * 4;
  const int shrink_smem = (ring > part ? ring : part) + 1024;
  const int expand_smem = (kTcTileM * RT * 2) + (kTcBN * RT * 2) + 2 * (kTcTileM * kTcBK * 2) + 1024;
  auto ks = lora_shrink_tc_kernel<T, RT>;
  auto ke = lora_expand_tc_kernel<T, RT>;
  // at least the largest shrink launched at this RT (four projections: the larger of
  // the 2-stage ring and the K-split partial tile)
  static const bool smem_ok =
      ensure_smem_tc(ks, (4 * RT <= 128 ? 4 : 3) * (kTcTileM * kTcBK * 2 + 4 * RT * kTcBK * 2) + 1024) &&
      ensure_smem_tc(ke, expand_smem);
  if (!smem_ok) return cudaErrorNotSupported;
  const long long tiles = (a.S + kTcTileM - 1) / kTcTileM + (long long)a.bs;
  if (tiles > 65535) return cudaErrorNotSupported;
  int blocks = 0;
  for (int m = 0; m < nm; ++m) blocks += (a.mod[m].out_dim + kTcBN - 1) / kTcBN;
  // K splits: enough shrink CTAs for two per SM, at least 4 K blocks each, a cluster of <= 8
  int splits = (int)(2 * tc_sm_count() / tiles);
  splits = splits < 1 ? 1 : splits > 8 ? 8 : splits;
  while (splits > 1 && a.in_dim / kTcBK < 4 * splits) --splits;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)splits, (unsigned)tiles);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = shrink_smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, ks, a);
  if (e != cudaSuccess) return e;
  return launch_kernel(ke, dim3((unsigned)blocks, (unsigned)tiles), dim3(kTcThreads), expand_smem, st, true, a);
}

template <typename T>
cudaError_t launch_prefill_r(PrefillArgs& a, cudaStream_t st, bool pdl) {
  return a.R == 16 ? launch_prefill_t<T, 16>(a, st, pdl)
       : a.R == 32 ? launch_prefill_t<T, 32>(a, st, pdl)
                   : launch_prefill_t<T, 64>(a, st, pdl);
}

}  // namespace

cudaError_t launch_apply_prefill(const PrefillLaunch& l, int dtype, cudaStream_t st, bool pdl) {
  if (dtype != kBF16 && dtype != kF16) return cudaErrorNotSupported;
  if (l.n_mod < 1 || l.n_mod > kMaxPrefillModules || l.in_dim % kTcBK != 0) return cudaErrorNotSupported;
  if (l.R != 16 && l.R != 32 && l.R != 64) return cudaErrorNotSupported;
  PrefillArgs a{};
  a.n_mod = l.n_mod;
  a.mid = l.mid;
  a.mid_stride = l.mid_stride;
  a.seg_indptr = l.seg_indptr;
  a.weight_indices = l.weight_indices;
  a.lora_ranks = l.lora_ranks;
  a.scalings = l.scalings;
  a.scalings_dtype = l.scalings_dtype;
  a.bs = l.bs;
  a.S = l.S;
  a.in_dim = l.in_dim;
  a.R = l.R;
  a.num_slots = l.num_slots;
  a.status = l.status;
  const uint32_t R = (uint32_t)l.R;
  bool ok = encode_2d(&a.x_map, l.x, dtype, (uint64_t)l.in_dim, (uint64_t)l.S, (uint64_t)l.x_stride, kTcBK, kTcTileM) &&
            encode_2d(&a.mid_map, l.mid, dtype, (uint64_t)l.n_mod * R, (uint64_t)l.S, (uint64_t)l.mid_stride, R,
                      kTcTileM);
  for (int m = 0; m < l.n_mod && ok; ++m) {
    a.mod[m] = l.mod[m];
    ok = encode_2d(&a.a_map[m], l.mod[m].a, dtype, (uint64_t)l.in_dim, (uint64_t)l.num_slots * R, (uint64_t)l.in_dim,
                   kTcBK, R) &&
         encode_2d(&a.b_map[m], l.mod[m].b, dtype, R, (uint64_t)l.num_slots * l.mod[m].out_dim, R, R, kTcBN) &&
         encode_2d(&a.y_map[m], l.mod[m].y, dtype, (uint64_t)l.mod[m].out_dim, (uint64_t)l.S,
                   (uint64_t)l.mod[m].y_stride, kTcBK, kTcTileM);
  }
  if (!ok) return cudaErrorNotSupported;
  return dtype == kBF16 ? launch_prefill_r<__nv_bfloat16>(a, st, pdl) : launch_prefill_r<__half>(a, st, pdl);
}

}  // namespace mlora
