// CUDA-core segment shrink / expand for short segments (decode).
//
// shrink:  mid[t, n] = T( sum_k x[t, k] * A[slot, n, k] ),  n < rank
//          (kernels/sgemm_lora_a.py:119-183 GEMV, :11-115 GEMM; the oracle is
//           backend/torch_backend.py:17-49). Columns >= rank and rank-0 slots
//           are left untouched, as sgemm_lora_a.py:148-149,156-157 do.
// expand:  y[t, o] = T( T(scale * sum_{k<rank} mid[t, k] * B[slot, o, k]) + y[t, o] )
//          (kernels/sgemm_lora_b.py:94-153 / :11-90; torch_backend.py:51-90),
//          in place, honouring y's row stride (layers.py:82-83).
//
// Design (B200): one CTA owns one (slot, rank-row group) for shrink and one
// (slot, output column block) for expand. The slot's weight rows are loaded
// with 128-bit loads into registers BEFORE griddepcontrol.wait, so under
// programmatic dependent launch the weight stream of this kernel overlaps the
// tail of the previous kernel. Activations (x, mid, y) are read after the
// wait with L2-only loads. Each slot's weights are read once per launch no
// matter how many segments route to it.
#include "common.cuh"
#include "kernels.h"
#include "routing.cuh"

namespace mlora {

constexpr int kSegCap = 256;  // segments gathered per pass
constexpr int kTT = 8;        // tokens per tile

// ---------------------------------------------------------------------------
// shrink
// ---------------------------------------------------------------------------
// T: activation/weight type; OutT: mid type (T, or f32 for TP partial sums)
// V: elements per load; NT threads; RPC rank rows per CTA; CH chunks per
// thread per k-block (k-block = NT*CH chunks).
template <typename T, typename OutT, int V, int NT, int RPC, int CH>
__global__ void __launch_bounds__(NT) shrink_kernel(const ShrinkArgs p) {
  constexpr int NW = NT / 32;
  __shared__ SlotSegments<kSegCap> sl;
  __shared__ int s_rows[kTT];
  __shared__ float s_red[NW][kTT * RPC];

  const int slot = blockIdx.y;
  const int row0 = blockIdx.x * RPC;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;

  int rank = __ldg(p.lora_ranks + slot);
  if (rank < 0 || rank > p.max_rank) {
    if (blockIdx.x == 0 && tid == 0) flag_error(p.status, kErrRankRange);
    rank = rank < 0 ? 0 : p.max_rank;
  }
  const int rows_eff = min(p.max_rank, rank * p.stack_num);
  if (row0 >= rows_eff) {
    pdl_exit_early();
    return;
  }
  const int nrows = min(RPC, rows_eff - row0);

  const int nchunk = p.in_dim / V;  // V divides in_dim (host-checked)
  constexpr int KB = NT * CH;
  const int nkb = (nchunk + KB - 1) / KB;
  const T* __restrict__ wbase =
      static_cast<const T*>(p.w) + (int64_t)slot * p.w_slot_stride + (int64_t)row0 * p.w_row_stride;
  const T* __restrict__ xbase = static_cast<const T*>(p.x);

  // ---- prologue: adapter weights (stable for the whole step) ----
  Chunk<T, V> a[RPC][CH];
  auto load_a = [&](int kb) {
#pragma unroll
    for (int r = 0; r < RPC; ++r)
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const int c = kb * KB + j * NT + tid;
        if (r < nrows && c < nchunk)
          a[r][j].ldg(wbase + (int64_t)r * p.w_row_stride + (int64_t)c * V);
        else
          a[r][j].zero();
      }
  };
  if (nkb == 1) load_a(0);
  collect_slot_segments<kSegCap>(sl, slot, 0, p.weight_indices, p.seg_indptr, p.bs, p.S,
                                 p.num_slots, p.status);
  pdl_trigger();
  pdl_wait();  // x comes from the previous kernel
  __syncthreads();

  while (true) {
    const int ntok = sl.cum[sl.n];
    for (int q0 = 0; q0 < ntok; q0 += kTT) {
      const int nt = min(kTT, ntok - q0);
      if (tid < nt) s_rows[tid] = slot_token_row(sl, q0 + tid);
      __syncthreads();
      float acc[kTT][RPC];
#pragma unroll
      for (int t = 0; t < kTT; ++t)
#pragma unroll
        for (int r = 0; r < RPC; ++r) acc[t][r] = 0.f;
      for (int kb = 0; kb < nkb; ++kb) {
        if (nkb > 1) load_a(kb);
#pragma unroll
        for (int t = 0; t < kTT; ++t) {
          if (t < nt) {
            const T* xr = xbase + (int64_t)s_rows[t] * p.x_stride;
#pragma unroll
            for (int j = 0; j < CH; ++j) {
              const int c = kb * KB + j * NT + tid;
              if (c < nchunk) {
                Chunk<T, V> xc;
                xc.ldcg(xr + (int64_t)c * V);
                float xf[V];
                xc.to_f(xf);
#pragma unroll
                for (int r = 0; r < RPC; ++r) {
                  float af[V];
                  a[r][j].to_f(af);
                  float s = 0.f;
#pragma unroll
                  for (int e = 0; e < V; ++e) s = fmaf(xf[e], af[e], s);
                  acc[t][r] += s;
                }
              }
            }
          }
        }
      }
      // CTA reduction: warp shuffle, then across warps in fixed order
#pragma unroll
      for (int t = 0; t < kTT; ++t)
#pragma unroll
        for (int r = 0; r < RPC; ++r) {
          const float v = warp_sum(acc[t][r]);
          if (lane == 0) s_red[warp][t * RPC + r] = v;
        }
      __syncthreads();
      if (tid < kTT * RPC) {
        const int t = tid / RPC, r = tid % RPC;
        if (t < nt && r < nrows) {
          float s = 0.f;
#pragma unroll
          for (int w = 0; w < NW; ++w) s += s_red[w][tid];
          OutT* o = static_cast<OutT*>(p.out) + (int64_t)s_rows[t] * p.out_stride + row0 + r;
          *o = Num<OutT>::from_f(s);
        }
      }
      __syncthreads();
    }
    if (sl.next >= p.bs) break;
    const int from = sl.next;
    __syncthreads();
    collect_slot_segments<kSegCap>(sl, slot, from, p.weight_indices, p.seg_indptr, p.bs, p.S,
                                   p.num_slots, p.status);
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// expand
// ---------------------------------------------------------------------------
// MidT: type of mid as stored (T, or f32 partial sums that are rounded to T on
// read so the result equals the unsharded path). OPT consecutive outputs per
// thread; RCH chunks of V rank columns held per output (rank block = RCH*V).
template <typename T, typename MidT, int V, int NT, int OPT, int RCH>
__global__ void __launch_bounds__(NT) expand_kernel(const ExpandArgs p) {
  constexpr int RB = RCH * V;  // rank columns per block
  __shared__ SlotSegments<kSegCap> sl;
  __shared__ int s_rows[kTT];
  __shared__ __align__(16) float s_mid[kTT][RB];

  const int slot = blockIdx.y;
  const int tid = threadIdx.x;
  const int o0 = (blockIdx.x * NT + tid) * OPT;

  int rank = __ldg(p.lora_ranks + slot);
  if (rank < 0 || rank > p.max_rank) {
    if (blockIdx.x == 0 && tid == 0) flag_error(p.status, kErrRankRange);
    rank = rank < 0 ? 0 : p.max_rank;
  }
  if (rank == 0) {
    pdl_exit_early();
    return;
  }
  float scale;
  switch (p.scalings_dtype) {
    case kBF16: scale = __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(p.scalings) + slot)); break;
    case kF16: scale = __half2float(__ldg(static_cast<const __half*>(p.scalings) + slot)); break;
    default: scale = __ldg(static_cast<const float*>(p.scalings) + slot); break;
  }
  const int nrb = (rank + RB - 1) / RB;
  const T* __restrict__ wbase = static_cast<const T*>(p.w) + (int64_t)slot * p.w_slot_stride;

  // ---- prologue: B rows of this thread's outputs ----
  Chunk<T, V> b[OPT][RCH];
  auto load_b = [&](int rb) {
#pragma unroll
    for (int i = 0; i < OPT; ++i)
#pragma unroll
      for (int c = 0; c < RCH; ++c) {
        const int k = rb * RB + c * V;
        if (o0 + i < p.out_dim && k < rank)
          b[i][c].ldg(wbase + (int64_t)(o0 + i) * p.w_row_stride + k);
        else
          b[i][c].zero();
      }
  };
  if (nrb == 1) load_b(0);
  collect_slot_segments<kSegCap>(sl, slot, 0, p.weight_indices, p.seg_indptr, p.bs, p.S,
                                 p.num_slots, p.status);
  pdl_trigger();
  pdl_wait();  // mid and y come from earlier kernels
  __syncthreads();

  const MidT* __restrict__ mbase = static_cast<const MidT*>(p.mid);
  T* __restrict__ ybase = static_cast<T*>(p.y);
  while (true) {
    const int ntok = sl.cum[sl.n];
    for (int q0 = 0; q0 < ntok; q0 += kTT) {
      const int nt = min(kTT, ntok - q0);
      if (tid < nt) s_rows[tid] = slot_token_row(sl, q0 + tid);
      __syncthreads();
      float acc[kTT][OPT];
#pragma unroll
      for (int t = 0; t < kTT; ++t)
#pragma unroll
        for (int i = 0; i < OPT; ++i) acc[t][i] = 0.f;
      for (int rb = 0; rb < nrb; ++rb) {
        if (nrb > 1) {
          load_b(rb);
          __syncthreads();  // previous block's s_mid reads are done
        }
        // mid tile -> smem as fp32, zero past rank (weights past rank may be stale)
        for (int e = tid; e < kTT * RB; e += NT) {
          const int t = e / RB, k = rb * RB + e % RB;
          float v = 0.f;
          if (t < nt && k < rank) {
            v = ldcg_f<MidT>(mbase + (int64_t)s_rows[t] * p.mid_stride + k);
            v = round_to<T>(v);
          }
          s_mid[t][e % RB] = v;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < OPT; ++i)
#pragma unroll
          for (int c = 0; c < RCH; ++c) {
            float bf[V];
            b[i][c].to_f(bf);
            const int kc = rb * RB + c * V;
#pragma unroll
            for (int e = 0; e < V; ++e)
              if (kc + e >= rank) bf[e] = 0.f;  // stale tail past rank
#pragma unroll
            for (int t = 0; t < kTT; ++t) {
              if (t < nt) {
                float s = 0.f;
#pragma unroll
                for (int e = 0; e < V; ++e) s = fmaf(s_mid[t][c * V + e], bf[e], s);
                acc[t][i] += s;
              }
            }
          }
      }
      // epilogue: scale, round to T, add residual, round, store
#pragma unroll
      for (int t = 0; t < kTT; ++t) {
        if (t < nt) {
          T* yr = ybase + (int64_t)s_rows[t] * p.y_stride + o0;
          if (o0 + OPT <= p.out_dim && p.y_vec_ok) {
            if constexpr (OPT * sizeof(T) == 4) {
              uint32_t u = __ldcg(reinterpret_cast<const unsigned int*>(yr));
              T v[OPT];
              memcpy(v, &u, 4);
#pragma unroll
              for (int i = 0; i < OPT; ++i)
                v[i] = Num<T>::from_f(round_to<T>(acc[t][i] * scale) + Num<T>::to_f(v[i]));
              memcpy(&u, v, 4);
              *reinterpret_cast<uint32_t*>(yr) = u;
            } else if constexpr (OPT * sizeof(T) == 8) {
              uint2 u = __ldcg(reinterpret_cast<const uint2*>(yr));
              T v[OPT];
              memcpy(v, &u, 8);
#pragma unroll
              for (int i = 0; i < OPT; ++i)
                v[i] = Num<T>::from_f(round_to<T>(acc[t][i] * scale) + Num<T>::to_f(v[i]));
              memcpy(&u, v, 8);
              *reinterpret_cast<uint2*>(yr) = u;
            } else {
#pragma unroll
              for (int i = 0; i < OPT; ++i)
                yr[i] = Num<T>::from_f(round_to<T>(acc[t][i] * scale) + ldcg_f<T>(yr + i));
            }
          } else {
#pragma unroll
            for (int i = 0; i < OPT; ++i)
              if (o0 + i < p.out_dim)
                yr[i] = Num<T>::from_f(round_to<T>(acc[t][i] * scale) + ldcg_f<T>(yr + i));
          }
        }
      }
      __syncthreads();
    }
    if (sl.next >= p.bs) break;
    const int from = sl.next;
    __syncthreads();
    collect_slot_segments<kSegCap>(sl, slot, from, p.weight_indices, p.seg_indptr, p.bs, p.S,
                                   p.num_slots, p.status);
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// host dispatch
// ---------------------------------------------------------------------------
namespace {

template <typename T, typename OutT, int V>
cudaError_t shrink_dispatch_vec(const ShrinkArgs& a, cudaStream_t st, bool pdl) {
  const int nchunk = a.in_dim / V;
  const int rpc = a.max_rank <= 32 ? 2 : 4;
  const dim3 grid((a.max_rank + rpc - 1) / rpc, a.num_slots);
  // choose threads and chunks per thread so one k-block covers the row
  auto go = [&](auto kern, int nt) { return launch_kernel(kern, grid, dim3(nt), 0, st, pdl, a); };
  if (rpc == 2) {
    if (nchunk <= 128) return go(shrink_kernel<T, OutT, V, 128, 2, 1>, 128);
    if (nchunk <= 256) return go(shrink_kernel<T, OutT, V, 256, 2, 1>, 256);
    if (nchunk <= 512) return go(shrink_kernel<T, OutT, V, 256, 2, 2>, 256);
    if (nchunk <= 1024) return go(shrink_kernel<T, OutT, V, 256, 2, 4>, 256);
    return go(shrink_kernel<T, OutT, V, 512, 2, 4>, 512);
  }
  if (nchunk <= 128) return go(shrink_kernel<T, OutT, V, 128, 4, 1>, 128);
  if (nchunk <= 256) return go(shrink_kernel<T, OutT, V, 256, 4, 1>, 256);
  if (nchunk <= 512) return go(shrink_kernel<T, OutT, V, 256, 4, 2>, 256);
  if (nchunk <= 1024) return go(shrink_kernel<T, OutT, V, 256, 4, 4>, 256);
  return go(shrink_kernel<T, OutT, V, 512, 4, 4>, 512);
}

template <typename T, typename OutT>
cudaError_t shrink_dispatch(const ShrinkArgs& a, cudaStream_t st, bool pdl) {
  constexpr int V = 16 / sizeof(T);
  if (a.vec_ok) return shrink_dispatch_vec<T, OutT, V>(a, st, pdl);
  const dim3 grid((a.max_rank + 1) / 2, a.num_slots);
  return launch_kernel(shrink_kernel<T, OutT, 1, 256, 2, 4>, grid, dim3(256), 0, st, pdl, a);
}

template <typename T, typename MidT, int V>
cudaError_t expand_dispatch_vec(const ExpandArgs& a, cudaStream_t st, bool pdl) {
  constexpr int OPT = sizeof(T) == 4 ? 2 : 2;
  constexpr int NT = 256;
  const dim3 grid((a.out_dim + NT * OPT - 1) / (NT * OPT), a.num_slots);
  const int rch = (a.max_rank + V - 1) / V;
  if (rch <= 1) return launch_kernel(expand_kernel<T, MidT, V, NT, OPT, 1>, grid, dim3(NT), 0, st, pdl, a);
  if (rch <= 2) return launch_kernel(expand_kernel<T, MidT, V, NT, OPT, 2>, grid, dim3(NT), 0, st, pdl, a);
  if (rch <= 4) return launch_kernel(expand_kernel<T, MidT, V, NT, OPT, 4>, grid, dim3(NT), 0, st, pdl, a);
  return launch_kernel(expand_kernel<T, MidT, V, NT, OPT, 8>, grid, dim3(NT), 0, st, pdl, a);
}

template <typename T, typename MidT>
cudaError_t expand_dispatch(const ExpandArgs& a, cudaStream_t st, bool pdl) {
  constexpr int V = 16 / sizeof(T);
  if (a.vec_ok) return expand_dispatch_vec<T, MidT, V>(a, st, pdl);
  constexpr int NT = 256;
  const dim3 grid((a.out_dim + NT - 1) / NT, a.num_slots);
  return launch_kernel(expand_kernel<T, MidT, 1, NT, 1, 16>, grid, dim3(NT), 0, st, pdl, a);
}

}  // namespace

cudaError_t launch_shrink(const ShrinkArgs& a, int dtype, bool out_f32, cudaStream_t st, bool pdl) {
  switch (dtype) {
    case kBF16:
      return out_f32 ? shrink_dispatch<__nv_bfloat16, float>(a, st, pdl)
                     : shrink_dispatch<__nv_bfloat16, __nv_bfloat16>(a, st, pdl);
    case kF16:
      return out_f32 ? shrink_dispatch<__half, float>(a, st, pdl) : shrink_dispatch<__half, __half>(a, st, pdl);
    case kF32:
      return shrink_dispatch<float, float>(a, st, pdl);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_expand(const ExpandArgs& a, int dtype, bool mid_f32, cudaStream_t st, bool pdl) {
  switch (dtype) {
    case kBF16:
      return mid_f32 ? expand_dispatch<__nv_bfloat16, float>(a, st, pdl)
                     : expand_dispatch<__nv_bfloat16, __nv_bfloat16>(a, st, pdl);
    case kF16:
      return mid_f32 ? expand_dispatch<__half, float>(a, st, pdl) : expand_dispatch<__half, __half>(a, st, pdl);
    case kF32:
      return expand_dispatch<float, float>(a, st, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace mlora
