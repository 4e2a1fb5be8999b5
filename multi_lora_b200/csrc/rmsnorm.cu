// Vectorised one-pass RMSNorm (kernels/rmsnorm.py:18-45,48-92 of the reference):
//   y[r, :] = T( (x_f32 * rsqrt(sum(x_f32^2) / H + eps)) * w_f32 )
// Rows are addressed with the reference's two-level stride
// (row r -> (r / inner) * stride_outer + (r % inner) * stride_inner,
// rmsnorm.py:59-74) so the q/k column slices of a fused qkv output are read in
// place. A group of G threads owns one row; each thread keeps its CPT chunks of
// the row in registers, so x is read from HBM exactly once. The norm weight is
// loaded before griddepcontrol.wait (it is constant for the step).
//
// Fused add (optional, the residual add in front of a decoder layer's norm):
// each chunk of the row is replaced by T(x + add) as it is loaded, written back
// to the residual row, and the rounded sum is what gets normalised; the result
// is bit-identical to a separate add followed by this RMSNorm, with one read
// of the row instead of a write and a re-read.
#include "common.cuh"
#include "kernels.h"

namespace mlora {

// a = T(a + b), element by element, in the chunk's packed form
template <typename T, int V>
__device__ __forceinline__ void add_round(Chunk<T, V>& a, const Chunk<T, V>& b) {
  float fa[V], fb[V];
  a.to_f(fa);
  b.to_f(fb);
  if constexpr (V * sizeof(T) == 16) {
    T o[V];
#pragma unroll
    for (int e = 0; e < V; ++e) o[e] = Num<T>::from_f(fa[e] + fb[e]);
    memcpy(&a.u, o, 16);
  } else {
    a.v = Num<T>::from_f(fa[0] + fb[0]);
  }
}

template <typename T, int V>
__device__ __forceinline__ void store_chunk(T* p, const Chunk<T, V>& a) {
  if constexpr (V * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(p) = a.u;
  } else {
    *p = a.v;
  }
}

// The V norm weights of chunk `c` (element offset k = c * V) as fp32. With
// `vec` (w 16-byte aligned, chunks of 4 or 8) one or two vector loads
// instead of V scalar ones: at 8192 columns the scalar loads were 8192 load
// instructions per block.
template <int V>
__device__ __forceinline__ void load_w_chunk(const void* w, int w_dtype, int64_t k, bool vec, float (&out)[V]) {
  if constexpr (V == 4 || V == 8) {
    if (vec) {
      if (w_dtype == kF32) {
        const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(w) + k);
#pragma unroll
        for (int i = 0; i < V / 4; ++i) {
          const float4 f = __ldg(src + i);
          out[4 * i] = f.x;
          out[4 * i + 1] = f.y;
          out[4 * i + 2] = f.z;
          out[4 * i + 3] = f.w;
        }
        return;
      }
      const uint16_t* w16 = static_cast<const uint16_t*>(w) + k;
      uint32_t h[V / 2];
      if constexpr (V == 8) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(w16));
        h[0] = u.x;
        h[1] = u.y;
        h[2] = u.z;
        h[3] = u.w;
      } else {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(w16));
        h[0] = u.x;
        h[1] = u.y;
      }
#pragma unroll
      for (int i = 0; i < V / 2; ++i) {
        if (w_dtype == kBF16) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&h[i]));
          out[2 * i] = f.x;
          out[2 * i + 1] = f.y;
        } else {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
          out[2 * i] = f.x;
          out[2 * i + 1] = f.y;
        }
      }
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < V; ++e) {
    switch (w_dtype) {
      case kBF16: out[e] = __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(w) + k + e)); break;
      case kF16: out[e] = __half2float(__ldg(static_cast<const __half*>(w) + k + e)); break;
      default: out[e] = __ldg(static_cast<const float*>(w) + k + e); break;
    }
  }
}

template <typename T, int V, int NT, int G, int CPT>
__global__ void __launch_bounds__(NT) rmsnorm_kernel(const RmsNormArgs p) {
  constexpr int RPB = NT / G;       // rows per block
  constexpr int WPG = G / 32;       // warps per row group
  __shared__ float s_part[RPB][WPG > 0 ? WPG : 1];

  const int tid = threadIdx.x;
  const int grp = tid / G, gt = tid % G;
  const int lane = tid & 31, wig = gt >> 5;
  const int64_t row = (int64_t)blockIdx.x * RPB + grp;
  const bool row_ok = row < p.rows;
  const int nchunk = p.hidden / V;
  constexpr int BLK = G * CPT;
  const int nblk = (nchunk + BLK - 1) / BLK;

  // norm weight (stable): converted once to fp32 per chunk
  float wf[CPT][V];
  auto load_w = [&](int blk) {
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int c = blk * BLK + j * G + gt;
#pragma unroll
      for (int e = 0; e < V; ++e) wf[j][e] = 0.f;
      if (c < nchunk) load_w_chunk<V>(p.w, p.w_dtype, (int64_t)c * V, p.w_vec != 0, wf[j]);
    }
  };
  if (nblk == 1) load_w(0);
  pdl_trigger();
  pdl_wait();

  const T* xr = static_cast<const T*>(p.x);
  if (row_ok) xr += (row / p.inner) * p.stride_outer + (row % p.inner) * p.stride_inner;
  T* yr = static_cast<T*>(p.y) + (row_ok ? row * p.y_stride : 0);
  const bool fused = p.add != nullptr;
  const T* ar = static_cast<const T*>(p.add) + (fused && row_ok ? row * p.add_stride : 0);
  T* rr = static_cast<T*>(p.res) + (fused && row_ok ? row * p.res_stride : 0);

  Chunk<T, V> xc[CPT];
  float ss = 0.f;
  for (int blk = 0; blk < nblk; ++blk) {
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int c = blk * BLK + j * G + gt;
      if (row_ok && c < nchunk) {
        xc[j].ldcg(xr + (int64_t)c * V);
        if (fused) {  // the residual add: T(x + add), kept and written back
          Chunk<T, V> ac;
          ac.ldcg(ar + (int64_t)c * V);
          add_round(xc[j], ac);
          store_chunk(rr + (int64_t)c * V, xc[j]);
        }
      } else {
        xc[j].zero();
      }
      float f[V];
      xc[j].to_f(f);
#pragma unroll
      for (int e = 0; e < V; ++e) ss = fmaf(f[e], f[e], ss);
    }
  }
  ss = warp_sum(ss);
  if constexpr (WPG > 1) {
    if (lane == 0) s_part[grp][wig] = ss;
    __syncthreads();
    ss = 0.f;
#pragma unroll
    for (int w = 0; w < WPG; ++w) ss += s_part[grp][w];
  }
  // Reference: var = sum / n_cols; rstd = rsqrt(var + eps)  (rmsnorm.py:40-41)
  const float rstd = rsqrtf(ss / (float)p.hidden + p.eps);
  if (!row_ok) return;

  for (int blk = 0; blk < nblk; ++blk) {
    if (nblk > 1) load_w(blk);
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int c = blk * BLK + j * G + gt;
      if (c >= nchunk) continue;
      if (nblk > 1) xc[j].ldcg((fused ? rr : xr) + (int64_t)c * V);  // the rounded sum this thread wrote
      float f[V];
      xc[j].to_f(f);
      if constexpr (V * sizeof(T) == 16) {
        T o[V];
#pragma unroll
        for (int e = 0; e < V; ++e) o[e] = Num<T>::from_f((f[e] * rstd) * wf[j][e]);
        uint4 u;
        memcpy(&u, o, 16);
        *reinterpret_cast<uint4*>(yr + (int64_t)c * V) = u;
      } else {
#pragma unroll
        for (int e = 0; e < V; ++e) yr[(int64_t)c * V + e] = Num<T>::from_f((f[e] * rstd) * wf[j][e]);
      }
    }
  }
}

namespace {

template <typename T, int V>
cudaError_t rms_dispatch(const RmsNormArgs& a, cudaStream_t st, bool pdl) {
  const int nchunk = a.hidden / V;
  auto go = [&](auto kern, int nt, int g) {
    const int rpb = nt / g;
    const dim3 grid((unsigned)((a.rows + rpb - 1) / rpb));
    return launch_kernel(kern, grid, dim3(nt), 0, st, pdl, a);
  };
  if (nchunk <= 32) return go(rmsnorm_kernel<T, V, 256, 32, 1>, 256, 32);
  if (nchunk <= 64) return go(rmsnorm_kernel<T, V, 256, 32, 2>, 256, 32);
  if (nchunk <= 128) return go(rmsnorm_kernel<T, V, 256, 32, 4>, 256, 32);
  if (nchunk <= 256) return go(rmsnorm_kernel<T, V, 256, 64, 4>, 256, 64);
  if (nchunk <= 512) return go(rmsnorm_kernel<T, V, 256, 256, 2>, 256, 256);
  if (nchunk <= 1024) return go(rmsnorm_kernel<T, V, 256, 256, 4>, 256, 256);
  if (nchunk <= 2048) return go(rmsnorm_kernel<T, V, 512, 512, 4>, 512, 512);
  return go(rmsnorm_kernel<T, V, 1024, 1024, 4>, 1024, 1024);  // loops blocks past 4096 chunks
}

}  // namespace

cudaError_t launch_rmsnorm(const RmsNormArgs& a, int dtype, cudaStream_t st, bool pdl) {
  switch (dtype) {
    case kBF16: return a.vec_ok ? rms_dispatch<__nv_bfloat16, 8>(a, st, pdl) : rms_dispatch<__nv_bfloat16, 1>(a, st, pdl);
    case kF16: return a.vec_ok ? rms_dispatch<__half, 8>(a, st, pdl) : rms_dispatch<__half, 1>(a, st, pdl);
    case kF32: return a.vec_ok ? rms_dispatch<float, 4>(a, st, pdl) : rms_dispatch<float, 1>(a, st, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace mlora
