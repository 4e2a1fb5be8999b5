// Fused apply_lora for short segments (decode): shrink and expand in ONE launch.
//
// Semantics are those of LoRABackend.apply_lora (backend/base.py:60-89 of the
// reference): mid = T(x @ A[slot, :rank].T) with fp32 accumulation
// (sgemm_lora_a.py:119-183), then
// y = T(T(scaling * mid @ B[slot, :, :rank].T) + y) (sgemm_lora_b.py:94-153).
// Up to four projections that share x and the routing (q/k/v, gate/up) can
// go in one launch (blockIdx.z selects the projection).
//
// Layout on the GPU: one thread-block CLUSTER per (adapter slot, projection),
// CS = 8 or 16 CTAs. CTA j of the cluster
//   1. owns k-slice j of the input dim: one thread issues TMA bulk copies of
//      A[slot, :rank, slice] and of its output block B[slot, block, :rank] into
//      shared memory (an mbarrier counts the bytes) BEFORE
//      griddepcontrol.wait, so under programmatic dependent launch the weight
//      stream overlaps the previous kernel;
//   2. after the wait it bulk-copies the slot's x rows (its slice) and y rows
//      (its output block) and computes split-K partials of mid;
//   3. pushes its partials into every peer CTA's shared memory with st.async
//      (distributed shared memory; each receiver's mbarrier counts the bytes),
//      so no cluster-wide barrier sits on the critical path; each CTA sums the
//      CS partials in a fixed order (deterministic) and rounds to T once, as
//      the reference stores mid in x's dtype;
//   4. adds the scaled delta of its output block into y.
// Each slot's A and B are read from HBM exactly once per launch. No global
// scratch, no atomics. Every wait is bounded (status bit on timeout).
#include <cooperative_groups.h>

#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace mlora {

constexpr int kFusedNT = 256;
constexpr int kFusedTT = 8;       // tokens per tile
constexpr int kFusedScan = 256;   // segment indices scanned per pass

// Segment list of one slot for up to kFusedScan scanned segment indices.
struct FusedSegs {
  int start[kFusedScan];
  int cum[kFusedScan + 1];
  int n;
};

// Warp 0 scans segment indices [from, min(bs, from + kFusedScan)) with every
// load of the pass issued up front (one memory round trip).
__device__ __forceinline__ void fused_scan(FusedSegs& sl, int slot, int from, const FusedArgs& p) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  constexpr int NB = kFusedScan / 32;
  int w[NB], st[NB], en[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int idx = from + b * 32 + lane;
    w[b] = -1;
    st[b] = en[b] = 0;
    if (idx < p.bs) {
      w[b] = __ldg(p.weight_indices + idx);
      st[b] = __ldg(p.seg_indptr + idx);
      en[b] = __ldg(p.seg_indptr + idx + 1);
    }
  }
  int n = 0, total = 0;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int idx = from + b * 32 + lane;
    bool match = false;
    int len = 0;
    if (idx < p.bs) {
      if (w[b] < 0 || w[b] >= p.num_slots) {
        if (slot == 0 && blockIdx.x == 0) flag_error(p.status, kErrSlotRange);
      } else if (w[b] == slot) {
        if (st[b] < 0 || en[b] < st[b] || en[b] > p.S) {
          if (blockIdx.x == 0) flag_error(p.status, kErrIndptr);
        } else if (en[b] > st[b]) {
          match = true;
          len = en[b] - st[b];
        }
      }
    }
    const unsigned m = __ballot_sync(0xffffffffu, match);
    int incl = len;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (match) {
      const int pos = n + __popc(m & ((1u << lane) - 1u));
      sl.start[pos] = st[b];
      sl.cum[pos] = total + incl - len;
    }
    n += __popc(m);
    total += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) {
    sl.n = n;
    sl.cum[n] = total;
  }
}

__device__ __forceinline__ int fused_token_row(const FusedSegs& sl, int q) {
  int lo = 0, hi = sl.n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (sl.cum[mid] <= q) lo = mid; else hi = mid - 1;
  }
  return sl.start[lo] + (q - sl.cum[lo]);
}

// RM: rank rows covered by the shrink thread grid (16, 32 or 64; >= R);
// KG = NT / RM threads per rank row.
template <typename T, int RM>
__global__ void __launch_bounds__(kFusedNT) apply_fused_kernel(const FusedArgs p) {
  constexpr int NT = kFusedNT;
  constexpr int V = 8;            // elements per 16-byte chunk (bf16/f16)
  constexpr int KG = NT / RM;     // threads per rank row in the shrink
  constexpr int TT = kFusedTT;
  constexpr int Q4 = RM / 4;      // 16-byte pieces per partial row
  __shared__ FusedSegs sl;
  __shared__ int s_rows[TT];
  __shared__ __align__(16) float s_part[TT][RM];
  __shared__ __align__(16) float s_mid[TT][RM];
  __shared__ __align__(8) uint64_t bar_w, bar_x, bar_p;
  extern __shared__ __align__(128) unsigned char s_dyn[];

  cg::cluster_group cluster = cg::this_cluster();
  const int cs = (int)cluster.num_blocks();
  const int j = (int)cluster.block_rank();
  const int slot = blockIdx.y;
  const int tid = threadIdx.x;
  const int R = p.R;
  FusedModule m = p.mod[0];
#pragma unroll
  for (int i = 1; i < kMaxFusedModules; ++i)
    if (i == (int)blockIdx.z) m = p.mod[i];

  int rank = __ldg(p.lora_ranks + slot);
  if (rank < 0 || rank > R) {
    if (j == 0 && tid == 0 && blockIdx.z == 0) flag_error(p.status, kErrRankRange);
    rank = rank < 0 ? 0 : R;
  }
  if (rank == 0) {  // base model: no delta, mid untouched (uniform per cluster)
    pdl_trigger();
    return;
  }
  fused_scan(sl, slot, 0, p);
  __syncthreads();
  if (sl.n == 0 && p.bs <= kFusedScan) {  // slot unused by this batch (uniform per cluster)
    pdl_trigger();
    return;
  }

  // shared memory: A [R][ks] | B [ob_max][R] | x [TT][ks] | y [TT][ob_max] | partials in [cs][TT][RM]
  const int k0 = j * p.ks;                       // multiple of V
  const int kend = min(p.in_dim, k0 + p.ks);
  const int klen = kend > k0 ? kend - k0 : 0;    // multiple of V
  const int c_end = klen / V;
  const int o_lo = min(m.out_dim, j * m.ob);
  const int o_hi = min(m.out_dim, o_lo + m.ob);
  const int olen = o_hi - o_lo;
  T* s_a = reinterpret_cast<T*>(s_dyn);
  T* s_b = s_a + (size_t)R * p.ks;
  T* s_x = s_b + (size_t)p.ob_max * R;
  T* s_y = s_x + (size_t)TT * p.ks;
  float* s_recv = reinterpret_cast<float*>(s_y + (size_t)TT * p.ob_max);

  // ---- prologue: adapter weights (stable for the step) into shared memory ----
  if (tid == 0) {
    mbar_init(&bar_w, 1);
    mbar_init(&bar_x, 1);
    mbar_init(&bar_p, 1);
    fence_barrier_init();
  }
  __syncthreads();
  cluster_arrive_release();  // this CTA runs and its barriers exist; peers wait before pushing to it
  const T* __restrict__ a_src = static_cast<const T*>(m.a) + (int64_t)slot * R * p.in_dim + k0;
  const T* __restrict__ b_src = static_cast<const T*>(m.b) + ((int64_t)slot * m.out_dim + o_lo) * R;
  const bool b_dense = rank == R;  // B rows hold exactly the rank: one contiguous block
  if (tid == 0) {
    const uint32_t a_bytes = (uint32_t)rank * klen * sizeof(T);
    const uint32_t b_bytes = b_dense ? (uint32_t)olen * R * sizeof(T) : 0u;
    mbar_arrive_expect_tx(&bar_w, a_bytes + b_bytes);
    if (klen > 0)
      for (int n = 0; n < rank; ++n)
        bulk_copy_g2s(s_a + (size_t)n * p.ks, a_src + (int64_t)n * p.in_dim, klen * sizeof(T), &bar_w);
    if (b_bytes > 0) bulk_copy_g2s(s_b, b_src, b_bytes, &bar_w);
  }
  const int rc = (rank + V - 1) / V;  // B chunks per row that hold rank columns
  if (!b_dense) {  // rows of R with only `rank` valid columns: 16-byte copies per thread
    for (int e = tid; e < olen * rc; e += NT) {
      const int row = e / rc, c = e - row * rc;
      cp_async16(s_b + (size_t)row * R + c * V, b_src + (int64_t)row * R + c * V);
    }
  }
  float scale;
  switch (p.scalings_dtype) {
    case kBF16: scale = __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(p.scalings) + slot)); break;
    case kF16: scale = __half2float(__ldg(static_cast<const __half*>(p.scalings) + slot)); break;
    default: scale = __ldg(static_cast<const float*>(p.scalings) + slot); break;
  }
  pdl_trigger();
  pdl_wait();  // x and y come from earlier kernels

  const T* __restrict__ xbase = static_cast<const T*>(p.x);
  T* __restrict__ ybase = static_cast<T*>(m.y);
  bool ok = true;
  uint32_t x_phase = 0, p_phase = 0;
  bool first = true;
  int tiles_left = 0;
  for (int from = 0; from < p.bs; from += kFusedScan) {
    if (from > 0) {
      __syncthreads();
      fused_scan(sl, slot, from, p);
      __syncthreads();
    }
    const int ntok = sl.cum[sl.n];
    for (int q0 = 0; q0 < ntok; q0 += TT) {
      const int nt = min(TT, ntok - q0);
      if (tid < nt) s_rows[tid] = fused_token_row(sl, q0 + tid);
      __syncthreads();
      if (tid == 0) {  // this tile's x rows (k-slice) and y rows (output block)
        fence_proxy_async_smem();
        const uint32_t y_bytes = m.y_tma ? (uint32_t)nt * olen * sizeof(T) : 0u;
        mbar_arrive_expect_tx(&bar_x, (uint32_t)nt * klen * sizeof(T) + y_bytes);
        for (int t = 0; t < nt; ++t) {
          if (klen > 0)
            bulk_copy_g2s(s_x + (size_t)t * p.ks, xbase + (int64_t)s_rows[t] * p.x_stride + k0, klen * sizeof(T),
                          &bar_x);
          if (y_bytes > 0 && olen > 0)
            bulk_copy_g2s(s_y + (size_t)t * p.ob_max, ybase + (int64_t)s_rows[t] * m.y_stride + o_lo,
                          olen * sizeof(T), &bar_x);
        }
      }
      if (first) ok = mbar_wait(&bar_w, 0, p.status) && ok;
      ok = mbar_wait(&bar_x, x_phase, p.status) && ok;
      x_phase ^= 1u;
      // split-K partials of this CTA's slice, one token at a time (decode tiles
      // hold few tokens); the KG threads of a rank row reduce by shuffles
      {
        const int n = tid / KG, kg = tid % KG;
        const uint4* arow = reinterpret_cast<const uint4*>(s_a + (size_t)n * p.ks);
        for (int t = 0; t < nt; ++t) {
          const uint4* xrow = reinterpret_cast<const uint4*>(s_x + (size_t)t * p.ks);
          float acc = 0.f;
          if (ok && n < rank) {
            for (int c = kg; c < c_end; c += KG) {
              float af[V], xf[V];
              unpack16<T>(arow[c], af);
              unpack16<T>(xrow[c], xf);
#pragma unroll
              for (int e = 0; e < V; ++e) acc = fmaf(xf[e], af[e], acc);
            }
          }
#pragma unroll
          for (int o = KG / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
          if (kg == 0) s_part[t][n] = acc;
        }
      }
      if (first && !b_dense) cp_async_wait_all();
      __syncthreads();  // s_part complete (and this CTA's B block, on the 16-byte-copy path)
      if (first) cluster_wait_acquire();  // every peer runs and has its barriers initialised
      first = false;
      // push this CTA's partials into slot j of every peer's receive buffer
      if (tid == 0) mbar_arrive_expect_tx(&bar_p, (uint32_t)cs * nt * RM * sizeof(float));
      {
        const uint32_t my_recv = smem_addr(s_recv + (size_t)j * TT * RM);
        const uint32_t my_bar = smem_addr(&bar_p);
        for (int e = tid; e < cs * nt * Q4; e += NT) {
          const int q = e / (nt * Q4), r = e - q * (nt * Q4);
          const int t = r / Q4, k4 = (r - t * Q4) * 4;
          const float4 v = *reinterpret_cast<const float4*>(&s_part[t][k4]);
          st_async_v4(cluster_map(my_recv + (uint32_t)(t * RM + k4) * 4u, (uint32_t)q), v.x, v.y, v.z, v.w,
                      cluster_map(my_bar, (uint32_t)q));
        }
      }
      ok = mbar_wait(&bar_p, p_phase, p.status) && ok;
      p_phase ^= 1u;
      for (int e = tid; e < TT * RM; e += NT) {
        const int t = e / RM, k = e - t * RM;
        float v = 0.f;
        if (t < nt && k < rank) {
          for (int q = 0; q < cs; ++q) v += s_recv[((size_t)q * TT + t) * RM + k];
          if (j == 0 && m.mid != nullptr)
            static_cast<T*>(m.mid)[(int64_t)s_rows[t] * m.mid_stride + k] = Num<T>::from_f(v);
          v = round_to<T>(v);
        }
        s_mid[t][k] = v;
      }
      __syncthreads();  // s_mid complete
      // expand: this CTA's output block; consecutive threads own consecutive outputs
      if (ok) {
        for (int o = o_lo + tid; o < o_hi; o += NT) {
          const uint4* brow = reinterpret_cast<const uint4*>(s_b + (size_t)(o - o_lo) * R);
          for (int t = 0; t < nt; ++t) {
            float acc = 0.f;
            for (int c = 0; c < rc; ++c) {
              float bf[V];
              unpack16<T>(brow[c], bf);
              const float4 m0 = *reinterpret_cast<const float4*>(&s_mid[t][c * V]);
              const float4 m1 = *reinterpret_cast<const float4*>(&s_mid[t][c * V + 4]);
              const float mv[V] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
#pragma unroll
              for (int e = 0; e < V; ++e)  // stale weights past the rank may be NaN: masked
                acc = fmaf(mv[e], (c * V + e < rank) ? bf[e] : 0.f, acc);
            }
            T* yp = ybase + (int64_t)s_rows[t] * m.y_stride + o;
            const float yold = m.y_tma ? Num<T>::to_f(s_y[(size_t)t * p.ob_max + (o - o_lo)]) : ldcg_f<T>(yp);
            *yp = Num<T>::from_f(round_to<T>(acc * scale) + yold);
          }
        }
      }
      tiles_left = (q0 + TT < ntok) || (from + kFusedScan < p.bs) ? 1 : 0;
      if (tiles_left) cluster.sync();  // peers finished reading s_recv before the next pushes
      else __syncthreads();
    }
  }
  // Never leave with copies in flight into this CTA's shared memory: weights
  // that no tile consumed (a slot with no tokens past the first scan pass),
  // or copies whose wait timed out, are drained here (bounded again).
  if (first) {
    cluster_wait_acquire();  // pairs the prologue arrive
    mbar_wait(&bar_w, 0, p.status);
    if (!b_dense) cp_async_wait_all();
  }
  if (!ok && tid == 0) {  // ok is only cleared inside a tile
    mbar_wait(&bar_x, x_phase ^ 1u, p.status);
    mbar_wait(&bar_p, p_phase ^ 1u, p.status);
  }
}

namespace {

template <typename T, int RM>
cudaError_t go_fused(const FusedArgs& a, int cs, size_t smem, cudaStream_t st, bool pdl) {
  auto kern = apply_fused_kernel<T, RM>;
  // Function attributes are set once per instance (largest shared memory so far);
  // whether a cluster shape can be placed at all is cached per (cs, smem KiB).
  static std::mutex mu;
  static int smem_set = 0;
  static bool nonportable_set = false;
  static std::map<std::pair<int, int>, bool> placeable;
  {
    std::lock_guard<std::mutex> lock(mu);
    cudaError_t e;
    if (cs > 8 && !nonportable_set) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return e;
      nonportable_set = true;
    }
    const int kib = (int)((smem + 1023) / 1024);
    if (kib * 1024 > smem_set) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kib * 1024);
      if (e != cudaSuccess) return e;
      smem_set = kib * 1024;
    }
    auto key = std::make_pair(cs, kib);
    auto it = placeable.find(key);
    if (it == placeable.end()) {
      cudaLaunchConfig_t q = {};
      q.gridDim = dim3(cs, 1, 1);
      q.blockDim = dim3(kFusedNT);
      q.dynamicSmemBytes = (size_t)kib * 1024;
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = cs;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = 1;
      q.attrs = qa;
      q.numAttrs = 1;
      int clusters = 0;
      e = cudaOccupancyMaxActiveClusters(&clusters, kern, &q);
      if (e != cudaSuccess) {
        (void)cudaGetLastError();
        clusters = 0;
      }
      it = placeable.emplace(key, clusters > 0).first;
    }
    if (!it->second) return cudaErrorNotSupported;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cs, a.num_slots, a.n_mod);
  cfg.blockDim = dim3(kFusedNT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace

// Picks the cluster size so the per-CTA shared memory fits; returns
// cudaErrorNotSupported when the shape is outside the fused kernel's range
// (the caller then runs shrink and expand separately).
cudaError_t launch_apply_fused(FusedArgs a, int dtype, cudaStream_t st, bool pdl) {
  if (dtype != kBF16 && dtype != kF16) return cudaErrorNotSupported;
  if (a.n_mod < 1 || a.n_mod > kMaxFusedModules) return cudaErrorNotSupported;
  if (a.R > 64 || a.R % 8 != 0 || a.in_dim % 8 != 0) return cudaErrorNotSupported;
  const int rm = a.R <= 16 ? 16 : a.R <= 32 ? 32 : 64;
  for (int cs : {8, 16}) {
    int ks = (a.in_dim + cs - 1) / cs;
    ks = (ks + 7) / 8 * 8;
    int ob_max = 8;
    for (int i = 0; i < a.n_mod; ++i) {
      FusedModule& m = a.mod[i];
      m.ob = ((m.out_dim + cs - 1) / cs + 7) / 8 * 8;
      ob_max = m.ob > ob_max ? m.ob : ob_max;
      m.y_tma = (reinterpret_cast<uintptr_t>(m.y) % 16 == 0) && (m.y_stride % 8 == 0) && (m.out_dim % 8 == 0);
    }
    const size_t smem = (size_t)2 * ((size_t)a.R * ks + (size_t)ob_max * a.R + (size_t)kFusedTT * ks +
                                     (size_t)kFusedTT * ob_max) +
                        (size_t)4 * cs * kFusedTT * rm;
    if (smem > 200 * 1024) continue;
    a.ks = ks;
    a.ob_max = ob_max;
    cudaError_t e;
    if (dtype == kBF16)
      e = rm == 16 ? go_fused<__nv_bfloat16, 16>(a, cs, smem, st, pdl)
        : rm == 32 ? go_fused<__nv_bfloat16, 32>(a, cs, smem, st, pdl)
                   : go_fused<__nv_bfloat16, 64>(a, cs, smem, st, pdl);
    else
      e = rm == 16 ? go_fused<__half, 16>(a, cs, smem, st, pdl)
        : rm == 32 ? go_fused<__half, 32>(a, cs, smem, st, pdl)
                   : go_fused<__half, 64>(a, cs, smem, st, pdl);
    if (e != cudaErrorNotSupported) return e;
  }
  return cudaErrorNotSupported;
}

}  // namespace mlora
