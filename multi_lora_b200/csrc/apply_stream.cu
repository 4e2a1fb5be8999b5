// Streaming apply_lora for decode-sized batches: shrink and expand as two
// persistent, warp-specialised kernels chained by programmatic dependent launch.
//
// Semantics are those of LoRABackend.apply_lora (backend/base.py:60-89 of the
// reference): mid = T(x @ A[slot, :rank].T) with fp32 accumulation
// (sgemm_lora_a.py:119-183), then
// y = T(T(scaling * mid @ B[slot, :, :rank].T) + y) (sgemm_lora_b.py:94-153),
// for up to four projections that share x and the routing.
//
// Work decomposition. Every CTA rebuilds the batch's slot -> token lists from
// the routing tables in shared memory (a counting sort, stable in segment
// order so that every CTA cuts the same tiles; slots of rank 0 or with no
// tokens drop out) and cuts each slot's tokens into tiles of up to kStreamTM
// rows. Items are then dealt round-robin to one CTA per SM:
//   shrink kernel: item = (tile, projection); it streams A[slot, :rank, :] and
//     the tile's x rows through the shared-memory ring in chunks of KC input
//     columns and accumulates mid for the tile over the whole input dim, so
//     the reduction is inside one CTA (fixed order, no atomics, no scratch);
//     the rounded mid rows go to the caller's mid buffer (columns < rank).
//   expand kernel: item = (tile, projection, OC-row block of B); it streams
//     B[slot, block, :], the tile's y rows (block columns) and mid rows, and
//     writes the updated y values straight from registers to the caller's rows.
// One producer warp fills a kStreamStages-deep shared-memory ring with 1-D
// TMA bulk copies (lane 0 arms the stage's full mbarrier with the byte count,
// the lanes issue one row copy each: a single issuing thread was measured at
// ~75-100 ns per bulk copy, too slow for row-sized pieces); eight consumer
// warps run mma.sync m16n8k16 tiles and release stages on empty mbarriers.
// The weights of the first ring fills are requested BEFORE griddepcontrol.wait,
// so under programmatic dependent launch they stream while the previous
// kernel finishes; x, y and mid are only read after the wait. The expand
// kernel is launched right behind the shrink kernel and prefetches its B
// blocks while the shrink runs; its wait is the shrink -> expand dependency.
// Each CTA needs ~100 KB of shared memory, so a shrink CTA and an expand CTA
// share an SM. Every mbarrier wait is bounded (status bit on timeout).
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "mma.cuh"
#include "tma.cuh"
#include "xchg.cuh"

namespace mlora {

constexpr int kStreamConsumers = 8;                          // consumer warps
constexpr int kStreamThreads = (kStreamConsumers + 1) * 32;  // + one producer warp
constexpr int kStreamTM = 8;                                 // tokens per tile
constexpr int kStreamStages = 2;        // expand ring
constexpr int kStreamShrinkStages = 2;  // shrink ring (stages twice as wide: half the row copies per byte)
constexpr int kStreamShrinkSplit = 4;   // CTAs per shrink item (a cluster splitting the input dim)

// Input columns per shrink chunk and B rows per expand block: ~16 KB of
// weights per ring stage at every rank.
__host__ __device__ constexpr int stream_kc(int rm) { return 8192 / rm; }

__host__ __device__ constexpr int align128(int b) { return (b + 127) / 128 * 128; }

template <int RM>
struct ShrinkStage {
  static constexpr int KC = 2 * stream_kc(RM);
  static constexpr int KCP = KC + 8;  // padded row (odd number of 16-byte units: ldmatrix conflict-free)
  static constexpr int A_BYTES = align128(RM * KCP * 2);
  static constexpr int X_BYTES = align128(kStreamTM * KCP * 2);
  static constexpr int BYTES = A_BYTES + X_BYTES;
};

template <int RM>
struct ExpandStage {
  static constexpr int OC = 2 * stream_kc(RM);
  static constexpr int OCP = OC + 8;
  static constexpr int MP = RM + 8;
  static constexpr int B_BYTES = align128(OC * RM * 2 + 16);  // + slack: a half k-step may read 16 B past the block
  static constexpr int Y_BYTES = align128(kStreamTM * OCP * 2);
  static constexpr int M_BYTES = align128(kStreamTM * MP * 4);  // rows of T, or of fp32 (mid_f32)
  static constexpr int BYTES = B_BYTES + Y_BYTES + M_BYTES;
};

// Routing arrays in dynamic shared memory behind the ring.
struct StreamRouting {
  int* cnt;     // [num_slots] tokens routed to the slot (0 if unused or rank 0)
  int* fill;    // [num_slots] rows placed so far
  int* off;     // [num_slots] first entry of the slot in tok
  int* toff;    // [num_slots + 1] first tile of the slot; toff[num_slots] = tiles
  int* rank;    // [num_slots] rank clamped to [0, R]
  float* scale; // [num_slots]
  int* tok;     // [S] token rows grouped by slot
};

__host__ __device__ inline int stream_routing_bytes(int num_slots, int S) {
  return 4 * (6 * num_slots + 1 + S);
}

__device__ __forceinline__ StreamRouting stream_routing(unsigned char* base, int num_slots) {
  StreamRouting r;
  int* p = reinterpret_cast<int*>(base);
  r.cnt = p;
  r.fill = p + num_slots;
  r.off = p + 2 * num_slots;
  r.rank = p + 3 * num_slots;
  r.scale = reinterpret_cast<float*>(p + 4 * num_slots);
  r.toff = p + 5 * num_slots;
  r.tok = p + 6 * num_slots + 1;
  return r;
}

// Counting sort of the batch's tokens by slot, stable in segment order.
// Reads only routing tables and ranks/scalings, which no kernel of the step writes.
__device__ void stream_build_routing(const StreamArgs& p, const StreamRouting& rt, bool want_scale) {
  __shared__ int s_overflow;
  const int tid = threadIdx.x, nt = blockDim.x;
  const bool reporter = blockIdx.x == 0;
  for (int s = tid; s < p.num_slots; s += nt) {
    int r = __ldg(p.lora_ranks + s);
    if (r < 0 || r > p.R) {
      if (reporter) flag_error(p.status, kErrRankRange);
      r = r < 0 ? 0 : p.R;
    }
    rt.rank[s] = r;
    rt.cnt[s] = 0;
    rt.fill[s] = 0;
    if (want_scale) {
      float sc;
      switch (p.scalings_dtype) {
        case kBF16: sc = __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(p.scalings) + s)); break;
        case kF16: sc = __half2float(__ldg(static_cast<const __half*>(p.scalings) + s)); break;
        default: sc = __ldg(static_cast<const float*>(p.scalings) + s); break;
      }
      rt.scale[s] = sc;
    }
  }
  __syncthreads();
  for (int i = tid; i < p.bs; i += nt) {
    const int w = __ldg(p.weight_indices + i);
    const int st = __ldg(p.seg_indptr + i), en = __ldg(p.seg_indptr + i + 1);
    if (w < 0 || w >= p.num_slots) {
      if (reporter) flag_error(p.status, kErrSlotRange);
      continue;
    }
    if (st < 0 || en < st || en > p.S) {
      if (reporter) flag_error(p.status, kErrIndptr);
      continue;
    }
    if (en > st && rt.rank[w] > 0) atomicAdd(&rt.cnt[w], en - st);
  }
  __syncthreads();
  if (tid < 32) {  // exclusive scans: token offsets and tile offsets per slot
    int tok_base = 0, tile_base = 0;
    for (int s0 = 0; s0 < p.num_slots; s0 += 32) {
      const int s = s0 + tid;
      const int c = s < p.num_slots ? rt.cnt[s] : 0;
      const int t = (c + kStreamTM - 1) / kStreamTM;
      int ic = c, it = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int vc = __shfl_up_sync(0xffffffffu, ic, o);
        const int vt = __shfl_up_sync(0xffffffffu, it, o);
        if (tid >= o) {
          ic += vc;
          it += vt;
        }
      }
      if (s < p.num_slots) {
        rt.off[s] = tok_base + ic - c;
        rt.toff[s] = tile_base + it - t;
      }
      tok_base += __shfl_sync(0xffffffffu, ic, 31);
      tile_base += __shfl_sync(0xffffffffu, it, 31);
    }
    if (tid == 0) {
      // valid routing covers each row at most once; more rows than S means
      // overlapping segments: flag it and do no work (the token list holds S rows)
      s_overflow = tok_base > p.S;
      if (s_overflow) flag_error(p.status, kErrIndptr);
      rt.toff[p.num_slots] = s_overflow ? 0 : tile_base;
    }
  }
  __syncthreads();
  if (s_overflow) return;
  // Token lists in segment order, identical in every CTA (tiles of a slot are
  // cut from this order, and different CTAs must agree on them): warp 0 walks
  // the segments 32 at a time; lanes of one slot (match_any) place their rows
  // after the slot's earlier segments.
  if (tid < 32) {
    const int lane = tid;
    for (int s0 = 0; s0 < p.bs; s0 += 32) {
      const int i = s0 + lane;
      int w = -1, st = 0, en = 0;
      if (i < p.bs) {
        w = __ldg(p.weight_indices + i);
        st = __ldg(p.seg_indptr + i);
        en = __ldg(p.seg_indptr + i + 1);
        if (w < 0 || w >= p.num_slots || st < 0 || en < st || en > p.S || rt.rank[w] == 0) w = -1;
      }
      const int len = w >= 0 ? en - st : 0;
      const unsigned peers = __match_any_sync(0xffffffffu, w >= 0 ? w : -1 - lane);
      const unsigned lower = peers & ((1u << lane) - 1u);
      int pre = 0;  // rows of this slot's segments on lower lanes
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const int v = __shfl_sync(0xffffffffu, len, k);
        if ((lower >> k) & 1u) pre += v;
      }
      const int base = w >= 0 ? rt.fill[w] : 0;
      __syncwarp();
      if (w >= 0) {
        for (int row = st; row < en; ++row) rt.tok[rt.off[w] + base + pre + (row - st)] = row;
        if (lane == 31 - __clz(peers)) rt.fill[w] = base + pre + len;  // the slot's last lane in this pass
      }
      __syncwarp();
    }
  }
  __syncthreads();
}

struct StreamTile {
  int slot, start, nt, rank;
};

// Tile index -> slot (binary search over the tile offsets), first token entry and row count.
__device__ __forceinline__ StreamTile stream_tile(const StreamRouting& rt, int num_slots, int tile) {
  int lo = 0, hi = num_slots - 1;
  while (lo < hi) {  // last slot whose first tile <= tile
    const int mid = (lo + hi + 1) >> 1;
    if (rt.toff[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  StreamTile t;  // (slots without tiles share their toff with a later slot, so the last match owns `tile`)
  t.slot = lo;
  const int k = tile - rt.toff[lo];
  t.start = rt.off[lo] + k * kStreamTM;
  t.nt = min(kStreamTM, rt.cnt[lo] - k * kStreamTM);
  t.rank = rt.rank[lo];
  return t;
}

// ---------------------------------------------------------------------------
// shared pieces of the two kernels
// ---------------------------------------------------------------------------
__device__ __forceinline__ StreamModule stream_module(const StreamArgs& p, int m) {
  StreamModule r = p.mod[0];
#pragma unroll
  for (int i = 1; i < kMaxStreamModules; ++i)
    if (i == m) r = p.mod[i];
  return r;
}

// ---------------------------------------------------------------------------
// shrink
// ---------------------------------------------------------------------------
// XCHG: the row-parallel peer exchange (p.xchg) is on; a separate instance,
// so the plain kernels carry none of its code.
template <typename T, int RM, bool XCHG>
__global__ void __launch_bounds__(kStreamThreads, 1) lora_shrink_stream_kernel(const StreamArgs p) {
  using SS = ShrinkStage<RM>;
  constexpr int NC = kStreamConsumers, NS = kStreamShrinkStages, TM = kStreamTM, KS = kStreamShrinkSplit;
  constexpr int KC = SS::KC, KCP = SS::KCP;
  constexpr uint32_t PB = TM * RM * 4;  // one CTA's fp32 partial tile
  extern __shared__ __align__(128) unsigned char s_dyn[];
  __shared__ __align__(8) uint64_t full[NS], empty[NS], bar_red[2], bar_free[2];
  __shared__ __align__(16) float s_red[NC][TM][RM];
  __shared__ __align__(16) float s_recv[2][KS][TM][RM];  // used in cluster rank 0

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const StreamRouting rt = stream_routing(s_dyn + NS * SS::BYTES, p.num_slots);
  stream_build_routing(p, rt, false);
  const int tiles = rt.toff[p.num_slots];
  const int n_items = tiles * p.n_mod;
  // one thread-block cluster of KS CTAs per item: CTA `crank` streams its share
  // of the input dim; the partial tiles meet in CTA 0 (distributed shared memory)
  const int crank = (int)(blockIdx.x % KS), cl = (int)(blockIdx.x / KS), NCL = (int)(gridDim.x / KS);
  const int my_items = cl < n_items ? (n_items - 1 - cl) / NCL + 1 : 0;  // the same for the whole cluster
  if (my_items == 0) {
    // CTA 0 waits even here: the grid must not complete before the previous
    // kernel (with the exchange on, the previous call's expand advances the
    // epoch the next call reads)
    pdl_exit_early();
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NC);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_red[s], 1);
      mbar_init(&bar_free[s], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  cluster_arrive_release();
  cluster_wait_acquire();  // every CTA's barriers exist before any remote operation
  pdl_trigger();           // the expand kernel may launch now and prefetch its weights

  const int nch = (p.in_dim + KC - 1) / KC;
  const int c_lo = crank * nch / KS, cnt = (crank + 1) * nch / KS - c_lo;  // this CTA's chunks per item
  const int total = my_items * cnt;                                         // ring fills of this CTA
  if (warp == NC) {
    // ---------------- producer warp: lane 0 arms the stage, every lane issues copies ----------------
    auto stage_a = [&](int s) { return reinterpret_cast<T*>(s_dyn + s * SS::BYTES); };
    auto stage_x = [&](int s) { return reinterpret_cast<T*>(s_dyn + s * SS::BYTES + SS::A_BYTES); };
    auto issue_a = [&](int f) {
      const int s = f % NS;
      const int item = cl + (f / cnt) * NCL, c = c_lo + f % cnt;
      const StreamTile t = stream_tile(rt, p.num_slots, item / p.n_mod);
      const int k0 = c * KC, kcl = min(KC, p.in_dim - k0);
      if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(t.rank + t.nt) * kcl * sizeof(T));
      __syncwarp();
      const T* a = static_cast<const T*>(stream_module(p, item % p.n_mod).a) + ((int64_t)t.slot * p.R) * p.in_dim + k0;
      for (int n = lane; n < t.rank; n += 32)
        bulk_copy_g2s(stage_a(s) + n * KCP, a + (int64_t)n * p.in_dim, kcl * sizeof(T), &full[s]);
    };
    auto issue_x = [&](int f) {
      const int s = f % NS;
      const int item = cl + (f / cnt) * NCL, c = c_lo + f % cnt;
      const StreamTile t = stream_tile(rt, p.num_slots, item / p.n_mod);
      const int k0 = c * KC, kcl = min(KC, p.in_dim - k0);
      const T* x = static_cast<const T*>(p.x) + k0;
      for (int r = lane; r < t.nt; r += 32)
        bulk_copy_g2s(stage_x(s) + r * KCP, x + (int64_t)rt.tok[t.start + r] * p.x_stride, kcl * sizeof(T),
                      &full[s]);
    };
    const int pre = min(NS, total);
    for (int f = 0; f < pre; ++f) issue_a(f);  // weights: before the wait
    pdl_wait();                                 // x comes from earlier kernels
    for (int f = 0; f < pre; ++f) issue_x(f);
    for (int f = pre; f < total; ++f) {
      if (!mbar_wait(&empty[f % NS], ((f / NS) - 1) & 1, p.status)) break;
      issue_a(f);
      issue_x(f);
    }
  } else {
    // ---------------- consumers ----------------
    const int ctid = tid;  // 0 .. NC*32-1
    const int g = lane >> 2, cq = lane & 3;
    bool ok = true;
    int f = 0;
    uint32_t epoch = 0;
    if (XCHG) {  // partials go to peers tagged with this call's epoch
      pdl_wait();
      epoch = xchg_epoch(p.xchg);
    }
    const uint32_t recv0 = smem_addr(&s_recv[0][0][0][0]);
    for (int j = 0; j < my_items; ++j) {
      const int item = cl + j * NCL;
      const int m = item % p.n_mod;
      const int par = j & 1;
      const StreamTile t = stream_tile(rt, p.num_slots, item / p.n_mod);
      // Transposed tiles: the slot's rank rows are the MMA's M side (16 per
      // tile), the tile's tokens its N side. Inside a 16-feature step the lane
      // that owns MMA columns {2c, 2c+1, 2c+8, 2c+9} takes features 4c..4c+3
      // of both operands (the step's sum does not depend on the order), so
      // each operand is one 8-byte shared-memory load per row; two accumulator
      // chains take alternate steps. Rank rows past the rank (stale stage
      // rows) only reach partial columns >= rank, which are never written
      // out; token columns >= nt are zero.
      constexpr int MT = RM / 16;
      float acc0[MT][4], acc1[MT][4];
#pragma unroll
      for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc0[i][e] = acc1[i][e] = 0.f;
      const bool xv = g < t.nt;
      for (int c = 0; c < cnt; ++c, ++f) {
        const int s = f % NS;
        if (ok) ok = mbar_wait(&full[s], (f / NS) & 1, p.status);  // after a timeout: no more waits
        if (ok) {
          const int ksteps = min(KC, p.in_dim - (c_lo + c) * KC) / 16;
          const T* xl = reinterpret_cast<const T*>(s_dyn + s * SS::BYTES + SS::A_BYTES) + g * KCP + 4 * cq;
          const T* al = reinterpret_cast<const T*>(s_dyn + s * SS::BYTES) + g * KCP + 4 * cq;
          auto kstep = [&](int off, float (&acc)[MT][4]) {  // off = first feature of the step
            uint2 xb = make_uint2(0u, 0u);
            if (xv) xb = *reinterpret_cast<const uint2*>(xl + off);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              if (mt == 0 || mt * 16 < t.rank) {  // rank >= 1: the first rank tile always runs
                const uint2 lo = *reinterpret_cast<const uint2*>(al + mt * 16 * KCP + off);
                const uint2 hi = *reinterpret_cast<const uint2*>(al + (mt * 16 + 8) * KCP + off);
                mma_16816<T>(acc[mt], lo.x, hi.x, lo.y, hi.y, xb.x, xb.y);
              }
            }
          };
          for (int kk = warp; kk < ksteps; kk += 2 * NC) {
            kstep(kk * 16, acc0);
            if (kk + NC < ksteps) kstep((kk + NC) * 16, acc1);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // this CTA's partial: the warps' tiles summed in warp order ...
      // (D[rank row][token]: rows g and g + 8 of each rank tile, tokens 2c and 2c + 1)
#pragma unroll
      for (int u = 0; u < 2; ++u) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          s_red[warp][2 * cq + u][mt * 16 + g] = acc0[mt][u] + acc1[mt][u];
          s_red[warp][2 * cq + u][mt * 16 + 8 + g] = acc0[mt][2 + u] + acc1[mt][2 + u];
        }
      }
      named_barrier(1, NC * 32);
      // ... pushed into slot `crank` of CTA 0's receive buffer (once CTA 0 has
      // released that buffer from item j - 2)
      if (j >= 2 && crank != 0 && ok) ok = mbar_wait(&bar_free[par], ((j >> 1) - 1) & 1, p.status);
      {
        const uint32_t dst = cluster_map(recv0 + (uint32_t)((par * KS + crank) * TM * RM) * 4u, 0);
        const uint32_t bar = cluster_map(smem_addr(&bar_red[par]), 0);
        for (int e = ctid; e < TM * RM / 4; e += NC * 32) {
          const int r = e / (RM / 4), c4 = (e % (RM / 4)) * 4;
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int w = 0; w < NC; ++w) {
            const float4 u = *reinterpret_cast<const float4*>(&s_red[w][r][c4]);
            v.x += u.x;
            v.y += u.y;
            v.z += u.z;
            v.w += u.w;
          }
          st_async_v4(dst + (uint32_t)(r * RM + c4) * 4u, v.x, v.y, v.z, v.w, bar);
        }
      }
      named_barrier(1, NC * 32);  // s_red may be overwritten by the next item
      if (crank == 0) {
        // CTA 0: the KS partials in cluster order, one rounding to T, rows of this tile only
        if (ctid == 0) mbar_arrive_expect_tx(&bar_red[par], (uint32_t)KS * PB);
        if (ok) ok = mbar_wait(&bar_red[par], (j >> 1) & 1, p.status);
        if (ok) {
          for (int e = ctid; e < t.nt * t.rank; e += NC * 32) {
            const int r = e / t.rank, k = e - r * t.rank;
            float v = 0.f;
#pragma unroll
            for (int q = 0; q < KS; ++q) v += s_recv[par][q][r][k];
            const int row = rt.tok[t.start + r];
            if (XCHG) {  // this rank's partial value, tagged, into every rank's buffer (peer stores)
              if (row < p.xchg.rows) {
                const int64_t at = xchg_row(p.xchg, epoch, p.xchg.rank, row, p.R) + k;
                const unsigned long long w = ((unsigned long long)(epoch + 1u) << 32) | __float_as_uint(v);
#pragma unroll
                for (int q = 0; q < kMaxPeers; ++q)  // compile-time indices: no local copy of the arguments
                  if (q < p.xchg.tp) word_store_sys(p.xchg.recv[q] + at, w);
              }
              continue;
            }
            const int64_t at = (int64_t)row * p.mid_stride + m * p.R + k;
            if (p.mid_f32) static_cast<float*>(p.mid)[at] = v;  // a partial, summed across ranks later
            else static_cast<T*>(p.mid)[at] = Num<T>::from_f(v);
          }
        }
        named_barrier(1, NC * 32);  // done reading s_recv[par]
        if (ctid > 0 && ctid < KS) {  // release the buffer to the peers for item j + 2
          asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                           cluster_map(smem_addr(&bar_free[par]), (uint32_t)ctid))
                       : "memory");
        }
      }
    }
  }
  // no CTA leaves while a peer may still write into its shared memory
  cluster_arrive_release();
  cluster_wait_acquire();
}

// ---------------------------------------------------------------------------
// expand
// ---------------------------------------------------------------------------
template <typename T, int RM, bool XCHG>
__global__ void __launch_bounds__(kStreamThreads) lora_expand_stream_kernel(const StreamArgs p) {
  using ES = ExpandStage<RM>;
  constexpr int NC = kStreamConsumers, NS = kStreamStages;
  constexpr int OC = ES::OC, OCP = ES::OCP, MP = ES::MP;
  extern __shared__ __align__(128) unsigned char s_dyn[];
  __shared__ __align__(8) uint64_t full[NS], empty[NS];
  __shared__ int s_blocks[kMaxStreamModules + 1];  // prefix of OC blocks over the projections

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const StreamRouting rt = stream_routing(s_dyn + NS * ES::BYTES, p.num_slots);
  if (tid == 0) {
    int acc = 0;
    for (int m = 0; m < p.n_mod; ++m) {
      s_blocks[m] = acc;
      acc += (stream_module(p, m).out_dim + OC - 1) / OC;
    }
    s_blocks[p.n_mod] = acc;
  }
  stream_build_routing(p, rt, true);
  const int per_tile = s_blocks[p.n_mod];
  const int n_items = rt.toff[p.num_slots] * per_tile;
  const int G = gridDim.x;
  const int my_items = blockIdx.x < n_items ? (n_items - 1 - blockIdx.x) / G + 1 : 0;
  if (my_items == 0) {
    pdl_exit_early();  // as in the shrink: keep the call order
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NC);
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();
  constexpr bool xchg = XCHG;  // mid: the sum of every rank's partials, polled tile by tile

  struct Item {
    StreamTile t;
    StreamModule m;
    int mi, o0, ocl;
  };
  auto decode = [&](int j) {
    const int item = blockIdx.x + j * G;
    Item it;
    it.t = stream_tile(rt, p.num_slots, item / per_tile);
    const int r = item % per_tile;
    int m = 0;
    while (m + 1 < p.n_mod && s_blocks[m + 1] <= r) ++m;
    it.mi = m;
    it.m = stream_module(p, m);
    it.o0 = (r - s_blocks[m]) * OC;
    it.ocl = min(OC, it.m.out_dim - it.o0);
    return it;
  };
  auto stage_b = [&](int s) { return reinterpret_cast<T*>(s_dyn + s * ES::BYTES); };
  auto stage_y = [&](int s) { return reinterpret_cast<T*>(s_dyn + s * ES::BYTES + ES::B_BYTES); };
  auto stage_m = [&](int s) { return reinterpret_cast<T*>(s_dyn + s * ES::BYTES + ES::B_BYTES + ES::Y_BYTES); };
  const uint32_t mid_es = p.mid_f32 ? 4u : (uint32_t)sizeof(T);  // bytes per mid element

  if (warp == NC) {
    // ---------------- producer warp: lane 0 arms the stage, every lane issues copies ----------------
    auto issue_b = [&](int j) {
      const int s = j % NS;
      const Item it = decode(j);
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[s], (uint32_t)(it.ocl * p.R + it.t.nt * it.ocl) * sizeof(T) +
                                            (xchg ? 0u : (uint32_t)it.t.nt * p.R * mid_es));
        const T* b = static_cast<const T*>(it.m.b) + ((int64_t)it.t.slot * it.m.out_dim + it.o0) * p.R;
        bulk_copy_g2s(stage_b(s), b, (uint32_t)it.ocl * p.R * sizeof(T), &full[s]);
      }
      __syncwarp();
    };
    auto issue_ym = [&](int j) {
      const int s = j % NS;
      const Item it = decode(j);
      const T* y = static_cast<const T*>(it.m.y) + it.o0;
      const T* mid = static_cast<const T*>(p.mid) + it.mi * p.R;
      for (int r = lane; r < 2 * it.t.nt; r += 32) {
        const int t = r >> 1;
        const int64_t row = rt.tok[it.t.start + t];
        if ((r & 1) != 0 && xchg) continue;  // mid comes from the peers' partials, read by the consumers
        if ((r & 1) == 0) bulk_copy_g2s(stage_y(s) + t * OCP, y + row * it.m.y_stride, it.ocl * sizeof(T), &full[s]);
        else if (p.mid_f32)  // fp32 rows (MP floats apart in the stage)
          bulk_copy_g2s(reinterpret_cast<float*>(stage_m(s)) + t * MP,
                        static_cast<const float*>(p.mid) + row * p.mid_stride + it.mi * p.R, p.R * 4u, &full[s]);
        else bulk_copy_g2s(stage_m(s) + t * MP, mid + row * p.mid_stride, p.R * sizeof(T), &full[s]);
      }
    };
    const int pre = min(NS, my_items);
    for (int j = 0; j < pre; ++j) issue_b(j);  // adapter weights: before the wait
    pdl_wait();                                 // mid (shrink kernel) and y (base projection)
    for (int j = 0; j < pre; ++j) issue_ym(j);
    for (int j = pre; j < my_items; ++j) {
      if (!mbar_wait(&empty[j % NS], ((j / NS) - 1) & 1, p.status)) break;
      issue_b(j);
      issue_ym(j);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2, cq = lane & 3;
  const int brow = lane & 7, bhalf = (lane >> 3) & 1;
  bool ok = true;
  // exchange: thread 0 reads the call's epoch (after the wait: the previous
  // call has advanced it), takes this CTA's ticket in the call's count right
  // away (the atomic waits for the load; its result is used only at exit) and
  // hands the epoch to the consumers
  __shared__ uint32_t s_epoch;
  uint32_t ticket = 0u;
  if (xchg && tid == 0) {
    pdl_wait();
    s_epoch = load_epoch(p.xchg.ctr);
    ticket = xchg_ticket(p.xchg.ctr, s_epoch);
  }
  __shared__ int s_xfail;  // exchange: a lane's poll ran out (the item is skipped, stages still drained)
  if (tid == 0) s_xfail = 0;
  named_barrier(1, NC * 32);
  if (xchg) pdl_wait();  // (thread 0 waited already) mid and y come from earlier kernels
  const uint32_t epoch = xchg ? s_epoch : 0u;
  bool xgood = true;
  for (int j = 0; j < my_items; ++j) {
    const int s = j % NS;
    const Item it = decode(j);
    if (ok) ok = mbar_wait(&full[s], (j / NS) & 1, p.status);  // after a timeout: no more waits
    const int rank = it.t.rank, nt = it.t.nt;
    {
      // ok differs between threads only after a copy-wait timeout; every barrier below is reached by all
      const bool run = ok && xgood;
      const float scale = rt.scale[it.t.slot];
      // A operand: the tile's mid rows; columns >= rank (stale in the caller's buffer) are zeroed in registers
      uint32_t am[RM / 16][4];
      const int mrow = (lane & 15) < nt ? (lane & 15) : 0;
      const uint32_t ma = smem_addr(stage_m(s)) + (uint32_t)(mrow * MP + (lane >> 4) * 8) * 2u;
      const float* mf = reinterpret_cast<const float*>(stage_m(s)) + g * MP + 2 * cq;  // fp32 rows (mid_f32)
      const unsigned long long* xr = nullptr;  // exchange: this rank's buffer, row of token g (from rank 0)
      if (xchg && g < nt) {
        const int row = rt.tok[it.t.start + g];
        unsigned long long* own = p.xchg.recv[0];
#pragma unroll
        for (int q = 1; q < kMaxPeers; ++q)
          if (q == p.xchg.rank) own = p.xchg.recv[q];
        xr = row < p.xchg.rows ? own + xchg_row(p.xchg, epoch, 0, row, p.R) : nullptr;
      }
      const int64_t xq = (int64_t)p.xchg.rows * p.R;  // words between two ranks' partial rows
      const uint32_t tag = epoch + 1u;
      uint64_t t0 = 0;
      bool lane_ok = true;
#pragma unroll
      for (int kk = 0; kk < RM / 16; ++kk) {
        if (xchg) {  // mid = the ranks' partials (polled until tagged with this call) in rank order, rounded to T
          float2 v0 = make_float2(0.f, 0.f), v2 = v0;
          const int c0 = kk * 16 + 2 * cq;
          if (xr != nullptr && run) {
            for (int q = 0; q < p.xchg.tp && lane_ok; ++q) {
              float a, b;
              if (c0 < rank) {
                lane_ok = poll_pair(xr + q * xq + c0, tag, c0, rank, a, b, t0);
                v0.x += a;
                v0.y += b;
              }
              if (c0 + 8 < rank && lane_ok) {
                lane_ok = poll_pair(xr + q * xq + c0 + 8, tag, c0 + 8, rank, a, b, t0);
                v2.x += a;
                v2.y += b;
              }
            }
          }
          am[kk][0] = pack_round2<T>(v0.x, v0.y);
          am[kk][1] = 0u;
          am[kk][2] = pack_round2<T>(v2.x, v2.y);
          am[kk][3] = 0u;
        } else if (p.mid_f32) {  // fragment built from fp32 rows, each pair rounded to T (rows g < nt; g + 8 >= nt)
          float2 v0 = make_float2(0.f, 0.f), v2 = v0;
          if (g < nt) {
            v0 = *reinterpret_cast<const float2*>(mf + kk * 16);
            v2 = *reinterpret_cast<const float2*>(mf + kk * 16 + 8);
          }
          am[kk][0] = pack_round2<T>(v0.x, v0.y);
          am[kk][1] = 0u;
          am[kk][2] = pack_round2<T>(v2.x, v2.y);
          am[kk][3] = 0u;
        } else {
          ldsm_x4(ma + (uint32_t)kk * 32u, am[kk][0], am[kk][1], am[kk][2], am[kk][3]);
        }
        const int c0 = kk * 16 + 2 * cq, c1 = c0 + 8;
        const uint32_t m0 = (c0 < rank ? 0x0000ffffu : 0u) | (c0 + 1 < rank ? 0xffff0000u : 0u);
        const uint32_t m1 = (c1 < rank ? 0x0000ffffu : 0u) | (c1 + 1 < rank ? 0xffff0000u : 0u);
        am[kk][0] &= m0;
        am[kk][1] &= m0;
        am[kk][2] &= m1;
        am[kk][3] &= m1;
      }
      if (xchg) {  // every lane's partials arrived, or the item is skipped (and reported): all consumers vote
        if (!lane_ok) {
          s_xfail = 1;
          flag_error(p.status, kErrTimeout);
        }
        named_barrier(1, NC * 32);
        xgood = s_xfail == 0;
      }
      const bool compute = run && xgood;
      const int ksteps = (rank + 15) / 16;
      const uint32_t ba = smem_addr(stage_b(s));
      T* ys = stage_y(s);
      auto tile_mma = [&](int nb, float (&acc)[4]) {
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < RM / 16; ++kk) {
          if (kk < ksteps) {
            uint32_t b0, b1;
            ldsm_x2(ba + (uint32_t)((nb * 8 + brow) * p.R + kk * 16 + bhalf * 8) * 2u, b0, b1);
            // B columns >= rank (stale, or past the row when R % 16 == 8) contribute zero
            const int c0 = kk * 16 + 2 * cq, c1 = c0 + 8;
            b0 &= (c0 < rank ? 0x0000ffffu : 0u) | (c0 + 1 < rank ? 0xffff0000u : 0u);
            b1 &= (c1 < rank ? 0x0000ffffu : 0u) | (c1 + 1 < rank ? 0xffff0000u : 0u);
            mma_16816<T>(acc, am[kk][0], am[kk][1], am[kk][2], am[kk][3], b0, b1);
          }
        }
      };
      // y = T(T(scale * acc) + y): read from the staged tile, written straight
      // to the caller's row (token g of the tile), so the stage is free as soon
      // as this warp has computed
      T* const yg = static_cast<T*>(it.m.y) + (int64_t)rt.tok[it.t.start + (g < nt ? g : 0)] * it.m.y_stride + it.o0;
      auto tile_store = [&](int nb, const float (&acc)[4]) {
        if (g < nt) {
          const int o = nb * 8 + 2 * cq;
          const uint32_t u = *reinterpret_cast<const uint32_t*>(ys + g * OCP + o);
          const uint32_t d = pack_round2<T>(acc[0] * scale, acc[1] * scale);  // T(scaling * delta)
          *reinterpret_cast<uint32_t*>(yg + o) =
              pack_round2<T>(Pack2<T>::lo(d) + Pack2<T>::lo(u), Pack2<T>::hi(d) + Pack2<T>::hi(u));
        }
      };
      const int ntl = compute ? it.ocl / 8 : 0;  // nothing written for a skipped item
      if (rank % 16 == 0) {
        // Whole 16-column k-steps (every rank column is valid, no masks): the
        // loop is issue-bound, so its addresses advance by fixed strides with
        // no per-tile test. Two output tiles per iteration: independent
        // tensor-core chains overlap their latencies.
        const uint32_t tile_bytes = 8u * (uint32_t)p.R * sizeof(T);
        uint32_t bad = ba + (uint32_t)((warp * 8 + brow) * p.R + bhalf * 8) * 2u;
        const T* yl = ys + g * OCP + warp * 8 + 2 * cq;
        T* yo = yg + warp * 8 + 2 * cq;
        const bool lane_out = g < nt;
        auto mma_at = [&](uint32_t baddr, float (&acc)[4]) {
          acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
#pragma unroll
          for (int kk = 0; kk < RM / 16; ++kk) {
            if (RM == 16 || kk < ksteps) {  // rank >= 16 here: the first k-step always runs
              uint32_t b0, b1;
              ldsm_x2(baddr + (uint32_t)kk * 32u, b0, b1);
              mma_16816<T>(acc, am[kk][0], am[kk][1], am[kk][2], am[kk][3], b0, b1);
            }
          }
        };
        auto store_at = [&](T* y, const T* sy, const float (&acc)[4]) {  // y = T(T(scale * acc) + y)
          const uint32_t u = *reinterpret_cast<const uint32_t*>(sy);
          const uint32_t d = pack_round2<T>(acc[0] * scale, acc[1] * scale);
          *reinterpret_cast<uint32_t*>(y) =
              pack_round2<T>(Pack2<T>::lo(d) + Pack2<T>::lo(u), Pack2<T>::hi(d) + Pack2<T>::hi(u));
        };
        for (int nb = warp; nb < ntl; nb += 2 * NC) {
          float acc0[4], acc1[4];
          const bool two = nb + NC < ntl;
          mma_at(bad, acc0);
          if (two) mma_at(bad + NC * tile_bytes, acc1);
          if (lane_out) {
            store_at(yo, yl, acc0);
            if (two) store_at(yo + 8 * NC, yl + 8 * NC, acc1);
          }
          bad += 2 * NC * tile_bytes;
          yl += 16 * NC;
          yo += 16 * NC;
        }
      } else {
        // two output tiles per iteration: independent tensor-core chains overlap their latencies
        for (int nb = warp; nb < ntl; nb += 2 * NC) {
          float acc0[4], acc1[4];
          const bool two = nb + NC < ntl;
          tile_mma(nb, acc0);
          if (two) tile_mma(nb + NC, acc1);
          tile_store(nb, acc0);
          if (two) tile_store(nb + NC, acc1);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp has read the stage
  }
  if (xchg && tid == 0) xchg_advance(p.xchg.ctr, ticket, (uint32_t)min(G, n_items));
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

int stream_sm_count() {
  static int n = [] {
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
bool ensure_smem(K kern, int bytes, int& set, std::mutex& mu) {
  std::lock_guard<std::mutex> lock(mu);
  if (bytes <= set) return true;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  set = bytes;
  return true;
}

template <typename T, int RM, bool XCHG>
cudaError_t launch_stream_rmx(const StreamArgs& a, cudaStream_t st, bool pdl) {
  static std::mutex mu;
  static int set_s = 0, set_e = 0;
  const int route = align128(stream_routing_bytes(a.num_slots, a.S));
  const int smem_s = kStreamShrinkStages * ShrinkStage<RM>::BYTES + route;
  const int smem_e = kStreamStages * ExpandStage<RM>::BYTES + route;
  auto ks = lora_shrink_stream_kernel<T, RM, XCHG>;
  auto ke = lora_expand_stream_kernel<T, RM, XCHG>;
  if (!ensure_smem(ks, smem_s, set_s, mu) || !ensure_smem(ke, smem_e, set_e, mu)) return cudaErrorNotSupported;
  const dim3 grid(stream_sm_count());
  if (a.phase == 2)  // expand only: mid comes from the caller (e.g. all-reduced shrink partials)
    return launch_kernel(ke, grid, dim3(kStreamThreads), smem_e, st, pdl, a);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(stream_sm_count() / kStreamShrinkSplit * kStreamShrinkSplit));
  cfg.blockDim = dim3(kStreamThreads);
  cfg.dynamicSmemBytes = smem_s;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kStreamShrinkSplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, ks, a);
  if (e != cudaSuccess || a.phase == 1) return e;
  // the expand kernel always follows with the programmatic attribute: its wait is the shrink -> expand edge
  return launch_kernel(ke, grid, dim3(kStreamThreads), smem_e, st, true, a);
}

template <typename T, int RM>
cudaError_t launch_stream_rm(const StreamArgs& a, cudaStream_t st, bool pdl) {
  return a.xchg.tp > 0 ? launch_stream_rmx<T, RM, true>(a, st, pdl) : launch_stream_rmx<T, RM, false>(a, st, pdl);
}

}  // namespace

constexpr int kStreamMaxRoutingBytes = 48 * 1024;

// Returns cudaErrorNotSupported when the shape is outside this path (the caller
// then uses another one).
cudaError_t launch_apply_stream(const StreamArgs& a, int dtype, cudaStream_t st, bool pdl) {
  if (dtype != kBF16 && dtype != kF16) return cudaErrorNotSupported;
  if (a.n_mod < 1 || a.n_mod > kMaxStreamModules || a.R > 64 || a.R % 8 != 0 || (a.phase != 2 && a.in_dim % 16 != 0))
    return cudaErrorNotSupported;
  if (stream_routing_bytes(a.num_slots, a.S) > kStreamMaxRoutingBytes) return cudaErrorNotSupported;
  const int rm = a.R <= 16 ? 16 : a.R <= 32 ? 32 : 64;
  if (dtype == kBF16)
    return rm == 16 ? launch_stream_rm<__nv_bfloat16, 16>(a, st, pdl)
         : rm == 32 ? launch_stream_rm<__nv_bfloat16, 32>(a, st, pdl)
                    : launch_stream_rm<__nv_bfloat16, 64>(a, st, pdl);
  return rm == 16 ? launch_stream_rm<__half, 16>(a, st, pdl)
       : rm == 32 ? launch_stream_rm<__half, 32>(a, st, pdl)
                  : launch_stream_rm<__half, 64>(a, st, pdl);
}

}  // namespace mlora
