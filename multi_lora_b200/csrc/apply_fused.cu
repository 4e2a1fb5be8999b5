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
//   1. owns k-slice j of the input dim: its threads copy A[slot, :rank, slice]
//      into padded shared-memory rows with 16-byte cp.async pieces, and one
//      thread copies its output block B[slot, block, :rank] with one TMA bulk
//      copy (an mbarrier counts the bytes), BEFORE griddepcontrol.wait, so
//      under programmatic dependent launch the weight stream overlaps the
//      previous kernel;
//   2. after the wait it loads the slot's x rows (its slice) and y rows (its
//      output block) and computes split-K partials of mid with warp-level
//      tensor-core tiles (mma.sync m16n8k16: up to 8 tokens per tile cost the
//      same as one, where a scalar loop would grow with the token count);
//   3. pushes its partials into every peer CTA's shared memory with st.async
//      (distributed shared memory; each receiver's mbarrier counts the bytes),
//      so no cluster-wide barrier sits on the critical path; each CTA sums the
//      CS partials in a fixed order (deterministic) and rounds to T once, as
//      the reference stores mid in x's dtype;
//   4. computes the delta of its output block with the same tensor-core tiles
//      (A operand = mid rounded to T, exactly what the reference multiplies)
//      and adds it, scaled, into y.
// Each slot's A and B are read from HBM exactly once per launch. No global
// scratch, no atomics. Every wait is bounded (status bit on timeout).
//
// Row-parallel instance (XCHG, tensor parallelism with the partials summed
// over peer memory, xchg.cuh): between steps 3 and 4 the cluster's fp32
// partial of mid (this rank's share of the input dim) goes to every rank's
// receive buffer as tagged words, split over the cluster's CTAs by
// destination; then every CTA polls its tile's words from all ranks in its
// own buffer, sums them in rank order and rounds to T once. One CTA per
// cluster reads the rank's epoch, hands it to the cluster with its first
// partial push and takes the cluster's ticket; the holder of the last ticket
// advances the epoch as it exits. A CTA
// that waits on a peer's CTAs must not wait behind a wave of its own grid,
// so this instance launches only when the grid fits in one wave.
#include <cooperative_groups.h>

#include <map>
#include <mutex>
#include <cstdlib>
#include <utility>

#include "common.cuh"
#include "kernels.h"
#include "mma.cuh"
#include "tma.cuh"
#include "xchg.cuh"

namespace cg = cooperative_groups;

namespace mlora {

constexpr int kFusedNT = 256;
constexpr int kFusedTT = 6;       // tokens per tile (6: a q/k/v CTA fits 4 per SM; 7+ tokens in a slot are rare in decode)
constexpr int kFusedScan = 256;   // segment indices scanned per pass

// Segment list of one slot for up to kFusedScan scanned segment indices.
struct FusedSegs {
  int start[kFusedScan];
  int cum[kFusedScan + 1];
  int n;
};

// Warp 0 scans segment indices [from, min(bs, from + kFusedScan)) with every
// load of the pass issued up front (one memory round trip). With `rows`, the
// token rows of the pass's first kFusedTT tokens are written there too.
__device__ __forceinline__ void fused_scan(FusedSegs& sl, int slot, int from, const FusedArgs& p,
                                           int* rows = nullptr) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  constexpr int NB = kFusedScan / 32;
  const int nbv = min(NB, (p.bs - from + 31) / 32);  // batches that hold segments (warp-uniform)
  int w[NB], st[NB], en[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    const int idx = from + b * 32 + lane;
    w[b] = -1;
    st[b] = en[b] = 0;
    if (b < nbv && idx < p.bs) {
      w[b] = __ldg(p.weight_indices + idx);
      st[b] = __ldg(p.seg_indptr + idx);
      en[b] = __ldg(p.seg_indptr + idx + 1);
    }
  }
  int n = 0, total = 0;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    if (b >= nbv) break;
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
      const int q0 = total + incl - len;  // the segment's first token within the slot
      sl.start[pos] = st[b];
      sl.cum[pos] = q0;
      if (rows != nullptr)
        for (int q = q0; q < q0 + len && q < kFusedTT; ++q) rows[q] = st[b] + (q - q0);
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

// Walks the flat indices start, start + step, ... of a [rows][cols] space
// as (r, c) pairs with two divisions in all instead of one per step.
struct FlatWalk {
  int r, c, dr, dc, cols;
  __device__ __forceinline__ FlatWalk(int start, int step, int cols_) : cols(cols_) {
    r = start / cols;
    c = start - r * cols;
    dr = step / cols;
    dc = step - dr * cols;
  }
  __device__ __forceinline__ void next() {
    r += dr;
    c += dc;
    if (c >= cols) {
      c -= cols;
      ++r;
    }
  }
};

// Shared-memory row stride (elements) for a row of `k` elements that
// ldmatrix reads conflict-free: an odd number of 16-byte units.
__host__ __device__ __forceinline__ int padded_row(int k) { return ((k / 8) % 2 == 0) ? k + 8 : k; }

// The exchange's fields, copied from the kernel parameters into the first
// kXchgSmem bytes of dynamic shared memory when the CTA starts: the gather
// then reads them without a constant-cache miss on its critical path.
struct XchgShared {
  unsigned long long* recv[kMaxPeers];
  uint32_t* ctr;
  int tp, rank, rows;
};
constexpr int kXchgSmem = 128;
static_assert(sizeof(XchgShared) <= kXchgSmem, "exchange fields");

// Row-parallel gather of one tile (the XCHG instance): with the shrink on
// (phases 0 and 1) this rank's partial -- the cluster's cs partials summed in
// CTA order -- is published to every rank as tagged words, the destinations
// split over the cluster's CTAs (phase 0 keeps its own value in registers
// instead of storing it to itself); with the expand on (phases 0 and 2) mid =
// every rank's partial summed in rank order from 0.f (the same on every rank,
// as an all-reduce gives), rounded to T once. A partial that does not arrive
// within the wait limit sets `s_xfail` and the timeout bit; the caller then
// skips the expand.
template <typename T, int RM>
__device__ __forceinline__ void xchg_gather(const XchgShared& xg, int R, uint32_t* status, bool shrink_on,
                                            bool expand_on, uint32_t epoch, int cs, int j, int nt, int rank,
                                            const float* s_recv, const int* s_rows, T (*s_mid)[RM + 8],
                                            int& s_xfail) {
  constexpr int NT = kFusedNT, TT = kFusedTT;
  static_assert(TT * RM <= 2 * NT, "two gather elements per thread");
  const int tid = threadIdx.x;
  const int tp = xg.tp, me = xg.rank, rows = xg.rows;
  float loc[2] = {0.f, 0.f};
  if (shrink_on) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int e = tid + i * NT;
      const int t = e / RM, k = e - t * RM;
      if (e < TT * RM && t < nt && k < rank) {
        float v = 0.f;
        for (int q = 0; q < cs; ++q) v += s_recv[((size_t)q * TT + t) * RM + k];
        loc[i] = v;
        const int row = s_rows[t];
        if (row < rows) {
          const int64_t at = xchg_offset(epoch, tp, rows, me, row, R) + k;
          const unsigned long long w = tagged_word(epoch, v);
          for (int q = j; q < tp; q += cs)  // this CTA's destinations
            if (q != me || !expand_on) word_store_sys(xg.recv[q] + at, w);
        }
      }
    }
  }
  if (!expand_on) return;
  const uint32_t tag = epoch + 1u;
  const unsigned long long* own = xg.recv[me];
  const int64_t xq = (int64_t)rows * R;  // words between two ranks' partial rows
  const bool skip = *reinterpret_cast<volatile int*>(&s_xfail) != 0;
  bool good = true;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int e = tid + i * NT;
    if (e < TT * RM) {
      const int t = e / RM, k = e - t * RM;
      float v = 0.f;
      if (t < nt && k < rank && !skip && s_rows[t] < rows) {
        const unsigned long long* base = own + xchg_offset(epoch, tp, rows, 0, s_rows[t], R) + k;
        unsigned long long wv[kMaxPeers];
#pragma unroll
        for (int q = 0; q < kMaxPeers; ++q) {  // every load issued before the first poll
          wv[q] = 0ull;
          if (q < tp && (q != me || !shrink_on)) wv[q] = word_load(base + q * xq);
        }
#pragma unroll
        for (int q = 0; q < kMaxPeers; ++q) {
          if (q < tp) {
            float pq = loc[i];
            if (q != me || !shrink_on) {
              unsigned long long a = wv[q];
              if ((uint32_t)(a >> 32) != tag && good) {  // not there yet: wait (bounded), out of line
                a = poll_until(base + q * xq, tag);
                good = (uint32_t)(a >> 32) == tag;
              }
              pq = __uint_as_float((uint32_t)a);
            }
            v += pq;
          }
        }
      }
      s_mid[t][k] = Num<T>::from_f(v);
    }
  }
  if (!good) {
    s_xfail = 1;
    flag_error(status, kErrTimeout);
  }
}

// RM: rank columns covered by the tiles (16, 32 or 64; >= R). Register caps
// (48 / 64 / 85) keep 5 / 4 / 3 CTAs per SM resident, without spills; fewer
// registers measured faster at RM 16 (the decode shapes are latency-bound).
// The exchange instance at RM 16 needs 64 (4 CTAs per SM) to stay unspilled.
template <typename T, int RM, bool XCHG>
__global__ void __launch_bounds__(kFusedNT, RM == 16 ? (XCHG ? 4 : 5) : RM == 32 ? 4 : 3)
    apply_fused_kernel(const FusedArgs p) {
  constexpr int NT = kFusedNT;
  constexpr int NW = NT / 32;
  constexpr int TT = kFusedTT;    // tokens per tile (the shrink's MMA N; the expand's M rows TT..15 are zero)
  constexpr int Q4 = RM / 4;      // 16-byte pieces per partial row
  constexpr int MP = RM + 8;      // padded row of the bf16/f16 mid tile
  __shared__ FusedSegs sl;
  __shared__ int s_rows[TT];
  __shared__ __align__(16) T s_mid[16][MP];
  __shared__ __align__(8) uint64_t bar_w, bar_p;
  extern __shared__ __align__(128) unsigned char s_dyn[];

  cg::cluster_group cluster = cg::this_cluster();
  const int cs = (int)cluster.num_blocks();
  const int j = (int)cluster.block_rank();
  const int slot = blockIdx.y;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int R = p.R;
  FusedModule m = p.mod[0];
#pragma unroll
  for (int i = 1; i < kMaxFusedModules; ++i)
    if (i == (int)blockIdx.z) m = p.mod[i];

  // one memory round trip: warp 0 scans the routing while warp 1 reads rank and scaling
  __shared__ int s_rank;
  __shared__ float s_scale;
  if (tid == 32) {
    s_rank = __ldg(p.lora_ranks + slot);
    switch (p.scalings_dtype) {
      case kBF16: s_scale = __bfloat162float(__ldg(static_cast<const __nv_bfloat16*>(p.scalings) + slot)); break;
      case kF16: s_scale = __half2float(__ldg(static_cast<const __half*>(p.scalings) + slot)); break;
      default: s_scale = __ldg(static_cast<const float*>(p.scalings) + slot); break;
    }
  }
  XchgShared& sx = *reinterpret_cast<XchgShared*>(s_dyn);  // XCHG only
  if (XCHG && tid >= 64 && tid < 64 + kMaxPeers) {  // warp 2 is idle during the scan
    const int q = tid - 64;
    unsigned long long* r = p.xchg.recv[0];
#pragma unroll
    for (int i = 1; i < kMaxPeers; ++i)
      if (q == i) r = p.xchg.recv[i];
    sx.recv[q] = r;
  }
  if (XCHG && tid == 64 + kMaxPeers) {
    sx.ctr = p.xchg.ctr;
    sx.tp = p.xchg.tp;
    sx.rank = p.xchg.rank;
    sx.rows = p.xchg.rows;
  }
  fused_scan(sl, slot, 0, p, s_rows);  // also the first tile's token rows
  __syncthreads();
  int rank = s_rank;
  const float scale = s_scale;
  if (rank < 0 || rank > R) {
    if (j == 0 && tid == 0 && blockIdx.z == 0) flag_error(p.status, kErrRankRange);
    rank = rank < 0 ? 0 : R;
  }
  // base model (rank 0: no delta, mid untouched) or a slot this batch does not
  // use: the whole cluster leaves (uniform per cluster)
  if (rank == 0 || (sl.n == 0 && p.bs <= kFusedScan)) {
    if (XCHG && p.phase != 1) {
      pdl_trigger();
      if (j == 0 && tid == 0) {  // the cluster's ticket
        pdl_wait();  // the previous call has finished counting
        xchg_advance(sx.ctr, xchg_ticket(sx.ctr, load_epoch(sx.ctr)), gridDim.y * gridDim.z);
      }
    } else {
      pdl_exit_early();
    }
    return;
  }
  // row-parallel phases: 1 publishes this rank's partial and stops, 2 skips the
  // shrink (every rank's partial, this one's included, comes from the buffer)
  const bool shrink_on = !XCHG || p.phase != 2;
  const bool expand_on = !XCHG || p.phase != 1;

  // shared memory: (XCHG) fields [kXchgSmem bytes] | A [R][kp] | B [ob_max][R] | x [TT][kp] | y [TT][ob_max] |
  //                warp partials [NW][TT][RM] f32 | partials in [cs][TT][RM] f32 |
  //                (XCHG) the epoch, 16 bytes
  const int kp = padded_row(p.ks);
  const int k0 = j * p.ks;                       // multiple of 16
  const int kend = min(p.in_dim, k0 + p.ks);
  const int klen = kend > k0 ? kend - k0 : 0;    // multiple of 8
  const int ksteps = (klen + 15) / 16;
  const int o_lo = min(m.out_dim, j * m.ob);
  const int o_hi = min(m.out_dim, o_lo + m.ob);
  const int olen = o_hi - o_lo;
  T* s_a = reinterpret_cast<T*>(s_dyn + (XCHG ? kXchgSmem : 0));
  T* s_b = s_a + (size_t)R * kp;
  T* s_x = s_b + (size_t)p.ob_max * R;
  T* s_y = s_x + (size_t)TT * kp;
  float* s_wred = reinterpret_cast<float*>(s_y + (size_t)TT * p.ob_max);
  float* s_recv = s_wred + (size_t)NW * TT * RM;

  // ---- prologue: adapter weights (stable for the step) into shared memory ----
  if (tid == 0) {
    mbar_init(&bar_w, 1);
    mbar_init(&bar_p, 1);
    fence_barrier_init();
  }
  for (int e = tid; e < 16 * MP; e += NT) (&s_mid[0][0])[e] = Num<T>::from_f(0.f);
  __shared__ int s_xfail;  // XCHG: a peer's partial never arrived (sticky: later tiles skip too)
  if (XCHG && tid == 0) s_xfail = 0;
  if (klen % 16 != 0)  // half k-step at the slice end: zero the 8 pad columns of the rank rows
    for (int e = tid; e < rank * 8; e += NT) s_a[(size_t)(e / 8) * kp + klen + (e % 8)] = Num<T>::from_f(0.f);
  __syncthreads();
  cluster_arrive_release();  // this CTA runs and its barriers exist; peers wait before pushing to it
  const T* __restrict__ a_src = static_cast<const T*>(m.a) + (int64_t)slot * R * p.in_dim + k0;
  const T* __restrict__ b_src = static_cast<const T*>(m.b) + ((int64_t)slot * m.out_dim + o_lo) * R;
  const bool b_dense = rank == R;  // B rows hold exactly the rank: one contiguous block
  // Weights: the contiguous B block as ONE bulk copy (rank == max_rank); the
  // A rows (and a B block with stale columns) as 16-byte cp.async pieces over
  // every thread -- a 1-D bulk copy costs ~80-100 ns of issue time, so one
  // thread issuing a copy per A row put ~1.5 us on the critical path.
  if (tid == 0) {
    const uint32_t b_bytes = b_dense && expand_on ? (uint32_t)olen * R * sizeof(T) : 0u;
    mbar_arrive_expect_tx(&bar_w, b_bytes);
    if (b_bytes > 0) bulk_copy_g2s(s_b, b_src, b_bytes, &bar_w);
  }
  if (klen > 0 && shrink_on)
    for (FlatWalk w(tid, NT, klen / 8); w.r < rank; w.next())
      cp_async16(s_a + (size_t)w.r * kp + w.c * 8, a_src + (int64_t)w.r * p.in_dim + w.c * 8);
  const int rc = (rank + 7) / 8;  // 16-byte B chunks per row that hold rank columns
  if (!b_dense && expand_on) {  // rows of R with only `rank` valid columns: 16-byte copies per thread
    for (int e = tid; e < olen * rc; e += NT) {
      const int row = e / rc, c = e - row * rc;
      cp_async16(s_b + (size_t)row * R + c * 8, b_src + (int64_t)row * R + c * 8);
    }
  }
  cp_async_commit();  // group: this CTA's weights
  pdl_trigger();
  pdl_wait();  // x and y come from earlier kernels
  // The call's epoch: thread 0 of the cluster's CTA 0 reads it (after the
  // wait: the previous call has advanced it) and hands it to the cluster in
  // its first partial push, so the call counts one ticket per cluster.
  const uint32_t eg = XCHG && j == 0 && tid == 0 ? load_epoch(sx.ctr) : 0u;
  uint32_t ticket = 0u;  // the cluster's ticket, taken with the first push

  const T* __restrict__ xbase = static_cast<const T*>(p.x);
  T* __restrict__ ybase = static_cast<T*>(m.y);
  const uint32_t sb_addr = smem_addr(s_b);
  const uint32_t smid_addr = smem_addr(&s_mid[0][0]);
  const int g = lane >> 2, cq = lane & 3;
  bool ok = true;
  uint32_t p_phase = 0;
  bool first = true;
  bool b_pending = true;  // bar_w (the dense B block) not yet waited on
  for (int from = 0; from < p.bs; from += kFusedScan) {
    if (from > 0) {
      __syncthreads();
      fused_scan(sl, slot, from, p);
      __syncthreads();
    }
    const int ntok = sl.cum[sl.n];
    for (int q0 = 0; q0 < ntok; q0 += TT) {
      const int nt = min(TT, ntok - q0);
      const bool scanned_rows = from == 0 && q0 == 0;  // written by the first scan (barrier passed)
      if (!scanned_rows && tid < nt) s_rows[tid] = fused_token_row(sl, q0 + tid);
      if (klen % 16 != 0)  // pad columns: disjoint from the x rows loaded below
        for (int e = tid; e < TT * 8; e += NT) s_x[(size_t)(e / 8) * kp + klen + (e % 8)] = Num<T>::from_f(0.f);
      if (!scanned_rows) __syncthreads();
      if (m.y_tma && olen > 0 && expand_on) {  // this tile's y rows (output block), needed only by the expand
        for (FlatWalk w(tid, NT, olen / 8); w.r < nt; w.next())
          cp_async16(s_y + (size_t)w.r * p.ob_max + w.c * 8,
                     ybase + (int64_t)s_rows[w.r] * m.y_stride + o_lo + w.c * 8);
      }
      cp_async_commit();  // group: this tile's y rows (possibly empty)
      {  // this tile's x rows (k-slice): plain 16-byte loads by every thread (L2 hits)
        if (klen > 0 && shrink_on)
          for (FlatWalk w(tid, NT, klen / 8); w.r < nt; w.next()) {
            const uint4 v =
                __ldcg(reinterpret_cast<const uint4*>(xbase + (int64_t)s_rows[w.r] * p.x_stride + k0) + w.c);
            *reinterpret_cast<uint4*>(s_x + (size_t)w.r * kp + w.c * 8) = v;
          }
      }
      if (first) cp_async_wait<1>();  // the weights group (this tile's y group may still be in flight)
      __syncthreads();  // x tile and A rows complete
      if (first && !b_dense) {  // B rows (cp.async, landed): zero the stale columns past the rank
        for (int e = tid; e < olen * (R - rank); e += NT) {
          const int row = e / (R - rank), c = rank + e % (R - rank);
          s_b[(size_t)row * R + c] = Num<T>::from_f(0.f);
        }
      }

      // ---- shrink: split-K partials of this CTA's slice on tensor cores ----
      // Transposed tiles: the slot's rank rows are the MMA's M side (16 per
      // tile), the tile's tokens its N side. Within a 16-feature step the lane
      // that owns MMA columns {2c, 2c+1, 2c+8, 2c+9} takes features 4c..4c+3
      // of both operands (the sum over the step does not depend on the order),
      // so every operand is one 8-byte shared-memory load per row. Rank rows
      // past the rank (stale or unset shared memory) only reach partial
      // columns >= rank, which the gather drops; token columns >= nt are zero.
      {
        constexpr int MT = RM / 16;
        float acc0[MT][4], acc1[MT][4];
#pragma unroll
        for (int i = 0; i < MT; ++i)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc0[i][e] = acc1[i][e] = 0.f;
        const bool xv = g < nt;
        // per-lane rows: token g of x, rank rows g and g + 8 of each rank tile
        const T* const xl = s_x + (size_t)g * kp + 4 * cq;
        const T* const al = s_a + (size_t)g * kp + 4 * cq;
        auto kstep = [&](int off, float (&acc)[MT][4]) {  // off = first feature of the step
          uint2 xb = make_uint2(0u, 0u);
          if (xv) xb = *reinterpret_cast<const uint2*>(xl + off);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            if (mt == 0 || mt * 16 < rank) {  // rank >= 1: the first rank tile always runs
              const uint2 lo = *reinterpret_cast<const uint2*>(al + (size_t)(mt * 16) * kp + off);
              const uint2 hi = *reinterpret_cast<const uint2*>(al + (size_t)(mt * 16 + 8) * kp + off);
              mma_16816<T>(acc[mt], lo.x, hi.x, lo.y, hi.y, xb.x, xb.y);
            }
          }
        };
        if (ok && shrink_on) {
          // two accumulator chains (alternate steps) halve the dependent MMA chain
          for (int kk = warp; kk < ksteps; kk += 2 * NW) {
            kstep(kk * 16, acc0);
            if (kk + NW < ksteps) kstep((kk + NW) * 16, acc1);
          }
        }
        // D[rank row][token]: rows g and g + 8 of each rank tile, tokens 2c and 2c + 1
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int t = 2 * cq + u;
          if (t < nt) {
            float* wr = s_wred + ((size_t)warp * TT + t) * RM;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              wr[mt * 16 + g] = acc0[mt][u] + acc1[mt][u];
              wr[mt * 16 + 8 + g] = acc0[mt][2 + u] + acc1[mt][2 + u];
            }
          }
        }
      }
      __syncthreads();  // warp partials complete
      const bool epoch_push = XCHG && first;  // the first push carries the epoch
      if (first) cluster_wait_acquire();  // every peer runs and has its barriers initialised
      first = false;
      if (XCHG && epoch_push && j == 0 && tid == 0 && p.phase != 1)
        ticket = xchg_ticket(sx.ctr, eg);  // the epoch load has long returned
      // ---- push this CTA's partial (its warps' partials summed in warp order) into
      //      slot j of every peer's receive buffer (phase 2: zeros, for the epoch) ----
      {
        if (tid == 0)
          mbar_arrive_expect_tx(&bar_p, (uint32_t)cs * nt * RM * sizeof(float) + (epoch_push ? 16u : 0u));
        if (epoch_push && j == 0 && tid == 0) {  // the epoch, into every CTA's slot after the partials
          const uint32_t dst = smem_addr(s_recv + (size_t)cs * TT * RM);
          const uint32_t bar = smem_addr(&bar_p);
          for (int q = 0; q < cs; ++q)
            st_async_v4(cluster_map(dst, (uint32_t)q), __uint_as_float(eg), 0.f, 0.f, 0.f,
                        cluster_map(bar, (uint32_t)q));
        }
        if (tid < nt * Q4) {
          const int t = tid / Q4, k4 = (tid - t * Q4) * 4;
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int w = 0; w < NW; ++w) {
            const float4 u = *reinterpret_cast<const float4*>(s_wred + ((size_t)w * TT + t) * RM + k4);
            v.x += u.x;
            v.y += u.y;
            v.z += u.z;
            v.w += u.w;
          }
          const uint32_t dst = smem_addr(s_recv + ((size_t)j * TT + t) * RM + k4);
          const uint32_t bar = smem_addr(&bar_p);
          for (int q = 0; q < cs; ++q)
            st_async_v4(cluster_map(dst, (uint32_t)q), v.x, v.y, v.z, v.w, cluster_map(bar, (uint32_t)q));
        }
        ok = mbar_wait(&bar_p, p_phase, p.status) && ok;
        p_phase ^= 1u;
      }
      if constexpr (XCHG) {
        const uint32_t epoch = __float_as_uint(s_recv[(size_t)cs * TT * RM]);
        xchg_gather<T, RM>(sx, R, p.status, shrink_on, expand_on, epoch, cs, j, nt, rank, s_recv, s_rows, s_mid,
                           s_xfail);
      } else {
        // ---- gather: mid = sum of the cs partials in CTA order, rounded to T once ----
        for (int e = tid; e < TT * RM; e += NT) {
          const int t = e / RM, k = e - t * RM;
          float v = 0.f;
          if (t < nt && k < rank) {
            for (int q = 0; q < cs; ++q) v += s_recv[((size_t)q * TT + t) * RM + k];
            if (j == 0 && m.mid != nullptr)
              static_cast<T*>(m.mid)[(int64_t)s_rows[t] * m.mid_stride + k] = Num<T>::from_f(v);
          }
          s_mid[t][k] = Num<T>::from_f(v);
        }
      }
      if (b_pending) {  // the dense B block, needed from here on, landed during the shrink
        ok = mbar_wait(&bar_w, 0, p.status) && ok;
        b_pending = false;
      }
      if (m.y_tma && olen > 0) cp_async_wait<0>();  // y rows staged during the shrink and exchange
      __syncthreads();  // s_mid, B and the staged y rows complete
      // ---- expand: this CTA's output block on tensor cores, fused scaling + residual ----
      if (ok && expand_on && (!XCHG || s_xfail == 0)) {
        uint32_t am[RM / 16][4];
#pragma unroll
        for (int kk = 0; kk < RM / 16; ++kk)
          ldsm_x4(smid_addr + (uint32_t)((lane & 15) * MP + kk * 16 + (lane >> 4) * 8) * 2u, am[kk][0], am[kk][1],
                  am[kk][2], am[kk][3]);
        const int brow = lane & 7, bhalf = (lane >> 3) & 1;
        const int ntiles = (olen + 7) / 8;
        const int ksteps_r = (rank + 15) / 16;
        auto tile_mma = [&](int nb, float (&acc)[4]) {
          acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
#pragma unroll
          for (int kk = 0; kk < RM / 16; ++kk) {
            if (kk < ksteps_r) {
              uint32_t b0, b1 = 0u;
              if (kk * 16 + 16 <= R) {
                ldsm_x2(sb_addr + (uint32_t)((nb * 8 + brow) * R + kk * 16 + bhalf * 8) * 2u, b0, b1);
              } else {  // R % 16 == 8: only the first 8 columns of this k-step exist in a B row
                ldsm_x1(sb_addr + (uint32_t)((nb * 8 + brow) * R + kk * 16) * 2u, b0);
              }
              mma_16816<T>(acc, am[kk][0], am[kk][1], am[kk][2], am[kk][3], b0, b1);
            }
          }
        };
        // per-lane rows (token g of the tile), hoisted out of the tile loop
        T* const yrow = ybase + (int64_t)(g < nt ? s_rows[g] : 0) * m.y_stride + o_lo;
        const T* const syrow = s_y + (size_t)g * p.ob_max;
        const bool vec = m.y_tma != 0;
        auto tile_store = [&](int nb, const float (&acc)[4]) {
          if (g < nt) {  // row g of the tile: outputs ol, ol + 1 of the block
            const int ol = nb * 8 + 2 * cq;
            const uint32_t d = pack_round2<T>(acc[0] * scale, acc[1] * scale);  // T(scaling * delta)
            if (vec && ol + 1 < olen) {
              const uint32_t u = *reinterpret_cast<const uint32_t*>(syrow + ol);
              *reinterpret_cast<uint32_t*>(yrow + ol) =
                  pack_round2<T>(Pack2<T>::lo(d) + Pack2<T>::lo(u), Pack2<T>::hi(d) + Pack2<T>::hi(u));
            } else {
              if (ol < olen) yrow[ol] = Num<T>::from_f(Pack2<T>::lo(d) + ldcg_f<T>(yrow + ol));
              if (ol + 1 < olen) yrow[ol + 1] = Num<T>::from_f(Pack2<T>::hi(d) + ldcg_f<T>(yrow + ol + 1));
            }
          }
        };
        if (vec && R % 16 == 0) {
          // Common shape (aligned y rows, 16-column k-steps): the loop is
          // issue-bound, so its addresses advance by fixed strides and no
          // per-tile bound or shape test is left in it. Two output tiles per
          // iteration: independent tensor-core chains overlap their latencies.
          const uint32_t tile_bytes = 8u * (uint32_t)R * sizeof(T);
          uint32_t ba = sb_addr + (uint32_t)((warp * 8 + brow) * R + bhalf * 8) * 2u;
          T* yp = yrow + warp * 8 + 2 * cq;
          const T* sp = syrow + warp * 8 + 2 * cq;
          const bool lane_out = g < nt;
          auto mma_at = [&](uint32_t baddr, float (&acc)[4]) {
            acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
#pragma unroll
            for (int kk = 0; kk < RM / 16; ++kk) {
              if (RM == 16 || kk < ksteps_r) {  // rank >= 1: the first k-step always runs
                uint32_t b0, b1;
                ldsm_x2(baddr + (uint32_t)kk * 32u, b0, b1);
                mma_16816<T>(acc, am[kk][0], am[kk][1], am[kk][2], am[kk][3], b0, b1);
              }
            }
          };
          auto store_at = [&](T* y, const T* sy, const float (&acc)[4]) {
            const uint32_t d = pack_round2<T>(acc[0] * scale, acc[1] * scale);  // T(scaling * delta)
            const uint32_t u = *reinterpret_cast<const uint32_t*>(sy);
            *reinterpret_cast<uint32_t*>(y) =
                pack_round2<T>(Pack2<T>::lo(d) + Pack2<T>::lo(u), Pack2<T>::hi(d) + Pack2<T>::hi(u));
          };
          for (int nb = warp; nb < ntiles; nb += 2 * NW) {
            float acc0[4], acc1[4];
            const bool two = nb + NW < ntiles;
            mma_at(ba, acc0);
            if (two) mma_at(ba + NW * tile_bytes, acc1);
            if (lane_out) {
              store_at(yp, sp, acc0);
              if (two) store_at(yp + 8 * NW, sp + 8 * NW, acc1);
            }
            ba += 2 * NW * tile_bytes;
            yp += 16 * NW;
            sp += 16 * NW;
          }
        } else {
          for (int nb = warp; nb < ntiles; nb += 2 * NW) {
            float acc0[4], acc1[4];
            const bool two = nb + NW < ntiles;
            tile_mma(nb, acc0);
            if (two) tile_mma(nb + NW, acc1);
            tile_store(nb, acc0);
            if (two) tile_store(nb + NW, acc1);
          }
        }
      }
      const bool more = (q0 + TT < ntok) || (from + kFusedScan < p.bs);
      if (more) cluster.sync();  // peers finished reading s_recv before the next pushes
      else __syncthreads();
    }
  }
  // Never leave with copies in flight into this CTA's shared memory: weights
  // that no tile consumed (a slot with no tokens past the first scan pass),
  // or copies whose wait timed out, are drained here (bounded again).
  if (first) cluster_wait_acquire();  // pairs the prologue arrive
  if (b_pending) mbar_wait(&bar_w, 0, p.status);
  cp_async_wait<0>();
  if (!ok && tid == 0) mbar_wait(&bar_p, p_phase ^ 1u, p.status);  // ok is only cleared inside a tile
  if (XCHG && j == 0 && tid == 0 && p.phase != 1) {
    if (first) ticket = xchg_ticket(sx.ctr, load_epoch(sx.ctr));  // no tile of this slot in any scan pass
    xchg_advance(sx.ctr, ticket, gridDim.y * gridDim.z);
  }
}

namespace {

template <typename T, int RM, bool XCHG>
struct FusedLauncher {
  std::mutex mu;
  int smem_set = 0;
  bool nonportable_set = false;
  std::map<std::pair<int, int>, int> occ;  // (cs, smem KiB) -> resident CTAs per SM (0: cannot place)

  // Resident CTAs per SM for this shape (0 when a cluster of cs cannot be placed).
  int occupancy(int cs, size_t smem) {
    std::lock_guard<std::mutex> lock(mu);
    auto kern = apply_fused_kernel<T, RM, XCHG>;
    const int kib = (int)((smem + 1023) / 1024);
    auto key = std::make_pair(cs, kib);
    auto it = occ.find(key);
    if (it != occ.end()) return it->second;
    int result = 0;
    if (cs > 8 && !nonportable_set) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        (void)cudaGetLastError();
        return occ[key] = 0;
      }
      nonportable_set = true;
    }
    if (kib * 1024 > smem_set) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kib * 1024) != cudaSuccess) {
        (void)cudaGetLastError();
        return occ[key] = 0;
      }
      smem_set = kib * 1024;
    }
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
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &q) != cudaSuccess) {
      (void)cudaGetLastError();
      clusters = 0;
    }
    int per_sm = 0;
    if (clusters > 0 &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kFusedNT, (size_t)kib * 1024) != cudaSuccess) {
      (void)cudaGetLastError();
      per_sm = 0;
    }
    result = clusters > 0 ? (per_sm > 0 ? per_sm : 1) : 0;
    return occ[key] = result;
  }

  cudaError_t launch(const FusedArgs& a, int cs, size_t smem, cudaStream_t st, bool pdl) {
    auto kern = apply_fused_kernel<T, RM, XCHG>;
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
};

template <typename T, int RM, bool XCHG>
FusedLauncher<T, RM, XCHG>& launcher() {
  static FusedLauncher<T, RM, XCHG> l;
  return l;
}

size_t fused_smem(const FusedArgs& a, int rm, int ks, int ob_max, int cs) {
  const int kp = padded_row(ks);
  return (size_t)2 * ((size_t)a.R * kp + (size_t)ob_max * a.R + (size_t)kFusedTT * kp + (size_t)kFusedTT * ob_max) +
         (size_t)4 * ((size_t)(kFusedNT / 32) * kFusedTT * rm + (size_t)cs * kFusedTT * rm);
}

int sm_count() {
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

template <typename T, int RM, bool XCHG>
cudaError_t launch_rmx(FusedArgs a, cudaStream_t st, bool pdl) {
  auto& l = launcher<T, RM, XCHG>();
  // Cluster size: fewest waves of CTAs for the whole launch (every slot counted,
  // since which slots the batch uses is only known on the device); ties go to
  // the size closest to 8 (8, 16, 4, 2): on B200, clusters of 16 at the same
  // wave count measured slower (twice the CTAs and partial pushes per slot).
  int best_cs = 0, best_waves = 1 << 30;
  size_t best_smem = 0;
  FusedArgs best = a;
  static const int forced_cs = [] {
    const char* v = getenv("MLORA_FUSED_CLUSTER");  // tuning: force 2, 4, 8 or 16 CTAs per cluster
    const int c = v != nullptr ? atoi(v) : 0;
    return (c == 2 || c == 4 || c == 8 || c == 16) ? c : 0;
  }();
  for (int cs : {2, 4, 8, 16}) {
    if (forced_cs != 0 && cs != forced_cs) continue;
    FusedArgs c = a;
    const int ks = ((a.in_dim + cs - 1) / cs + 15) / 16 * 16;
    int ob_max = 8;
    for (int i = 0; i < c.n_mod; ++i) {
      FusedModule& m = c.mod[i];
      m.ob = ((m.out_dim + cs - 1) / cs + 7) / 8 * 8;
      ob_max = m.ob > ob_max ? m.ob : ob_max;
      m.y_tma = (reinterpret_cast<uintptr_t>(m.y) % 16 == 0) && (m.y_stride % 8 == 0) && (m.out_dim % 8 == 0);
    }
    const size_t smem = fused_smem(c, RM, ks, ob_max, cs) + (XCHG ? kXchgSmem + 16 : 0);  // + fields, epoch slot
    if (smem > 200 * 1024) continue;
    const int per_sm = l.occupancy(cs, smem);
    if (per_sm <= 0) continue;
    const long long ctas = (long long)c.n_mod * c.num_slots * cs;
    const int waves = (int)((ctas + (long long)sm_count() * per_sm - 1) / ((long long)sm_count() * per_sm));
    if (XCHG && waves > 1) continue;  // its CTAs wait on peers' CTAs: the whole grid must be resident
    auto pref = [](int c) { return c == 8 ? 0 : c == 16 ? 1 : c == 4 ? 2 : 3; };
    if (waves < best_waves || (waves == best_waves && pref(cs) < pref(best_cs))) {
      c.ks = ks;
      c.ob_max = ob_max;
      best = c;
      best_cs = cs;
      best_waves = waves;
      best_smem = smem;
    }
  }
  if (best_cs == 0) return cudaErrorNotSupported;
  return l.launch(best, best_cs, best_smem, st, pdl);
}

template <typename T, int RM>
cudaError_t launch_rm(const FusedArgs& a, cudaStream_t st, bool pdl) {
  return a.xchg.tp > 0 ? launch_rmx<T, RM, true>(a, st, pdl) : launch_rmx<T, RM, false>(a, st, pdl);
}

}  // namespace

// Returns cudaErrorNotSupported when the shape is outside the fused kernel's
// range (the caller then runs shrink and expand separately).
cudaError_t launch_apply_fused(FusedArgs a, int dtype, cudaStream_t st, bool pdl) {
  if (dtype != kBF16 && dtype != kF16) return cudaErrorNotSupported;
  if (a.n_mod < 1 || a.n_mod > kMaxFusedModules) return cudaErrorNotSupported;
  if (a.R > 64 || a.R % 8 != 0 || a.in_dim % 8 != 0) return cudaErrorNotSupported;
  if (a.xchg.tp > 0 && (a.n_mod != 1 || a.phase < 0 || a.phase > 2)) return cudaErrorNotSupported;
  const int rm = a.R <= 16 ? 16 : a.R <= 32 ? 32 : 64;
  if (dtype == kBF16)
    return rm == 16 ? launch_rm<__nv_bfloat16, 16>(a, st, pdl)
         : rm == 32 ? launch_rm<__nv_bfloat16, 32>(a, st, pdl)
                    : launch_rm<__nv_bfloat16, 64>(a, st, pdl);
  return rm == 16 ? launch_rm<__half, 16>(a, st, pdl)
       : rm == 32 ? launch_rm<__half, 32>(a, st, pdl)
                  : launch_rm<__half, 64>(a, st, pdl);
}

}  // namespace mlora
