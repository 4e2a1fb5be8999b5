// Slot-grouped routing inside one CTA.
//
// The reference walks segments one by one (backend/torch_backend.py:38-49,
// kernels/sgemm_lora_a.py:250-262: one program per segment). Here one CTA owns
// one adapter slot and gathers every segment that routes to it, so the
// slot's weights are read from HBM once per launch however many segments
// share the adapter. Segment boundaries come from seg_indptr exactly as in
// torch_backend.py:38-41 ([indptr[i], indptr[i+1]), empty segments skipped).
#pragma once

#include "common.cuh"

namespace mlora {

// Segment list of one slot, built in shared memory in passes of CAP entries.
template <int CAP>
struct SlotSegments {
  int start[CAP];    // first token row of each matching segment
  int cum[CAP + 1];  // exclusive prefix of segment lengths; cum[n] = tokens
  int n;             // segments in this pass
  int next;          // first segment index not yet scanned (bs when done)
};

// Warp 0 scans weight_indices[from, bs) in order and appends the non-empty
// segments that route to `slot` until CAP would overflow. Invalid routing
// (slot index out of range, indptr decreasing or past S) is reported in
// `status` and that segment is skipped. Caller must __syncthreads() after.
template <int CAP>
__device__ __forceinline__ void collect_slot_segments(
    SlotSegments<CAP>& sl, int slot, int from, const int32_t* __restrict__ widx,
    const int32_t* __restrict__ indptr, int bs, int S, int num_slots, uint32_t* status) {
  const int lane = threadIdx.x & 31;
  if (threadIdx.x >= 32) return;
  int n = 0;
  int total = 0;
  int i = from;
  for (; i < bs; i += 32) {
    const int idx = i + lane;
    bool match = false;
    int st = 0, len = 0;
    if (idx < bs) {
      const int w = __ldg(widx + idx);
      if (w < 0 || w >= num_slots) {
        // report once, from the CTA that owns slot 0 and the first column
        if (slot == 0 && blockIdx.x == 0) flag_error(status, kErrSlotRange);
      } else if (w == slot) {
        st = __ldg(indptr + idx);
        const int en = __ldg(indptr + idx + 1);
        if (st < 0 || en < st || en > S) {
          if (blockIdx.x == 0) flag_error(status, kErrIndptr);
        } else if (en > st) {
          match = true;
          len = en - st;
        }
      }
    }
    const unsigned m = __ballot_sync(0xffffffffu, match);
    const int cnt = __popc(m);
    if (n + cnt > CAP) break;  // warp-uniform; resume from i next pass
    // inclusive scan of lengths across the warp
    int incl = len;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (match) {
      const int pos = n + __popc(m & ((1u << lane) - 1u));
      sl.start[pos] = st;
      sl.cum[pos] = total + incl - len;
    }
    n += cnt;
    total += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) {
    sl.n = n;
    sl.cum[n] = total;
    sl.next = i < bs ? i : bs;
  }
}

// Token row of the q-th token (0-based) of the current pass.
template <int CAP>
__device__ __forceinline__ int slot_token_row(const SlotSegments<CAP>& sl, int q) {
  // largest j with cum[j] <= q (segments are non-empty, so cum is strictly increasing)
  int lo = 0, hi = sl.n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (sl.cum[mid] <= q) lo = mid; else hi = mid - 1;
  }
  return sl.start[lo] + (q - sl.cum[lo]);
}

}  // namespace mlora
