// Row-parallel peer exchange: device side shared by the streaming pair
// (apply_stream.cu) and the fused decode kernel (apply_fused.cu).
//
// Every partial value goes to every rank as one 8-byte word {fp32 bits, tag}
// with tag = epoch + 1 of the call; the reader polls its words until the tag
// is this call's. The epoch is the number of calls this rank has completed;
// the words alternate between two halves by epoch parity, so a rank one call
// ahead never overwrites words still being read (to be two calls ahead it
// would need this rank's partials of the call in between, which this rank
// publishes only after its current call has finished).
#pragma once

#include <stdint.h>

#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace mlora {

__device__ __forceinline__ void word_store_sys(unsigned long long* w, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(w), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long word_load(const unsigned long long* w) {
  unsigned long long a;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(a) : "l"(w) : "memory");
  return a;
}
__device__ __forceinline__ void word_load_pair(const unsigned long long* w, unsigned long long& a,
                                               unsigned long long& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(w) : "memory");
}
// The word carrying `v` for the call of `epoch`.
__device__ __forceinline__ unsigned long long tagged_word(uint32_t epoch, float v) {
  return ((unsigned long long)(epoch + 1u) << 32) | __float_as_uint(v);
}
// The call's epoch: read after griddepcontrol.wait, when every earlier call's
// last kernel (which advances the counter) has completed.
__device__ __forceinline__ uint32_t xchg_epoch(const PeerXchg& x) {
  return *reinterpret_cast<volatile const uint32_t*>(x.ctr);
}
// Offset (words) of partial row `row` from rank `from` in a receive buffer
// of `tp` ranks x `rows` rows x R words per half.
__device__ __forceinline__ int64_t xchg_offset(uint32_t epoch, int tp, int rows, int from, int row, int R) {
  return ((int64_t)(epoch & 1u) * tp * rows + (int64_t)from * rows + row) * R;
}
__device__ __forceinline__ int64_t xchg_row(const PeerXchg& x, uint32_t epoch, int from, int row, int R) {
  return xchg_offset(epoch, x.tp, x.rows, from, row, R);
}
// Polls the word at `w` (already loaded once into `a`) until it carries
// `tag`; bounded by kWaitLimitNs from `t0` (0: not started). Returns false
// on timeout.
__device__ __forceinline__ bool poll_word(const unsigned long long* w, unsigned long long a, uint32_t tag, float& v,
                                          uint64_t& t0) {
  while ((uint32_t)(a >> 32) != tag) {
    if (t0 == 0) t0 = global_timer_ns();
    else if (global_timer_ns() - t0 > kWaitLimitNs) return false;
    a = word_load(w);
  }
  v = __uint_as_float((uint32_t)a);
  return true;
}
// Slow path of a poll, kept out of line (the common case, a word that has
// already arrived, costs a tag compare in the caller): reloads the word at
// `w` until it carries `tag` or kWaitLimitNs have passed; returns the last
// word read (the caller checks its tag).
static __device__ __noinline__ unsigned long long poll_until(const unsigned long long* w, uint32_t tag) {
  const uint64_t t0 = global_timer_ns();
  unsigned long long a = word_load(w);
  while ((uint32_t)(a >> 32) != tag && global_timer_ns() - t0 <= kWaitLimitNs) a = word_load(w);
  return a;
}
// Two adjacent words (columns c, c + 1 of one rank's row), polled until both
// carry `tag` (each column only if it is below `live`); bounded by
// kWaitLimitNs from `t0`. Returns false on timeout.
__device__ __forceinline__ bool poll_pair(const unsigned long long* w, uint32_t tag, int c, int live, float& v0,
                                          float& v1, uint64_t& t0) {
  unsigned long long a, b;
  word_load_pair(w, a, b);
  const bool need0 = c < live, need1 = c + 1 < live;
  while ((need0 && (uint32_t)(a >> 32) != tag) || (need1 && (uint32_t)(b >> 32) != tag)) {
    if (t0 == 0) t0 = global_timer_ns();
    else if (global_timer_ns() - t0 > kWaitLimitNs) return false;
    word_load_pair(w, a, b);
  }
  v0 = need0 ? __uint_as_float((uint32_t)a) : 0.f;
  v1 = need1 ? __uint_as_float((uint32_t)b) : 0.f;
  return true;
}
// A CTA's ticket in the count of the call's last kernel, taken once the CTA
// has read the epoch: both branches depend on the loaded value, so the atomic
// cannot overtake the load (the epoch this CTA uses is the one before any
// advance), and the caller consumes the ticket only at its exit, so the
// atomic's round trip hides behind the CTA's work. Nothing needs a fence: the
// next call reads the counters after griddepcontrol.wait, which makes this
// grid's stores visible.
// (`ctr`: the rank's counters, PeerXchg::ctr.)
__device__ __forceinline__ uint32_t xchg_ticket(uint32_t* ctr, uint32_t epoch) {
  if (epoch != 0xFFFFFFFFu) return atomicAdd(&ctr[1], 1u);
  return atomicInc(&ctr[1], 0xFFFFFFFFu);  // the same increment (the counter never reaches the bound)
}
// The holder of the last of `counted` tickets resets the count and advances
// the epoch (an increment whose result nobody waits for).
__device__ __forceinline__ void xchg_advance(uint32_t* ctr, uint32_t ticket, uint32_t counted) {
  if (ticket == counted - 1u) {
    ctr[1] = 0u;
    atomicAdd(&ctr[0], 1u);
  }
}
__device__ __forceinline__ uint32_t load_epoch(const uint32_t* ctr) { return *reinterpret_cast<volatile const uint32_t*>(ctr); }

}  // namespace mlora
