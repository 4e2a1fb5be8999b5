// Shared device helpers for the multi-LoRA sm_100a kernels.
//
// Element types are the three the reference pool supports (bf16 / f16 / f32,
// multi_lora/pool.py:336-343 takes any torch float dtype). All arithmetic is
// done in fp32 and rounded once on store, as the reference Triton kernels do
// (kernels/sgemm_lora_a.py:324, kernels/sgemm_lora_b.py:572-579).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mlora {

// Element type codes shared with include/mlora_b200.h.
enum DType : int { kBF16 = 0, kF16 = 1, kF32 = 2 };

// Bits a kernel ORs into the optional device status word when it meets
// metadata that would make it read or write out of bounds. The access is
// skipped; the host reads the word and raises.
enum StatusBits : uint32_t {
  kErrSlotRange = 1u << 0,    // weight_indices[i] outside [0, num_slots)
  kErrRankRange = 1u << 1,    // lora_ranks[s] outside [0, max_rank]
  kErrIndptr = 1u << 2,       // seg_indptr[i] > seg_indptr[i+1] or past S
  kErrScatterRange = 1u << 3, // scatter descriptor outside its buffers
};

__device__ __forceinline__ void flag_error(uint32_t* status, uint32_t bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// Programmatic dependent launch. A kernel launched with the programmatic
// stream-serialisation attribute may start while the previous kernel in the
// stream is still running; everything before pdl_wait() must only touch data
// that no still-running kernel writes (adapter weights, routing metadata,
// norm weights). Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Early exit of a CTA that touches nothing earlier kernels write. CTA 0 of
// the grid still waits for the previous kernel (every CTA that works waits on
// its own path), so a grid never completes before its predecessor: a kernel
// that waits for this one also waits for every kernel before it, even when no
// CTA of this grid had work.
__device__ __forceinline__ void pdl_exit_early() {
  pdl_trigger();
  if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 0) pdl_wait();
}

template <typename T>
struct Num;
template <>
struct Num<__nv_bfloat16> {
  static constexpr bool is_bf16 = true;
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <>
struct Num<__half> {
  static constexpr bool is_bf16 = false;
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <>
struct Num<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};

// Two 16-bit elements packed in one 32-bit word (element 0 in the low half).
template <typename T>
struct Pack2;
template <>
struct Pack2<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(__nv_bfloat16 a, __nv_bfloat16 b) {
    return (uint32_t)__bfloat16_as_ushort(a) | ((uint32_t)__bfloat16_as_ushort(b) << 16);
  }
  static __device__ __forceinline__ float lo(uint32_t u) { return __bfloat162float(__ushort_as_bfloat16((unsigned short)(u & 0xffffu))); }
  static __device__ __forceinline__ float hi(uint32_t u) { return __bfloat162float(__ushort_as_bfloat16((unsigned short)(u >> 16))); }
};
template <>
struct Pack2<__half> {
  static __device__ __forceinline__ uint32_t pack(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
  }
  static __device__ __forceinline__ float lo(uint32_t u) { return __half2float(__ushort_as_half((unsigned short)(u & 0xffffu))); }
  static __device__ __forceinline__ float hi(uint32_t u) { return __half2float(__ushort_as_half((unsigned short)(u >> 16))); }
};

// Two fp32 values rounded to T and packed (element 0 in the low half).
template <typename T>
__device__ __forceinline__ uint32_t pack_round2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack_round2<__nv_bfloat16>(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack_round2<__half>(float lo, float hi) {
  const __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Round an fp32 value through element type T and back (the value a tensor of
// dtype T would hold).
template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return Num<T>::to_f(Num<T>::from_f(v));
}

// ---------------------------------------------------------------------------
// Chunked loads: a "chunk" is V consecutive elements. V = 16 / sizeof(T) is
// one 128-bit access; V = 1 is the scalar path used for unaligned shapes.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& u, float* f);

template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void unpack16<__half>(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h;
    memcpy(&h, &w[i], 4);
    const float2 v = __half22float2(h);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}
template <>
__device__ __forceinline__ void unpack16<float>(const uint4& u, float* f) {
  f[0] = __uint_as_float(u.x);
  f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z);
  f[3] = __uint_as_float(u.w);
}

// Raw storage of one chunk, kept packed in registers until it is used.
template <typename T, int V>
struct Chunk {
  static_assert(V * sizeof(T) == 16, "vector chunk must be 16 bytes");
  uint4 u;
  __device__ __forceinline__ void zero() { u = make_uint4(0, 0, 0, 0); }
  // read-only data (adapter weights): non-coherent path
  __device__ __forceinline__ void ldg(const T* p) { u = __ldg(reinterpret_cast<const uint4*>(p)); }
  // data written by an earlier kernel (activations): L2 only
  __device__ __forceinline__ void ldcg(const T* p) { u = __ldcg(reinterpret_cast<const uint4*>(p)); }
  __device__ __forceinline__ void to_f(float* f) const { unpack16<T>(u, f); }
};
template <typename T>
struct Chunk<T, 1> {
  T v;
  __device__ __forceinline__ void zero() { v = Num<T>::from_f(0.f); }
  __device__ __forceinline__ void ldg(const T* p) { v = __ldg(p); }
  __device__ __forceinline__ void ldcg(const T* p) { v = __ldcg(p); }
  __device__ __forceinline__ void to_f(float* f) const { f[0] = Num<T>::to_f(v); }
};

// Scalar load of one element with the L2-only policy (activations).
template <typename T>
__device__ __forceinline__ float ldcg_f(const T* p) {
  return Num<T>::to_f(__ldcg(p));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace mlora
