// Shared helpers for the ddtree_b200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ddtree_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "ddtree_b200 is built for sm_100a only"
#endif

#define DDT_FULL_MASK 0xffffffffu

namespace ddt {

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? DDT_OK : DDT_ERR_CUDA;
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---- order-preserving keys ------------------------------------------------
// key(x) grows with x; positive NaN maps above +inf.  -0 and +0 get the same key (they
// compare equal, so ties between them resolve by index as torch's do).
__device__ __forceinline__ uint32_t f32_key(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u << 1) == 0u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_f32(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}
__device__ __forceinline__ uint32_t bf16_key(uint16_t b) {
  if ((b & 0x7fffu) == 0u) b = 0u;
  return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
}
__device__ __forceinline__ float key_bf16(uint32_t k) {
  uint32_t b = (k & 0x8000u) ? (k & 0x7fffu) : (~k & 0xffffu);
  return __uint_as_float(b << 16);
}
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// ---- warp / block reductions ---------------------------------------------
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(DDT_FULL_MASK, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(DDT_FULL_MASK, v, o);
  return v;
}

// Bounded spin helpers use the global nanosecond timer so a lost arrival ends the
// wait with an error status instead of hanging the GPU.
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

}  // namespace ddt
