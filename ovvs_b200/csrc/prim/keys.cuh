// Candidate keys: one uint64 per (distance, row id) that orders exactly like the reference's
// top-k total order (src/prim/cpu/cpu_prims.cpp:24-32): numeric ascending, -0 == +0, NaN after
// every number, ties by lower id. High 32 bits: order-preserving image of the fp32 value (NaN ->
// 0xFFFFFFFF); low 32 bits: row id. kEmptyKey (NaN, 0xFFFFFFFF) sorts after every real
// candidate and marks an empty slot.
#pragma once

#include <cstdint>

namespace ovvs {
namespace keys {

constexpr uint64_t kEmptyKey = ~0ull;
constexpr uint32_t kEmptyId = 0xFFFFFFFFu;

__host__ __device__ __forceinline__ uint32_t order_bits(float v) {
#ifdef __CUDA_ARCH__
  uint32_t u = __float_as_uint(v);
#else
  uint32_t u;
  __builtin_memcpy(&u, &v, 4);
#endif
  if (v != v) return 0xFFFFFFFFu;
  if (v == 0.0f) u = 0u;  // -0 ties with +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Inverse of order_bits for non-NaN images (the sign of zero is not recoverable: +0).
__host__ __device__ __forceinline__ float order_value(uint32_t o) {
  if (o == 0xFFFFFFFFu) return __builtin_nanf("");
  const uint32_t u = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
#endif
}

__host__ __device__ __forceinline__ uint64_t make_key(float v, uint32_t id) {
  return (static_cast<uint64_t>(order_bits(v)) << 32) | id;
}

__host__ __device__ __forceinline__ uint32_t key_id(uint64_t k) { return static_cast<uint32_t>(k); }
__host__ __device__ __forceinline__ float key_value(uint64_t k) {
  return order_value(static_cast<uint32_t>(k >> 32));
}

}  // namespace keys
}  // namespace ovvs
