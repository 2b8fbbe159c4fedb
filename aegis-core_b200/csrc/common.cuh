#pragma once
// Small helpers shared by every translation unit of libaegis_capi.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace aegis {

// ceil(a / b) for a >= 0, b > 0, without the overflow of (a + b - 1) / b near
// the type's maximum (an M or N of 2^31 - 1 is a valid problem).
template <class T>
__host__ __device__ constexpr T ceil_div(T a, T b) { return a / b + (a % b != 0 ? 1 : 0); }

// 16-bit element traits: f16 and bf16 share every kernel; only the
// conversions differ.
template <class T> struct Elem;
template <> struct Elem<__half> {
  static constexpr bool kBf16 = false;
  __device__ __forceinline__ static float to_f32(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_f32(float x) { return __float2half_rn(x); }
  __device__ __forceinline__ static float2 pair_to_f32(uint32_t v) {
    return __half22float2(*reinterpret_cast<const __half2*>(&v));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr bool kBf16 = true;
  __device__ __forceinline__ static float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_f32(float x) { return __float2bfloat16_rn(x); }
  // bf16 -> f32 is exact: the bf16 bits are the high half of the f32 bits.
  __device__ __forceinline__ static float2 pair_to_f32(uint32_t v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};

// Bits of the per-device status word (kernel watchdogs, see status.h).
enum StatusBits : unsigned {
  kStatusTimeoutProducer = 1u << 0,
  kStatusTimeoutMma = 1u << 1,
  kStatusTimeoutEpilogue = 1u << 2,
  kStatusTimeoutDrain = 1u << 3,
  kStatusTimeoutSelftest = 1u << 4,
};

// Default limit of every bounded wait inside a kernel (nanoseconds of
// %globaltimer). A pipeline wait never legitimately lasts more than a few
// hundred microseconds; two seconds also covers time slicing with other
// contexts on a shared GPU.
inline constexpr long long kDefaultWaitLimitNs = 2000000000ll;

// Split-K slot sums: p[0] + p[stride] + ... + p[(S-1)*stride] in that fixed
// order (the first slot taken as is, each next one added, exactly as a plain
// sequential loop does), with the L2 loads issued BATCH at a time (the last
// batch predicated) so S slots cost ceil(S/BATCH) round trips instead of S.
// BATCH = 8 for floats, 4 for float4 (16 data registers in flight, so a
// reduce kernel keeps its occupancy).
__device__ __forceinline__ void add_slot(float& acc, float v, bool first) { acc = first ? v : acc + v; }
__device__ __forceinline__ void add_slot(float4& acc, const float4& v, bool first) {
  if (first) {
    acc = v;
  } else {
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
}
// `stride` and S * stride fit in 32 bits (split-K workspaces are capped far
// below 2^31 elements).
template <class V, int BATCH = sizeof(V) == 16 ? 4 : 8>
__device__ __forceinline__ V sum_slots_t(const V* p, int stride, int S) {
  V acc{};
  for (int q = 0; q < S; q += BATCH, p += BATCH * stride) {
    V v[BATCH];
#pragma unroll
    for (int j = 0; j < BATCH; ++j)
      if (q + j < S) v[j] = __ldcg(p + j * stride);
#pragma unroll
    for (int j = 0; j < BATCH; ++j)
      if (q + j < S) add_slot(acc, v[j], q + j == 0);
  }
  return acc;
}

}  // namespace aegis
