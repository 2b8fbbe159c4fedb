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
// sequential loop does), with the L2 loads issued eight at a time so S slots
// cost about S/8 round trips instead of S.
__device__ __forceinline__ float sum_slots(const float* p, long long stride, int S) {
  float acc = 0.f;
  int q = 0;
  for (; q + 8 <= S; q += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __ldcg(p + (long long)(q + j) * stride);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc = (q + j == 0) ? v[j] : acc + v[j];
  }
  for (; q < S; ++q) {
    const float v = __ldcg(p + (long long)q * stride);
    acc = (q == 0) ? v : acc + v;
  }
  return acc;
}
__device__ __forceinline__ float4 sum_slots4(const float4* p, long long stride, int S) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  int q = 0;
  for (; q + 8 <= S; q += 8) {
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __ldcg(p + (long long)(q + j) * stride);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (q + j == 0) {
        acc = v[j];
      } else {
        acc.x += v[j].x; acc.y += v[j].y; acc.z += v[j].z; acc.w += v[j].w;
      }
    }
  }
  for (; q < S; ++q) {
    const float4 v = __ldcg(p + (long long)q * stride);
    if (q == 0) {
      acc = v;
    } else {
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
  }
  return acc;
}

}  // namespace aegis
