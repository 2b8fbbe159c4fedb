// Seeded host data for tests and benchmarks (libaegis_datagen.so, not part of
// the C ABI). The reference generates every GEMM input on the host with
// std::mt19937(seed) and std::uniform_real_distribution<float>(-1, 1), A then
// B from one engine, each value rounded to f16 (src/bench/harness.cu:48-54);
// the decode configuration uses std::normal_distribution<float>. Using the
// same libstdc++ engine and distributions here gives bit-identical inputs.
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <new>
#include <random>

namespace {

// IEEE binary32 -> binary16, round to nearest even (overflow -> Inf, NaN kept).
uint16_t f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t absx = x & 0x7fffffffu;
  if (absx > 0x7f800000u) return uint16_t(sign | 0x7e00u);  // NaN
  if (absx >= 0x47800000u) {                                  // >= 65536: overflow or Inf
    // 65520 and above rounds to Inf; below rounds within range (handled next).
    return uint16_t(sign | 0x7c00u);
  }
  if (absx >= 0x38800000u) {  // normal f16 range (>= 2^-14)
    const uint32_t mant = absx & 0x7fffffu;
    const uint32_t exp = (absx >> 23) - 127 + 15;
    uint32_t h = (exp << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;  // may carry into Inf: correct
    return uint16_t(sign | h);
  }
  // Subnormal f16 (or zero): value = mant * 2^-24.
  if (absx < 0x33000000u) return uint16_t(sign);  // < 2^-25: rounds to 0
  const uint32_t e = absx >> 23;                  // biased f32 exponent
  const uint32_t mant = (absx & 0x7fffffu) | 0x800000u;
  const uint32_t shift = 126u - e;  // value = mant * 2^(e-150); in 2^-24 units: mant >> (126 - e)
  uint32_t h = mant >> shift;
  const uint32_t rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1u);
  if (rem > half || (rem == half && (h & 1u))) ++h;
  return uint16_t(sign | h);
}

// IEEE binary32 -> bfloat16, round to nearest even (NaN kept quiet).
uint16_t f32_to_bf16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return uint16_t((x >> 16) | 0x40u);
  const uint32_t lsb = (x >> 16) & 1u;
  x += 0x7fffu + lsb;
  return uint16_t(x >> 16);
}

struct Engine {
  std::mt19937 rng;
};

}  // namespace

extern "C" {

__attribute__((visibility("default"))) void* datagen_engine_new(unsigned seed) {
  return new (std::nothrow) Engine{std::mt19937(seed)};
}

__attribute__((visibility("default"))) void datagen_engine_free(void* e) { delete static_cast<Engine*>(e); }

// kind 0: uniform_real_distribution<float>(p0, p1); kind 1: normal_distribution<float>(p0, p1).
// dtype 0: f16, 1: bf16, 2: float32 (out is float*). Draws n values in order.
__attribute__((visibility("default"))) int datagen_fill(void* eng, int kind, float p0, float p1, int dtype, void* out,
                                                        size_t n) {
  if (!eng || !out || kind < 0 || kind > 1 || dtype < 0 || dtype > 2) return -1;
  std::mt19937& rng = static_cast<Engine*>(eng)->rng;
  auto emit = [&](auto& dist) {
    if (dtype == 2) {
      float* o = static_cast<float*>(out);
      for (size_t i = 0; i < n; ++i) o[i] = dist(rng);
    } else {
      uint16_t* o = static_cast<uint16_t*>(out);
      if (dtype == 0)
        for (size_t i = 0; i < n; ++i) o[i] = f32_to_f16(dist(rng));
      else
        for (size_t i = 0; i < n; ++i) o[i] = f32_to_bf16(dist(rng));
    }
  };
  if (kind == 0) {
    std::uniform_real_distribution<float> d(p0, p1);
    emit(d);
  } else {
    std::normal_distribution<float> d(p0, p1);
    emit(d);
  }
  return 0;
}

// Raw conversions (tests compare them with numpy's).
__attribute__((visibility("default"))) void datagen_f32_to_16(const float* in, uint16_t* out, size_t n, int bf16) {
  for (size_t i = 0; i < n; ++i) out[i] = bf16 ? f32_to_bf16(in[i]) : f32_to_f16(in[i]);
}

}  // extern "C"
