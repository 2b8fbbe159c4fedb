// Per-thread split-K scratch table (see scratch.h).
#include "scratch.h"

#include <bit>
#include <cstdint>
#include <unordered_map>

namespace aegis::scratch {
namespace {

constexpr unsigned kMinClassLog2 = 16;  // 64 KiB

// (stream, device, kind, class) packed for hashing. A stream handle is unique
// per device while it lives; the device is kept for the legacy handles 0/1/2,
// which name a different stream on every device.
struct Key {
  uintptr_t stream;
  uint32_t tag;  // device << 16 | kind << 8 | log2(class)
  bool operator==(const Key& o) const { return stream == o.stream && tag == o.tag; }
};

struct KeyHash {
  size_t operator()(const Key& k) const {
    return std::hash<uintptr_t>{}(k.stream) ^ (size_t(k.tag) * 0x9E3779B97F4A7C15ull);
  }
};

thread_local std::unordered_map<Key, void*, KeyHash> t_held;

unsigned class_log2(size_t bytes) {
  const unsigned l = unsigned(std::bit_width(bytes - 1));  // ceil(log2(bytes)) for bytes >= 2
  return l < kMinClassLog2 ? kMinClassLog2 : l;
}

}  // namespace

cudaError_t acquire(cudaStream_t stream, size_t bytes, Kind kind, void** out) {
  *out = nullptr;
  if (bytes == 0 || bytes > (size_t(1) << 40)) return cudaErrorInvalidValue;
  int dev = 0;
  if (const cudaError_t e = cudaGetDevice(&dev); e != cudaSuccess) return e;
  const unsigned lg = class_log2(bytes);
  const Key key{reinterpret_cast<uintptr_t>(stream), (uint32_t(dev) << 16) | (uint32_t(kind) << 8) | lg};
  if (const auto it = t_held.find(key); it != t_held.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  // New key: never allocate into a graph being captured.
  cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
  if (const cudaError_t e = cudaStreamIsCapturing(stream, &capturing); e != cudaSuccess) return e;
  if (capturing != cudaStreamCaptureStatusNone) return cudaErrorStreamCaptureUnsupported;
  const size_t cls = size_t(1) << lg;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, cls);
  if (e == cudaSuccess) e = cudaMemsetAsync(p, 0, cls, stream);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return e;
  }
  t_held.emplace(key, p);
  *out = p;
  return cudaSuccess;
}

size_t held() { return t_held.size(); }

}  // namespace aegis::scratch
