// Per-device status word (see status.h).
#include "status.h"

#include <mutex>

#include "gpu_target.h"

namespace aegis::status {
namespace {

std::mutex g_mu;
unsigned* g_word[gpu::kMaxDevices] = {};

}  // namespace

cudaError_t word(unsigned** out) {
  *out = nullptr;
  int dev = 0;
  if (const cudaError_t e = cudaGetDevice(&dev); e != cudaSuccess) return e;
  if (dev < 0 || dev >= gpu::kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_word[dev]) {
    unsigned* p = nullptr;
    if (const cudaError_t e = cudaMalloc(&p, 4 * sizeof(unsigned)); e != cudaSuccess) return e;
    if (const cudaError_t e = cudaMemset(p, 0, 4 * sizeof(unsigned)); e != cudaSuccess) {
      cudaFree(p);
      return e;
    }
    g_word[dev] = p;
  }
  *out = g_word[dev];
  return cudaSuccess;
}

cudaError_t take(unsigned* bits, unsigned* block) {
  *bits = 0;
  *block = 0;
  int dev = 0;
  if (const cudaError_t e = cudaGetDevice(&dev); e != cudaSuccess) return e;
  if (dev < 0 || dev >= gpu::kMaxDevices) return cudaSuccess;
  unsigned* p = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    p = g_word[dev];
  }
  if (!p) return cudaSuccess;
  unsigned h[4] = {};
  if (const cudaError_t e = cudaMemcpy(h, p, sizeof h, cudaMemcpyDeviceToHost); e != cudaSuccess) return e;
  if (h[0] != 0) {
    if (const cudaError_t e = cudaMemset(p, 0, sizeof h); e != cudaSuccess) return e;
  }
  *bits = h[0];
  *block = h[1];
  return cudaSuccess;
}

}  // namespace aegis::status
