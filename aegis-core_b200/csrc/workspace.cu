// Per-stream workspace cache (see workspace.h).
#include "workspace.h"

#include <vector>

namespace aegis::ws {
namespace {

struct Buffer {
  int dev;
  cudaStream_t stream;
  Use use;
  size_t bytes;
  void* ptr;
};

thread_local std::vector<Buffer> t_buffers;

size_t size_class(size_t bytes) {
  size_t c = size_t(64) << 10;
  while (c < bytes) c <<= 1;
  return c;
}

}  // namespace

cudaError_t get(cudaStream_t stream, size_t bytes, void** out, Use use) {
  *out = nullptr;
  if (bytes == 0) return cudaErrorInvalidValue;
  int dev = 0;
  if (const cudaError_t e = cudaGetDevice(&dev); e != cudaSuccess) return e;
  const size_t cls = size_class(bytes);
  for (const Buffer& b : t_buffers)
    if (b.dev == dev && b.stream == stream && b.use == use && b.bytes == cls) {
      *out = b.ptr;
      return cudaSuccess;
    }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (const cudaError_t e = cudaStreamIsCapturing(stream, &cap); e != cudaSuccess) return e;
  if (cap != cudaStreamCaptureStatusNone) return cudaErrorStreamCaptureUnsupported;
  void* p = nullptr;
  if (const cudaError_t e = cudaMalloc(&p, cls); e != cudaSuccess) return e;
  if (const cudaError_t e = cudaMemsetAsync(p, 0, cls, stream); e != cudaSuccess) {
    cudaFree(p);
    return e;
  }
  t_buffers.push_back({dev, stream, use, cls, p});
  *out = p;
  return cudaSuccess;
}

size_t allocations() { return t_buffers.size(); }

}  // namespace aegis::ws
