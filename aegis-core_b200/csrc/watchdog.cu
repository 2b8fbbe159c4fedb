// Watchdog self-test: one wait that nothing ever completes, bounded by the
// same ptx::mbar_wait_bounded every pipeline wait in this library uses. The
// kernel must give up after `limit_ns`, report it in a status word and
// return normally (no trap, no fault), leaving the context usable.
#include "common.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace aegis {
namespace {

__global__ void watchdog_selftest_kernel(unsigned* status, long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_addr(&bar), 1);
    abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Phase 0 never completes: nobody arrives on the barrier.
    const bool ok = ptx::mbar_wait_bounded(ptx::smem_addr(&bar), 0u, &abort_flag, status, kStatusTimeoutSelftest,
                                           limit_ns);
    if (ok) atomicOr(status + 2, 1u);  // would mean the wait "succeeded": reported as a failure by the host
  }
}

}  // namespace

cudaError_t watchdog_selftest(long long limit_ns, cudaStream_t stream, unsigned* bits_out) {
  *bits_out = 0;
  unsigned* d = nullptr;
  if (const cudaError_t e = cudaMalloc(&d, 4 * sizeof(unsigned)); e != cudaSuccess) return e;
  cudaError_t e = cudaMemsetAsync(d, 0, 4 * sizeof(unsigned), stream);
  if (e == cudaSuccess) {
    watchdog_selftest_kernel<<<1, 32, 0, stream>>>(d, limit_ns);
    e = cudaGetLastError();
  }
  unsigned h[4] = {};
  if (e == cudaSuccess) e = cudaMemcpyAsync(h, d, sizeof h, cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  cudaFree(d);
  if (e != cudaSuccess) return e;
  *bits_out = h[2] ? 0u : h[0];
  return cudaSuccess;
}

}  // namespace aegis
