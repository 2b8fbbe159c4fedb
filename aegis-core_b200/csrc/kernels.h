#pragma once
// Internal host entry points of the kernel families (not exported from the
// shared library; the C ABI and aegis::matmul reach them through the
// registry).
#include <cuda_runtime.h>

#include <string>

#include "aegis/gemm.h"

namespace aegis {

// C = beta * C over the batch (beta == 0: zeros, C not read): the alpha == 0
// path (reference src/matmul.cu:366-382).
cudaError_t scale_c(const gemm::GemmParams& p, cudaStream_t stream);

// The general kernel: any layout / ld / alignment / batch stride.
cudaError_t simt_run(const gemm::GemmParams& p, cudaStream_t stream);

// umma family, config index into gemm::UMMA_CONFIGS. Falls back to simt_run
// when the TMA path cannot address p or the device is not sm_100.
cudaError_t umma_run(int cfg, const gemm::GemmParams& p, cudaStream_t stream);
gemm::LaunchPlan umma_plan(int cfg, const gemm::GemmParams& p);
cudaError_t umma_attrs(int cfg, cudaFuncAttributes* attrs);
size_t umma_smem_bytes(int cfg);

// N-sharded GEMM with the all-gather of C fused into the epilogue (peer
// stores). c_ranks: every rank's C (device pointers valid on this device).
cudaError_t umma_nsharded(const gemm::GemmParams& local, void* const* c_ranks, int nranks, int col_offset,
                          cudaStream_t stream);

// gemv family, config index into gemm::GEMV_CONFIGS.
cudaError_t gemv_run(int cfg, const gemm::GemmParams& p, cudaStream_t stream);
gemm::LaunchPlan gemv_plan(int cfg, const gemm::GemmParams& p);
cudaError_t gemv_attrs(int cfg, cudaFuncAttributes* attrs);

// ummav family: decode GEMM on tensor cores (swap-AB, stream-K segments).
// Runs the CUDA-core gemv for problems it cannot take (ummav_applicable: an
// sm_100 device and a problem ummav_takes).
bool ummav_takes(const gemm::GemmParams& p);  // shape, layout and alignment only
bool ummav_applicable(const gemm::GemmParams& p);
cudaError_t ummav_run(int cfg, const gemm::GemmParams& p, cudaStream_t stream);
gemm::LaunchPlan ummav_plan(int cfg, const gemm::GemmParams& p);
cudaError_t ummav_attrs(int cfg, cudaFuncAttributes* attrs);
size_t ummav_smem_bytes(int cfg);

// Allocation-free decode GEMV: the gemv kernel with its split-K scratch in
// a fixed device array of this library (no cudaMalloc, cudaFree or other
// allocation on any call). One batch, M <= kNoAllocMaxM, N <= kNoAllocMaxN;
// *why names the reason of a rejection.
inline constexpr int kNoAllocMaxM = 16;
inline constexpr int kNoAllocMaxN = 65536;
cudaError_t gemv_run_noalloc(const gemm::GemmParams& p, cudaStream_t stream, const char** why);
// The plan gemv_run_noalloc would launch on the planning target; false when
// the problem's tickets do not fit the fixed array.
bool gemv_noalloc_plan(const gemm::GemmParams& p, gemm::LaunchPlan* out);

// Watchdog self-test kernel: one wait that nothing completes.
cudaError_t watchdog_selftest(long long limit_ns, cudaStream_t stream, unsigned* bits_out);

// Deterministic split-K plan (reference src/gemm/splitk.cuh:77-92 restated
// for large tiles): the S in [1, s_max] minimising
//   ceil(tiles*S / sms) * ceil(k_blocks / S) * t_block  +  S * reduce_cost
// (smallest S on ties). Pure function of its arguments.
int splitk_choose(long long tiles, int k_blocks, int sms, int min_blocks_per_split, double t_block_ns,
                  double reduce_ns_per_split, long long max_splits);

}  // namespace aegis
