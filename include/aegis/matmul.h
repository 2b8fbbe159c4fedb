#pragma once
// aegis::matmul: one entry point that runs the tuned winner for this device.
// Mirrors the reference's include/aegis/matmul.h (Riffe007/aegis-core,
// matmul.h:8-123) with B200 rules:
//
// Selection, against the winners compiled in for the device's arch
// (include/aegis/winners/sm_100a.h, written by the tuner's emit-header step),
// among the rows tuned on the call's operand type (f16 or bf16); when (N, K)
// has none of that type, the other 16-bit type's rows (the same kernel
// templates serve both types):
//   1. exact (M, N, K) match;
//   2. else the winner with the same N and K whose M is nearest in log2 (ties
//      go to the larger M);
//   3. else a built-in rule over this library's own kernels (there is no
//      vendor-library dispatch target): M <= 2 -> the CUDA-core decode GEMV;
//      M <= 16 -> the tensor-core decode stream (ummav) for row-major
//      operands the TMA path can address, else the CUDA-core GEMV; larger M
//      with TMA-addressable operands -> umma (CTA pairs when M and N exceed
//      128; split-K when the tiles cannot fill the SMs); otherwise the simt
//      kernel.
// Rows whose kernel the device cannot run (gemm::supported) are skipped.
// alpha == 0 runs the scale-C kernel (C = beta * C; beta == 0 writes zeros
// without reading C), as BLAS does.
//
// Workspace: the split-K partials come from a per-stream cache (allocated on
// the first call that needs its size class on a stream; make that first call
// outside stream capture). Later calls only launch: no allocation, no host
// synchronisation. Never exits: returns cudaSuccess or the error;
// matmul_last_error() describes the last failure on this host thread.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <span>
#include <string>

#include "aegis/gemm.h"

namespace aegis {

namespace detail {
enum class Dispatch { Aegis };
struct Winner {
  int M, N, K;
  const char* impl;               // registry name
  Dispatch dispatch = Dispatch::Aegis;
  double pct_of_cublas = 0;       // kernel % of cuBLAS (paired median; 0 = not measured)
  double ci_lo = 0, ci_hi = 0;    // paired CI of cuBLAS time / kernel time (0 = none)
  gemm::DType dtype = gemm::DType::F16;  // operand type the row was tuned on
};

struct Choice {
  enum class Kind { Aegis, Rule } kind = Kind::Rule;
  const Winner* winner = nullptr;             // the row chosen (Kind::Aegis)
  const gemm::KernelEntry* kernel = nullptr;  // what runs
  int filtered = 0;                           // rows of (N, K) skipped as unsupported
};
// Capability-aware selection among `table`'s rows for (N, K) (reference
// matmul.cu:432-467), falling back to the built-in rule for p.
Choice choose(std::span<const Winner> table, const gemm::GemmParams& p, const gemm::DeviceCaps& caps,
              std::string* why = nullptr);
// The built-in rule alone.
const gemm::KernelEntry* rule_for(const gemm::GemmParams& p, const gemm::DeviceCaps& caps);
// The winners table for the current device's arch (empty if none).
std::span<const Winner> winners_table();
}  // namespace detail

// Row-major f16 convenience form, the reference's signature (matmul.h:112-113).
cudaError_t matmul(const __half* A, const __half* B, __half* C, int M, int N, int K,
                   cudaStream_t stream = nullptr);
// The same for bf16 operands (no reference counterpart: the reference is f16-only).
cudaError_t matmul(const __nv_bfloat16* A, const __nv_bfloat16* B, __nv_bfloat16* C, int M, int N, int K,
                   cudaStream_t stream = nullptr);
// General form.
cudaError_t matmul(const gemm::GemmParams& p, cudaStream_t stream = nullptr);
// Text of the last failure on this host thread ("" if none).
const char* matmul_last_error();
// The impl matmul() would run for a packed row-major f16 problem of this shape.
const char* matmul_choice(int M, int N, int K);
// The impl matmul() would run for p.
const char* matmul_choice(const gemm::GemmParams& p);

}  // namespace aegis
