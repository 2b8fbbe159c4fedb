// C++ drop-in test: a program written against the reference's C++ API
// (include/aegis/matmul.h, include/aegis/gemm.h), linked statically against
// libaegis.a, as the reference's tests/test_matmul.cu links its libaegis.a.
//
//   matmul_test OUT_PREFIX [M N K]
//
// Inputs: std::mt19937(0) with uniform_real_distribution<float>(-1, 1), A
// drawn first, then B, each rounded to f16 (the reference harness's order,
// src/bench/harness.cu:48-54). Runs
//   1. aegis::matmul(const __half*, const __half*, __half*, M, N, K, stream),
//   2. aegis::matmul(const gemm::GemmParams&, stream) on the same data as bf16,
// writes the two C matrices to OUT_PREFIX.f16 / OUT_PREFIX.bf16 (raw 16-bit
// row-major) for the caller to check against the oracle, and prints one line
// of JSON with the dispatch choices and registry facts. Exit 0 on success.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "aegis/gemm.h"
#include "aegis/matmul.h"

namespace {

int fail(const char* what) {
  std::fprintf(stderr, "matmul_test: %s (%s)\n", what, aegis::matmul_last_error());
  return 1;
}

bool write_raw(const char* path, const void* p, size_t bytes) {
  FILE* f = std::fopen(path, "wb");
  if (!f) return false;
  const bool ok = std::fwrite(p, 1, bytes, f) == bytes;
  return std::fclose(f) == 0 && ok;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 2 && argc != 5) {
    std::fprintf(stderr, "usage: matmul_test OUT_PREFIX [M N K]\n");
    return 2;
  }
  const int M = argc == 5 ? std::atoi(argv[2]) : 512, N = argc == 5 ? std::atoi(argv[3]) : 512,
            K = argc == 5 ? std::atoi(argv[4]) : 512;
  std::mt19937 rng(0);
  std::uniform_real_distribution<float> u(-1.f, 1.f);
  std::vector<__half> hA(size_t(M) * K), hB(size_t(K) * N);
  std::vector<__nv_bfloat16> bA(hA.size()), bB(hB.size());
  for (size_t i = 0; i < hA.size(); ++i) {
    const float x = u(rng);
    hA[i] = __float2half(x);
    bA[i] = __float2bfloat16(x);
  }
  for (size_t i = 0; i < hB.size(); ++i) {
    const float x = u(rng);
    hB[i] = __float2half(x);
    bB[i] = __float2bfloat16(x);
  }
  const size_t a_bytes = hA.size() * 2, b_bytes = hB.size() * 2, c_bytes = size_t(M) * N * 2;
  void *dA, *dB, *dC;
  if (cudaMalloc(&dA, a_bytes) != cudaSuccess || cudaMalloc(&dB, b_bytes) != cudaSuccess ||
      cudaMalloc(&dC, c_bytes) != cudaSuccess)
    return fail("cudaMalloc");
  cudaStream_t s;
  if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return fail("cudaStreamCreate");
  std::vector<unsigned char> out(c_bytes);
  char path[4096];

  // 1. The reference's row-major f16 form.
  cudaMemcpy(dA, hA.data(), a_bytes, cudaMemcpyHostToDevice);
  cudaMemcpy(dB, hB.data(), b_bytes, cudaMemcpyHostToDevice);
  cudaMemset(dC, 0xff, c_bytes);  // NaN: every element must be written
  if (aegis::matmul(static_cast<const __half*>(dA), static_cast<const __half*>(dB), static_cast<__half*>(dC), M, N,
                    K, s) != cudaSuccess)
    return fail("aegis::matmul (f16 pointer form)");
  if (cudaStreamSynchronize(s) != cudaSuccess) return fail("synchronize");
  cudaMemcpy(out.data(), dC, c_bytes, cudaMemcpyDeviceToHost);
  std::snprintf(path, sizeof path, "%s.f16", argv[1]);
  if (!write_raw(path, out.data(), c_bytes)) return fail("write f16 result");
  const char* choice_f16 = aegis::matmul_choice(M, N, K);

  // 2. The general form with bf16 operands.
  cudaMemcpy(dA, bA.data(), a_bytes, cudaMemcpyHostToDevice);
  cudaMemcpy(dB, bB.data(), b_bytes, cudaMemcpyHostToDevice);
  cudaMemset(dC, 0xff, c_bytes);
  const aegis::gemm::GemmParams p = aegis::gemm::row_major_params(dA, dB, dC, M, N, K, aegis::gemm::DType::BF16);
  if (aegis::matmul(p, s) != cudaSuccess) return fail("aegis::matmul (GemmParams, bf16)");
  if (cudaStreamSynchronize(s) != cudaSuccess) return fail("synchronize");
  cudaMemcpy(out.data(), dC, c_bytes, cudaMemcpyDeviceToHost);
  std::snprintf(path, sizeof path, "%s.bf16", argv[1]);
  if (!write_raw(path, out.data(), c_bytes)) return fail("write bf16 result");

  // Invalid parameters are refused, not run (reference gemm::validate).
  aegis::gemm::GemmParams bad = p;
  bad.lda = K - 1;
  const bool refused = aegis::matmul(bad, s) == cudaErrorInvalidValue;

  const aegis::gemm::KernelEntry* e = aegis::gemm::find("umma_256x256x64_s7_c2");
  std::printf("{\"choice_f16\":\"%s\",\"choice_bf16\":\"%s\",\"registry\":%zu,\"find_pair\":%s,"
              "\"invalid_refused\":%s}\n",
              choice_f16, aegis::matmul_choice(p), aegis::gemm::registry().size(), e ? "true" : "false",
              refused ? "true" : "false");
  cudaFree(dA);
  cudaFree(dB);
  cudaFree(dC);
  cudaStreamDestroy(s);
  return 0;
}
