#pragma once
// cuBLASLt heuristic sweep for the "cublaslt_best" baseline: the library's
// best algorithm for a row-major C = A*B, as the reference measures it
// (src/bench/harness.cu:963-1031 LtPlan / Harness::cublaslt_best): ask the
// heuristic for its top candidates (FP32 compute and scale, 16-bit A/B/C,
// a bounded workspace), time each, keep the fastest that passes the check.
// One departure, stated by the reference as its dispatch rule
// (src/lt_algo.h:58-60): candidates whose split-K reduction keeps partials in
// reduced precision are dropped, so every baseline reduces in FP32 like the
// kernels it is compared with.
//
// Baseline code for the tuner and bench.py, not part of libaegis_capi.
#include <cublasLt.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <string>
#include <vector>

namespace aegis::tune {

class LtSweep {
 public:
  static constexpr int kMaxAlgos = 8;  // the reference's kLtMaxAlgos (harness.h:179)

  struct Algo {
    cublasLtMatmulAlgo_t algo;
    size_t workspace = 0;
    int rank = 0;  // position in the heuristic's list
    int id = -1, tile = -1, stages = -1, splitk = 1, reduction = 0;
  };

  // bf16: CUDA_R_16BF operands and output, else CUDA_R_16F.
  LtSweep(bool bf16, int M, int N, int K, size_t max_workspace) : M_(M), N_(N), K_(K) {
    if (cublasLtCreate(&lt_) != CUBLAS_STATUS_SUCCESS) return;
    const cudaDataType t = bf16 ? CUDA_R_16BF : CUDA_R_16F;
    // Row-major C[M,N] = A[M,K] * B[K,N] is column-major C^T[N,M] = B^T[N,K] * A^T[K,M].
    if (cublasLtMatmulDescCreate(&op_, CUBLAS_COMPUTE_32F, CUDA_R_32F) != CUBLAS_STATUS_SUCCESS ||
        cublasLtMatrixLayoutCreate(&lb_, t, N, K, N) != CUBLAS_STATUS_SUCCESS ||
        cublasLtMatrixLayoutCreate(&la_, t, K, M, K) != CUBLAS_STATUS_SUCCESS ||
        cublasLtMatrixLayoutCreate(&lc_, t, N, M, N) != CUBLAS_STATUS_SUCCESS)
      return;
    cublasLtMatmulPreference_t pref = nullptr;
    if (cublasLtMatmulPreferenceCreate(&pref) != CUBLAS_STATUS_SUCCESS) return;
    cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &max_workspace,
                                         sizeof max_workspace);
    cublasLtMatmulHeuristicResult_t res[kMaxAlgos] = {};
    int returned = 0;
    const cublasStatus_t st =
        cublasLtMatmulAlgoGetHeuristic(lt_, op_, lb_, la_, lc_, lc_, pref, kMaxAlgos, res, &returned);
    cublasLtMatmulPreferenceDestroy(pref);
    if (st != CUBLAS_STATUS_SUCCESS) return;
    for (int i = 0; i < returned; ++i) {
      if (res[i].state != CUBLAS_STATUS_SUCCESS) continue;
      Algo a;
      a.algo = res[i].algo;
      a.workspace = res[i].workspaceSize;
      a.rank = i;
      size_t w = 0;
      cublasLtMatmulAlgoConfigGetAttribute(&a.algo, CUBLASLT_ALGO_CONFIG_ID, &a.id, sizeof a.id, &w);
      cublasLtMatmulAlgoConfigGetAttribute(&a.algo, CUBLASLT_ALGO_CONFIG_TILE_ID, &a.tile, sizeof a.tile, &w);
      cublasLtMatmulAlgoConfigGetAttribute(&a.algo, CUBLASLT_ALGO_CONFIG_STAGES_ID, &a.stages, sizeof a.stages, &w);
      cublasLtMatmulAlgoConfigGetAttribute(&a.algo, CUBLASLT_ALGO_CONFIG_SPLITK_NUM, &a.splitk, sizeof a.splitk, &w);
      cublasLtMatmulAlgoConfigGetAttribute(&a.algo, CUBLASLT_ALGO_CONFIG_REDUCTION_SCHEME, &a.reduction,
                                           sizeof a.reduction, &w);
      if (a.splitk > 1 && a.reduction != int(CUBLASLT_REDUCTION_SCHEME_COMPUTE_TYPE)) {
        ++dropped_;  // partials below FP32
        continue;
      }
      algos_.push_back(a);
    }
    ok_ = true;
  }
  ~LtSweep() {
    if (lc_) cublasLtMatrixLayoutDestroy(lc_);
    if (la_) cublasLtMatrixLayoutDestroy(la_);
    if (lb_) cublasLtMatrixLayoutDestroy(lb_);
    if (op_) cublasLtMatmulDescDestroy(op_);
    if (lt_) cublasLtDestroy(lt_);
  }
  LtSweep(const LtSweep&) = delete;
  LtSweep& operator=(const LtSweep&) = delete;

  bool ok() const { return ok_; }
  int size() const { return int(algos_.size()); }
  int dropped() const { return dropped_; }
  const Algo& algo(int i) const { return algos_[size_t(i)]; }

  // Row-major C = A * B with candidate i; `ws` holds at least algo(i).workspace bytes.
  cublasStatus_t run(int i, const void* A, const void* B, void* C, void* ws, size_t ws_bytes,
                     cudaStream_t s) const {
    const float one = 1.f, zero = 0.f;
    const Algo& a = algos_[size_t(i)];
    return cublasLtMatmul(lt_, op_, &one, B, lb_, A, la_, &zero, C, lc_, C, lc_, &a.algo, ws, ws_bytes, s);
  }

  std::string describe(int i) const {
    const Algo& a = algos_[size_t(i)];
    char b[192];
    std::snprintf(b, sizeof b,
                  "{\"rank\":%d,\"algo_id\":%d,\"tile\":%d,\"stages\":%d,\"splitk\":%d,\"reduction\":%d,"
                  "\"workspace\":%zu}",
                  a.rank, a.id, a.tile, a.stages, a.splitk, a.reduction, a.workspace);
    return b;
  }

 private:
  int M_, N_, K_;
  bool ok_ = false;
  int dropped_ = 0;
  cublasLtHandle_t lt_ = nullptr;
  cublasLtMatmulDesc_t op_ = nullptr;
  cublasLtMatrixLayout_t la_ = nullptr, lb_ = nullptr, lc_ = nullptr;
  std::vector<Algo> algos_;
};

}  // namespace aegis::tune
