// TEST INFRASTRUCTURE ONLY (the checker, never the product). A C-callable
// bridge into the reference's own oracle, compiled together with the
// reference's unmodified src/bench/reference.cu (Riffe007/aegis-core) by
// oracle/Makefile into oracle/_ref/libaegis_ref.so. Tests use it to pin
// oracle.c, and bench.py's reference arm times it as the reference's CPU path.
// Only argument marshalling lives here: the arithmetic is the reference's
// aegis::bench::cpu_reference (reference.cu:69-105) and tolerance
// (reference.cu:186-194).
#include <cstdint>
#include <cstring>
#include <vector>

#include "bench/reference.h"

extern "C" {

struct ref_gemm {  // same layout as oracle_gemm in oracle.c (f16 only: the reference has no bf16)
  int M, N, K;
  int layout_a, layout_b;
  long long lda, ldb, ldc;
  float alpha, beta;
  int batch;
  long long stride_a, stride_b, stride_c;
  int dtype;
};

static void to_host(const ref_gemm* g, const uint16_t* A, size_t nA, const uint16_t* B, size_t nB, const uint16_t* C0,
                    size_t nC, aegis::bench::HostGemm* h) {
  aegis::gemm::GemmParams& p = h->p;
  p.M = g->M; p.N = g->N; p.K = g->K;
  p.layout_a = g->layout_a ? aegis::gemm::Layout::ColMajor : aegis::gemm::Layout::RowMajor;
  p.layout_b = g->layout_b ? aegis::gemm::Layout::ColMajor : aegis::gemm::Layout::RowMajor;
  p.lda = g->lda; p.ldb = g->ldb; p.ldc = g->ldc;
  p.alpha = g->alpha; p.beta = g->beta;
  p.batch = g->batch;
  p.stride_a = g->stride_a; p.stride_b = g->stride_b; p.stride_c = g->stride_c;
  h->A.resize(nA);
  h->B.resize(nB);
  h->C0.resize(C0 ? nC : 0);
  std::memcpy(h->A.data(), A, nA * 2);
  std::memcpy(h->B.data(), B, nB * 2);
  if (C0) std::memcpy(h->C0.data(), C0, nC * 2);
}

__attribute__((visibility("default"))) int ref_cpu_reference(const ref_gemm* g, const uint16_t* A, size_t nA,
                                                             const uint16_t* B, size_t nB, const uint16_t* C0,
                                                             size_t nC, double* out) {
  if (g->dtype != 0) return -1;
  aegis::bench::HostGemm h;
  to_host(g, A, nA, B, nB, C0, nC, &h);
  std::vector<double> r;
  aegis::bench::cpu_reference(h, r);
  std::memcpy(out, r.data(), r.size() * sizeof(double));
  return 0;
}

__attribute__((visibility("default"))) double ref_tolerance(const ref_gemm* g, const uint16_t* A, size_t nA,
                                                            const uint16_t* B, size_t nB, const uint16_t* C0,
                                                            size_t nC, double c) {
  aegis::bench::HostGemm h;
  to_host(g, A, nA, B, nB, C0, nC, &h);
  return aegis::bench::tolerance(h, c).tol;
}

}  // extern "C"
