/*
 * TEST INFRASTRUCTURE ONLY. This file is the checker, never the product:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load the library built from it (liboracle.so).
 *
 * CPU restatement of the reference's GEMM oracle (Riffe007/aegis-core):
 *   oracle_gemm_ref   <- aegis::bench::cpu_reference, src/bench/reference.cu:69-105
 *                        (one FP64 sum per output element in k order, B transposed
 *                        once per batch, then alpha*acc (+ beta*C0); alpha == 0
 *                        ignores A*B; beta == 0 never reads C0; rows split over
 *                        min(16, nthreads) threads only above 1e7 MACs, :99)
 *   oracle_tolerance  <- aegis::bench::tolerance, src/bench/reference.cu:186-194
 *                        (c*sqrt(K)*eps*max|A|*max|B|*|alpha| + eps*|beta|*max|C0|,
 *                        finite maxima, eps = 2^-10 for f16), plus the north-star
 *                        bound eps*K*max|A|*max|B|*|alpha| (+ the same beta term):
 *                        2^-10 as stated for f16 outputs; for bf16 outputs the
 *                        output type's eps 2^-7, since rounding an exact result to
 *                        bf16 alone can exceed 2^-10*K*max|A|*max|B| at small K
 *   oracle_compare    <- aegis::bench::compare, src/bench/reference.cu:196-247
 *                        (NaN must stay NaN, Inf/overflow the same Inf, finite
 *                        within `allowed`, C padding columns N..ldc-1 untouched)
 * Element decode is exact (f16 or bf16 -> double). The products are summed with
 * separate multiply and add (built with -ffp-contract=off), as the reference's
 * host build does on x86-64, so results equal the reference bit for bit; the
 * pinning tests compare this file with the reference's own function built
 * under oracle/_ref.
 * bf16 has no reference implementation (the reference is f16-only): the same
 * arithmetic with the bf16 decode, eps_bf16 = 2^-7.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_API __attribute__((visibility("default")))

typedef struct {
  int M, N, K;
  int layout_a, layout_b; /* 0 row-major, 1 column-major */
  long long lda, ldb, ldc;
  float alpha, beta;
  int batch;
  long long stride_a, stride_b, stride_c;
  int dtype; /* 0 f16, 1 bf16 */
} oracle_gemm;

typedef struct {
  int pass;
  long long checked, nan_mismatch, inf_mismatch, out_of_tol;
  double max_err, max_ratio;
  long long first_index; /* element index into `out` of the first failure, -1 if none */
  double first_got, first_want;
} oracle_result;

static double f16_to_double(uint16_t h) {
  const int sign = h >> 15, exp = (h >> 10) & 0x1f, mant = h & 0x3ff;
  double v;
  if (exp == 0) v = ldexp((double)mant, -24);
  else if (exp == 31) v = mant ? NAN : INFINITY;
  else v = ldexp((double)(mant | 0x400), exp - 25);
  return sign ? -v : v;
}

static double bf16_to_double(uint16_t h) {
  uint32_t x = (uint32_t)h << 16;
  float f;
  memcpy(&f, &x, 4);
  return (double)f;
}

static double decode(uint16_t h, int dtype) { return dtype == 1 ? bf16_to_double(h) : f16_to_double(h); }

ORACLE_API double oracle_decode(uint16_t h, int dtype) { return decode(h, dtype); }

typedef struct {
  const oracle_gemm* g;
  const uint16_t *A, *C0;
  const double* bt;
  double* out;
  int b, i0, i1;
} rows_job;

static void* rows_worker(void* arg) {
  const rows_job* j = (const rows_job*)arg;
  const oracle_gemm* g = j->g;
  const int ra = g->layout_a == 0;
  double* arow = (double*)malloc(sizeof(double) * (size_t)(g->K > 0 ? g->K : 1));
  for (int i = j->i0; i < j->i1; ++i) {
    for (int k = 0; k < g->K; ++k)
      arow[k] = decode(j->A[(size_t)(j->b * g->stride_a + (ra ? i * g->lda + k : i + k * g->lda))], g->dtype);
    for (int n = 0; n < g->N; ++n) {
      double acc = 0;
      const double* bj = j->bt + (size_t)n * g->K;
      if (g->alpha != 0.f)
        for (int k = 0; k < g->K; ++k) acc += arow[k] * bj[k];
      double v = g->alpha == 0.f ? 0.0 : (double)g->alpha * acc;
      if (g->beta != 0.f)
        v += (double)g->beta * decode(j->C0[(size_t)(j->b * g->stride_c + i * g->ldc + n)], g->dtype);
      j->out[((size_t)j->b * g->M + i) * g->N + n] = v;
    }
  }
  free(arow);
  return NULL;
}

/* out: batch*M*N doubles, packed b*M*N + i*N + j. nthreads <= 0: 1. Returns 0. */
ORACLE_API int oracle_gemm_ref(const oracle_gemm* g, const uint16_t* A, const uint16_t* B, const uint16_t* C0,
                               double* out, int nthreads) {
  if (g->M <= 0 || g->N <= 0 || g->K <= 0 || g->batch <= 0) return 0;
  const int rb = g->layout_b == 0;
  double* bt = (double*)malloc(sizeof(double) * (size_t)g->N * g->K);
  if (!bt) return -1;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 16) nthreads = 16;
  for (int b = 0; b < g->batch; ++b) {
    if (g->alpha != 0.f)
      for (int k = 0; k < g->K; ++k)
        for (int n = 0; n < g->N; ++n)
          bt[(size_t)n * g->K + k] =
              decode(B[(size_t)(b * g->stride_b + (rb ? k * g->ldb + n : k + n * g->ldb))], g->dtype);
    const double work = (double)g->M * g->N * g->K;
    const int parts = work < 1e7 ? 1 : (nthreads < g->M ? nthreads : g->M);
    pthread_t th[16];
    rows_job jobs[16];
    for (int t = 0; t < parts; ++t) {
      jobs[t].g = g;
      jobs[t].A = A;
      jobs[t].C0 = C0;
      jobs[t].bt = bt;
      jobs[t].out = out;
      jobs[t].b = b;
      jobs[t].i0 = (int)((long long)g->M * t / parts);
      jobs[t].i1 = (int)((long long)g->M * (t + 1) / parts);
      if (parts == 1) rows_worker(&jobs[t]);
      else pthread_create(&th[t], NULL, rows_worker, &jobs[t]);
    }
    if (parts > 1)
      for (int t = 0; t < parts; ++t) pthread_join(th[t], NULL);
  }
  free(bt);
  return 0;
}

/* Rows [r0, r1) of every batch only (the CPU-baseline sample of large
 * problems: rows are independent, reference.cu:83-102). out holds
 * batch*(r1-r0)*N doubles. */
ORACLE_API int oracle_gemm_ref_rows(const oracle_gemm* g, const uint16_t* A, const uint16_t* B, const uint16_t* C0,
                                    double* out, int r0, int r1, int nthreads) {
  if (r0 < 0 || r1 > g->M || r0 >= r1) return -1;
  oracle_gemm sub = *g;
  sub.M = r1 - r0;
  const int ra = g->layout_a == 0;
  const uint16_t* As = A + (ra ? (size_t)r0 * g->lda : (size_t)r0);
  const uint16_t* Cs = C0 ? C0 + (size_t)r0 * g->ldc : NULL;
  return oracle_gemm_ref(&sub, As, B, Cs, out, nthreads);
}

static double max_abs_finite(const uint16_t* v, size_t n, int dtype) {
  double m = 0;
  for (size_t i = 0; i < n; ++i) {
    const double x = fabs(decode(v[i], dtype));
    if (isfinite(x) && x > m) m = x;
  }
  return m;
}

/* kind 0: reference form c*sqrt(K)*eps*...; kind 1: north-star form 2^-10*K*... */
ORACLE_API double oracle_tolerance(const oracle_gemm* g, const uint16_t* A, size_t nA, const uint16_t* B, size_t nB,
                                   const uint16_t* C0, size_t nC, double c, int kind) {
  const double eps = g->dtype == 1 ? 0.0078125 : 9.765625e-4;
  const double ma = max_abs_finite(A, nA, g->dtype), mb = max_abs_finite(B, nB, g->dtype);
  const double mc = (g->beta != 0.f && C0) ? max_abs_finite(C0, nC, g->dtype) : 0.0;
  const double beta_term = eps * fabs((double)g->beta) * mc;
  if (kind == 1) return eps * (double)g->K * ma * mb * fabs((double)g->alpha) + beta_term;
  return c * sqrt((double)g->K) * eps * ma * mb * fabs((double)g->alpha) + beta_term;
}

ORACLE_API int oracle_compare(const oracle_gemm* g, const uint16_t* out, size_t n_out, const double* ref,
                              const uint16_t* C0, double allowed, oracle_result* r) {
  const double overflow = g->dtype == 1 ? 3.3961775292304e38 : 65520.0; /* round-to-nearest overflow threshold */
  const double maxfin = g->dtype == 1 ? 3.3895313892515355e38 : 65504.0;
  memset(r, 0, sizeof *r);
  r->first_index = -1;
#define FAIL_AT(idx, got, want)     \
  do {                              \
    if (r->first_index < 0) {       \
      r->first_index = (long long)(idx); \
      r->first_got = (got);         \
      r->first_want = (want);       \
    }                               \
  } while (0)
  for (int b = 0; b < g->batch; ++b)
    for (int i = 0; i < g->M; ++i) {
      for (int j = 0; j < g->N; ++j) {
        const size_t oi = (size_t)(b * g->stride_c + i * g->ldc + j);
        if (oi >= n_out) { ++r->out_of_tol; FAIL_AT(oi, NAN, NAN); continue; }
        const double o = decode(out[oi], g->dtype);
        const double w = ref[((size_t)b * g->M + i) * g->N + j];
        ++r->checked;
        if (isnan(w)) {
          if (!isnan(o)) { ++r->nan_mismatch; FAIL_AT(oi, o, w); }
          continue;
        }
        if (isinf(w) || fabs(w) >= overflow) {
          const int same_inf = isinf(o) && ((o > 0) == (w > 0));
          const int near_max = isfinite(o) && fabs(fabs(w) - maxfin) <= allowed;
          if (!same_inf && !(isfinite(w) && near_max)) { ++r->inf_mismatch; FAIL_AT(oi, o, w); }
          continue;
        }
        if (!isfinite(o)) {
          if (!(isinf(o) && fabs(w) + allowed >= overflow)) { ++r->inf_mismatch; FAIL_AT(oi, o, w); }
          continue;
        }
        const double err = fabs(o - w);
        if (err > r->max_err) r->max_err = err;
        const double ratio = allowed > 0 ? err / allowed : (err > 0 ? INFINITY : 0.0);
        if (ratio > r->max_ratio) r->max_ratio = ratio;
        if (err > allowed) { ++r->out_of_tol; FAIL_AT(oi, o, w); }
      }
      if (C0)
        for (long long j = g->N; j < g->ldc; ++j) {
          const size_t oi = (size_t)(b * g->stride_c + i * g->ldc + j);
          if (oi < n_out && out[oi] != C0[oi]) {
            ++r->out_of_tol;
            FAIL_AT(oi, decode(out[oi], g->dtype), decode(C0[oi], g->dtype));
          }
        }
    }
#undef FAIL_AT
  r->pass = r->nan_mismatch == 0 && r->inf_mismatch == 0 && r->out_of_tol == 0;
  return 0;
}
