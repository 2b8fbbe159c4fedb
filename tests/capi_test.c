/* C ABI test, strict C11 against include/aegis/aegis.h (the drop-in include
 * path), linked with libaegis_capi.so. Covers what the reference's C ABI test
 * covers (tests/capi_test.c there): error paths, the size-query protocol of
 * the manifest and hardware JSON, the struct_size rule, and GEMMs against a
 * double-precision CPU reference, for f16 and the ABI 1.4 bf16 entry points,
 * every layout pair, padded leading dimensions, alpha/beta and strided batch,
 * plus the registry, plan and watchdog entry points. Exit status 0 = pass.
 * Needs a GPU; built and run by tests/test_capi_gpu.py. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "aegis/aegis.h"

static int failures = 0;

#define EXPECT(cond, ...)                                  \
  do {                                                     \
    if (!(cond)) {                                         \
      fprintf(stderr, "FAIL %s:%d: ", __FILE__, __LINE__); \
      fprintf(stderr, __VA_ARGS__);                        \
      fputc('\n', stderr);                                 \
      ++failures;                                          \
    }                                                      \
  } while (0)

/* 16-bit encodings, round to nearest even; enough for test data in [-1, 1]. */
static uint16_t to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
  if (ax >= 0x47800000u) return (uint16_t)(sign | 0x7c00u);
  if (ax < 0x38800000u) { /* subnormal */
    if (ax < 0x33000000u) return (uint16_t)sign;
    const uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u, sh = 126u - e;
    uint32_t h = m >> sh;
    const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1u);
    if (rem > half || (rem == half && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
  }
  uint32_t h = (((ax >> 23) - 112u) << 10) | ((ax & 0x7fffffu) >> 13);
  const uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return (uint16_t)(sign | h);
}
static uint16_t to_bf16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  x += 0x7fffu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}
static double from_f16(uint16_t h) {
  const int e = (h >> 10) & 0x1f, m = h & 0x3ff;
  double v = e == 0 ? ldexp(m, -24) : (e == 31 ? (m ? NAN : INFINITY) : ldexp(m | 0x400, e - 25));
  return (h & 0x8000) ? -v : v;
}
static double from_bf16(uint16_t h) {
  const uint32_t x = (uint32_t)h << 16;
  float f;
  memcpy(&f, &x, 4);
  return f;
}

static uint32_t lcg = 12345u;
static float frand(void) { /* uniform in [-1, 1) */
  lcg = lcg * 1664525u + 1013904223u;
  return (float)((lcg >> 8) & 0xffffff) / 8388608.0f - 1.0f;
}

static void test_errors(aegis_context* ctx) {
  EXPECT(aegis_create(NULL, 0) == AEGIS_ERR_INVALID_ARGUMENT, "create(NULL)");
  aegis_context* bad = NULL;
  EXPECT(aegis_create(&bad, 9999) == AEGIS_ERR_NO_DEVICE && bad == NULL, "create(9999)");
  EXPECT(aegis_destroy(NULL) == AEGIS_OK, "destroy(NULL)");
  EXPECT(aegis_gemm_f16(ctx, NULL, NULL, NULL, 1, 1, 1) == AEGIS_ERR_INVALID_ARGUMENT, "gemm with NULL operands");
  EXPECT(strlen(aegis_last_error_string()) > 0, "invalid argument sets aegis_last_error_string");
  void* p = NULL;
  EXPECT(aegis_device_alloc(ctx, 64, &p) == AEGIS_OK && p, "alloc");
  EXPECT(aegis_gemm_f16(ctx, p, p, p, 0, 4, 4) == AEGIS_OK, "M = 0 is a no-op");
  EXPECT(aegis_gemm_bf16(ctx, NULL, NULL, NULL, 4, 0, 4) == AEGIS_OK, "N = 0 with NULL operands is a no-op");
  EXPECT(aegis_gemm_f16(ctx, p, p, p, -1, 4, 4) == AEGIS_ERR_INVALID_ARGUMENT, "M < 0");
  EXPECT(aegis_gemm_f16_ex(ctx, 7, AEGIS_ROW_MAJOR, 4, 4, 4, 1.f, p, 4, p, 4, 0.f, p, 4) ==
             AEGIS_ERR_INVALID_ARGUMENT, "bad layout");
  EXPECT(aegis_gemm_bf16_ex(ctx, AEGIS_ROW_MAJOR, AEGIS_ROW_MAJOR, 4, 4, 8, 1.f, p, 4, p, 4, 0.f, p, 4) ==
             AEGIS_ERR_INVALID_ARGUMENT, "lda < K");
  EXPECT(aegis_gemm_f16_strided_batched(ctx, 0, 0, 4, 4, 4, 1.f, p, 4, 16, p, 4, 16, 0.f, p, 4, 8, 2) ==
             AEGIS_ERR_INVALID_ARGUMENT, "overlapping C batches");
  EXPECT(aegis_gemm_f16(NULL, p, p, p, 4, 4, 4) == AEGIS_ERR_INVALID_ARGUMENT, "ctx = NULL");
  /* Sizes above 2^31 - 2^20 are refused before anything is read (index headroom). */
  EXPECT(aegis_gemm_f16(ctx, p, p, p, 2147483647, 8, 8) == AEGIS_ERR_INVALID_ARGUMENT, "M = 2^31 - 1");
  EXPECT(aegis_gemm_bf16(ctx, p, p, p, 8, 8, 2147483000) == AEGIS_ERR_INVALID_ARGUMENT, "K near 2^31");
  EXPECT(aegis_gemm_impl(ctx, "no_such_kernel", AEGIS_DTYPE_F16, 0, 0, 4, 4, 4, 1.f, p, 4, 0, p, 4, 0, 0.f, p, 4,
                         0, 1) == AEGIS_ERR_INVALID_ARGUMENT, "unknown impl");
  EXPECT(aegis_device_free(ctx, p) == AEGIS_OK, "free");
  EXPECT(strcmp(aegis_status_string(AEGIS_ERR_CUDA), "unknown status") != 0, "status string");
  EXPECT(aegis_abi_version() == AEGIS_ABI_VERSION_MAJOR * 1000 + AEGIS_ABI_VERSION_MINOR, "abi version");
  EXPECT(aegis_abi_version() == 1004, "ABI 1.4");
}

static void test_manifest_and_hw(void) {
  size_t needed = 0;
  EXPECT(aegis_device_manifest(0, NULL, 0, &needed) == AEGIS_OK && needed > 1, "manifest size query");
  char small[8];
  EXPECT(aegis_device_manifest(0, small, sizeof small, &needed) == AEGIS_ERR_BUFFER_TOO_SMALL, "small buffer");
  char* buf = malloc(needed);
  size_t again = 0;
  EXPECT(buf && aegis_device_manifest(0, buf, needed, &again) == AEGIS_OK, "manifest fill");
  EXPECT(again == needed && strlen(buf) + 1 == needed, "manifest size stable");
  EXPECT(strstr(buf, "\"measured_d2d_bw_gbps\"") && strstr(buf, "\"sm_arch\":100"), "manifest keys");
  EXPECT(aegis_device_manifest(-1, buf, needed, NULL) == AEGIS_ERR_NO_DEVICE, "manifest bad device");
  free(buf);

  EXPECT(aegis_hw_info_json(0, NULL, 0, &needed) == AEGIS_OK && needed > 1, "hw json size query");
  buf = malloc(needed);
  EXPECT(buf && aegis_hw_info_json(0, buf, needed, &again) == AEGIS_OK && again == needed, "hw json fill");
  EXPECT(strstr(buf, "\"schema\":\"aegis-hw/1\"") && strstr(buf, "\"core_types\"") && strstr(buf, "\"nvdec\""),
         "hw json keys");
  EXPECT(aegis_hw_info_json(-2, NULL, 0, &needed) == AEGIS_ERR_NO_DEVICE, "hw json bad device");
  EXPECT(aegis_hw_info_json(-1, NULL, 0, &needed) == AEGIS_OK, "hw json host only");
  free(buf);

  aegis_hw_gpu_info g;
  memset(&g, 0, sizeof g);
  EXPECT(aegis_hw_gpu(0, &g) == AEGIS_ERR_INVALID_ARGUMENT, "hw gpu: struct_size unset");
  g.struct_size = sizeof g;
  EXPECT(aegis_hw_gpu(0, &g) == AEGIS_OK && g.present == 1 && g.arch == 100 && g.sm_count > 0 &&
             g.smem_per_block_optin >= g.smem_per_block && g.name[0] != 0,
         "hw gpu struct");
  unsigned char old[64];
  memset(old, 0xab, sizeof old);
  uint32_t old_size = 16;
  memcpy(old, &old_size, sizeof old_size);
  EXPECT(aegis_hw_gpu(0, (aegis_hw_gpu_info*)old) == AEGIS_OK && old[16] == 0xab && old[63] == 0xab,
         "hw gpu: a 16-byte struct_size is respected");
  aegis_hw_cpu_info c;
  memset(&c, 0, sizeof c);
  c.struct_size = sizeof c;
  EXPECT(aegis_hw_cpu(&c) == AEGIS_OK && c.logical_cpus > 0 && c.performance_cores > 0, "hw cpu struct");
}

/* One general GEMM through the C ABI, checked against a double reference
 * with the bound 4*sqrt(K)*eps*|alpha| + eps*|beta| (inputs in [-1, 1]). */
static void test_gemm_general(aegis_context* ctx, int bf16, int la, int lb, int M, int N, int K, float alpha,
                              float beta, int batch, const char* impl) {
  const int64_t lda = (la == AEGIS_ROW_MAJOR ? K : M) + 3, ldb = (lb == AEGIS_ROW_MAJOR ? N : K) + 5;
  const int64_t ldc = N + 2;
  const int64_t sa = lda * (la == AEGIS_ROW_MAJOR ? M : K) + 1, sb = ldb * (lb == AEGIS_ROW_MAJOR ? K : N) + 7;
  const int64_t sc = ldc * M;
  const size_t nA = (size_t)(sa * batch), nB = (size_t)(sb * batch), nC = (size_t)(sc * batch);
  uint16_t* hA = malloc(nA * 2);
  uint16_t* hB = malloc(nB * 2);
  uint16_t* hC = malloc(nC * 2);
  uint16_t* hC0 = malloc(nC * 2);
  for (size_t i = 0; i < nA; ++i) hA[i] = bf16 ? to_bf16(frand()) : to_f16(frand());
  for (size_t i = 0; i < nB; ++i) hB[i] = bf16 ? to_bf16(frand()) : to_f16(frand());
  for (size_t i = 0; i < nC; ++i) hC0[i] = bf16 ? to_bf16(frand()) : to_f16(frand());
  void *dA = NULL, *dB = NULL, *dC = NULL;
  int s = aegis_device_alloc(ctx, nA * 2, &dA);
  if (s == AEGIS_OK) s = aegis_device_alloc(ctx, nB * 2, &dB);
  if (s == AEGIS_OK) s = aegis_device_alloc(ctx, nC * 2, &dC);
  if (s == AEGIS_OK) s = aegis_copy_to_device(ctx, dA, hA, nA * 2);
  if (s == AEGIS_OK) s = aegis_copy_to_device(ctx, dB, hB, nB * 2);
  if (s == AEGIS_OK) s = aegis_copy_to_device(ctx, dC, hC0, nC * 2);
  if (s == AEGIS_OK) {
    if (impl)
      s = aegis_gemm_impl(ctx, impl, bf16 ? AEGIS_DTYPE_BF16 : AEGIS_DTYPE_F16, la, lb, M, N, K, alpha, dA, lda, sa,
                          dB, ldb, sb, beta, dC, ldc, sc, batch);
    else if (batch == 1)
      s = bf16 ? aegis_gemm_bf16_ex(ctx, la, lb, M, N, K, alpha, dA, lda, dB, ldb, beta, dC, ldc)
               : aegis_gemm_f16_ex(ctx, la, lb, M, N, K, alpha, dA, lda, dB, ldb, beta, dC, ldc);
    else
      s = bf16 ? aegis_gemm_bf16_strided_batched(ctx, la, lb, M, N, K, alpha, dA, lda, sa, dB, ldb, sb, beta, dC,
                                                 ldc, sc, batch)
               : aegis_gemm_f16_strided_batched(ctx, la, lb, M, N, K, alpha, dA, lda, sa, dB, ldb, sb, beta, dC,
                                                ldc, sc, batch);
  }
  if (s == AEGIS_OK) s = aegis_synchronize(ctx);
  if (s == AEGIS_OK) s = aegis_copy_to_host(ctx, hC, dC, nC * 2);
  EXPECT(s == AEGIS_OK, "gemm_general %s: %s (%s)", impl ? impl : "dispatch", aegis_status_string(s),
         aegis_last_error_string());
  const double eps = bf16 ? 0.0078125 : 9.765625e-4;
  double worst = 0;
  for (int b = 0; s == AEGIS_OK && b < batch; ++b)
    for (int i = 0; i < M; ++i)
      for (int j = 0; j < N; ++j) {
        double ref = 0;
        for (int k = 0; k < K; ++k) {
          const uint16_t a = hA[b * sa + (la == AEGIS_ROW_MAJOR ? i * lda + k : i + k * lda)];
          const uint16_t x = hB[b * sb + (lb == AEGIS_ROW_MAJOR ? k * ldb + j : k + j * ldb)];
          ref += (bf16 ? from_bf16(a) : from_f16(a)) * (bf16 ? from_bf16(x) : from_f16(x));
        }
        const size_t c = (size_t)(b * sc + i * ldc + j);
        ref = (alpha == 0.f ? 0.0 : alpha * ref) + (beta != 0.f ? beta * (bf16 ? from_bf16(hC0[c]) : from_f16(hC0[c])) : 0.0);
        const double tol = 4.0 * sqrt((double)K) * eps * fabs(alpha) + eps * fabs(beta) + 1e-7;
        const double got = bf16 ? from_bf16(hC[c]) : from_f16(hC[c]);
        const double err = isfinite(got) ? fabs(got - ref) : INFINITY;
        if (err / tol > worst) worst = err / tol;
      }
  int pad_ok = 1;
  for (int b = 0; b < batch; ++b)
    for (int i = 0; i < M; ++i)
      for (int64_t j = N; j < ldc; ++j) pad_ok &= hC[b * sc + i * ldc + j] == hC0[b * sc + i * ldc + j];
  printf("%-4s %-24s %s %s%s %4dx%4dx%4d batch %d alpha %5.2f beta %5.2f err/tol=%.3f\n",
         worst <= 1.0 && pad_ok ? "ok" : "FAIL", impl ? impl : "dispatch", bf16 ? "bf16" : "f16 ",
         la == AEGIS_ROW_MAJOR ? "R" : "C", lb == AEGIS_ROW_MAJOR ? "R" : "C", M, N, K, batch, alpha, beta, worst);
  EXPECT(worst <= 1.0, "gemm_general err/tol %.3f", worst);
  EXPECT(pad_ok, "gemm_general wrote C padding");
  aegis_device_free(ctx, dA);
  aegis_device_free(ctx, dB);
  aegis_device_free(ctx, dC);
  free(hA);
  free(hB);
  free(hC);
  free(hC0);
}

static void test_registry_and_plan(aegis_context* ctx) {
  size_t needed = 0;
  EXPECT(aegis_registry_json(ctx, NULL, 0, &needed) == AEGIS_OK && needed > 2, "registry size query");
  char* buf = malloc(needed);
  EXPECT(buf && aegis_registry_json(ctx, buf, needed, NULL) == AEGIS_OK, "registry fill");
  EXPECT(strstr(buf, "\"umma_128x256x64_s4_ksm\"") && strstr(buf, "\"gemv_256x256_ksm\"") &&
             strstr(buf, "\"simt_64x64x16\""),
         "registry names");
  EXPECT(strstr(buf, "\"supported\":false") == NULL, "every registry entry runs on this B200: %s", buf);
  free(buf);
  char plan[256];
  EXPECT(aegis_gemm_plan_json(ctx, "umma_128x256x64_s4_ksm", AEGIS_DTYPE_BF16, 256, 256, 65536, plan, sizeof plan,
                              NULL) == AEGIS_OK && strstr(plan, "\"splits\":1,") == NULL,
         "tall-K plan splits: %s", plan);
  EXPECT(aegis_gemm_plan_json(ctx, NULL, AEGIS_DTYPE_BF16, 8192, 8192, 8192, plan, sizeof plan, NULL) == AEGIS_OK &&
             strstr(plan, "\"splits\":1,"),
         "8192^3 does not split: %s", plan);
  char choice[64];
  EXPECT(aegis_gemm_choice(ctx, 1, 4096, 4096, choice, sizeof choice, NULL) == AEGIS_OK &&
             (strncmp(choice, "ummav_", 6) == 0 || strncmp(choice, "gemv_", 5) == 0),
         "decode shape dispatches to a decode kernel: %s", choice);
  EXPECT(aegis_gemm_choice(ctx, 4096, 4096, 4096, choice, sizeof choice, NULL) == AEGIS_OK &&
             strncmp(choice, "umma_", 5) == 0,
         "square shape dispatches to umma: %s", choice);
}

static void test_watchdog(aegis_context* ctx) {
  EXPECT(aegis_watchdog_selftest(ctx, 10) == AEGIS_ERR_INVALID_ARGUMENT, "watchdog limit range");
  EXPECT(aegis_watchdog_selftest(ctx, 20000000) == AEGIS_OK, "watchdog: a wait that never completes returns: %s",
         aegis_last_error_string());
  EXPECT(aegis_synchronize(ctx) == AEGIS_OK, "context usable after the watchdog test");
}

int main(void) {
  aegis_context* ctx = NULL;
  if (aegis_create(&ctx, 0) != AEGIS_OK) {
    fprintf(stderr, "aegis_create: %s\n", aegis_last_error_string());
    return 1;
  }
  test_errors(ctx);
  test_manifest_and_hw();
  test_registry_and_plan(ctx);
  test_watchdog(ctx);
  const char* impls[] = {NULL, "umma_128x256x64_s4", "umma_128x128x64_s6", "umma_128x256x64_s4_ksm",
                         "umma_128x128x64_s6_ksm", "umma_256x256x64_s7_c2", "umma_256x256x64_s7_c2_ksm",
                         "umma_128x64x64_s8", "umma_128x64x64_s8_ksm",
                         "gemv_256x256_ksm", "gemv_64x256_ksm", "ummav_128x16x64_s11", "ummav_128x16x64_s6x2",
                         "simt_64x64x16"};
  for (int bf16 = 0; bf16 < 2; ++bf16)
    for (int la = 0; la < 2; ++la)
      for (int lb = 0; lb < 2; ++lb) {
        test_gemm_general(ctx, bf16, la, lb, 67, 45, 91, 1.f, 0.f, 1, NULL);
        test_gemm_general(ctx, bf16, la, lb, 13, 40, 130, -0.5f, 0.75f, 1, NULL);
        test_gemm_general(ctx, bf16, la, lb, 5, 33, 205, 2.f, 1.f, 3, NULL);
      }
  for (size_t i = 0; i < sizeof impls / sizeof impls[0]; ++i) {
    test_gemm_general(ctx, 0, AEGIS_ROW_MAJOR, AEGIS_ROW_MAJOR, 131, 260, 200, 1.f, 0.f, 1, impls[i]);
    test_gemm_general(ctx, 1, AEGIS_COL_MAJOR, AEGIS_ROW_MAJOR, 9, 100, 333, 0.5f, -1.f, 2, impls[i]);
  }
  /* alpha == 0: C = beta * C */
  test_gemm_general(ctx, 0, AEGIS_ROW_MAJOR, AEGIS_ROW_MAJOR, 20, 30, 40, 0.f, 0.5f, 1, NULL);
  EXPECT(aegis_destroy(ctx) == AEGIS_OK, "destroy");
  printf("%s (%d failures)\n", failures ? "capi_test: FAILED" : "capi_test: all passed", failures);
  return failures ? 1 : 0;
}
