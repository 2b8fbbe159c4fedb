// C ABI (include/aegis.h) over aegis::matmul. Mirrors the reference's
// src/capi.cpp (context, thread-local error detail, run_gemm error mapping,
// size-query protocol) and adds the ABI 1.4 entry points.
//
// Every entry point validates its arguments and turns CUDA and launch errors
// into status codes. Nothing here exits the process.
#include "aegis.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <new>
#include <string>

#include "aegis/gemm.h"
#include "aegis/matmul.h"
#include "capi_error.h"
#include "common.cuh"
#include "gpu_target.h"
#include "kernels.h"
#include "status.h"

struct aegis_context {
  int device = 0;
  cudaStream_t own = nullptr;     // created by aegis_create
  cudaStream_t stream = nullptr;  // own, or the caller's
  std::string last_error;
};

namespace {

thread_local std::string t_error;  // aegis_last_error_string()

int fail(int status, const std::string& detail) {
  t_error = detail;
  return status;
}

}  // namespace

namespace aegis::capi {
void set_error(const std::string& detail) { t_error = detail; }
}  // namespace aegis::capi

namespace {

int fail_arg(const char* fn, const char* what) { return fail(AEGIS_ERR_INVALID_ARGUMENT, std::string(fn) + ": " + what); }

int fail_cuda(aegis_context* ctx, cudaError_t e, const char* fn) {
  if (ctx) ctx->last_error = cudaGetErrorString(e);
  cudaGetLastError();  // clear a non-sticky error so it does not leak into the next call
  return fail(e == cudaErrorMemoryAllocation ? AEGIS_ERR_OUT_OF_MEMORY : AEGIS_ERR_CUDA,
              std::string(fn) + ": " + cudaGetErrorString(e));
}

int enter(aegis_context* ctx, const char* fn) {
  if (!ctx) return fail_arg(fn, "context is NULL");
  const cudaError_t e = cudaSetDevice(ctx->device);
  return e == cudaSuccess ? AEGIS_OK : fail_cuda(ctx, e, fn);
}

int run_gemm(aegis_context* ctx, const aegis::gemm::GemmParams& p, const char* fn) {
  if (int s = enter(ctx, fn)) return s;
  if (aegis::gemm::validate(p) != cudaSuccess)
    return fail_arg(fn, "negative size or a size above 2^31 - 2^20, too-small leading dimension, null operand, "
                        "bad layout or overlapping C batches");
  if (aegis::gemm::is_empty(p)) return AEGIS_OK;
  const cudaError_t e = aegis::matmul(p, ctx->stream);
  if (e == cudaSuccess) return AEGIS_OK;
  ctx->last_error = cudaGetErrorString(e);
  cudaGetLastError();
  const std::string detail = aegis::matmul_last_error();
  if (e == cudaErrorMemoryAllocation) return fail(AEGIS_ERR_OUT_OF_MEMORY, detail);
  if (e == cudaErrorStreamCaptureUnsupported) return fail(AEGIS_ERR_CUDA, detail);
  return fail(AEGIS_ERR_LAUNCH_FAILED, detail);
}

bool to_layout(int l, aegis::gemm::Layout* out) {
  if (l == AEGIS_ROW_MAJOR) *out = aegis::gemm::Layout::RowMajor;
  else if (l == AEGIS_COL_MAJOR) *out = aegis::gemm::Layout::ColMajor;
  else return false;
  return true;
}

int gemm_general(aegis_context* ctx, aegis::gemm::DType dt, int layout_a, int layout_b, int M, int N, int K,
                 float alpha, const void* A, int64_t lda, int64_t stride_a, const void* B, int64_t ldb,
                 int64_t stride_b, float beta, void* C, int64_t ldc, int64_t stride_c, int batch, const char* fn) {
  aegis::gemm::GemmParams p;
  if (!to_layout(layout_a, &p.layout_a) || !to_layout(layout_b, &p.layout_b))
    return fail_arg(fn, "layout must be AEGIS_ROW_MAJOR or AEGIS_COL_MAJOR");
  p.A = A;
  p.B = B;
  p.C = C;
  p.M = M; p.N = N; p.K = K;
  p.lda = lda; p.ldb = ldb; p.ldc = ldc;
  p.alpha = alpha; p.beta = beta;
  p.batch = batch;
  p.stride_a = stride_a; p.stride_b = stride_b; p.stride_c = stride_c;
  p.dtype = dt;
  return run_gemm(ctx, p, fn);
}

int copy_out(const std::string& s, char* buf, size_t buf_len, size_t* needed) {
  if (needed) *needed = s.size() + 1;
  if (!buf && buf_len == 0) return AEGIS_OK;  // size query
  if (!buf) return fail(AEGIS_ERR_INVALID_ARGUMENT, "buf is NULL but buf_len is not 0");
  if (buf_len < s.size() + 1) return fail(AEGIS_ERR_BUFFER_TOO_SMALL, "buffer too small (see needed)");
  std::memcpy(buf, s.c_str(), s.size() + 1);
  return AEGIS_OK;
}

int nsharded(aegis_context* ctx, aegis::gemm::DType dt, int M, int N, int K, const void* A, int64_t lda,
             const void* B_shard, int64_t ldb, void* const* c_ranks, int64_t ldc, int nranks, int rank,
             const char* fn) {
  if (int s = enter(ctx, fn)) return s;
  if (nranks < 1 || nranks > 8 || rank < 0 || rank >= nranks) return fail_arg(fn, "need 1 <= nranks <= 8, 0 <= rank < nranks");
  if (M < 0 || N < 0 || K < 0) return fail_arg(fn, "negative size");
  if (M == 0 || N == 0 || K == 0) return AEGIS_OK;
  if (N % nranks != 0) return fail_arg(fn, "N must divide evenly by nranks");
  if (!c_ranks) return fail_arg(fn, "c_ranks is NULL");
  for (int i = 0; i < nranks; ++i)
    if (!c_ranks[i]) return fail_arg(fn, "a c_ranks entry is NULL");
  const int ns = N / nranks;
  aegis::gemm::GemmParams p;
  p.A = A;
  p.B = B_shard;
  p.C = c_ranks[rank];
  p.M = M; p.N = ns; p.K = K;
  p.lda = lda; p.ldb = ldb; p.ldc = ldc;
  p.dtype = dt;
  if (aegis::gemm::validate(p) != cudaSuccess || ldc < N)
    return fail_arg(fn, "null operand or too-small leading dimension (ldc must be >= N)");
  if (!aegis::gemm::tma_compatible(p))
    return fail_arg(fn, "A and B_shard must be 16-byte aligned with lda, ldb multiples of 8");
  const cudaError_t e = aegis::umma_nsharded(p, c_ranks, nranks, rank * ns, ctx->stream);
  if (e == cudaSuccess) return AEGIS_OK;
  ctx->last_error = cudaGetErrorString(e);
  cudaGetLastError();
  if (e == cudaErrorNotSupported) return fail(AEGIS_ERR_LAUNCH_FAILED, std::string(fn) + ": needs an sm_100 device");
  return fail(AEGIS_ERR_LAUNCH_FAILED, std::string(fn) + ": " + cudaGetErrorString(e));
}

}  // namespace

extern "C" {

int aegis_abi_version(void) { return AEGIS_ABI_VERSION_MAJOR * 1000 + AEGIS_ABI_VERSION_MINOR; }

const char* aegis_last_error_string(void) { return t_error.c_str(); }

const char* aegis_status_string(int status) {
  switch (status) {
    case AEGIS_OK: return "ok";
    case AEGIS_ERR_INVALID_ARGUMENT: return "invalid argument";
    case AEGIS_ERR_CUDA: return "CUDA error (see aegis_last_error)";
    case AEGIS_ERR_BUFFER_TOO_SMALL: return "buffer too small (see needed)";
    case AEGIS_ERR_NO_DEVICE: return "no such CUDA device";
    case AEGIS_ERR_OUT_OF_MEMORY: return "out of device memory";
    case AEGIS_ERR_LAUNCH_FAILED: return "kernel launch failed (see aegis_last_error_string)";
    default: return "unknown status";
  }
}

int aegis_create(aegis_context** out, int device) {
  if (!out) return fail_arg("aegis_create", "out is NULL");
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    cudaGetLastError();
    return fail(AEGIS_ERR_NO_DEVICE, "aegis_create: no such CUDA device");
  }
  auto* ctx = new (std::nothrow) aegis_context;
  if (!ctx) return fail(AEGIS_ERR_OUT_OF_MEMORY, "aegis_create: out of host memory");
  ctx->device = device;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->own, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    const int s = fail_cuda(nullptr, e, "aegis_create");
    delete ctx;
    return s;
  }
  ctx->stream = ctx->own;
  *out = ctx;
  return AEGIS_OK;
}

int aegis_destroy(aegis_context* ctx) {
  if (!ctx) return AEGIS_OK;
  int status = AEGIS_OK;
  if (cudaSetDevice(ctx->device) == cudaSuccess && ctx->own) {
    if (cudaStreamSynchronize(ctx->own) != cudaSuccess || cudaStreamDestroy(ctx->own) != cudaSuccess) {
      status = AEGIS_ERR_CUDA;
      cudaGetLastError();
    }
  }
  delete ctx;
  return status;
}

int aegis_set_stream(aegis_context* ctx, void* cuda_stream) {
  if (!ctx) return fail_arg("aegis_set_stream", "context is NULL");
  ctx->stream = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : ctx->own;
  return AEGIS_OK;
}

int aegis_synchronize(aegis_context* ctx) {
  if (int s = enter(ctx, "aegis_synchronize")) return s;
  const cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return fail_cuda(ctx, e, "aegis_synchronize");
  unsigned bits = 0, block = 0;
  if (const cudaError_t e2 = aegis::status::take(&bits, &block); e2 != cudaSuccess)
    return fail_cuda(ctx, e2, "aegis_synchronize");
  if (bits != 0) {
    char buf[160];
    std::snprintf(buf, sizeof buf,
                  "aegis_synchronize: kernel watchdog fired (status bits 0x%x, first block %u): a bounded wait "
                  "ran out; that launch's output is not valid",
                  bits, block ? block - 1 : 0);
    ctx->last_error = buf;
    return fail(AEGIS_ERR_CUDA, buf);
  }
  return AEGIS_OK;
}

const char* aegis_last_error(const aegis_context* ctx) { return ctx ? ctx->last_error.c_str() : ""; }

int aegis_device_alloc(aegis_context* ctx, size_t bytes, void** out) {
  if (!out || bytes == 0) return fail_arg("aegis_device_alloc", "out is NULL or bytes is 0");
  *out = nullptr;
  if (int s = enter(ctx, "aegis_device_alloc")) return s;
  const cudaError_t e = cudaMalloc(out, bytes);
  return e == cudaSuccess ? AEGIS_OK : fail_cuda(ctx, e, "aegis_device_alloc");
}

int aegis_device_free(aegis_context* ctx, void* ptr) {
  if (!ptr) return ctx ? AEGIS_OK : fail_arg("aegis_device_free", "context is NULL");
  if (int s = enter(ctx, "aegis_device_free")) return s;
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? AEGIS_OK : fail_cuda(ctx, e, "aegis_device_free");
}

static int copy(aegis_context* ctx, void* dst, const void* src, size_t bytes, cudaMemcpyKind kind, const char* fn) {
  if (!dst || !src) return fail_arg(fn, "NULL pointer");
  if (int s = enter(ctx, fn)) return s;
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, kind, ctx->stream);  // ordered after queued GEMMs
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  return e == cudaSuccess ? AEGIS_OK : fail_cuda(ctx, e, fn);
}

int aegis_copy_to_device(aegis_context* ctx, void* dst, const void* src, size_t bytes) {
  return copy(ctx, dst, src, bytes, cudaMemcpyHostToDevice, "aegis_copy_to_device");
}

int aegis_copy_to_host(aegis_context* ctx, void* dst, const void* src, size_t bytes) {
  return copy(ctx, dst, src, bytes, cudaMemcpyDeviceToHost, "aegis_copy_to_host");
}

int aegis_gemm_f16(aegis_context* ctx, const void* A, const void* B, void* C, int M, int N, int K) {
  return run_gemm(ctx, aegis::gemm::row_major_params(A, B, C, M, N, K, aegis::gemm::DType::F16), "aegis_gemm_f16");
}

int aegis_gemm_f16_strided_batched(aegis_context* ctx, int layout_a, int layout_b, int M, int N, int K, float alpha,
                                   const void* A, int64_t lda, int64_t stride_a, const void* B, int64_t ldb,
                                   int64_t stride_b, float beta, void* C, int64_t ldc, int64_t stride_c, int batch) {
  return gemm_general(ctx, aegis::gemm::DType::F16, layout_a, layout_b, M, N, K, alpha, A, lda, stride_a, B, ldb,
                      stride_b, beta, C, ldc, stride_c, batch, "aegis_gemm_f16_strided_batched");
}

int aegis_gemm_f16_ex(aegis_context* ctx, int layout_a, int layout_b, int M, int N, int K, float alpha, const void* A,
                      int64_t lda, const void* B, int64_t ldb, float beta, void* C, int64_t ldc) {
  return gemm_general(ctx, aegis::gemm::DType::F16, layout_a, layout_b, M, N, K, alpha, A, lda, 0, B, ldb, 0, beta, C,
                      ldc, 0, 1, "aegis_gemm_f16_ex");
}

int aegis_gemm_bf16(aegis_context* ctx, const void* A, const void* B, void* C, int M, int N, int K) {
  return run_gemm(ctx, aegis::gemm::row_major_params(A, B, C, M, N, K, aegis::gemm::DType::BF16), "aegis_gemm_bf16");
}

int aegis_gemm_bf16_strided_batched(aegis_context* ctx, int layout_a, int layout_b, int M, int N, int K, float alpha,
                                    const void* A, int64_t lda, int64_t stride_a, const void* B, int64_t ldb,
                                    int64_t stride_b, float beta, void* C, int64_t ldc, int64_t stride_c, int batch) {
  return gemm_general(ctx, aegis::gemm::DType::BF16, layout_a, layout_b, M, N, K, alpha, A, lda, stride_a, B, ldb,
                      stride_b, beta, C, ldc, stride_c, batch, "aegis_gemm_bf16_strided_batched");
}

int aegis_gemm_bf16_ex(aegis_context* ctx, int layout_a, int layout_b, int M, int N, int K, float alpha, const void* A,
                       int64_t lda, const void* B, int64_t ldb, float beta, void* C, int64_t ldc) {
  return gemm_general(ctx, aegis::gemm::DType::BF16, layout_a, layout_b, M, N, K, alpha, A, lda, 0, B, ldb, 0, beta, C,
                      ldc, 0, 1, "aegis_gemm_bf16_ex");
}

int aegis_gemm_choice(aegis_context* ctx, int M, int N, int K, char* buf, size_t buf_len, size_t* needed) {
  if (M <= 0 || N <= 0 || K <= 0) return fail_arg("aegis_gemm_choice", "M, N and K must be positive");
  if (int s = enter(ctx, "aegis_gemm_choice")) return s;
  return copy_out(aegis::matmul_choice(M, N, K), buf, buf_len, needed);
}

int aegis_gemm_bf16_nsharded(aegis_context* ctx, int M, int N, int K, const void* A, int64_t lda, const void* B_shard,
                             int64_t ldb, void* const* c_ranks, int64_t ldc, int nranks, int rank) {
  return nsharded(ctx, aegis::gemm::DType::BF16, M, N, K, A, lda, B_shard, ldb, c_ranks, ldc, nranks, rank,
                  "aegis_gemm_bf16_nsharded");
}

int aegis_gemm_f16_nsharded(aegis_context* ctx, int M, int N, int K, const void* A, int64_t lda, const void* B_shard,
                            int64_t ldb, void* const* c_ranks, int64_t ldc, int nranks, int rank) {
  return nsharded(ctx, aegis::gemm::DType::F16, M, N, K, A, lda, B_shard, ldb, c_ranks, ldc, nranks, rank,
                  "aegis_gemm_f16_nsharded");
}

int aegis_ipc_get_handle(aegis_context* ctx, const void* dptr, void* handle) {
  if (!dptr || !handle) return fail_arg("aegis_ipc_get_handle", "NULL pointer");
  if (int s = enter(ctx, "aegis_ipc_get_handle")) return s;
  static_assert(sizeof(cudaIpcMemHandle_t) == AEGIS_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dptr));
  if (e != cudaSuccess) return fail_cuda(ctx, e, "aegis_ipc_get_handle");
  std::memcpy(handle, &h, sizeof h);
  return AEGIS_OK;
}

int aegis_ipc_open_handle(aegis_context* ctx, const void* handle, void** dptr) {
  if (!handle || !dptr) return fail_arg("aegis_ipc_open_handle", "NULL pointer");
  *dptr = nullptr;
  if (int s = enter(ctx, "aegis_ipc_open_handle")) return s;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  const cudaError_t e = cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? AEGIS_OK : fail_cuda(ctx, e, "aegis_ipc_open_handle");
}

int aegis_ipc_close_handle(aegis_context* ctx, void* dptr) {
  if (!dptr) return fail_arg("aegis_ipc_close_handle", "NULL pointer");
  if (int s = enter(ctx, "aegis_ipc_close_handle")) return s;
  const cudaError_t e = cudaIpcCloseMemHandle(dptr);
  return e == cudaSuccess ? AEGIS_OK : fail_cuda(ctx, e, "aegis_ipc_close_handle");
}

int aegis_gemm_impl(aegis_context* ctx, const char* impl, int dtype, int layout_a, int layout_b, int M, int N, int K,
                    float alpha, const void* A, int64_t lda, int64_t stride_a, const void* B, int64_t ldb,
                    int64_t stride_b, float beta, void* C, int64_t ldc, int64_t stride_c, int batch) {
  const char* fn = "aegis_gemm_impl";
  if (!impl) return fail_arg(fn, "impl is NULL");
  if (dtype != AEGIS_DTYPE_F16 && dtype != AEGIS_DTYPE_BF16) return fail_arg(fn, "dtype must be AEGIS_DTYPE_F16 or AEGIS_DTYPE_BF16");
  if (int s = enter(ctx, fn)) return s;
  const aegis::gemm::KernelEntry* e = aegis::gemm::find(impl);
  if (!e || !e->run) return fail_arg(fn, "no such kernel configuration in the registry");
  aegis::gemm::GemmParams p;
  if (!to_layout(layout_a, &p.layout_a) || !to_layout(layout_b, &p.layout_b))
    return fail_arg(fn, "layout must be AEGIS_ROW_MAJOR or AEGIS_COL_MAJOR");
  p.A = A; p.B = B; p.C = C;
  p.M = M; p.N = N; p.K = K;
  p.lda = lda; p.ldb = ldb; p.ldc = ldc;
  p.alpha = alpha; p.beta = beta;
  p.batch = batch;
  p.stride_a = stride_a; p.stride_b = stride_b; p.stride_c = stride_c;
  p.dtype = dtype == AEGIS_DTYPE_BF16 ? aegis::gemm::DType::BF16 : aegis::gemm::DType::F16;
  if (aegis::gemm::validate(p) != cudaSuccess)
    return fail_arg(fn, "negative size or a size above 2^31 - 2^20, too-small leading dimension, null operand, "
                        "bad layout or overlapping C batches");
  if (aegis::gemm::is_empty(p)) return AEGIS_OK;
  const cudaError_t err = e->run(p, ctx->stream);
  if (err == cudaSuccess) return AEGIS_OK;
  ctx->last_error = cudaGetErrorString(err);
  cudaGetLastError();
  const std::string detail = std::string(fn) + ": launch " + impl + ": " + cudaGetErrorString(err);
  if (err == cudaErrorMemoryAllocation) return fail(AEGIS_ERR_OUT_OF_MEMORY, detail);
  if (err == cudaErrorStreamCaptureUnsupported) return fail(AEGIS_ERR_CUDA, detail);
  return fail(AEGIS_ERR_LAUNCH_FAILED, detail);
}

int aegis_registry_json(aegis_context* ctx, char* buf, size_t buf_len, size_t* needed) {
  if (int s = enter(ctx, "aegis_registry_json")) return s;
  const aegis::gemm::DeviceCaps caps = aegis::gemm::current_caps();
  std::string j = "[";
  bool first = true;
  for (const aegis::gemm::KernelEntry& e : aegis::gemm::registry()) {
    std::string why;
    const bool ok = aegis::gemm::supported(e, caps, &why);
    if (!first) j += ",";
    first = false;
    j += std::string("{\"name\":\"") + e.name + "\",\"config\":" + e.config + ",\"tune_max_m\":" +
         std::to_string(e.tune_max_m) + ",\"regs\":" + std::to_string(e.req.regs) + ",\"smem_bytes\":" +
         std::to_string(e.req.smem_bytes) + ",\"supported\":" + (ok ? "true" : "false") + ",\"why\":\"" + why + "\"}";
  }
  j += "]";
  return copy_out(j, buf, buf_len, needed);
}

int aegis_gemm_plan_json(aegis_context* ctx, const char* impl, int dtype, int M, int N, int K, char* buf,
                         size_t buf_len, size_t* needed) {
  const char* fn = "aegis_gemm_plan_json";
  if (M <= 0 || N <= 0 || K <= 0) return fail_arg(fn, "M, N and K must be positive");
  if (M > aegis::gemm::kMaxDim || N > aegis::gemm::kMaxDim || K > aegis::gemm::kMaxDim)
    return fail_arg(fn, "M, N and K must be at most 2^31 - 2^20");
  if (dtype != AEGIS_DTYPE_F16 && dtype != AEGIS_DTYPE_BF16) return fail_arg(fn, "bad dtype");
  if (int s = enter(ctx, fn)) return s;
  static const char dummy[16] alignas(16) = {};
  aegis::gemm::GemmParams p = aegis::gemm::row_major_params(
      dummy, dummy, const_cast<char*>(dummy), M, N, K,
      dtype == AEGIS_DTYPE_BF16 ? aegis::gemm::DType::BF16 : aegis::gemm::DType::F16);
  const char* name = impl ? impl : aegis::matmul_choice(p);
  aegis::gemm::LaunchPlan pl;
  if (!aegis::gemm::find(name)) return fail_arg(fn, "no such kernel configuration in the registry");
  if (!aegis::gemm::launch_plan(name, p, &pl)) pl = aegis::gemm::LaunchPlan{};
  char b[384];
  std::snprintf(b, sizeof b, "{\"impl\":\"%s\",\"splits\":%d,\"k_chunk\":%d,\"tiles\":%lld,\"grid\":%u,\"kdir_wave\":%d}", name,
                pl.splits, pl.k_chunk, pl.tiles, pl.grid, pl.kdir_wave);
  return copy_out(b, buf, buf_len, needed);
}

int aegis_plan_simulated_json(int arch, int sm_count, const char* impl, int dtype, int M, int N, int K, char* buf,
                              size_t buf_len, size_t* needed) {
  const char* fn = "aegis_plan_simulated_json";
  if (M <= 0 || N <= 0 || K <= 0) return fail_arg(fn, "M, N and K must be positive");
  if (M > aegis::gemm::kMaxDim || N > aegis::gemm::kMaxDim || K > aegis::gemm::kMaxDim)
    return fail_arg(fn, "M, N and K must be at most 2^31 - 2^20");
  if (dtype != AEGIS_DTYPE_F16 && dtype != AEGIS_DTYPE_BF16) return fail_arg(fn, "bad dtype");
  if (arch <= 0 || sm_count <= 0 || sm_count > 4096) return fail_arg(fn, "arch and sm_count must be positive");
  // A B200's per-CTA limits, with the given compute capability and SM count.
  aegis::gpu::Target model;
  model.cc = arch;
  model.sms = sm_count;
  model.smem_optin = 232448;
  model.regs_per_cta = 65536;
  model.threads_per_cta = 1024;
  const aegis::gpu::PlanOn scope(model);
  static const char dummy[16] alignas(16) = {};
  const aegis::gemm::GemmParams p = aegis::gemm::row_major_params(
      dummy, dummy, const_cast<char*>(dummy), M, N, K,
      dtype == AEGIS_DTYPE_BF16 ? aegis::gemm::DType::BF16 : aegis::gemm::DType::F16);
  const aegis::gemm::DeviceCaps caps = aegis::gemm::current_caps();
  const aegis::detail::Choice c = aegis::detail::choose(aegis::detail::winners_table(), p, caps);
  const char* chosen = c.kernel ? c.kernel->name : "none";
  const char* name = impl ? impl : chosen;
  aegis::gemm::LaunchPlan pl;
  if (impl && std::strcmp(impl, "gemv_noalloc") == 0) {
    // The plan of aegis_gemv_noalloc (not a registry kernel).
    if (M > aegis::kNoAllocMaxM || N > aegis::kNoAllocMaxN || !aegis::gemv_noalloc_plan(p, &pl))
      return fail_arg(fn, "outside the limits of aegis_gemv_noalloc");
  } else {
    if (!aegis::gemm::find(name)) return fail_arg(fn, "no such kernel configuration in the registry");
    if (!aegis::gemm::launch_plan(name, p, &pl)) pl = aegis::gemm::LaunchPlan{};
  }
  char b[384];
  std::snprintf(b, sizeof b,
                "{\"impl\":\"%s\",\"splits\":%d,\"k_chunk\":%d,\"tiles\":%lld,\"grid\":%u,\"kdir_wave\":%d,\"dispatch\":\"%s\","
                "\"kind\":\"%s\"}",
                name, pl.splits, pl.k_chunk, pl.tiles, pl.grid, pl.kdir_wave, chosen,
                c.kind == aegis::detail::Choice::Kind::Aegis ? "winner" : "rule");
  return copy_out(b, buf, buf_len, needed);
}

int aegis_gemv_noalloc(aegis_context* ctx, int dtype, int layout_a, int layout_b, int M, int N, int K, float alpha,
                       const void* A, int64_t lda, const void* B, int64_t ldb, float beta, void* C, int64_t ldc) {
  const char* fn = "aegis_gemv_noalloc";
  if (dtype != AEGIS_DTYPE_F16 && dtype != AEGIS_DTYPE_BF16) return fail_arg(fn, "dtype must be AEGIS_DTYPE_F16 or AEGIS_DTYPE_BF16");
  aegis::gemm::GemmParams p;
  if (!to_layout(layout_a, &p.layout_a) || !to_layout(layout_b, &p.layout_b))
    return fail_arg(fn, "layout must be AEGIS_ROW_MAJOR or AEGIS_COL_MAJOR");
  if (int s = enter(ctx, fn)) return s;
  p.A = A; p.B = B; p.C = C;
  p.M = M; p.N = N; p.K = K;
  p.lda = lda; p.ldb = ldb; p.ldc = ldc;
  p.alpha = alpha; p.beta = beta;
  p.dtype = dtype == AEGIS_DTYPE_BF16 ? aegis::gemm::DType::BF16 : aegis::gemm::DType::F16;
  const char* why = "";
  const cudaError_t e = aegis::gemv_run_noalloc(p, ctx->stream, &why);
  if (e == cudaSuccess) return AEGIS_OK;
  cudaGetLastError();
  if (e == cudaErrorInvalidValue)
    return fail_arg(fn, *why ? why : "negative size, too-small leading dimension or null operand");
  ctx->last_error = cudaGetErrorString(e);
  return fail(AEGIS_ERR_LAUNCH_FAILED, std::string(fn) + ": " + (*why ? why : "") + " " + cudaGetErrorString(e));
}

int aegis_watchdog_selftest(aegis_context* ctx, int64_t timeout_ns) {
  if (timeout_ns < 100000 || timeout_ns > 10000000000ll)
    return fail_arg("aegis_watchdog_selftest", "timeout_ns must be in [1e5, 1e10]");
  if (int s = enter(ctx, "aegis_watchdog_selftest")) return s;
  unsigned bits = 0;
  const cudaError_t e = aegis::watchdog_selftest(timeout_ns, ctx->stream, &bits);
  if (e != cudaSuccess) return fail_cuda(ctx, e, "aegis_watchdog_selftest");
  if (!(bits & aegis::kStatusTimeoutSelftest))
    return fail(AEGIS_ERR_CUDA, "aegis_watchdog_selftest: the bounded wait did not report its expiry");
  return AEGIS_OK;
}

}  // extern "C"
