/*
 * aegis-b200: C ABI of the B200 (sm_100a) GEMM/GEMV library.
 *
 * This header is the drop-in boundary. Every ABI 1.3 entry point keeps the
 * name, signature, argument meaning and status codes of the reference's
 * include/aegis/aegis.h (Riffe007/aegis-core, include/aegis/aegis.h:37-194),
 * so existing C and Rust callers (rust/aegis-sys binds this file through
 * include/aegis/aegis.h) link against libaegis_capi.so unchanged. ABI 1.4
 * only adds functions; no ABI 1.3 struct or signature changes.
 *
 * Conventions (same as the reference):
 *   - Every function returns AEGIS_OK (0) or a negative AEGIS_ERR_* status.
 *     Nothing exits or aborts the process.
 *   - aegis_last_error_string() holds the detail of the last failure on the
 *     calling thread (kept until the next failure); aegis_last_error(ctx) the
 *     last CUDA error text a context saw.
 *   - GEMM operands are device pointers to 16-bit IEEE binary16 (f16) or
 *     bfloat16 (bf16) bit patterns (uint16_t on the host), from any CUDA
 *     allocator in this process.
 *   - A context is used by one host thread at a time. Calls are asynchronous
 *     on the context's stream.
 *   - Size queries use (buf = NULL, buf_len = 0, &needed).
 */
#ifndef AEGIS_B200_AEGIS_H
#define AEGIS_B200_AEGIS_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define AEGIS_API __declspec(dllexport)
#else
#define AEGIS_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (reference include/aegis/aegis.h:39-46). */
#define AEGIS_OK 0
#define AEGIS_ERR_INVALID_ARGUMENT (-1) /* null pointer, negative size, bad layout or ld */
#define AEGIS_ERR_CUDA (-2)             /* a CUDA call failed, or a kernel watchdog fired */
#define AEGIS_ERR_BUFFER_TOO_SMALL (-3) /* see the `needed` out-parameter */
#define AEGIS_ERR_NO_DEVICE (-4)        /* device index out of range / no GPU */
#define AEGIS_ERR_OUT_OF_MEMORY (-5)
#define AEGIS_ERR_LAUNCH_FAILED (-6)    /* a kernel could not be launched */

/* ABI version (reference aegis.h:49-51): 1.4 = 1.3 plus the bf16, N-sharded,
 * IPC and watchdog entry points below. */
#define AEGIS_ABI_VERSION_MAJOR 1
#define AEGIS_ABI_VERSION_MINOR 4
/* major * 1000 + minor. Replaces reference aegis.h:51. */
AEGIS_API int aegis_abi_version(void);

/* Static text for a status code; never NULL. Replaces reference aegis.h:54. */
AEGIS_API const char* aegis_status_string(int status);

/* Detail of the last failed call on this thread ("" if none). Replaces
 * reference aegis.h:59. */
AEGIS_API const char* aegis_last_error_string(void);

/* One device plus one stream: a private non-blocking stream, or the caller's
 * (aegis_set_stream). Replaces reference aegis.h:63. */
typedef struct aegis_context aegis_context;

/* Replaces reference aegis.h:65. AEGIS_ERR_NO_DEVICE for a bad index. */
AEGIS_API int aegis_create(aegis_context** out, int device);
/* Waits for the context's own stream, then frees it. NULL is a no-op.
 * Replaces reference aegis.h:66. */
AEGIS_API int aegis_destroy(aegis_context* ctx);

/* Use a caller-owned cudaStream_t (as void*); NULL goes back to the
 * context's own stream. A caller's stream is never destroyed. Replaces
 * reference aegis.h:70. */
AEGIS_API int aegis_set_stream(aegis_context* ctx, void* cuda_stream);

/* Waits for the work queued on the context's stream. Also reports a kernel
 * watchdog that fired since the last check on this device (a bounded wait
 * inside a kernel gave up; the output of that launch is not valid) as
 * AEGIS_ERR_CUDA with the detail in aegis_last_error_string(). Replaces
 * reference aegis.h:73. */
AEGIS_API int aegis_synchronize(aegis_context* ctx);

/* Last CUDA error text this context saw ("" if none). Replaces reference
 * aegis.h:76. */
AEGIS_API const char* aegis_last_error(const aegis_context* ctx);

/* Synchronous device-memory helpers, ordered after the context's queued work.
 * Replace reference aegis.h:79-82. */
AEGIS_API int aegis_device_alloc(aegis_context* ctx, size_t bytes, void** out);
AEGIS_API int aegis_device_free(aegis_context* ctx, void* ptr); /* NULL is a no-op */
AEGIS_API int aegis_copy_to_device(aegis_context* ctx, void* dst, const void* src, size_t bytes);
AEGIS_API int aegis_copy_to_host(aegis_context* ctx, void* dst, const void* src, size_t bytes);

/* C[M,N] = A[M,K] * B[K,N]: packed row-major, f16 in, FP32 accumulate, f16
 * out (alpha 1, beta 0). M, N or K == 0: AEGIS_OK, nothing launched.
 * Replaces reference aegis.h:91-92. */
AEGIS_API int aegis_gemm_f16(aegis_context* ctx, const void* A, const void* B, void* C,
                             int M, int N, int K);

/* General GEMM. For each batch b < batch:
 *   C_b = alpha * A_b * B_b + beta * C_b
 *   A_b = A + b * stride_a (M x K), B_b = B + b * stride_b (K x N),
 *   C_b = C + b * stride_c (M x N, row-major, ldc >= N).
 * AEGIS_ROW_MAJOR: X[r * ld + c] (ld >= cols); AEGIS_COL_MAJOR: X[r + c * ld]
 * (ld >= rows). Leading dimensions and strides count elements.
 * alpha == 0: A*B is not evaluated (C = beta * C); beta == 0: C is not read.
 * Otherwise NaN and Inf propagate. Any alignment is accepted (operands that
 * the TMA path cannot address take the general kernel). Empty sizes: no-op.
 * Negative sizes, too-small ld, null operands, overlapping C batches:
 * AEGIS_ERR_INVALID_ARGUMENT. Replaces reference aegis.h:108-121. */
#define AEGIS_ROW_MAJOR 0
#define AEGIS_COL_MAJOR 1

AEGIS_API int aegis_gemm_f16_ex(aegis_context* ctx, int layout_a, int layout_b, int M, int N, int K,
                                float alpha, const void* A, int64_t lda, const void* B, int64_t ldb,
                                float beta, void* C, int64_t ldc);

AEGIS_API int aegis_gemm_f16_strided_batched(aegis_context* ctx, int layout_a, int layout_b, int M,
                                             int N, int K, float alpha, const void* A, int64_t lda,
                                             int64_t stride_a, const void* B, int64_t ldb,
                                             int64_t stride_b, float beta, void* C, int64_t ldc,
                                             int64_t stride_c, int batch);

/* Name of the kernel configuration aegis_gemm_f16 runs for this shape on the
 * context's device (a registry name such as "umma_128x256x64_s4"), copied
 * NUL-terminated into buf. Replaces reference aegis.h:126-127. */
AEGIS_API int aegis_gemm_choice(aegis_context* ctx, int M, int N, int K, char* buf,
                                size_t buf_len, size_t* needed);

/* JSON device manifest: properties plus a measured device-to-device copy
 * bandwidth ("measured_d2d_bw_gbps"), measured on the first call per device
 * and cached for the process. Replaces reference aegis.h:136. */
AEGIS_API int aegis_device_manifest(int device, char* buf, size_t buf_len, size_t* needed);

/* Hardware description as JSON (schema "aegis-hw/1"). device = -1 describes
 * the host only and makes no CUDA call. A size query snapshots the document
 * for the calling thread; the next fill on that thread returns the same
 * snapshot. Replaces reference aegis.h:155. */
AEGIS_API int aegis_hw_info_json(int device, char* buf, size_t buf_len, size_t* needed);

/* GPU part as a struct. Set struct_size = sizeof(aegis_hw_gpu_info) first; at
 * most struct_size bytes are written. Same layout as reference
 * aegis.h:157-178. Unknown fields: -1. */
typedef struct aegis_hw_gpu_info {
  uint32_t struct_size;
  int32_t present;
  int32_t device;
  int32_t arch;                  /* major * 10 + minor */
  int32_t sm_count;
  int32_t regs_per_sm;
  int64_t smem_per_sm;
  int64_t smem_per_block;
  int64_t smem_per_block_optin;
  int64_t l2_bytes;
  int64_t memory_bytes;
  int32_t unified;
  int32_t tma_hardware;          /* 1: arch >= 90 */
  int32_t tma_built;             /* 1: this library compiled its TMA tier */
  int32_t nvml;                  /* 1: NVML answered for this device */
  int32_t max_sm_clock_mhz;      /* -1: unknown */
  int32_t max_mem_clock_mhz;     /* -1: unknown */
  double power_limit_w;          /* < 0: not readable */
  char name[128];
} aegis_hw_gpu_info;
/* Replaces reference aegis.h:179. */
AEGIS_API int aegis_hw_gpu(int device, aegis_hw_gpu_info* out);

/* Host CPU part as a struct (struct_size as above). Same layout as reference
 * aegis.h:183-191; the ARM ISA flags read 0 on x86 hosts. */
typedef struct aegis_hw_cpu_info {
  uint32_t struct_size;
  int32_t logical_cpus;
  int32_t clusters;
  int32_t core_types;
  int32_t performance_cores;
  int64_t performance_max_khz;   /* -1: unknown */
  int32_t neon, fp16, dotprod, sve, sve2, i8mm, bf16;
} aegis_hw_cpu_info;
/* Replaces reference aegis.h:192. */
AEGIS_API int aegis_hw_cpu(aegis_hw_cpu_info* out);

/* ---- ABI 1.4 additions: bfloat16 ------------------------------------------
 * The same three entry points with bfloat16 operands: bf16 in, FP32
 * accumulate, bf16 out, identical argument rules. No counterpart in the
 * reference (it is f16-only); they mirror aegis_gemm_f16 (aegis.h:91),
 * aegis_gemm_f16_ex (aegis.h:111) and aegis_gemm_f16_strided_batched
 * (aegis.h:115) argument for argument. */
AEGIS_API int aegis_gemm_bf16(aegis_context* ctx, const void* A, const void* B, void* C,
                              int M, int N, int K);
AEGIS_API int aegis_gemm_bf16_ex(aegis_context* ctx, int layout_a, int layout_b, int M, int N,
                                 int K, float alpha, const void* A, int64_t lda, const void* B,
                                 int64_t ldb, float beta, void* C, int64_t ldc);
AEGIS_API int aegis_gemm_bf16_strided_batched(aegis_context* ctx, int layout_a, int layout_b,
                                              int M, int N, int K, float alpha, const void* A,
                                              int64_t lda, int64_t stride_a, const void* B,
                                              int64_t ldb, int64_t stride_b, float beta, void* C,
                                              int64_t ldc, int64_t stride_c, int batch);

/* ---- ABI 1.4 additions: N-sharded (column-parallel) GEMM -------------------
 * One process (or thread) per GPU, `nranks` ranks on one node. Rank `rank`
 * holds all of A (M x K, row-major, lda) and its column shard of B,
 * B_r = B[:, rank*Ns : (rank+1)*Ns] stored as a row-major K x Ns matrix with
 * leading dimension ldb (Ns = N / nranks; N must divide evenly). It computes
 * C[:, rank*Ns : (rank+1)*Ns] = A * B_r and the kernel's epilogue stores every
 * finished tile straight into the C of EVERY rank (its own and its peers', over
 * NVLink), so the all-gather of C happens tile by tile inside the GEMM.
 * c_ranks[i] is rank i's C (M x N, row-major, ldc) as a pointer valid on this
 * context's device (aegis_ipc_open_handle for i != rank).
 * Ordering, because every rank writes into every rank's C:
 *   - after the call, every rank must pass a cross-rank barrier ordered after
 *     it on its stream (e.g. a one-element NCCL all-reduce) before any rank
 *     reads its C;
 *   - before a call that writes into a C buffer some rank may still be reading
 *     (a copy-out of the previous result, a consumer kernel), every rank must
 *     pass a cross-rank barrier ordered after those reads, or the next call's
 *     peer stores can overwrite C while it is read. Alternating two C buffers
 *     does not remove this: the barrier must follow the reads of the buffer
 *     about to be reused.
 * No counterpart in the reference (it has no multi-GPU code). */
AEGIS_API int aegis_gemm_bf16_nsharded(aegis_context* ctx, int M, int N, int K, const void* A,
                                       int64_t lda, const void* B_shard, int64_t ldb,
                                       void* const* c_ranks, int64_t ldc, int nranks, int rank);
AEGIS_API int aegis_gemm_f16_nsharded(aegis_context* ctx, int M, int N, int K, const void* A,
                                      int64_t lda, const void* B_shard, int64_t ldb,
                                      void* const* c_ranks, int64_t ldc, int nranks, int rank);

/* CUDA IPC helpers for the N-sharded GEMM: export a device allocation of this
 * context's device as an opaque AEGIS_IPC_HANDLE_BYTES-byte handle, open a
 * peer's handle as a local pointer, close it. No counterpart in the reference. */
#define AEGIS_IPC_HANDLE_BYTES 64
AEGIS_API int aegis_ipc_get_handle(aegis_context* ctx, const void* dptr, void* handle);
AEGIS_API int aegis_ipc_open_handle(aegis_context* ctx, const void* handle, void** dptr);
AEGIS_API int aegis_ipc_close_handle(aegis_context* ctx, void* dptr);

/* ---- ABI 1.4 additions: kernel registry ------------------------------------
 * The general GEMM of aegis_gemm_*_strided_batched run by one named kernel
 * configuration of the registry (e.g. "umma_128x256x64_s4_ksm", "gemv_64x256_ksm",
 * "simt_64x64x16") instead of the dispatcher's choice; a configuration that
 * cannot address the operands runs the general kernel, as the dispatcher
 * would. dtype: AEGIS_DTYPE_F16 or AEGIS_DTYPE_BF16. Unknown impl:
 * AEGIS_ERR_INVALID_ARGUMENT. Replaces the reference's C++-only registry
 * lookup gemm::find + KernelEntry::run (include/aegis/gemm.h:109-134), which
 * its bench_gemm --impl and aegis_tune tools call (bench/bench_gemm.cu:46-55). */
#define AEGIS_DTYPE_F16 0
#define AEGIS_DTYPE_BF16 1
AEGIS_API int aegis_gemm_impl(aegis_context* ctx, const char* impl, int dtype, int layout_a, int layout_b, int M,
                              int N, int K, float alpha, const void* A, int64_t lda, int64_t stride_a,
                              const void* B, int64_t ldb, int64_t stride_b, float beta, void* C, int64_t ldc,
                              int64_t stride_c, int batch);

/* The registry as JSON: [{"name":..,"config":{..},"supported":true|false,
 * "why":".."},...] for the context's device. Replaces gemm::registry() and
 * gemm::supported() (reference include/aegis/gemm.h:121-134). */
AEGIS_API int aegis_registry_json(aegis_context* ctx, char* buf, size_t buf_len, size_t* needed);

/* The launch a kernel configuration makes for a packed row-major problem on
 * the context's device, as JSON {"impl":..,"splits":S,"k_chunk":..,"tiles":..,
 * "grid":..}; impl NULL: the dispatcher's choice. Replaces the reference's
 * gemm::gemv_launch_plan (include/aegis/gemm.h:273-280), widened to every
 * split-K family. */
AEGIS_API int aegis_gemm_plan_json(aegis_context* ctx, const char* impl, int dtype, int M, int N, int K, char* buf,
                                   size_t buf_len, size_t* needed);

/* aegis_gemm_plan_json without a device or a context: the dispatcher's choice
 * and the launch plan for a packed row-major problem on a simulated device of
 * compute capability `arch` (major*10 + minor; 100 for B200) with `sm_count`
 * SMs and B200's other limits. JSON as aegis_gemm_plan_json plus
 * "kind":"winner" (a tuned winners row chose it) or "rule" (the built-in
 * rule), and "dispatch" (the chosen kernel; `impl` only replaces the kernel
 * whose plan is reported; impl "gemv_noalloc" reports the plan of
 * aegis_gemv_noalloc below). Runs nothing on any GPU; for planning tools and
 * tests of the dispatch rules on machines without one. No reference
 * counterpart (the reference tests dispatch on its device only,
 * tests/test_matmul.cu). */
AEGIS_API int aegis_plan_simulated_json(int arch, int sm_count, const char* impl, int dtype, int M, int N, int K,
                                        char* buf, size_t buf_len, size_t* needed);

/* ---- ABI 1.4 addition: decode GEMV that allocates nothing -------------------
 * C = alpha * A * B + beta * C for decode shapes, like aegis_gemm_*_ex with
 * row- or column-major A and B (layout_a, layout_b), one batch, M <= 16 and
 * N <= 65536; dtype AEGIS_DTYPE_F16 or AEGIS_DTYPE_BF16. Larger problems:
 * AEGIS_ERR_INVALID_ARGUMENT with the reason in aegis_last_error_string().
 * The regular entry points take their split-K scratch from a per-stream cache
 * that calls cudaMalloc the first time a stream needs it. This one is for
 * callers that cannot allow that: engines that give all device memory to
 * their own allocator at start-up and forbid later allocations, code that
 * runs while a CUDA graph is being captured, and processes on a hard memory
 * budget. It calls no cudaMalloc, cudaFree or other allocating routine: its
 * scratch is a fixed 4 MiB + 16 KiB array inside this library, which every
 * GPU that loads the library holds until the process exits (a plan that
 * would need more uses fewer K splits). The first call on a device looks up
 * that array's device address, so make it before any stream capture. Every
 * call shares the array: calls whose kernels overlap on the GPU (concurrent
 * streams) race and must be serialised by the caller. It runs the CUDA-core
 * gemv kernel (deterministic split-K); results match the regular entry points
 * within the library's tolerance.
 * No counterpart in the reference, which has no allocation-free path. */
AEGIS_API int aegis_gemv_noalloc(aegis_context* ctx, int dtype, int layout_a, int layout_b, int M, int N, int K,
                                 float alpha, const void* A, int64_t lda, const void* B, int64_t ldb, float beta,
                                 void* C, int64_t ldc);

/* ---- ABI 1.4 addition: watchdog self-test ----------------------------------
 * Every wait inside this library's kernels is bounded. This runs one small
 * kernel whose wait can never complete, with the given limit (1e5..1e10 ns),
 * and returns AEGIS_OK if the kernel gave up, returned and reported it (the
 * context stays usable), or AEGIS_ERR_CUDA otherwise. No counterpart in the
 * reference (its kernels trap instead). */
AEGIS_API int aegis_watchdog_selftest(aegis_context* ctx, int64_t timeout_ns);

#ifdef __cplusplus
}
#endif

#endif /* AEGIS_B200_AEGIS_H */
