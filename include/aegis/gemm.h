#pragma once
// aegis-b200 C++ GEMM interface: the problem description every kernel takes,
// the kernel registry, and the per-family configuration tables.
//
// Mirrors the reference's include/aegis/gemm.h (Riffe007/aegis-core):
//   GemmParams / row_major_params / validate / is_empty  (gemm.h:46-73)
//   KernelReq / KernelEntry / DeviceCaps / registry()     (gemm.h:91-134)
// with one addition, GemmParams::dtype (f16 or bf16; the reference is
// f16-only), and new B200 kernel families in place of the reference's
// sm_80/sm_90-style tiers:
//   umma_*   tcgen05 (TMEM accumulator) + TMA + mbarrier warp-specialised GEMM,
//            optionally with deterministic split-K (suffix _ksm);
//   gemv_*   decode GEMV for M <= 16, 128-bit weight streaming on CUDA cores,
//            deterministic split-K;
//   simt_*   the general kernel: any layout, leading dimension and alignment.
//
// Semantics (identical to the reference): for batch b in [0, batch)
//   C_b = alpha * A_b * B_b + beta * C_b,  FP32 accumulation,
// A_b = A + b*stride_a (M x K), B_b = B + b*stride_b (K x N), C_b = C + b*stride_c
// (M x N row-major, ldc >= N). alpha == 0: A*B does not contribute (NaN/Inf in
// A or B do not propagate). beta == 0: C is not read. Empty sizes: no-op.
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <span>
#include <string>
#include <string_view>

namespace aegis::gemm {

enum class Layout : int { RowMajor = 0, ColMajor = 1 };
enum class DType : int { F16 = 0, BF16 = 1 };

struct GemmParams {
  const void* A = nullptr;
  const void* B = nullptr;
  void* C = nullptr;
  int M = 0, N = 0, K = 0;
  Layout layout_a = Layout::RowMajor, layout_b = Layout::RowMajor;
  long long lda = 0, ldb = 0, ldc = 0;
  float alpha = 1.f, beta = 0.f;
  int batch = 1;
  long long stride_a = 0, stride_b = 0, stride_c = 0;
  DType dtype = DType::F16;
};

// Packed row-major NN, alpha 1, beta 0, one batch (reference gemm.h:59-66).
inline GemmParams row_major_params(const void* A, const void* B, void* C, int M, int N, int K,
                                   DType dt = DType::F16) {
  GemmParams p;
  p.A = A; p.B = B; p.C = C;
  p.M = M; p.N = N; p.K = K;
  p.lda = K; p.ldb = N; p.ldc = N;
  p.dtype = dt;
  return p;
}

// cudaSuccess, or cudaErrorInvalidValue for negative sizes, null operands with
// nonzero sizes, a bad layout/dtype, ld below the contiguous extent, negative
// A/B batch strides or overlapping C batches (reference registry.cu:13-30);
// and, beyond the reference, for M, N or K above kMaxDim, which leaves the
// kernels' 32-bit index arithmetic (row and k loops that step past the end)
// headroom below 2^31.
inline constexpr int kMaxDim = (1 << 30) + ((1 << 30) - (1 << 20));  // 2^31 - 2^20
cudaError_t validate(const GemmParams& p);
inline bool is_empty(const GemmParams& p) {
  return p.M == 0 || p.N == 0 || p.K == 0 || p.batch == 0;
}

// ---------------------------------------------------------------------------
// Registry (reference gemm.h:91-134).
// ---------------------------------------------------------------------------
// Legacy row-major f16 entry: C = A*B, packed (lda = K, ldb = N, ldc = N).
using LaunchFn = cudaError_t (*)(const void* A, const void* B, void* C, int M, int N, int K,
                                 cudaStream_t stream);
using AttrsFn = cudaError_t (*)(cudaFuncAttributes* attrs);
// General entry: validates p, launches asynchronously on `stream`.
using RunFn = cudaError_t (*)(const GemmParams& p, cudaStream_t stream);

struct KernelReq {
  int min_arch = 0;       // major*10 + minor; the umma family needs exactly sm_100 (arch 100)
  bool tma = false;       // uses cp.async.bulk.tensor
  bool tcgen05 = false;   // uses tcgen05 / TMEM
  size_t smem_bytes = 0;  // dynamic + static smem per block
  int threads = 0;
  int regs = -1;          // filled from cudaFuncGetAttributes
};

struct KernelEntry {
  const char* name;
  const char* config;  // JSON of the template parameters
  LaunchFn launch;
  AttrsFn attrs;
  RunFn run;
  int tune_max_m = 0;  // > 0: the tuner only times shapes with M <= this
  KernelReq req{};
};

struct DeviceCaps {
  int arch = 0;
  bool tma_built = true;
  size_t smem_per_block_optin = 0;
  int regs_per_block = 0;
  int max_threads_per_block = 0;
};
DeviceCaps current_caps();
bool supported(const KernelEntry& e, const DeviceCaps& caps, std::string* why = nullptr);

std::span<const KernelEntry> registry();
const KernelEntry* find(std::string_view name);

// ---------------------------------------------------------------------------
// umma family: tcgen05.mma kind::f16 (f16 or bf16 operands, FP32 accumulator
// in TMEM), BK = 64 (one 128-byte swizzle row of 16-bit elements per
// k-block), STAGES-deep TMA ring, persistent tile walk, two TMEM accumulators
// (the epilogue of a tile overlaps the main loop of the next).
// CTAS = 1: one CTA per SM, BM = 128 rows (cta_group::1).
// CTAS = 2: a cluster of two CTAs on two SMs shares one BM = 256 tile
//           (cta_group::2: each CTA loads half of A and half of B; the leader
//           issues M = 256 MMAs into both CTAs' TMEM). No TMA multicast.
// SPLITK: 0 = never split K; 1 = split K by the SM count when the tile count
// alone cannot fill the GPU (partials reduced in a fixed order, bit-identical
// across runs). Name: umma_<BM>x<BN>x<BK>_s<STAGES>[_c2][_ksm].
// ---------------------------------------------------------------------------
// KWAVE: walk K last to first in every odd wave of resident tiles of the
// problem's raster, so consecutive waves meet at the same end of K and reuse
// the operand blocks still in L2 (name suffix _kw).
struct UmmaConfig { int BM, BN, BK, STAGES, SPLITK, CTAS, KWAVE = 0; };
// Ring depth of the CTA-pair configs: 7 x 32 KB stages fill the 227 KB of
// shared memory a CTA may use.
inline constexpr int kUmmaPairStages = 7;
inline constexpr UmmaConfig UMMA_CONFIGS[] = {
    {128, 256, 64, 4, 0, 1},
    {128, 128, 64, 6, 0, 1},
    {128, 256, 64, 4, 1, 1},
    {128, 128, 64, 6, 1, 1},
    {256, 256, 64, kUmmaPairStages, 0, 2},
    {256, 256, 64, kUmmaPairStages, 1, 2},
    // Small problems: 128 x 64 tiles, an 8-deep ring of 24 KB stages (twice
    // the CTAs of 128 x 128 tiles, and K = 512 fully in flight).
    {128, 64, 64, 8, 0, 1},
    {128, 64, 64, 8, 1, 1},
    // CTA pairs with the by-wave K walk: less DRAM traffic on multi-wave grids.
    {256, 256, 64, kUmmaPairStages, 0, 2, 1},
};
std::span<const KernelEntry> umma_entries();

// ---------------------------------------------------------------------------
// gemv family (decode, M <= 16 per row tile; any M runs): weights B streamed
// with 16-byte loads, LPR lanes per B row (BN = 8*LPR columns per CTA), the
// other threads stacked along K; FP32 FMA on CUDA cores; per-CTA fixed-order
// tree reduction through shared memory; deterministic split-K sized by the SM
// count. Name: gemv_<BN>x<THREADS>_ksm.
// ---------------------------------------------------------------------------
struct GemvConfig { int BN, THREADS; };
inline constexpr GemvConfig GEMV_CONFIGS[] = {
    {256, 256}, {128, 256}, {64, 256}, {32, 256},
};
std::span<const KernelEntry> gemv_entries();

// ---------------------------------------------------------------------------
// ummav family (decode, M <= 16, row-major operands the TMA path can address;
// anything else runs the gemv family): C^T = B^T * A^T on tensor cores, the
// weights as the 128-row tcgen05 operand and the activation rows padded to 16,
// a STAGES-deep TMA ring, CTAS_PER_SM CTAs per SM, an even k-block split over
// all CTAs (stream-K segments) with an ordered ticket fix-up. Deterministic.
// Name: ummav_128x16x64_s<STAGES>[x<CTAS_PER_SM>].
// ---------------------------------------------------------------------------
struct UmmavConfig { int STAGES, CTAS_PER_SM; };
inline constexpr UmmavConfig UMMAV_CONFIGS[] = {
    {11, 1},
    {6, 2},
};
std::span<const KernelEntry> ummav_entries();

// ---------------------------------------------------------------------------
// simt family: the general kernel (any layout, ld, alignment, batch stride).
// Name: simt_<BM>x<BN>x<BK>.
// ---------------------------------------------------------------------------
std::span<const KernelEntry> simt_entries();

// Split-K partials beyond this lower S (reference gemm.h:268).
inline constexpr long long kSplitKMaxWorkspace = 256ll << 20;

// The launch an umma/gemv entry makes for p on the current device (or the
// thread's simulated one): effective splits and CTA count.
struct LaunchPlan {
  int splits = 1;
  int k_chunk = 0;       // K rows per split
  long long tiles = 0;   // output tiles (all batches)
  unsigned grid = 0;     // CTAs launched
  int kdir_wave = 0;     // umma: tiles per wave of the by-wave k-walk (0: every tile walks K forward)
};
bool launch_plan(const char* impl, const GemmParams& p, LaunchPlan* out);
int split_count(const char* impl, const GemmParams& p);

// Whether the umma (TMA) path can address p: 16-byte aligned base pointers,
// leading dimensions and batch strides that are multiples of 8 elements,
// non-zero batch strides for batched operands. Otherwise umma entries run the
// simt kernel (reference mma_tma.cu:297-305 plays the same role).
bool tma_compatible(const GemmParams& p);

}  // namespace aegis::gemm
