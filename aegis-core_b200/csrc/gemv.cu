// Decode GEMV family (gemv_*): C[M,N] = alpha * A[M,K] * B[K,N] + beta * C for
// small M, memory-bound on the weights B.
//
// Replaces the reference's decode kernels (src/gemm/gemv.cu:105-236 and the
// mma.sync gemv_tc.cu:152-197) with a B200 streaming design on CUDA cores:
//   - CTA = 256 threads over a BN-column x MT-row output tile and one K slice
//     (split-K). LPR = BN/8 lanes cover one B row with 16-byte loads (8
//     elements each), so a warp reads 32/LPR rows x BN*2 contiguous bytes per
//     load instruction; the RG = 256/LPR row groups stride down the slice.
//     U independent 16-byte loads per thread are in flight before any math,
//     and the main loop has no barrier: each warp streams on its own.
//   - The grid is sized to about four CTAs per SM (one wave); each CTA walks
//     its K slice in batches of RG*U rows.
//   - A's rows for the CTA's K slice are staged once in shared memory as FP32
//     [k][MT] and read as broadcasts.
//   - FP32 FMA into MT x 8 accumulators per thread, k ascending.
//   - Reduction: row groups inside a warp by a fixed shuffle-xor tree, then
//     the 8 warps through shared memory in warp order 0..7.
//   - Split-K, deterministic. With S = 2, 4 or 8 splits the tile's S CTAs form one
//     thread-block cluster (split = cluster rank): each leaves its FP32
//     partial in its own shared memory, and after a cluster barrier rank 0
//     sums ranks 0..S-1 in order over distributed shared memory and applies
//     alpha/beta. With more splits (reference src/gemm/splitk.cuh:155-222):
//     every CTA of a tile writes its FP32 partial slot, fences, takes a
//     ticket on the tile's counter; the CTA that draws the last ticket sums
//     slots 0..S-1 in order, applies alpha/beta, and resets the counter to 0.
//     Either way the order is fixed and nothing spins on another CTA.
// No tensor cores: the shape is memory-bound.
#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>

#include "common.cuh"
#include "gpu_target.h"
#include "kernels.h"
#include "ptx.cuh"
#include "scratch.h"

namespace aegis {

using gemm::DType;
using gemm::GemmParams;
using gemm::Layout;

namespace {

constexpr int GThreads = 256;
constexpr int kSmemFloats = 8192;  // 32 KiB: A chunk, then the cross-warp reduction (aliased)

// Rows per thread per batch (= independent 16-byte weight loads in flight):
// bounded by the registers the MT x 8 accumulators leave.
__host__ __device__ constexpr int gemv_rows_per_thread(int MT) {
  return MT <= 2 ? 8 : (MT == 4 ? 4 : (MT == 8 ? 4 : 2));
}
// Resident CTAs per SM each instantiation is compiled for (its register
// budget: four CTAs of 256 threads leave 64 registers a thread).
__host__ __device__ constexpr int gemv_ctas_per_sm(int MT) { return MT <= 4 ? 4 : (MT == 8 ? 2 : 1); }

struct GemvArgs {
  const void* A;
  const void* B;
  void* C;
  int M, N, K;
  int ra, rb;                // A / B row-major
  long long lda, ldb, ldc, sa, sb, sc;
  float alpha, beta;
  int tiles_n, tiles_m;
  int S, kc;                 // splits, rows per split
  unsigned* counters;        // per tile (S > 1, ticket fix-up)
  float* partials;           // tiles x S x MT x BN (S > 1, ticket fix-up)
  int batch0;
  int cluster;               // 1: launched in clusters of S CTAs (S = 2, 4, 8), fix-up in shared memory
};

template <int MT>
__device__ __forceinline__ void fma8(float (&acc)[MT][8], const float (&b)[8], const float* arow) {
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const float av = arow[m];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[m][j] = fmaf(av, b[j], acc[m][j]);
  }
}

template <class T>
__device__ __forceinline__ void unpack8(const uint4& v, float (&b)[8]) {
  using E = Elem<T>;
  const float2 p0 = E::pair_to_f32(v.x), p1 = E::pair_to_f32(v.y), p2 = E::pair_to_f32(v.z),
               p3 = E::pair_to_f32(v.w);
  b[0] = p0.x; b[1] = p0.y; b[2] = p1.x; b[3] = p1.y;
  b[4] = p2.x; b[5] = p2.y; b[6] = p3.x; b[7] = p3.y;
}

// VECB: B row-major with 16-byte-aligned rows (base, ldb); otherwise element loads
// (row- or column-major B, any alignment).
template <class T, int LPR, int MT, bool VECB>
__global__ void __launch_bounds__(GThreads, gemv_ctas_per_sm(MT)) gemv_kernel(GemvArgs a) {
  using E = Elem<T>;
  constexpr int BN = 8 * LPR;
  constexpr int RG = GThreads / LPR;
  constexpr int U = gemv_rows_per_thread(MT);            // 16-byte loads in flight per thread
  static_assert(8 * MT * BN <= kSmemFloats, "cross-warp reduction must fit the shared buffer");
  __shared__ __align__(16) float sm[kSmemFloats];
  __shared__ int s_last;

  const int tid = int(threadIdx.x);
  const int l = tid % LPR, g = tid / LPR;
  const int split = int(blockIdx.x % a.S);
  const int nt = int(blockIdx.x / a.S);
  const int mt = int(blockIdx.y);
  const long long b = a.batch0 + blockIdx.z;
  const int n0 = nt * BN, m0 = mt * MT;
  const int k_begin = split * a.kc;
  const int k_end = k_begin + min(a.kc, a.K - k_begin);  // no k_begin + kc overflow near 2^31
  const T* A = static_cast<const T*>(a.A) + b * a.sa;
  const T* B = static_cast<const T*>(a.B) + b * a.sb;
  const int n = n0 + l * 8;  // first of this thread's 8 columns
  const int ncols = max(0, min(8, a.N - n));

  float acc[MT][8];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[m][j] = 0.f;

  // The CTA's first batch of weight rows (rows k_begin .. +RG*U, its BN
  // columns) into L2 while the previous grid on the stream ends
  // (ptx::prefetch_l2: a hint, safe before the wait). One prefetch per 64
  // bytes, spread over the CTA's threads independently of the load mapping.
  if constexpr (VECB) {
    constexpr int P = LPR >= 4 ? LPR / 4 : 1;  // 64-byte pieces per row
    const int rows = min(RG * U, k_end - k_begin);
#pragma unroll 1
    for (int i = tid; i < rows * P; i += GThreads) {
      const int col = n0 + (i % P) * 32;
      if (col < a.N) ptx::prefetch_l2(B + (long long)(k_begin + i / P) * a.ldb + col);
    }
  }
  // Programmatic dependent launch: nothing global is read before the grids
  // this one depends on have completed (their writes are then visible).
  ptx::griddep_wait();

  // This CTA's A rows, staged as FP32 [k][MT] in chunks of the shared buffer
  // (8192 / MT rows each; one chunk when the K slice fits); each chunk's
  // weights stream in batches of U rows per
  // thread: all U loads of a batch are issued before any of its math, and no
  // barrier sits inside the batch loop, so the warps of the CTA (and the
  // other CTAs on the SM) keep loads in flight while one warp computes.
  constexpr int CH = (kSmemFloats / MT) / RG * RG;  // rows per chunk
  auto load_batch = [&](uint4 (&bv)[U], int base, int c1) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = base + u * RG;
      bv[u] = make_uint4(0u, 0u, 0u, 0u);
      if (k < c1 && ncols > 0) {
        const long long gk = k;
        if constexpr (VECB) {
          const T* src = B + gk * a.ldb + n;
          if (ncols == 8) {
            bv[u] = __ldg(reinterpret_cast<const uint4*>(src));
          } else {
            uint16_t h[8] = {};
            for (int j = 0; j < ncols; ++j) h[j] = reinterpret_cast<const uint16_t*>(src)[j];
            bv[u] = make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16),
                               h[4] | (uint32_t(h[5]) << 16), h[6] | (uint32_t(h[7]) << 16));
          }
        } else {
          uint16_t h[8] = {};
          for (int j = 0; j < ncols; ++j) {
            const T* src = a.rb ? B + gk * a.ldb + n + j : B + gk + (long long)(n + j) * a.ldb;
            h[j] = *reinterpret_cast<const uint16_t*>(src);
          }
          bv[u] = make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16),
                             h[4] | (uint32_t(h[5]) << 16), h[6] | (uint32_t(h[7]) << 16));
        }
      }
    }
  };
  bool released = false;
  for (int c0 = k_begin; c0 < k_end; c0 += CH) {
    const int c1 = min(k_end, c0 + CH);
    uint4 bv[U];
    // The chunk's first batch of weights is requested before its A rows are
    // staged, so the two global latencies overlap.
    load_batch(bv, c0 + g, c1);
    if (c0 != k_begin) __syncthreads();  // the previous chunk's A rows are consumed
    for (int i = tid; i < (c1 - c0) * MT; i += GThreads) {
      const int kk = i / MT, m = i % MT;
      const int gm = m0 + m, gk = c0 + kk;
      float v = 0.f;
      if (gm < a.M) v = E::to_f32(a.ra ? A[(long long)gm * a.lda + gk] : A[gm + (long long)gk * a.lda]);
      sm[kk * MT + m] = v;
    }
    __syncthreads();
    if (!released) {
      // The next grid on the stream may launch and run up to its own
      // griddepcontrol.wait while this one streams its weights.
      ptx::griddep_launch_dependents();
      released = true;
    }
    for (int base = c0 + g; base < c1; base += RG * U) {
      if (base != c0 + g) load_batch(bv, base, c1);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int k = base + u * RG;
        if (k < c1) {
          float bf[8];
          unpack8<T>(bv[u], bf);
          fma8<MT>(acc, bf, &sm[(k - c0) * MT]);
        }
      }
    }
  }
  if (!released) ptx::griddep_launch_dependents();

  // Row groups inside the warp: fixed shuffle-xor tree over the lane bits above LPR.
#pragma unroll
  for (int off = LPR; off < 32; off <<= 1)
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[m][j] += __shfl_xor_sync(0xffffffffu, acc[m][j], off);

  // The 8 warps through shared memory, summed in warp order.
  __syncthreads();  // A chunk no longer needed: reuse the buffer
  const int warp = tid / 32, wl = tid % 32;
  if (wl < LPR) {
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int j = 0; j < 8; ++j) sm[(warp * MT + m) * BN + wl * 8 + j] = acc[m][j];
  }
  __syncthreads();
  constexpr int ELEMS = MT * BN;
  float tilev[ceil_div(ELEMS, GThreads)];
#pragma unroll
  for (int r = 0; r < ceil_div(ELEMS, GThreads); ++r) {
    const int e = tid + r * GThreads;
    float s = 0.f;
    if (e < ELEMS) {
      s = sm[e];
#pragma unroll
      for (int w = 1; w < 8; ++w) s += sm[w * ELEMS + e];
    }
    tilev[r] = s;
  }

  T* C = static_cast<T*>(a.C) + b * a.sc;
  auto store = [&](int e, float v) {
    const int m = e / BN, c = e % BN;
    const int gm = m0 + m, gn = n0 + c;
    if (gm >= a.M || gn >= a.N) return;
    T* q = C + (long long)gm * a.ldc + gn;
    float x = a.alpha * v;
    if (a.beta != 0.f) x += a.beta * E::to_f32(*q);
    *q = E::from_f32(x);
  };

  if (a.S == 1) {
#pragma unroll
    for (int r = 0; r < ceil_div(ELEMS, GThreads); ++r) {
      const int e = tid + r * GThreads;
      if (e < ELEMS) store(e, tilev[r]);
    }
    return;
  }
  if (a.cluster) {
    // The tile's S CTAs are one cluster, rank = split (grid x = tiles_n * S,
    // cluster dims (S, 1, 1)). Every thread of every CTA passes both
    // barriers: the first publishes each CTA's partial (release/acquire at
    // cluster scope), the second keeps every CTA resident until rank 0 has
    // read its shared memory.
    __syncthreads();  // every warp is done reading the cross-warp sums
#pragma unroll
    for (int r = 0; r < ceil_div(ELEMS, GThreads); ++r) {
      const int e = tid + r * GThreads;
      if (e < ELEMS) sm[e] = tilev[r];
    }
    ptx::cluster_sync();
    if (ptx::cluster_ctarank() == 0) {
#pragma unroll
      for (int r = 0; r < ceil_div(ELEMS, GThreads); ++r) {
        const int e = tid + r * GThreads;
        if (e >= ELEMS) continue;
        const uint32_t local = ptx::smem_addr(&sm[e]);
        float v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q < a.S) v[q] = ptx::ld_shared_cluster_f32(ptx::map_to_rank(local, uint32_t(q)));
        float sum = v[0];
#pragma unroll
        for (int q = 1; q < 8; ++q)
          if (q < a.S) sum += v[q];
        store(e, sum);
      }
    }
    ptx::cluster_sync();
    return;
  }
  const long long tile = ((long long)blockIdx.z * a.tiles_m + mt) * a.tiles_n + nt;
  float* slot0 = a.partials + tile * a.S * ELEMS;
#pragma unroll
  for (int r = 0; r < ceil_div(ELEMS, GThreads); ++r) {
    const int e = tid + r * GThreads;
    if (e < ELEMS) __stcg(slot0 + (long long)split * ELEMS + e, tilev[r]);
  }
  __threadfence();  // the partial is visible device-wide before the ticket
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(a.counters + tile, 1u) == unsigned(a.S - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();  // acquire the other CTAs' partials
  // Slots 0..S-1 summed in order; eight loads in flight at a time (the last
  // CTA's sum is the kernel's tail).
#pragma unroll
  for (int r = 0; r < ceil_div(ELEMS, GThreads); ++r) {
    const int e = tid + r * GThreads;
    if (e >= ELEMS) continue;
    float s = 0.f;
    for (int q0 = 0; q0 < a.S; q0 += 8) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = q0 + j < a.S ? __ldcg(slot0 + (long long)(q0 + j) * ELEMS + e) : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (q0 + j < a.S) s = (q0 + j == 0) ? v[j] : s + v[j];
    }
    store(e, s);
  }
  if (tid == 0) a.counters[tile] = 0;  // ready for the next launch (graph replays need no reset)
}

// --------------------------------------------------------------- host side
int mt_for(int M, int BN) {
  const int cap = 1024 / BN;  // MT * BN <= 1024 (reduction buffer)
  int mt = 1;
  while (mt < M && mt < 16 && mt < cap) mt <<= 1;
  return mt;
}

struct GPlan {
  int LPR, MT, S, kc, tiles_n, tiles_m;
  long long tiles;
};

// Cluster split-K fix-up (the kernel's a.cluster path) for S = 2, 4 or 8.
// Against the global-ticket fix-up on a B200 (graph windows, three
// alternating runs): clusters of 2, 4 and 8 were 1-4.5% faster or level;
// 112 clusters of 5 (M = 1, N x K = 14336 x 4096, BN = 128) were 11% slower,
// so other split counts keep the ticket fix-up. AEGIS_GEMV_CLUSTER=0 turns
// it off (global-ticket fix-up for every S, no split trimming), read once,
// for A/B measurement.
bool gemv_clusters_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("AEGIS_GEMV_CLUSTER");
    return !(e && e[0] == '0');
  }();
  return on;
}
constexpr int kMaxClusterSplits = 8;

// The clusters of S CTAs the device can hold at once for `kernel`
// (cudaOccupancyMaxActiveClusters), cached per (device, kernel, S); 0 when
// the query fails. A cluster must fit one GPC, so clusters of S CTAs can hold
// fewer CTAs than the per-SM limit suggests: a launch uses the cluster fix-up
// only when all its clusters fit at once.
int max_active_clusters(const void* kernel, int S) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const auto key = std::make_tuple(dev, kernel, S);
  std::lock_guard<std::mutex> lock(mu);
  if (const auto it = cache.find(key); it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(S));
  cfg.blockDim = dim3(GThreads);
  cfg.dynamicSmemBytes = 0;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = unsigned(S);
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();  // the query failed: no cluster fix-up, nothing left pending
    n = 0;
  }
  return cache[key] = n;
}

GPlan plan_for(int cfg, const GemmParams& p) {
  const gemm::GemvConfig& c = gemm::GEMV_CONFIGS[cfg];
  GPlan pl{};
  pl.LPR = c.BN / 8;
  pl.MT = mt_for(p.M, c.BN);
  pl.tiles_n = ceil_div(p.N, c.BN);
  pl.tiles_m = ceil_div(p.M, pl.MT);
  pl.tiles = (long long)pl.tiles_n * pl.tiles_m * p.batch;
  const gpu::Target* d = gpu::planning_target();
  const int sms = d ? d->sms : 148;
  // Split K so that tiles x splits fills one wave (gemv_ctas_per_sm CTAs per
  // SM: ~128 KB of weight loads in flight per SM at MT <= 2), with at least
  // 64 rows a split, and the partials within the workspace cap. A split's A
  // rows need not fit the shared buffer: the kernel stages them in chunks
  // (capping the split there had forced extra splits, a second wave, e.g.
  // M = 16, K x N = 4096 x 14336 on 74 SMs).
  const long long target = (long long)sms * gemv_ctas_per_sm(pl.MT);
  long long S = std::max<long long>(1, target / pl.tiles);  // rounded down: never a second wave
  // Nine splits become eight, the largest cluster fix-up (portable cluster
  // size), at MT <= 2: a ninth of the CTAs for a tail without the global
  // ticket round trips. Measured on a B200 (graph windows): M = 1, K x N =
  // 4096 x 4096, BN = 64: 10.09 -> 9.31 us; M = 2: 12.24 -> 12.02 us. Not
  // kept: ten splits to eight (BN = 256, N = 14336: 0.7% slower) and nine to
  // eight at M = 4 (15.87 -> 16.34 us: the longer slices cost more than the
  // tail saves).
  if (gemv_clusters_enabled() && pl.MT <= 2 && S == 9) S = 8;
  S = std::min<long long>(S, std::max(1, ceil_div(p.K, 64)));
  // Rows per split: ceil(K / S) rounded up to 16, in 64-bit (K may be near
  // 2^31); a split of all of K when rounding would pass K.
  auto rows_for = [&](long long splits) {
    const long long kc = ceil_div(ceil_div<long long>(p.K, splits), 16ll) * 16;
    return int(std::min<long long>(kc, p.K));
  };
  int kc = rows_for(S);
  const long long slot = pl.tiles * pl.MT * c.BN * (long long)sizeof(float);
  const long long cap = std::max<long long>(1, gemm::kSplitKMaxWorkspace / std::max<long long>(1, slot));
  if (ceil_div(p.K, kc) > cap) kc = rows_for(cap);  // fewer, longer splits: the partials' workspace cap
  pl.S = ceil_div(p.K, kc);
  pl.kc = kc;
  return pl;
}

bool vec_b_ok(const GemmParams& p) {
  return p.layout_b == Layout::RowMajor && (reinterpret_cast<uintptr_t>(p.B) & 15u) == 0 && p.ldb % 8 == 0 &&
         (p.batch <= 1 || p.stride_b % 8 == 0);
}

template <class T, int LPR, bool VECB>
const void* kernel_mt(int MT) {
  switch (MT) {
    case 1: return reinterpret_cast<const void*>(&gemv_kernel<T, LPR, 1, VECB>);
    case 2: return reinterpret_cast<const void*>(&gemv_kernel<T, LPR, 2, VECB>);
    case 4: return reinterpret_cast<const void*>(&gemv_kernel<T, LPR, 4, VECB>);
    case 8:
      if constexpr (LPR <= 16) return reinterpret_cast<const void*>(&gemv_kernel<T, LPR, 8, VECB>);
      break;
    case 16:
      if constexpr (LPR <= 8) return reinterpret_cast<const void*>(&gemv_kernel<T, LPR, 16, VECB>);
      break;
  }
  return nullptr;
}

// The gemv_kernel instantiation for these parameters (nullptr: none).
template <class T>
const void* kernel_for(bool vec, int LPR, int MT) {
  auto by_lpr = [&](auto vecb) -> const void* {
    constexpr bool V = decltype(vecb)::value;
    switch (LPR) {
      case 32: return kernel_mt<T, 32, V>(MT);
      case 16: return kernel_mt<T, 16, V>(MT);
      case 8: return kernel_mt<T, 8, V>(MT);
      case 4: return kernel_mt<T, 4, V>(MT);
    }
    return nullptr;
  };
  return vec ? by_lpr(std::true_type{}) : by_lpr(std::false_type{});
}

const void* kernel_for(DType dt, bool vec, int LPR, int MT) {
  return dt == DType::BF16 ? kernel_for<__nv_bfloat16>(vec, LPR, MT) : kernel_for<__half>(vec, LPR, MT);
}

// Launched with programmatic stream serialization: the grid may start while
// the previous grid on the stream drains; it waits (griddepcontrol.wait)
// before its first global read and lets its own dependents launch once its
// weight loads are in flight. a.cluster: clusters of a.S CTAs along x.
cudaError_t launch(const void* kernel, const GemvArgs& a, dim3 grid, cudaStream_t s) {
  if (!kernel) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(GThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (a.cluster) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = unsigned(a.S);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  GemvArgs args = a;
  void* params[] = {&args};
  return cudaLaunchKernelExC(&cfg, kernel, params);
}

constexpr int kMaxGridZ = 65535;

}  // namespace

cudaError_t gemv_run(int cfg, const GemmParams& p, cudaStream_t stream) {
  if (const cudaError_t e = gemm::validate(p); e != cudaSuccess) return e;
  if (gemm::is_empty(p)) return cudaSuccess;
  if (p.alpha == 0.f) return scale_c(p, stream);
  const GPlan pl = plan_for(cfg, p);
  if (pl.tiles_m > 65535) return cudaErrorInvalidConfiguration;
  GemvArgs a{};
  a.A = p.A;
  a.B = p.B;
  a.C = p.C;
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.ra = p.layout_a == Layout::RowMajor;
  a.rb = p.layout_b == Layout::RowMajor;
  a.lda = p.lda;
  a.ldb = p.ldb;
  a.ldc = p.ldc;
  a.sa = p.stride_a;
  a.sb = p.stride_b;
  a.sc = p.stride_c;
  a.alpha = p.alpha;
  a.beta = p.beta;
  a.tiles_n = pl.tiles_n;
  a.tiles_m = pl.tiles_m;
  a.S = pl.S;
  a.kc = pl.kc;
  const long long grid_x = (long long)pl.tiles_n * pl.S;
  if (grid_x > 0x7fffffffll) return cudaErrorInvalidConfiguration;
  const bool vec = vec_b_ok(p);
  const void* kernel = kernel_for(p.dtype, vec, pl.LPR, pl.MT);
  const bool cluster_ok =
      gemv_clusters_enabled() && (pl.S == 2 || pl.S == 4 || pl.S == kMaxClusterSplits);
  const int cluster_cap = cluster_ok && kernel ? max_active_clusters(kernel, pl.S) : 0;
  for (int b0 = 0; b0 < p.batch; b0 += kMaxGridZ) {
    const int nb = std::min(kMaxGridZ, p.batch - b0);
    a.batch0 = b0;
    a.cluster = cluster_ok && (long long)pl.tiles_n * pl.tiles_m * nb <= cluster_cap;
    if (pl.S > 1 && !a.cluster) {
      // Tile indices restart per launch (blockIdx.z), so each launch of a
      // batch chunk reuses the same counter/partial slots, in stream order.
      const long long tiles = (long long)pl.tiles_n * pl.tiles_m * nb;
      void* cnt = nullptr;
      void* part = nullptr;
      if (const cudaError_t e = scratch::acquire(stream, size_t(tiles) * sizeof(unsigned), scratch::Kind::Tickets, &cnt);
          e != cudaSuccess)
        return e;
      const size_t pbytes = size_t(tiles) * pl.S * pl.MT * (8 * pl.LPR) * sizeof(float);
      if (const cudaError_t e = scratch::acquire(stream, pbytes, scratch::Kind::Partials, &part); e != cudaSuccess) return e;
      a.counters = static_cast<unsigned*>(cnt);
      a.partials = static_cast<float*>(part);
    }
    const dim3 grid(unsigned(grid_x), unsigned(pl.tiles_m), unsigned(nb));
    const cudaError_t e = launch(kernel, a, grid, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

gemm::LaunchPlan gemv_plan(int cfg, const GemmParams& p) {
  const GPlan pl = plan_for(cfg, p);
  gemm::LaunchPlan r;
  r.splits = pl.S;
  r.k_chunk = pl.kc;
  r.tiles = pl.tiles;
  r.grid = unsigned((long long)pl.tiles_n * pl.S * pl.tiles_m * p.batch);
  return r;
}

cudaError_t gemv_attrs(int cfg, cudaFuncAttributes* attrs) {
  switch (gemm::GEMV_CONFIGS[cfg].BN / 8) {
    case 32: return cudaFuncGetAttributes(attrs, &gemv_kernel<__half, 32, 1, true>);
    case 16: return cudaFuncGetAttributes(attrs, &gemv_kernel<__half, 16, 1, true>);
    case 8: return cudaFuncGetAttributes(attrs, &gemv_kernel<__half, 8, 1, true>);
    default: return cudaFuncGetAttributes(attrs, &gemv_kernel<__half, 4, 1, true>);
  }
}

// --------------------------------------------------------------- allocation-free entry
// The decode GEMV above takes its split-K tickets and partials from the
// per-stream workspace cache, which calls cudaMalloc the first time a stream
// needs a size class. Some callers cannot allow that: engines that hand all
// device memory to their own allocator at start-up and forbid allocations
// afterwards, code that runs while a CUDA graph is being captured (where
// cudaMalloc is not allowed, and the cache refuses a first use), and
// processes on a hard memory budget where a late allocation may fail. For
// them, gemv_run_noalloc runs the same kernel with its scratch in the
// fixed array below, which the CUDA module reserves on every GPU that loads
// this library, for the life of the process.
//
// Capacity: kNoAllocPartialBytes of FP32 partials and kNoAllocCounterBytes of
// tickets. A plan whose partials would not fit uses fewer splits; problems
// beyond kNoAllocMaxM rows, kNoAllocMaxN columns or one batch are rejected.
// Every call shares the array and leaves its contents behind: the tickets
// are cleared on the stream before each launch; calls whose kernels overlap
// on the GPU (several streams at once) race on the array.
namespace {

constexpr size_t kNoAllocPartialBytes = size_t(4) << 20;  // 4 MiB
constexpr size_t kNoAllocCounterBytes = size_t(16) << 10;   // 4096 tickets
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocPartialBytes + kNoAllocCounterBytes];

std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[gpu::kMaxDevices] = {};

// The device address of g_noalloc_scratch on the current device, looked up
// once per device (with that device current). In host code the symbol itself
// is only a host-side stand-in; it must never be passed to a kernel.
cudaError_t noalloc_scratch(unsigned char** out) {
  *out = nullptr;
  int dev = 0;
  if (const cudaError_t e = cudaGetDevice(&dev); e != cudaSuccess) return e;
  if (dev < 0 || dev >= gpu::kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch); e != cudaSuccess) return e;
    g_noalloc_ptr[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

// The plan of the CUDA-core GEMV config that ummav_run falls back to for
// this M (gemv_256 up to M = 4, gemv_128 up to 8, else gemv_64), with fewer,
// longer splits when its partials would not fit the fixed array. On a B200
// (148 SMs) the regular plan's partials stay under ~2.4 MiB, so only devices
// with several hundred SMs take the second branch; aegis_plan_simulated_json
// reports this plan for a modelled device ("gemv_noalloc"). False when the
// tickets would not fit.
bool noalloc_plan(const GemmParams& p, GPlan* out) {
  GPlan pl = plan_for(p.M <= 4 ? 0 : (p.M <= 8 ? 1 : 2), p);
  const long long slot_bytes = pl.tiles * pl.MT * (8 * pl.LPR) * (long long)sizeof(float);
  if ((long long)pl.S * slot_bytes > (long long)kNoAllocPartialBytes) {
    const long long s_fit = std::max<long long>(1, (long long)kNoAllocPartialBytes / slot_bytes);
    pl.kc = int(std::min<long long>(ceil_div(ceil_div<long long>(p.K, s_fit), 16ll) * 16, p.K));
    pl.S = ceil_div(p.K, pl.kc);
  }
  *out = pl;
  return pl.tiles * (long long)sizeof(unsigned) <= (long long)kNoAllocCounterBytes;
}

}  // namespace

bool gemv_noalloc_plan(const GemmParams& p, gemm::LaunchPlan* out) {
  GPlan pl{};
  const bool ok = noalloc_plan(p, &pl);
  out->splits = pl.S;
  out->k_chunk = pl.kc;
  out->tiles = pl.tiles;
  out->grid = unsigned((long long)pl.tiles_n * pl.S * pl.tiles_m);
  return ok;
}

cudaError_t gemv_run_noalloc(const GemmParams& p, cudaStream_t stream, const char** why) {
  *why = "";
  if (const cudaError_t e = gemm::validate(p); e != cudaSuccess) {
    *why = "invalid GEMM parameters";
    return e;
  }
  if (gemm::is_empty(p)) return cudaSuccess;
  if (p.batch != 1 || p.M > kNoAllocMaxM || p.N > kNoAllocMaxN) {
    *why = "the allocation-free GEMV takes one batch, M <= 16 and N <= 65536";
    return cudaErrorInvalidValue;
  }
  if (p.alpha == 0.f) return scale_c(p, stream);
  GPlan pl{};
  if (!noalloc_plan(p, &pl)) {
    *why = "too many output tiles for the fixed ticket array";
    return cudaErrorInvalidValue;
  }
  GemvArgs a{};
  a.A = p.A;
  a.B = p.B;
  a.C = p.C;
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.ra = p.layout_a == Layout::RowMajor;
  a.rb = p.layout_b == Layout::RowMajor;
  a.lda = p.lda;
  a.ldb = p.ldb;
  a.ldc = p.ldc;
  a.alpha = p.alpha;
  a.beta = p.beta;
  a.tiles_n = pl.tiles_n;
  a.tiles_m = pl.tiles_m;
  a.S = pl.S;
  a.kc = pl.kc;
  if (pl.S > 1) {
    unsigned char* scratch = nullptr;
    if (const cudaError_t e = noalloc_scratch(&scratch); e != cudaSuccess) {
      *why = "cudaGetSymbolAddress of the fixed scratch array failed";
      return e;
    }
    a.partials = reinterpret_cast<float*>(scratch);
    a.counters = reinterpret_cast<unsigned*>(scratch + kNoAllocPartialBytes);
    // Tickets must read zero at launch (a completed launch leaves them zero;
    // clearing here also covers a launch that never completed).
    if (const cudaError_t e = cudaMemsetAsync(a.counters, 0, size_t(pl.tiles) * sizeof(unsigned), stream);
        e != cudaSuccess)
      return e;
  }
  const dim3 grid(unsigned((long long)pl.tiles_n * pl.S), unsigned(pl.tiles_m), 1u);
  return launch(kernel_for(p.dtype, vec_b_ok(p), pl.LPR, pl.MT), a, grid, stream);
}

}  // namespace aegis
