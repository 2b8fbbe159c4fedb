// Host side of the umma family: TMA tensor maps, the split-K plan, the
// deterministic split-K reduction kernel, and the run() entry points.
//
// Split-K (tall-K shapes whose tiles cannot fill the SMs): S CTAs per output
// tile each run the same main loop over a K slice and write FP32 partials to
// workspace slot s ([s][batch][M][N]); a second kernel sums slots 0..S-1 in
// that fixed order per element and applies alpha/beta. Results are bitwise
// identical run to run. The reference gets the same guarantee with an
// ordered ticket in the last CTA of each tile (src/gemm/splitk.cuh:155-222);
// with 128x256 tiles and up to ~74 splits the last CTA would read megabytes
// alone, so here every SM shares the (L2-resident) reduction.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "gpu_target.h"
#include "kernels.h"
#include "status.h"
#include "umma_launch.cuh"
#include "tma_map.h"
#include "scratch.h"

namespace aegis {

using gemm::DType;
using gemm::GemmParams;
using gemm::Layout;

int splitk_choose(long long tiles, int k_blocks, int sms, int min_blocks_per_split, double t_block_ns,
                  double reduce_ns_per_split, long long max_splits) {
  if (sms < 1 || tiles < 1 || k_blocks < 1) return 1;
  long long s_max = k_blocks / std::max(1, min_blocks_per_split);
  s_max = std::min<long long>(s_max, max_splits);
  s_max = std::min<long long>(s_max, 1024);
  if (s_max < 1) s_max = 1;
  int best = 1;
  double best_cost = 0;
  for (long long S = 1; S <= s_max; ++S) {
    const long long kc = (k_blocks + S - 1) / S;
    const long long s_eff = (k_blocks + kc - 1) / kc;  // splits actually launched
    if (s_eff != S) continue;
    const long long waves = (tiles * S + sms - 1) / sms;
    const double cost = double(waves) * double(kc) * t_block_ns + (S > 1 ? double(S) * reduce_ns_per_split : 0.0);
    if (S == 1 || cost < best_cost) {
      best = int(S);
      best_cost = cost;
    }
  }
  return best;
}

namespace {

struct Maps {
  CUtensorMap a, b;
};

// A: row-major -> K-major box {64 k, 128 m}; col-major -> M-major boxes {64 m, 64 k}.
// B: row-major -> N-major boxes {64 n, 64 k}; col-major -> K-major box {64 k, BN n}.
// `bbox`: the B box width along N for K-major B (BN, or BN/2 for CTA pairs).
bool make_maps(const GemmParams& p, int bbox, Maps* m) {
  const bool ar = p.layout_a == Layout::RowMajor, br = p.layout_b == Layout::RowMajor;
  const long long ba = p.batch > 1 && p.stride_a != 0 ? p.batch : 1;
  const long long bb = p.batch > 1 && p.stride_b != 0 ? p.batch : 1;
  const bool okA = ar ? encode_map(&m->a, p.dtype, p.A, p.K, p.M, p.lda, ba, p.stride_a, umma::BM)
                      : encode_map(&m->a, p.dtype, p.A, p.M, p.K, p.lda, ba, p.stride_a, umma::BK);
  const bool okB = br ? encode_map(&m->b, p.dtype, p.B, p.N, p.K, p.ldb, bb, p.stride_b, umma::BK)
                      : encode_map(&m->b, p.dtype, p.B, p.K, p.N, p.ldb, bb, p.stride_b, bbox);
  return okA && okB;
}

// ---------------------------------------------------------------- split-K reduce
// out[b][m][n] = alpha * (P[0] + ... + P[S-1]) (+ beta * C) in a fixed order:
// the S slots form G consecutive groups of per = ceil(S/G) slots; each group is
// summed in slot order by its own threads, then the group sums are added in
// group order. G is the smallest power of two with per <= 8, at most 8, so a
// group costs one batch of L2 loads up to S = 64. G and the order depend on S
// only: results are bitwise identical run to run and on every rank of an
// N-sharded call. A block is 256 threads = G groups x 256/G units (float4 when
// N % 4 == 0, else float).
constexpr int kReduceThreads = 256;
constexpr int kReduceMaxGroups = 8;

inline int reduce_groups(int S) {
  int G = 1;
  while (G < kReduceMaxGroups && (S + G - 1) / G > 8) G *= 2;
  return G;
}

template <class T, bool VEC4>
__global__ void __launch_bounds__(kReduceThreads, 4) splitk_reduce_kernel(const float* __restrict__ part, int S,
                                                                       int lg_groups, int batch, int M, int N,
                                                                       T* __restrict__ C, long long ldc,
                                                                       long long stride_c, float alpha, float beta) {
  using E = Elem<T>;
  using V = std::conditional_t<VEC4, float4, float>;
  constexpr int W = VEC4 ? 4 : 1;
  __shared__ V group_sum[kReduceThreads];
  // Launched as a programmatic dependent of the GEMM that wrote the partials:
  // nothing is read before that grid has completed.
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  // 32-bit indexing: the host guarantees S * batch * M * N < 2^31.
  const int plane_v = batch * M * N / W;  // one slot, in V units
  const int nw = N / W;
  const int total = plane_v;
  const int G = 1 << lg_groups;
  const int U = kReduceThreads >> lg_groups;  // units per pass
  const int per = (S + G - 1) / G;
  const int g = int(threadIdx.x) >> (8 - lg_groups), u = int(threadIdx.x) & (U - 1);
  const int q0 = g * per, q1 = min(S, q0 + per);
  const V* base = reinterpret_cast<const V*>(part) + q0 * plane_v;
  for (int t = int(blockIdx.x) * U + u, t_end = ((total + U - 1) / U) * U; t < t_end; t += int(gridDim.x) * U) {
    V acc{};
    // Partials are dense [S][batch][M][N]: unit t of slot q is base[q * plane_v + t].
    if (t < total && q0 < q1) acc = sum_slots_t<V>(base + t, plane_v, q1 - q0);
    if (G > 1) {  // block-uniform
      group_sum[threadIdx.x] = acc;
      __syncthreads();
      if (g == 0) {
        for (int k = 1; k < G && k * per < S; ++k) add_slot(acc, group_sum[k * U + u], false);
      }
      __syncthreads();  // group_sum is reused by the next pass
    }
    if (g != 0 || t >= total) continue;
    const int bm = t / nw, n = (t - bm * nw) * W;
    const int m = bm % M, b = bm / M;
    T* c = C + b * stride_c + (long long)m * ldc + n;
    if constexpr (VEC4) {
      float v[4] = {alpha * acc.x, alpha * acc.y, alpha * acc.z, alpha * acc.w};
      if (beta != 0.f) {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] += beta * E::to_f32(c[j]);
      }
      if ((reinterpret_cast<uintptr_t>(c) & 7u) == 0) {
        uint2 w;
        w.x = E::pack(v[0], v[1]);
        w.y = E::pack(v[2], v[3]);
        *reinterpret_cast<uint2*>(c) = w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) c[j] = E::from_f32(v[j]);
      }
    } else {
      float v = alpha * acc;
      if (beta != 0.f) v += beta * E::to_f32(*c);
      *c = E::from_f32(v);
    }
  }
}

template <class T>
cudaError_t launch_reduce(const float* part, int S, const GemmParams& p, cudaStream_t s) {
  const gpu::Target* d = gpu::this_device();
  const int sms = d ? d->sms : 148;
  const bool vec = p.N % 4 == 0;
  const long long plane = (long long)p.batch * p.M * p.N;
  if ((long long)S * plane >= (1ll << 31)) return cudaErrorInvalidValue;  // beyond the workspace cap
  const int G = reduce_groups(S);
  int lg = 0;
  while ((1 << lg) < G) ++lg;
  const int U = kReduceThreads >> lg;
  const long long total = vec ? plane / 4 : plane;
  const int blocks = int(std::max<long long>(1, std::min<long long>((total + U - 1) / U, (long long)sms * 8)));
  T* C = static_cast<T*>(p.C);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(blocks));
  cfg.blockDim = dim3(kReduceThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return vec ? cudaLaunchKernelEx(&cfg, &splitk_reduce_kernel<T, true>, part, S, lg, p.batch, p.M, p.N, C, p.ldc,
                                  p.stride_c, p.alpha, p.beta)
             : cudaLaunchKernelEx(&cfg, &splitk_reduce_kernel<T, false>, part, S, lg, p.batch, p.M, p.N, C, p.ldc,
                                  p.stride_c, p.alpha, p.beta);
}

// ---------------------------------------------------------------- planning
// Units one launch can take (one cluster each, grid.x < 2^31). Far above
// any problem that fits in device memory; larger plans are refused.
constexpr long long kMaxUnits = 1ll << 29;

struct Plan {
  int BM = 128, BN = 256, STAGES = 4, CTAS = 1;
  int splits = 1, kb_per_split = 0, kb_total = 0;
  int tiles_m = 0, tiles_n = 0;
  int group_m = umma::kGroupM;
  bool steal = true;  // more units than resident CTAs (pairs)
  long long tiles = 0, units = 0;
  int grid = 0;
  int slots = 0;      // units resident at once (CTAs, or pairs for cta_group::2)
  bool kwave = false;  // the config walks K by wave (UmmaConfig::KWAVE)
};

// Raster group (tile rows walked together before moving along N): 8, or 4
// for tall grids of CTA pairs at most 8 tiles wide (a 16384 x 2048 grid, an
// 8-rank N-shard of 16384^3: 1.2% faster with 4 on a B200, where a group's
// A panels and all of B no longer share L2 at 8). The AEGIS_UMMA_GROUP_M
// environment variable overrides it, read once, for tuning sweeps; values
// outside [1, 64] are ignored.
int group_for(int ctas, int tiles_m, int tiles_n) {
  static const int forced = [] {
    const char* s = std::getenv("AEGIS_UMMA_GROUP_M");
    const int v = s ? std::atoi(s) : 0;
    return v >= 1 && v <= 64 ? v : 0;
  }();
  if (forced) return forced;
  return ctas == 2 && tiles_n <= 8 && tiles_m >= 32 ? 4 : umma::kGroupM;
}

// The k-walk rule of a launch whose tiles are the columns [col0, col0 +
// tiles_n) of a full problem tiles_n_full tile columns wide: by wave (in the
// full problem's raster) when the config asks for it and the full problem is
// unsplit, one batch and more than one wave of slots.
void set_kdir(umma::Args* a, const Plan& pl, int batch, int tiles_n_full, int col0) {
  a->kdir_wave = 0;
  a->kdir_tiles_n = tiles_n_full;
  a->kdir_col0 = col0;
  a->kdir_group = group_for(pl.CTAS, pl.tiles_m, tiles_n_full);  // the full problem's raster
  if (pl.kwave && pl.splits == 1 && batch == 1 && pl.slots > 0 &&
      (long long)pl.tiles_m * tiles_n_full > pl.slots)
    a->kdir_wave = pl.slots;
}

// CTA pairs that can be resident at once on the current device (both CTAs of
// a cluster must sit in one GPC), queried once per device; sms/2 if the query
// is unavailable (sizing tests on a simulated device).
int pair_slots(int sms) {
  static std::mutex mu;
  static int cached[gpu::kMaxDevices] = {};
  const gpu::Target* d = gpu::planning_target();
  if (!d || d->modelled) return sms;
  int dev = d->ordinal;
  if (dev < 0 || dev >= gpu::kMaxDevices) return sms;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int n = 0;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(2 * sms));
    cfg.blockDim = dim3(umma::kThreads);
    cfg.dynamicSmemBytes = umma::LayoutPair<256, gemm::kUmmaPairStages>::ALLOC;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    auto* kern = &umma::umma2_gemm_kernel<__nv_bfloat16, 256, gemm::kUmmaPairStages, false, true, umma::kEpiStore>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(umma::LayoutPair<256, gemm::kUmmaPairStages>::ALLOC)) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sms;
    }
    cached[dev] = std::min(n, sms);
  }
  return cached[dev];
}

Plan make_plan(int cfg, const GemmParams& p) {
  const gemm::UmmaConfig& c = gemm::UMMA_CONFIGS[cfg];
  Plan pl;
  pl.BM = c.BM;
  pl.BN = c.BN;
  pl.STAGES = c.STAGES;
  pl.CTAS = c.CTAS;
  pl.kwave = c.KWAVE != 0;
  pl.tiles_m = ceil_div(p.M, c.BM);
  pl.tiles_n = ceil_div(p.N, c.BN);
  pl.group_m = group_for(c.CTAS, pl.tiles_m, pl.tiles_n);
  pl.kb_total = ceil_div(p.K, umma::BK);
  pl.tiles = (long long)p.batch * pl.tiles_m * pl.tiles_n;
  const gpu::Target* d = gpu::planning_target();
  // Tile slots: one per SM, or one per resident pair of SMs for cta_group::2.
  const int sms = d ? (c.CTAS == 2 ? pair_slots(d->sms / 2) : d->sms) : 0;
  int S = 1;
  if (c.SPLITK && sms > 0 && pl.tiles < sms) {
    // One k-block is BK/16 = 4 MMAs of 128 x BN x 16 (about 128 cycles each at
    // BN = 256 on one SM, ~1.85 GHz). The reduction moves 8 bytes per output
    // element per split (write + read FP32) at ~5 TB/s.
    const double t_block_ns = 4.0 * 128.0 * (double(c.BN) / 256.0) / 1.85;
    const double out_elems = double(p.batch) * p.M * p.N;
    const double reduce_ns = out_elems * 8.0 / 5.0e3;
    const long long cap = std::max<long long>(1, gemm::kSplitKMaxWorkspace / (long long)std::max(1.0, out_elems * 4));
    S = splitk_choose(pl.tiles, pl.kb_total, sms, 4, t_block_ns, reduce_ns, cap);
    // AEGIS_UMMA_SPLITS overrides the model for tuning sweeps (read on every
    // plan; clamped to [1, k-blocks / 4] and the workspace cap).
    if (const char* env = std::getenv("AEGIS_UMMA_SPLITS")) {
      const long long v = std::atoll(env);
      if (v >= 1) S = int(std::max<long long>(1, std::min<long long>({v, pl.kb_total / 4, cap})));
    }
  }
  pl.slots = sms;
  pl.kb_per_split = ceil_div(pl.kb_total, S);
  pl.splits = ceil_div(pl.kb_total, pl.kb_per_split);
  pl.units = pl.tiles * pl.splits;
  // One CTA (pair: one cluster of two) per unit: the CTAs that fit run and
  // take the rest in launch order (tile_sched.cuh).
  pl.grid = int(std::max<long long>(1, std::min<long long>(pl.units, kMaxUnits))) * c.CTAS;
  // When every unit has a resident CTA (pair) from the start there is nothing
  // to take: no cluster-launch-control request (its failed answer would only
  // delay the CTAs' exit). If fewer CTAs turn out resident, the others still
  // start later and run their own units.
  pl.steal = sms <= 0 || pl.units > sms;
  return pl;
}

umma::Args make_args(const GemmParams& p, const Plan& pl) {
  umma::Args a{};
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.batch = p.batch;
  a.a_batched = p.batch > 1 && p.stride_a != 0;
  a.b_batched = p.batch > 1 && p.stride_b != 0;
  a.tiles_m = pl.tiles_m;
  a.tiles_n = pl.tiles_n;
  a.group_m = pl.group_m;
  a.steal = pl.steal ? 1 : 0;
  a.splits = pl.splits;
  a.kb_per_split = pl.kb_per_split;
  a.kb_total = pl.kb_total;
  a.units = pl.units;
  a.C = p.C;
  a.ldc = p.ldc;
  a.stride_c = p.stride_c;
  a.alpha = p.alpha;
  a.beta = p.beta;
  a.wait_limit_ns = kDefaultWaitLimitNs;
  set_kdir(&a, pl, p.batch, pl.tiles_n, 0);
  return a;
}

cudaError_t launch(const GemmParams& p, const umma::LaunchKey& k, const Maps& m, const umma::Args& a, int grid,
                   cudaStream_t s) {
  return p.dtype == DType::BF16 ? umma::launch_family<__nv_bfloat16>(k, m.a, m.b, a, grid, s)
                                : umma::launch_family<__half>(k, m.a, m.b, a, grid, s);
}

// The N-sharded GEMM runs UMMA_CONFIGS[4]: CTA pairs, 256 x 256 tiles, no
// split-K (measured equal to or faster than one-CTA 128 x 256 tiles at
// 4096^3 .. 16384^3).
constexpr int kNshardConfig = 4;
static_assert(gemm::UMMA_CONFIGS[kNshardConfig].CTAS == 2 && gemm::UMMA_CONFIGS[kNshardConfig].BN == 256 &&
                  !gemm::UMMA_CONFIGS[kNshardConfig].SPLITK,
              "the N-sharded path needs the non-split CTA-pair config");

bool device_is_sm100() {
  const gpu::Target* d = gpu::this_device();
  return d && d->cc == 100;
}

}  // namespace

cudaError_t umma_run(int cfg, const GemmParams& p, cudaStream_t stream) {
  if (const cudaError_t e = gemm::validate(p); e != cudaSuccess) return e;
  if (gemm::is_empty(p)) return cudaSuccess;
  if (p.alpha == 0.f) return scale_c(p, stream);
  if (!gemm::tma_compatible(p) || !device_is_sm100()) return simt_run(p, stream);
  const Plan pl = make_plan(cfg, p);
  if (pl.units > kMaxUnits) return cudaErrorInvalidValue;
  Maps maps;
  if (!make_maps(p, pl.CTAS == 2 ? pl.BN / 2 : pl.BN, &maps)) return simt_run(p, stream);  // TMA refused the geometry
  umma::Args a = make_args(p, pl);
  if (const cudaError_t e = status::word(&a.status); e != cudaSuccess) return e;
  umma::LaunchKey k{pl.BN, pl.STAGES, p.layout_a == Layout::ColMajor, p.layout_b == Layout::RowMajor,
                    umma::kEpiStore, pl.CTAS == 2};
  if (pl.splits == 1) return launch(p, k, maps, a, pl.grid, stream);
  // Split-K: partials, then the ordered reduction.
  void* part = nullptr;
  const size_t bytes = size_t(pl.splits) * p.batch * size_t(p.M) * p.N * sizeof(float);
  if (const cudaError_t e = scratch::acquire(stream, bytes, scratch::Kind::Partials, &part); e != cudaSuccess) return e;
  a.partials = static_cast<float*>(part);
  k.epi = umma::kEpiPartial;
  if (const cudaError_t e = launch(p, k, maps, a, pl.grid, stream); e != cudaSuccess) return e;
  return p.dtype == DType::BF16 ? launch_reduce<__nv_bfloat16>(a.partials, pl.splits, p, stream)
                                : launch_reduce<__half>(a.partials, pl.splits, p, stream);
}

gemm::LaunchPlan umma_plan(int cfg, const GemmParams& p) {
  const Plan pl = make_plan(cfg, p);
  gemm::LaunchPlan r;
  r.splits = pl.splits;
  r.k_chunk = int(std::min<long long>((long long)pl.kb_per_split * umma::BK, p.K));
  r.tiles = pl.tiles;
  r.grid = unsigned(pl.grid);
  umma::Args a{};
  set_kdir(&a, pl, p.batch, pl.tiles_n, 0);
  r.kdir_wave = a.kdir_wave;
  return r;
}

cudaError_t umma_attrs(int cfg, cudaFuncAttributes* attrs) {
  const gemm::UmmaConfig& c = gemm::UMMA_CONFIGS[cfg];
  return umma::attrs_family<__half>(c.BN, c.STAGES, c.CTAS == 2, attrs);
}

size_t umma_smem_bytes(int cfg) {
  const gemm::UmmaConfig& c = gemm::UMMA_CONFIGS[cfg];
  if (c.CTAS == 2) return size_t(umma::LayoutPair<256, gemm::kUmmaPairStages>::ALLOC);
  // Split-K configs also launch the partial-store epilogue, with its staging.
  const int epi = c.SPLITK ? umma::kEpiPartial : umma::kEpiStore;
  if (c.BN == 64) return size_t(umma::Layout<64, 8>::alloc_for(epi));
  return c.BN == 256 ? size_t(umma::Layout<256, 4>::alloc_for(epi)) : size_t(umma::Layout<128, 6>::alloc_for(epi));
}

cudaError_t umma_nsharded(const GemmParams& local, void* const* c_ranks, int nranks, int col_offset,
                          cudaStream_t stream) {
  if (nranks < 1 || nranks > umma::kMaxPeers || !c_ranks) return cudaErrorInvalidValue;
  if (!gemm::tma_compatible(local) || !device_is_sm100()) return cudaErrorNotSupported;
  if (local.layout_a != Layout::RowMajor || local.layout_b != Layout::RowMajor || local.batch != 1)
    return cudaErrorInvalidValue;
  const Plan pl = make_plan(kNshardConfig, local);  // CTA pairs, 256 x 256 tiles, no split
  if (pl.units > kMaxUnits) return cudaErrorInvalidValue;
  Maps maps;
  if (!make_maps(local, pl.CTAS == 2 ? pl.BN / 2 : pl.BN, &maps)) return cudaErrorNotSupported;
  umma::Args a = make_args(local, pl);
  if (const cudaError_t e = status::word(&a.status); e != cudaSuccess) return e;
  a.col_offset = col_offset;
  for (int i = 0; i < nranks; ++i)
    if (!c_ranks[i]) return cudaErrorInvalidValue;
  // The epilogue stores each finished tile into this rank's C, then each warp
  // copies its rows to the other ranks with row-contiguous stores
  // (push_warp_rows), overlapping the next tile's main loop.
  a.peers[0] = local.C;
  int np = 1;
  for (int i = 0; i < nranks; ++i)
    if (c_ranks[i] != local.C) {
      if (np >= nranks) return cudaErrorInvalidValue;  // local.C must be one of c_ranks
      a.peers[np++] = c_ranks[i];
    }
  a.npeers = np;  // entries equal to local.C are this rank's own C
  bool vec = local.ldc % 8 == 0 && col_offset % 8 == 0;
  for (int i = 0; i < np; ++i) vec = vec && (reinterpret_cast<uintptr_t>(a.peers[i]) & 15u) == 0;
  a.peer_vec = vec ? 1 : 0;
  // The k-walk of each tile follows the full problem's raster, so every
  // element is summed in the order of the 1-GPU GEMM: possible when this
  // rank's columns start and (unless it is the last rank) end on tile
  // boundaries; otherwise forward only.
  const int n_full = local.N * nranks;
  const bool aligned = col_offset % pl.BN == 0 && (local.N % pl.BN == 0 || col_offset + local.N == n_full);
  set_kdir(&a, pl, 1, ceil_div(n_full, pl.BN), aligned ? col_offset / pl.BN : 0);
  if (!aligned) a.kdir_wave = 0;
  const umma::LaunchKey k{pl.BN, pl.STAGES, false, true, umma::kEpiPeers, pl.CTAS == 2};
  return launch(local, k, maps, a, pl.grid, stream);
}

}  // namespace aegis
