// Decode GEMM on tensor cores (ummav family): C[M,N] = alpha*A[M,K]*B[K,N] +
// beta*C for M <= 16, row-major A and B, computed transposed as
//   C^T[N, M] = B^T[N, K] * A^T[K, M]
// so the weights B fill the 128-row MMA operand and the few activation rows
// (padded to 16 by TMA zero fill) are the 16-column operand:
// tcgen05.mma.cta_group::1.kind::f16 with M = 128 (weight columns), N = 16,
// K = 16, FP32 accumulators in TMEM.
//
// Why tensor cores here. The reference's decode kernels stream B through
// CUDA cores (src/gemm/gemv.cu) or mma.sync (src/gemm/gemv_tc.cu). On B200 a
// CUDA-core GEMV needs M FP32 FMAs per weight element; at M = 16 and 6.5 TB/s
// that is ~52 TFMA/s, above the ~36 TFMA/s the CUDA cores deliver, so the
// kernel would be compute-bound. Here the tensor core does the arithmetic and
// the kernel is a pure TMA weight stream: producer warp -> mbarrier ring ->
// one MMA thread -> epilogue warps, as in the umma kernel.
//
// Work split (deterministic stream-K): the N/128 column tiles x K/64
// k-blocks form one linear sequence; CTA c takes k-blocks
// [T*c/G, T*(c+1)/G) of it (T total, G CTAs), cut into segments at tile
// boundaries. A tile covered by one segment is stored directly; otherwise each
// segment writes an FP32 partial slot and takes a ticket (per 32-column
// quarter of the tile, one epilogue warp each), and the warp drawing the last
// ticket sums the slots in segment order and applies alpha/beta (the reference's ordered-ticket rule,
// src/gemm/splitk.cuh:155-222). The partition depends only on the shape and
// G, so results are bitwise identical run to run. Nothing waits on another
// CTA; every mbarrier wait is bounded.
#include <algorithm>

#include "common.cuh"
#include "gpu_target.h"
#include "kernels.h"
#include "ptx.cuh"
#include "status.h"
#include "tma_map.h"
#include "scratch.h"

namespace aegis {
namespace ummav {

constexpr int BMN = 128;  // weight columns per tile (MMA M)
constexpr int MPAD = 16;  // activation rows (MMA N)
constexpr int BK = 64;
constexpr int kThreads = 192;

struct Args {
  int M, N, K;
  int tiles, kb;        // column tiles, k-blocks per tile
  unsigned total;       // tiles * kb (the host keeps total * grid below 2^32)
  void* C;
  long long ldc;
  float alpha, beta;
  float* partials;      // [tiles][maxseg][MPAD][BMN]
  unsigned* counters;   // [tiles][4]: one ticket per (tile, epilogue warp)
  int maxseg;
  unsigned* status;
  long long wait_limit_ns;
};

template <int STAGES>
struct Layout {
  static constexpr int B_BYTES = BMN * BK * 2;   // 16 KB: weights, two [64 k][64 n] boxes
  static constexpr int A_BYTES = MPAD * BK * 2;  // 2 KB: activations [16 m][64 k]
  static constexpr int STAGE_TX = B_BYTES + A_BYTES;
  static constexpr int B_OFF = 0;
  static constexpr int A_OFF = STAGES * B_BYTES;
  static constexpr int BAR_OFF = A_OFF + STAGES * A_BYTES;
  static constexpr int NBARS = 2 * STAGES + 5;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int BYTES = MISC_OFF + 16;
  static constexpr int ALLOC = BYTES + 1024;
  static constexpr int TMEM_COLS = 32;  // two 16-column accumulators
  static_assert(A_OFF % 1024 == 0 && BAR_OFF % 8 == 0, "operand tiles stay 1024-byte aligned");
};

// 32-bit arithmetic throughout: total * gridDim.x < 2^32 (host check), and a
// 64-bit division by a run-time value is a long emulated sequence on the
// critical path of a microsecond-scale kernel.
__device__ __forceinline__ unsigned range_start(const Args& a, unsigned c) {
  return a.total * c / gridDim.x;
}

// The CTA whose range holds linear k-block x.
__device__ __forceinline__ int owner_of(const Args& a, unsigned x) {
  unsigned c = x * gridDim.x / a.total;
  while (c + 1 < gridDim.x && range_start(a, c + 1) <= x) ++c;
  while (c > 0 && range_start(a, c) > x) --c;
  return int(c);
}

struct Seg {
  int tile, kb0, nkb;
};

template <class T, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    ummav_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ Args a) {
  using L = Layout<STAGES>;
  using E = Elem<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = ptx::smem_addr(smem);
  const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31);
  const uint32_t bar0 = sbase + L::BAR_OFF;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int acc) { return bar0 + 8u * (2 * STAGES + acc); };
  auto tempty_bar = [&](int acc) { return bar0 + 8u * (2 * STAGES + 2 + acc); };
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      ptx::mbar_init(empty_bar(s), 1);
    }
    for (int acc = 0; acc < 2; ++acc) {
      ptx::mbar_init(tfull_bar(acc), 1);
      ptx::mbar_init(tempty_bar(acc), 128);
    }
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tensormap(&tmA);
    ptx::prefetch_tensormap(&tmB);
  }
  __syncthreads();  // barriers initialised
  // The producer starts streaming at once; TMEM is allocated meanwhile and its
  // address shared among warps 1..5 only (named barrier 1).
  uint32_t tmem_base = 0;
  if (warp != 0) {
    if (warp == 1) {
      ptx::tmem_alloc(ptx::smem_addr(tmem_slot), L::TMEM_COLS);
      ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    ptx::named_barrier(1, kThreads - 32);
    ptx::tc_fence_after();
    tmem_base = *tmem_slot;
  }
  const unsigned r0 = range_start(a, blockIdx.x), r1 = range_start(a, blockIdx.x + 1);
  auto next_seg = [&](unsigned pos) {
    Seg s;
    const unsigned t = pos / unsigned(a.kb);
    s.tile = int(t);
    s.kb0 = int(pos - t * unsigned(a.kb));
    s.nkb = int(min(unsigned(a.kb - s.kb0), r1 - pos));
    return s;
  };
  if (STAGES < 8 && warp == 0 && lane == 0) {
    // The weights of this CTA's first STAGES k-blocks into L2 while the
    // previous grid ends (ptx::tma_prefetch_3d: a hint, safe before the wait).
    // Shallow rings only. A/B on a B200 (graph windows, eight decode shapes):
    // with it the 6-stage config (two CTAs per SM) ran 4-8% faster, the
    // 11-stage one (one CTA per SM) ~2% slower on six of eight: its own ring
    // already covers the start, and the prefetches add L2 requests.
    int n = 0;
    for (unsigned pos = r0; pos < r1 && n < STAGES;) {
      const Seg sg = next_seg(pos);
      for (int i = 0; i < sg.nkb && n < STAGES; ++i, ++n) {
        const int k0 = (sg.kb0 + i) * BK;
        if (k0 + BK > a.K) break;  // whole boxes only (as the umma kernels)
        if (sg.tile * BMN + 64 <= a.N) ptx::tma_prefetch_3d(&tmB, sg.tile * BMN, k0, 0);
        if (sg.tile * BMN + 128 <= a.N) ptx::tma_prefetch_3d(&tmB, sg.tile * BMN + 64, k0, 0);
      }
      pos += sg.nkb;
    }
  }
  // Programmatic dependent launch: no global memory is read or written before
  // the grids this one depends on have completed.
  ptx::griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    // One lane runs the loop (no warp-wide shuffle or __syncwarp per k-block).
    uint32_t filled = 0, fill_parity = 0;
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (unsigned pos = r0; pos < r1 && ok;) {
        const Seg sg = next_seg(pos);
        for (int i = 0; i < sg.nkb; ++i) {
          ok = ptx::mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, a.status, kStatusTimeoutProducer,
                                      a.wait_limit_ns);
          if (!ok) break;
          const int k0 = (sg.kb0 + i) * BK;
          const uint32_t fb = full_bar(stage);
          ptx::mbar_arrive_expect_tx(fb, L::STAGE_TX);
          const uint32_t sb = sbase + L::B_OFF + stage * L::B_BYTES;
          ptx::tma_load_3d(sb, &tmB, fb, sg.tile * BMN, k0, 0);
          ptx::tma_load_3d(sb + 8192, &tmB, fb, sg.tile * BMN + 64, k0, 0);
          ptx::tma_load_3d(sbase + L::A_OFF + stage * L::A_BYTES, &tmA, fb, k0, 0, 0);
          filled |= 1u << stage;
          fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        pos += sg.nkb;
      }
    }
    __syncwarp();
    ptx::griddep_launch_dependents();  // every load is issued: dependents may start their prologue
    if (lane == 0)
      for (int s = 0; s < STAGES; ++s)
        if (filled & (1u << s))
          if (!ptx::mbar_wait_teardown(full_bar(s), (fill_parity >> s) & 1u, a.wait_limit_ns) && a.status)
            atomicOr(a.status, kStatusTimeoutDrain);
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (one lane)
    constexpr uint32_t idesc = ptx::umma_idesc_f16(Elem<T>::kBf16, /*a MN-major*/ true, /*b K-major*/ false, BMN, MPAD);
    if (lane == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (unsigned pos = r0; pos < r1 && ok;) {
        const Seg sg = next_seg(pos);
        ok = ptx::mbar_wait_bounded(tempty_bar(acc), acc_phase ^ 1u, abort_flag, a.status, kStatusTimeoutMma,
                                    a.wait_limit_ns);
        if (!ok) break;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * MPAD);
        for (int i = 0; i < sg.nkb; ++i) {
          ok = ptx::mbar_wait_bounded(full_bar(stage), phase, abort_flag, a.status, kStatusTimeoutMma,
                                      a.wait_limit_ns);
          if (!ok) break;
          ptx::tc_fence_after();
          const uint32_t sb = sbase + L::B_OFF + stage * L::B_BYTES;
          const uint32_t sa = sbase + L::A_OFF + stage * L::A_BYTES;
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks) {
            // Weights: N-major [k][n] rows of 128 B, 16 k-rows per step; activations: K-major, 32 B per step.
            const uint64_t wd = ptx::sdesc_sw128(sb + ks * 2048u, 8192u, 1024u);
            const uint64_t xd = ptx::sdesc_sw128(sa + ks * 32u, 16u, 1024u);
            ptx::umma_f16(d_tmem, wd, xd, idesc, (i > 0 || ks > 0) ? 1u : 0u);
          }
          ptx::umma_commit(empty_bar(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        ptx::umma_commit(tfull_bar(acc));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
        pos += sg.nkb;
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // weight column within the tile
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (unsigned pos = r0; pos < r1 && ok;) {
      const Seg sg = next_seg(pos);
      if (lane == 0)
        ok = ptx::mbar_wait_bounded(tfull_bar(acc), acc_phase, abort_flag, a.status, kStatusTimeoutEpilogue,
                                    a.wait_limit_ns);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      ptx::tc_fence_after();
      uint32_t r[16];
      ptx::tmem_ld_32x32b_x16(tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * MPAD), r);
      ptx::tmem_ld_wait(r);
      ptx::tc_fence_before();
      ptx::mbar_arrive(tempty_bar(acc));  // the values are in registers: free the accumulator
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;

      const unsigned tile_first = unsigned(sg.tile) * unsigned(a.kb);
      const int c_first = owner_of(a, tile_first);
      const int nseg = owner_of(a, tile_first + a.kb - 1) - c_first + 1;
      const int n = sg.tile * BMN + row;
      T* C = static_cast<T*>(a.C);
      if (nseg == 1) {
        if (n < a.N)
#pragma unroll
          for (int m = 0; m < MPAD; ++m) {
            if (m >= a.M) break;
            float x = a.alpha * __uint_as_float(r[m]);
            T* q = C + (long long)m * a.ldc + n;
            if (a.beta != 0.f) x += a.beta * E::to_f32(*q);
            *q = E::from_f32(x);
          }
      } else {
        // Each epilogue warp owns 32 weight columns of the tile and settles
        // them alone: its own partial rows, its own ticket on the
        // (tile, quarter) counter, its own ordered sum. No cross-warp barrier.
        const int seg = int(blockIdx.x) - c_first;
        float* slots = a.partials + (long long)sg.tile * a.maxseg * (MPAD * BMN);
        float* mine = slots + (long long)seg * (MPAD * BMN);
#pragma unroll
        for (int m = 0; m < MPAD; ++m)
          if (m < a.M) __stcg(mine + m * BMN + row, __uint_as_float(r[m]));
        __threadfence();  // this lane's partial is visible device-wide before the ticket
        __syncwarp();
        unsigned* counter = a.counters + (long long)sg.tile * 4 + quarter;
        int last = 0;
        if (lane == 0) last = atomicAdd(counter, 1u) == unsigned(nseg - 1);
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();  // acquire the other segments' partials
          // Sum segments 0..nseg-1 in order per element, in blocks of 8 rows x
          // 8 segments so 64 independent L2 loads are in flight per thread.
          for (int m0 = 0; m0 < a.M; m0 += 8) {
            float sum[8];
            for (int q0 = 0; q0 < nseg; q0 += 8) {
              float v[8][8];
#pragma unroll
              for (int u = 0; u < 8; ++u)
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  v[u][j] = (q0 + u < nseg && m0 + j < a.M)
                                ? __ldcg(slots + (long long)(q0 + u) * (MPAD * BMN) + (m0 + j) * BMN + row)
                                : 0.f;
#pragma unroll
              for (int u = 0; u < 8; ++u)
                if (q0 + u < nseg)
#pragma unroll
                  for (int j = 0; j < 8; ++j) sum[j] = (q0 + u == 0) ? v[u][j] : sum[j] + v[u][j];
            }
            if (n < a.N)
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                if (m0 + j >= a.M) break;
                float x = a.alpha * sum[j];
                T* qp = C + (long long)(m0 + j) * a.ldc + n;
                if (a.beta != 0.f) x += a.beta * E::to_f32(*qp);
                *qp = E::from_f32(x);
              }
          }
          __syncwarp();
          if (lane == 0) *counter = 0;  // ready for the next launch
        }
      }
      pos += sg.nkb;
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    if (lane == 0) {
      ptx::umma_commit(drain_bar);
      if (!ptx::mbar_wait_teardown(drain_bar, 0, a.wait_limit_ns) && a.status) atomicOr(a.status, kStatusTimeoutDrain);
    }
    __syncwarp();
    ptx::tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}


struct Plan {
  int tiles, kb, grid, maxseg;
  long long total;
};

// The grid G. When s whole-tile splits (s = resident slots / tiles, at
// least 1) still fill three quarters of the slots, G = tiles * s: CTA c
// covers [T*c/G, T*(c+1)/G), so every tile is cut into exactly s equal
// segments, and at s = 1 each CTA streams one whole tile and stores it
// directly, with no partials and no tickets (M = 1, K x N = 4096 x 14336: 112
// CTAs, each 1 MB of weights, as cuBLAS's own decode kernel streams it).
// Otherwise the slots share the k-blocks evenly (stream-K).
// maxseg: segments per tile, at most (a CTA covers floor or ceil of T/G).
Plan make_plan(int cfg, const gemm::GemmParams& p) {
  const gemm::UmmavConfig& c = gemm::UMMAV_CONFIGS[cfg];
  Plan pl;
  pl.tiles = ceil_div(p.N, BMN);
  pl.kb = ceil_div(p.K, BK);
  pl.total = (long long)pl.tiles * pl.kb;
  const gpu::Target* d = gpu::planning_target();
  const int sms = d ? d->sms : 148;
  const long long slots = (long long)sms * c.CTAS_PER_SM;
  const long long s = pl.tiles <= slots ? std::min<long long>(slots / pl.tiles, pl.kb) : 0;
  if (s >= 1 && 4 * pl.tiles * s >= 3 * slots)
    pl.grid = int(pl.tiles * s);
  else
    pl.grid = int(std::max<long long>(1, std::min<long long>(pl.total, slots)));
  const long long per = pl.total / pl.grid;  // smallest range
  pl.maxseg = int(std::min<long long>(pl.grid, (pl.kb + std::max<long long>(1, per) - 1) / std::max<long long>(1, per) + 1));
  return pl;
}

template <class T, int STAGES>
cudaError_t launch_s(const CUtensorMap& ta, const CUtensorMap& tb, const Args& a, int grid, cudaStream_t s) {
  auto* kern = &ummav_kernel<T, STAGES>;
  static gpu::SmemOptIn optin;
  constexpr size_t smem = size_t(Layout<STAGES>::ALLOC);
  if (const cudaError_t e = optin.ensure(reinterpret_cast<const void*>(kern), smem); e != cudaSuccess) return e;
  // Programmatic dependent launch: this grid's prologue (barrier set-up, TMEM
  // allocation, descriptor prefetch) may overlap the previous grid's tail on
  // the stream; the kernel waits (griddepcontrol.wait) before touching memory.
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, a);
}

// The instantiations gemm::UMMAV_CONFIGS lists.
template <class T>
cudaError_t launch(int stages, const CUtensorMap& ta, const CUtensorMap& tb, const Args& a, int grid,
                   cudaStream_t s) {
  if (stages == 11) return launch_s<T, 11>(ta, tb, a, grid, s);
  if (stages == 6) return launch_s<T, 6>(ta, tb, a, grid, s);
  return cudaErrorNotSupported;
}

}  // namespace ummav

bool ummav_takes(const gemm::GemmParams& p) {
  return p.M <= ummav::MPAD && p.batch == 1 && p.layout_a == gemm::Layout::RowMajor &&
         p.layout_b == gemm::Layout::RowMajor && gemm::tma_compatible(p);
}

bool ummav_applicable(const gemm::GemmParams& p) {
  const gpu::Target* d = gpu::this_device();
  return d && d->cc == 100 && ummav_takes(p);
}

cudaError_t ummav_run(int cfg, const gemm::GemmParams& p, cudaStream_t stream) {
  if (const cudaError_t e = gemm::validate(p); e != cudaSuccess) return e;
  if (gemm::is_empty(p)) return cudaSuccess;
  if (p.alpha == 0.f) return scale_c(p, stream);
  if (!ummav_applicable(p)) return gemv_run(p.M <= 4 ? 0 : (p.M <= 8 ? 1 : 2), p, stream);
  const ummav::Plan pl = ummav::make_plan(cfg, p);
  // The kernel's position arithmetic is 32-bit: total * grid < 2^32 (about
  // 2e11 weight elements at 296 CTAs, far beyond device memory).
  if ((unsigned long long)pl.total * (unsigned long long)pl.grid >= (1ull << 32))
    return gemv_run(p.M <= 4 ? 0 : (p.M <= 8 ? 1 : 2), p, stream);
  CUtensorMap ta, tb;
  if (!encode_map(&ta, p.dtype, p.A, p.K, p.M, p.lda, 1, 0, ummav::MPAD) ||
      !encode_map(&tb, p.dtype, p.B, p.N, p.K, p.ldb, 1, 0, ummav::BK))
    return gemv_run(p.M <= 4 ? 0 : (p.M <= 8 ? 1 : 2), p, stream);
  ummav::Args a{};
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.tiles = pl.tiles;
  a.kb = pl.kb;
  a.total = unsigned(pl.total);
  a.C = p.C;
  a.ldc = p.ldc;
  a.alpha = p.alpha;
  a.beta = p.beta;
  a.maxseg = pl.maxseg;
  a.wait_limit_ns = kDefaultWaitLimitNs;
  if (const cudaError_t e = status::word(&a.status); e != cudaSuccess) return e;
  if (pl.maxseg > 1) {
    void* cnt = nullptr;
    void* part = nullptr;
    if (const cudaError_t e = scratch::acquire(stream, size_t(pl.tiles) * 4 * sizeof(unsigned), scratch::Kind::Tickets, &cnt);
        e != cudaSuccess)
      return e;
    const size_t pbytes = size_t(pl.tiles) * pl.maxseg * ummav::MPAD * ummav::BMN * sizeof(float);
    if (const cudaError_t e = scratch::acquire(stream, pbytes, scratch::Kind::Partials, &part); e != cudaSuccess) return e;
    a.counters = static_cast<unsigned*>(cnt);
    a.partials = static_cast<float*>(part);
  }
  const int stages = gemm::UMMAV_CONFIGS[cfg].STAGES;
  return p.dtype == gemm::DType::BF16 ? ummav::launch<__nv_bfloat16>(stages, ta, tb, a, pl.grid, stream)
                                      : ummav::launch<__half>(stages, ta, tb, a, pl.grid, stream);
}

gemm::LaunchPlan ummav_plan(int cfg, const gemm::GemmParams& p) {
  const ummav::Plan pl = ummav::make_plan(cfg, p);
  gemm::LaunchPlan r;
  r.splits = pl.maxseg;
  r.k_chunk = int(std::min<long long>(pl.total / std::max(1, pl.grid), pl.kb) * ummav::BK);
  r.tiles = pl.tiles;
  r.grid = unsigned(pl.grid);
  return r;
}

cudaError_t ummav_attrs(int cfg, cudaFuncAttributes* attrs) {
  const bool deep = gemm::UMMAV_CONFIGS[cfg].STAGES == 11;
  const cudaError_t e = deep ? cudaFuncGetAttributes(attrs, &ummav::ummav_kernel<__half, 11>)
                             : cudaFuncGetAttributes(attrs, &ummav::ummav_kernel<__half, 6>);
  if (e == cudaSuccess) attrs->sharedSizeBytes += unsigned(ummav_smem_bytes(cfg));
  return e;
}

size_t ummav_smem_bytes(int cfg) {
  return gemm::UMMAV_CONFIGS[cfg].STAGES == 11 ? size_t(ummav::Layout<11>::ALLOC) : size_t(ummav::Layout<6>::ALLOC);
}

}  // namespace aegis
