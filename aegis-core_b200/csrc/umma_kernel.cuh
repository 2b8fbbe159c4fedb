#pragma once
// The tcgen05 GEMM kernel (umma family).
//
// C[M,N] (+)= A[M,K] * B[K,N] for one batch entry per tile, f16 or bf16
// operands, FP32 accumulation in tensor memory (TMEM).
//
// Replaces the reference's best large-GEMM kernel, gemm_mma_tma_kernel
// (src/gemm/mma_tma.cu:171-228: TMA box loads into an mbarrier ring feeding
// mma.sync from every warp), with the Blackwell structure:
//   warp 0      TMA producer: lane 0 alone fills a STAGES-deep ring of
//               (A tile, B tile) k-blocks, mbarrier complete_tx;
//   warp 1      allocates 2*BN TMEM columns; one lane issues tcgen05.mma
//               (M=128, N=BN, K=16) for every k-block and commits each stage
//               back to the producer and each finished accumulator to the
//               epilogue;
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//               lanes 32*(w%4)..+31, i.e. tile rows), FP32 -> alpha/beta ->
//               16-bit, stores to C; or FP32 partials (split-K); or the same
//               16-bit tile stored to every rank's C (N-sharded all-gather).
// Persistent with an in-order dynamic schedule (tile_sched.cuh): one CTA per
// unit is launched; the CTAs that fit run their own unit, then take the
// not-yet-started ones in launch order (cluster launch control), walking a
// grouped raster (Args::group_m M-tiles per group) so concurrently running
// tiles share A and B in L2. Two TMEM accumulators let the epilogue of one
// tile overlap the main loop of the next.
//
// Operand layouts in shared memory (128-byte swizzle, TMA writes them):
//   A row-major  (K-major): one box [128 rows][64 k]          16 KB
//   A col-major  (M-major): two boxes [64 k][64 m]             2 x 8 KB
//   B row-major  (N-major): BN/64 boxes [64 k][64 n]           BN/64 x 8 KB
//   B col-major  (K-major): one box [BN rows n][64 k]          BN*128 B
// Edges: TMA zero-fills out-of-range rows/columns/k (so K tails add zeros);
// the epilogue masks rows >= M and columns >= N.
//
// Every wait is bounded (ptx::mbar_wait_bounded): on expiry the CTA records
// a status bit, every role stops waiting, in-flight TMA copies and MMAs are
// drained (bounded), TMEM is freed, and the kernel returns.
#include <cuda.h>

#include <cstdint>

#include "common.cuh"
#include "ptx.cuh"
#include "tile_sched.cuh"

namespace aegis::umma {

inline constexpr int BM = 128;
inline constexpr int BK = 64;  // 64 16-bit elements = one 128-byte swizzle row
inline constexpr int kThreads = 192;
inline constexpr int kGroupM = 8;  // default raster group (tile rows)
inline constexpr int kMaxPeers = 8;

enum Epi : int { kEpiStore = 0, kEpiPartial = 1, kEpiPeers = 2 };

struct Args {
  int M, N, K;
  int batch;
  int a_batched, b_batched;  // use the batch coordinate for A / B loads
  int tiles_m, tiles_n;
  int group_m;      // tile rows per raster group (>= 1)
  int steal;        // more units than resident CTAs (pairs): take the rest by cluster launch control
  int splits, kb_per_split, kb_total;
  long long units;  // batch * tiles_m * tiles_n * splits
  void* C;
  long long ldc, stride_c;
  float alpha, beta;
  float* partials;           // kEpiPartial: [split][batch][M][N] FP32
  void* peers[kMaxPeers];    // kEpiPeers: this rank's C first, then every other rank's (row-major, ldc)
  int npeers, col_offset;    // kEpiPeers: ranks; this rank's first column
  int peer_vec;              // kEpiPeers: 16-byte pushes (aligned bases, ldc and col_offset % 8 == 0)
  unsigned* status;          // per-device watchdog word
  long long wait_limit_ns;
  // K-walk direction by wave: with kdir_wave > 0 a tile walks its k-blocks
  // last to first when its position in the full problem's grouped raster
  // (kdir_tiles_n tile columns, kdir_group rows per group; this launch's
  // tile column 0 is the full grid's column kdir_col0) lies in an odd wave of
  // kdir_wave tiles. Consecutive waves then meet at the same end of K, where
  // the operand blocks the previous wave read last are still in L2. The
  // direction is a function of the tile and the full problem only, so an
  // N-sharded rank sums each element in the same order as the 1-GPU GEMM.
  int kdir_wave, kdir_tiles_n, kdir_col0, kdir_group;
};

template <int BN, int STAGES>
struct Layout {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_TX = A_BYTES + B_BYTES;
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = STAGES * A_BYTES;
  static constexpr int BAR_OFF = STAGES * (A_BYTES + B_BYTES);
  static constexpr int NBARS = 2 * STAGES + 5;  // full[S], empty[S], tfull[2], tempty[2], drain
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int SCHED_OFF = (MISC_OFF + 16 + 15) / 16 * 16;  // tile schedule (tile_sched.cuh)
  static constexpr int BYTES = SCHED_OFF + SchedSmem::BYTES;
  static constexpr int ALLOC = BYTES + 1024;  // dynamic smem requested (1024-byte alignment slack)
  // Split-K partial store staging (kEpiPartial launches only): 4 KB per
  // epilogue warp (32 rows x 128 bytes) after the schedule state. The other
  // epilogues do not request it: the spare shared memory stays L1.
  static constexpr int EPI_WARP_BYTES = 4096;
  static constexpr int EPI_OFF = (BYTES + 127) / 128 * 128;
  static constexpr int ALLOC_STAGED = EPI_OFF + 4 * EPI_WARP_BYTES + 1024;
  static constexpr int alloc_for(int epi) { return epi == kEpiPartial ? ALLOC_STAGED : ALLOC; }
  static constexpr int TMEM_COLS = 2 * BN;
  static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "tiles must stay 1024-byte aligned");
  static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0,
                "TMEM allocation is a power of two of at least 32 columns");
};

struct Unit {
  int b, m0, n0, split, kb0, nkb;
  bool rev;  // walk k-blocks kb0 + nkb - 1 down to kb0
};

// Whether the tile at (tile row mi, tile column ni of this launch) walks K
// backwards (Args::kdir_wave). Tile counts stay below 2^29 (host-checked).
__device__ __forceinline__ bool k_reversed(const Args& a, unsigned mi, unsigned ni) {
  if (a.kdir_wave <= 0) return false;
  const unsigned g = unsigned(a.kdir_group);
  const unsigned gn = ni + unsigned(a.kdir_col0);
  const unsigned grp = mi / g, first_m = grp * g;
  const unsigned gsize = min(unsigned(a.tiles_m) - first_m, g);
  const unsigned idx = grp * g * unsigned(a.kdir_tiles_n) + gn * gsize + (mi - first_m);
  return ((idx / unsigned(a.kdir_wave)) & 1u) != 0;
}

// The i-th k-block a unit loads (0 <= i < nkb).
__device__ __forceinline__ int unit_kb(const Unit& u, int i) { return u.kb0 + (u.rev ? u.nkb - 1 - i : i); }

// Unit -> (split, batch, tile) in the grouped raster, for TM-row tiles. Units
// stay below 2^29 (the host refuses larger plans), so 32-bit unsigned
// arithmetic is exact; the split and batch divisions are skipped when there is
// one of them (a 64-bit division by a run-time value is a long emulated
// sequence, measured at ~0.7 us before a small GEMM's first load).
// Raster position `tile` (batch-major, then the grouped raster of each batch
// entry) -> batch, first row and first column; returns the tile's (row,
// column) index in the grid through mi, ni.
template <int TM, int BN>
__device__ __forceinline__ void decode_tile_tm(const Args& a, unsigned tile, Unit* r, unsigned* mi_out,
                                               unsigned* ni_out) {
  unsigned t = tile;
  r->b = 0;
  if (a.batch > 1) {
    const unsigned per_batch = unsigned(a.tiles_m) * unsigned(a.tiles_n);
    const unsigned b = tile / per_batch;
    r->b = int(b);
    t = tile - b * per_batch;
  }
  const unsigned span = unsigned(a.group_m) * unsigned(a.tiles_n);
  const unsigned grp = t / span;
  const unsigned first_m = grp * unsigned(a.group_m);
  const unsigned gsize = min(unsigned(a.tiles_m) - first_m, unsigned(a.group_m));
  const unsigned rr = t - grp * span;
  const unsigned ni = rr / gsize;
  const unsigned mi = first_m + (rr - ni * gsize);
  r->m0 = int(mi * unsigned(TM));
  r->n0 = int(ni * unsigned(BN));
  *mi_out = mi;
  *ni_out = ni;
}

template <int TM, int BN>
__device__ __forceinline__ Unit decode_unit_tm(const Args& a, long long unit) {
  const unsigned u = unsigned(unit);
  Unit r;
  unsigned tile = u, mi = 0, ni = 0;
  r.split = 0;
  r.rev = false;
  if (a.splits > 1) {
    tile = u / unsigned(a.splits);
    r.split = int(u - tile * unsigned(a.splits));
  }
  decode_tile_tm<TM, BN>(a, tile, &r, &mi, &ni);
  r.kb0 = r.split * a.kb_per_split;
  r.nkb = min(a.kb_total - r.kb0, a.kb_per_split);
  r.rev = k_reversed(a, mi, ni);
  return r;
}

template <int BN>
__device__ __forceinline__ Unit decode_unit(const Args& a, long long u) {
  return decode_unit_tm<BM, BN>(a, u);
}

// L2 prefetch of the first `n` k-blocks of a unit's operand boxes (the
// copies its producer issues first), before griddepcontrol.wait (see
// ptx::tma_prefetch_3d). A_ROWS x 64 of A and B_COLS x 64 of B per k-block,
// in the box shapes of the tensor maps. Only boxes that lie wholly inside the
// matrix are prefetched: with boxes mostly outside it (decode shapes, M of
// 1..16 in a 128-row box) the prefetches measured slower than none.
template <bool A_MN, bool B_MN, int A_ROWS, int B_COLS>
__device__ __forceinline__ void prefetch_first_blocks(const CUtensorMap* tmA, const CUtensorMap* tmB, int M, int N,
                                                      int K, int m0, int n0, int kb0, int n, int za, int zb) {
  for (int i = 0; i < n; ++i) {
    const int k0 = (kb0 + i) * BK;
    if (k0 + BK > K) break;
    if constexpr (A_MN) {
#pragma unroll
      for (int j = 0; j < A_ROWS / 64; ++j)
        if (m0 + 64 * (j + 1) <= M) ptx::tma_prefetch_3d(tmA, m0 + 64 * j, k0, za);
    } else {
      if (m0 + A_ROWS <= M) ptx::tma_prefetch_3d(tmA, k0, m0, za);
    }
    if constexpr (B_MN) {
#pragma unroll
      for (int j = 0; j < B_COLS / 64; ++j)
        if (n0 + 64 * (j + 1) <= N) ptx::tma_prefetch_3d(tmB, n0 + 64 * j, k0, zb);
    } else {
      if (n0 + B_COLS <= N) ptx::tma_prefetch_3d(tmB, k0, n0, zb);
    }
  }
}

// ------------------------------------------------------------- epilogue
template <class T>
__device__ __forceinline__ void store_row_chunk(T* dst, const float (&v)[32], int ncols) {
  using E = Elem<T>;
  if (ncols == 32 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w;
      w.x = E::pack(v[8 * q + 0], v[8 * q + 1]);
      w.y = E::pack(v[8 * q + 2], v[8 * q + 3]);
      w.z = E::pack(v[8 * q + 4], v[8 * q + 5]);
      w.w = E::pack(v[8 * q + 6], v[8 * q + 7]);
      d4[q] = w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < ncols) dst[i] = E::from_f32(v[i]);
  }
}

template <class T, int EPI>
__device__ __forceinline__ void epilogue_chunk(const Args& a, const Unit& u, int row, int col,
                                               const uint32_t (&r)[32]) {
  using E = Elem<T>;
  const int ncols = min(32, a.N - col);
  float v[32];
  if constexpr (EPI == kEpiPartial) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
    float* dst = a.partials + (((long long)u.split * a.batch + u.b) * a.M + row) * (long long)a.N + col;
    if (ncols == 32 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
      float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int q = 0; q < 8; ++q) d4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < ncols) dst[i] = v[i];
    }
  } else if constexpr (EPI == kEpiStore) {
    T* dst = static_cast<T*>(a.C) + (long long)u.b * a.stride_c + (long long)row * a.ldc + col;
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = a.alpha * __uint_as_float(r[i]);
    if (a.beta != 0.f) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < ncols) v[i] += a.beta * E::to_f32(dst[i]);
    }
    store_row_chunk<T>(dst, v, ncols);
  } else {  // kEpiPeers: plain C = A*B into this rank's C (push_warp_rows copies it to the peers)
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
    T* dst = static_cast<T*>(a.peers[0]) + (long long)row * a.ldc + a.col_offset + col;
    store_row_chunk<T>(dst, v, ncols);
  }
}

// kEpiPeers, after the warp has stored its 32 rows of the tile into this
// rank's C and released the accumulator: copies those rows into every other
// rank's C over NVLink. The rows are read back (L2) with the lanes across the
// columns, so each warp store writes 512 contiguous bytes of one row; stored
// straight from the TMEM layout (one row per lane) they were 16-byte pieces of
// 32 rows per instruction, a fraction of the link bandwidth once several
// peers share them. Eight rows' loads are in flight before their stores. The
// copy overlaps the main loop of the next tile (the epilogue warps are
// otherwise idle there).
template <class T, int BN>
__device__ __forceinline__ void push_warp_rows(const Args& a, const Unit& u, int row_first, int lane) {
  static_assert(BN == 256, "one 16-byte piece per lane per row");
  __syncwarp();  // the warp's own stores are visible to all its lanes
  if (a.npeers < 2) return;
  const int ncols = min(BN, a.N - u.n0);
  const T* src = static_cast<const T*>(a.peers[0]);
  const bool vec = a.peer_vec && ncols == BN;
#pragma unroll 1
  for (int i0 = 0; i0 < 32; i0 += 8) {
    if (vec) {
      uint4 v[8];
      long long off[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = row_first + i0 + i;
        off[i] = r < a.M ? (long long)r * a.ldc + a.col_offset + u.n0 + lane * 8 : -1;
        if (off[i] >= 0) v[i] = __ldcg(reinterpret_cast<const uint4*>(src + off[i]));
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (off[i] >= 0)
          for (int p = 1; p < a.npeers; ++p) *reinterpret_cast<uint4*>(static_cast<T*>(a.peers[p]) + off[i]) = v[i];
    } else {
      for (int i = 0; i < 8; ++i) {
        const int r = row_first + i0 + i;
        if (r >= a.M) break;
        const long long base = (long long)r * a.ldc + a.col_offset + u.n0;
        for (int c = lane; c < ncols; c += 32) {
          const T x = src[base + c];
          for (int p = 1; p < a.npeers; ++p) static_cast<T*>(a.peers[p])[base + c] = x;
        }
      }
    }
  }
}

// Warp-wide split-K partial store of one 32-column FP32 chunk through a 4 KB
// shared-memory buffer at `stage`: each lane holds one row (row_first + lane)
// in the TMEM layout; the chunk is written to shared memory row by row and
// stored back with the lanes across the columns, so each 16-byte store of the
// warp lands in whole 128-byte row segments (4 rows per instruction: 8x fewer
// store requests than 16-byte pieces of 32 rows). The 16-byte slots of a row
// are XOR-swizzled by the row, so both shared-memory passes take the minimum
// four wavefronts. Measured on a B200 (graph windows, cold L2, bitwise equal
// outputs): 256^2 x 65536 split-K 21.2 -> 20.6 us, 512^2 x 65536 43.0 -> 40.9
// us. 16-bit C stores stay per row: staged they were 3-6% slower on 512^3 to
// 2048^3 (the extra shared-memory round trip sits on the critical path of a
// one-tile CTA), and so were warps with fewer than 32 rows inside M. The
// caller takes this path only for full warps of full chunks (warp-uniform).
template <class T>
__device__ __forceinline__ void partial_chunk_staged(const Args& a, const Unit& u, int row_first, int lane, int col,
                                                     const uint32_t (&r)[32], uint32_t stage) {
  float* plane = a.partials + ((long long)u.split * a.batch + u.b) * a.M * (long long)a.N;
#pragma unroll
  for (int q = 0; q < 8; ++q)
    ptx::st_shared_v4(stage + uint32_t(lane * 128 + 16 * (q ^ (lane & 7))), r[4 * q], r[4 * q + 1], r[4 * q + 2],
                      r[4 * q + 3]);
  __syncwarp();
  const int q = lane & 7;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int rl = 4 * j + (lane >> 3);
    const uint4 v = ptx::ld_shared_v4(stage + uint32_t(rl * 128 + 16 * (q ^ (rl & 7))));
    *reinterpret_cast<uint4*>(plane + (long long)(row_first + rl) * a.N + col + 4 * q) = v;
  }
  __syncwarp();  // the buffer is rewritten by the next chunk
}

// Reads this warp's 32 rows of a BN-column accumulator from TMEM and hands
// each 32-column chunk to the epilogue. Two register buffers: the next
// chunk's TMEM load is in flight while the current one is converted and
// stored, so a tile costs about one load latency instead of BN/32 of them
// (tcgen05.wait::ld waits for every load this thread has issued, and only
// one is outstanding at each wait). ld and wait run on the whole warp.
// `stage`: this warp's 4 KB staging buffer for split-K partials
// (partial_chunk_staged), or 0 to store each row from its own lane.
template <class T, int EPI, int BN>
__device__ __forceinline__ void drain_rows(const Args& a, const Unit& u, int row, uint32_t t_row,
                                           uint32_t stage = 0) {
  static_assert(BN % 64 == 0, "chunks are taken in pairs");
  uint32_t r0[32], r1[32];
  const int lane = int(threadIdx.x & 31);
  const int row_first = row - lane;
  // Staged partial stores: the whole warp's 32 rows inside M, rows 16-byte
  // aligned (N % 4 == 0; the scratch base is 256-byte aligned). Warp-uniform.
  const bool staged = EPI == kEpiPartial && stage != 0 && row_first + 32 <= a.M && (a.N & 3) == 0;
  ptx::tmem_ld_32x32b_x32(t_row, r0);
#pragma unroll 1
  for (int c = 0; c < BN / 32; c += 2) {
    ptx::tmem_ld_wait(r0);
    ptx::tmem_ld_32x32b_x32(t_row + uint32_t((c + 1) * 32), r1);
    const int col0 = u.n0 + c * 32;
    if (staged && col0 + 32 <= a.N)
      partial_chunk_staged<T>(a, u, row_first, lane, col0, r0, stage);
    else if (row < a.M && col0 < a.N)
      epilogue_chunk<T, EPI>(a, u, row, col0, r0);
    ptx::tmem_ld_wait(r1);
    if (c + 2 < BN / 32) ptx::tmem_ld_32x32b_x32(t_row + uint32_t((c + 2) * 32), r0);
    const int col1 = col0 + 32;
    if (staged && col1 + 32 <= a.N)
      partial_chunk_staged<T>(a, u, row_first, lane, col1, r1, stage);
    else if (row < a.M && col1 < a.N)
      epilogue_chunk<T, EPI>(a, u, row, col1, r1);
  }
}

// ------------------------------------------------------------- kernel
template <class T, int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ Args a) {
  using L = Layout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = ptx::smem_addr(smem);
  const int warp = int(threadIdx.x >> 5);
  const int lane = int(threadIdx.x & 31);

  const uint32_t bar0 = sbase + L::BAR_OFF;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int acc) { return bar0 + 8u * (2 * STAGES + acc); };
  auto tempty_bar = [&](int acc) { return bar0 + 8u * (2 * STAGES + 2 + acc); };
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);
  const Sched sched{sbase + L::SCHED_OFF, abort_flag, a.status, a.wait_limit_ns};
  const long long first_unit = blockIdx.x;  // one CTA per unit; later units come from the schedule

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
    sched.init(1 + 4);  // consumers: the MMA lane, the four epilogue warps
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&tmA);
    ptx::prefetch_tensormap(&tmB);
    // The first unit's first k-blocks into L2 while the previous grid ends
    // (unsplit walks only: split-K units measured up to 6% slower with it).
    const Unit u = decode_unit<BN>(a, first_unit);
    if (a.splits == 1)
      prefetch_first_blocks<A_MN, B_MN, BM, BN>(&tmA, &tmB, a.M, a.N, a.K, u.m0, u.n0,
                                                u.rev ? u.kb0 + u.nkb - min(u.nkb, STAGES) : u.kb0,
                                                min(u.nkb, STAGES),
                                              a.a_batched ? u.b : 0, a.b_batched ? u.b : 0);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_addr(tmem_slot), L::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: the prologue above (barriers, TMEM,
  // descriptor prefetch) may overlap the previous grid on the stream; no
  // thread touches global memory before that grid has completed, and the
  // next grid may launch (its CTAs start as SMs free up).
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    // One lane runs the whole loop: a warp-wide shuffle or __syncwarp per
    // k-block measured ~100 cycles of the ~512 a k-block's MMAs take.
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t filled = 0, fill_parity = 0;  // per stage: ever filled / parity of the last fill
      bool ok = true;
      SchedOwner owner;
      for (long long unit = first_unit; ok && unit >= 0;) {
        if (a.steal) owner.request(sched);  // the next unit, answered while this one loads
        const Unit u = decode_unit<BN>(a, unit);
        const int za = a.a_batched ? u.b : 0, zb = a.b_batched ? u.b : 0;
        for (int i = 0; i < u.nkb; ++i) {
          ok = ptx::mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, a.status, kStatusTimeoutProducer,
                                      a.wait_limit_ns);
          if (!ok) break;
          const int k0 = unit_kb(u, i) * BK;
          const uint32_t fb = full_bar(stage);
          ptx::mbar_arrive_expect_tx(fb, L::STAGE_TX);
          const uint32_t sa = sbase + L::A_OFF + stage * L::A_BYTES;
          const uint32_t sb = sbase + L::B_OFF + stage * L::B_BYTES;
          if constexpr (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) ptx::tma_load_3d(sa + j * 8192, &tmA, fb, u.m0 + 64 * j, k0, za);
          } else {
            ptx::tma_load_3d(sa, &tmA, fb, k0, u.m0, za);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) ptx::tma_load_3d(sb + j * 8192, &tmB, fb, u.n0 + 64 * j, k0, zb);
          } else {
            ptx::tma_load_3d(sb, &tmB, fb, k0, u.n0, zb);
          }
          filled |= 1u << stage;
          fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        ok = owner.publish_next(sched, 1, false, &unit, kStatusTimeoutProducer);
      }
      // Teardown: every copy this CTA issued (and a schedule request still in
      // flight) has landed before shared memory is released (immediate on
      // the normal path: the MMA warp consumed them).
      owner.drain(sched);
      for (int s = 0; s < STAGES; ++s)
        if (filled & (1u << s))
          if (!ptx::mbar_wait_teardown(full_bar(s), (fill_parity >> s) & 1u, a.wait_limit_ns) && a.status)
            atomicOr(a.status, kStatusTimeoutDrain);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = ptx::umma_idesc_f16(Elem<T>::kBf16, A_MN, B_MN, BM, BN);
    // Descriptor strides (bytes): SBO = 8 rows of 128 B; LBO = distance between
    // 64-element chunks along M/N (MN-major only; 1 unit for K-major).
    constexpr uint32_t a_lbo = A_MN ? 8192u : 16u, b_lbo = B_MN ? 8192u : 16u;
    // Advance per K=16 step: 32 B inside the swizzled row (K-major), or 16
    // k-rows of 128 B (MN-major).
    constexpr uint32_t a_kstep = A_MN ? 2048u : 32u, b_kstep = B_MN ? 2048u : 32u;
    if (lane == 0) {  // one lane issues everything (see the producer)
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      int seq = 0;
      for (long long unit = first_unit; ok && unit >= 0;) {
        const Unit u = decode_unit<BN>(a, unit);
        ok = ptx::mbar_wait_bounded(tempty_bar(acc), acc_phase ^ 1u, abort_flag, a.status, kStatusTimeoutMma,
                                    a.wait_limit_ns);
        if (!ok) break;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int i = 0; i < u.nkb; ++i) {
          ok = ptx::mbar_wait_bounded(full_bar(stage), phase, abort_flag, a.status, kStatusTimeoutMma,
                                      a.wait_limit_ns);
          if (!ok) break;
          ptx::tc_fence_after();
          const uint32_t sa = sbase + L::A_OFF + stage * L::A_BYTES;
          const uint32_t sb = sbase + L::B_OFF + stage * L::B_BYTES;
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks) {
            const uint64_t ad = ptx::sdesc_sw128(sa + ks * a_kstep, a_lbo, 1024u);
            const uint64_t bd = ptx::sdesc_sw128(sb + ks * b_kstep, b_lbo, 1024u);
            ptx::umma_f16(d_tmem, ad, bd, idesc, (i > 0 || ks > 0) ? 1u : 0u);
          }
          ptx::umma_commit(empty_bar(stage));  // frees the stage once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        ptx::umma_commit(tfull_bar(acc));  // accumulator complete
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
        ok = sched_take(sched, seq, false, &unit, kStatusTimeoutMma);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    int seq = 0;
    for (long long unit = first_unit; unit >= 0;) {
      const Unit u = decode_unit<BN>(a, unit);
      bool ok = true;
      if (lane == 0)
        ok = ptx::mbar_wait_bounded(tfull_bar(acc), acc_phase, abort_flag, a.status, kStatusTimeoutEpilogue,
                                    a.wait_limit_ns);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      ptx::tc_fence_after();
      const int row = u.m0 + row_in_tile;
      const uint32_t t_row = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
      drain_rows<T, EPI, BN>(a, u, row, t_row,
                             EPI == kEpiPartial ? sbase + uint32_t(L::EPI_OFF + quarter * L::EPI_WARP_BYTES) : 0u);
      ptx::tc_fence_before();
      ptx::mbar_arrive(tempty_bar(acc));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
      if constexpr (EPI == kEpiPeers) push_warp_rows<T, BN>(a, u, u.m0 + quarter * 32, lane);
      long long next = -1;
      if (lane == 0) ok = sched_take(sched, seq, false, &next, kStatusTimeoutEpilogue);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      unit = __shfl_sync(0xffffffffu, next, 0);
    }
    if constexpr (EPI == kEpiPeers) __threadfence_system();  // peer stores complete before the kernel ends
  }

  // ------------------------------------------------ teardown
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    if (lane == 0) {
      // Every MMA this CTA issued has finished before TMEM is released.
      ptx::umma_commit(drain_bar);
      if (!ptx::mbar_wait_teardown(drain_bar, 0, a.wait_limit_ns) && a.status) atomicOr(a.status, kStatusTimeoutDrain);
    }
    __syncwarp();
    ptx::tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

}  // namespace aegis::umma
