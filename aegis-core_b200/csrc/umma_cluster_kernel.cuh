#pragma once
// Cluster split-K umma kernel (configs with the suffix _kcl).
//
// For problems whose tiles cannot fill the SMs (512^3, 1024^3): a cluster of
// S CTAs (S = 1, 2, 4 or 8, one per SM) computes one 128 x BN output tile,
// CTA r over the r-th of S even slices of the k-blocks, into its own TMEM
// accumulator. The partial tiles are reduced inside the cluster through
// distributed shared memory, in the same launch:
//   - tile rows are divided evenly among the S CTAs (CTA q owns rows
//     [q*128/S, (q+1)*128/S));
//   - each epilogue thread holds one tile row (tcgen05.ld 32x32b) and stores
//     it, FP32, into slot r of the owning CTA's receive buffer
//     (st.shared::cluster), then arrives on the owner's "received" mbarrier
//     with release at cluster scope;
//   - once all S x 128/S rows have arrived (acquire at cluster scope), the
//     owner's epilogue warps sum slots 0..S-1 in that fixed order per element,
//     apply alpha/beta and store the 16-bit result to C.
// The sum order depends only on S, which depends only on the shape, so the
// result is bitwise identical run to run. Compared with the _ksm configs,
// nothing goes through global memory and there is no second kernel; compared
// with one CTA per tile, each SM loads 1/S of the tile's A and B panels.
//
// The reference's split-K is an ordered ticket in the last CTA of each tile
// over global partial slots (src/gemm/splitk.cuh:155-222); the fixed slot
// order 0..S-1 is the same guarantee.
//
// Not persistent: one tile per cluster (the configs target problems with at
// most one wave of clusters). Barriers: a cluster barrier phase started after
// the prologue is completed before any remote store or arrive (every CTA's
// mbarriers exist), and a final cluster barrier keeps every CTA resident
// until no other CTA can still touch its shared memory. Every mbarrier wait is
// bounded as in the other umma kernels; the cluster barriers are reached on
// every path.
#include "umma_kernel.cuh"

namespace aegis::umma {

inline constexpr int kMaxClusterSplits = 8;  // portable cluster size

template <int BN, int STAGES>
struct LayoutCluster {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_TX = A_BYTES + B_BYTES;
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = STAGES * A_BYTES;
  static constexpr int RECV_OFF = STAGES * (A_BYTES + B_BYTES);
  // One FP32 tile row plus 16 bytes: the 16-byte stores of 8 consecutive rows
  // (one shared-memory wavefront) fall in distinct banks.
  static constexpr int RSTRIDE = BN * 4 + 16;
  static constexpr int RECV_BYTES = BM * RSTRIDE;  // S slots x 128/S rows
  static constexpr int BAR_OFF = RECV_OFF + RECV_BYTES;
  static constexpr int NBARS = 2 * STAGES + 3;  // full[S], empty[S], tfull, received, drain
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int BYTES = MISC_OFF + 16;
  static constexpr int ALLOC = BYTES + 1024;  // dynamic smem requested (1024-byte alignment slack)
  static constexpr int TMEM_COLS = BN;
  static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "tiles must stay 1024-byte aligned");
  static_assert(RSTRIDE % 16 == 0 && BAR_OFF % 8 == 0, "16-byte rows, 8-byte barriers");
  static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0,
                "TMEM allocation is a power of two of at least 32 columns");
  static_assert(ALLOC <= 232448, "fits the shared memory a CTA may use");
};

// Stores this thread's tile row (BN FP32 values from TMEM, 32 columns per
// load, the next load in flight while the current chunk is stored) to
// `dst`, a shared::cluster address in the owning CTA.
template <int BN>
__device__ __forceinline__ void send_row(uint32_t t_row, uint32_t dst) {
  static_assert(BN % 64 == 0, "chunks are taken in pairs");
  uint32_t r0[32], r1[32];
  ptx::tmem_ld_32x32b_x32(t_row, r0);
#pragma unroll
  for (int c = 0; c < BN / 32; c += 2) {
    ptx::tmem_ld_wait(r0);
    ptx::tmem_ld_32x32b_x32(t_row + uint32_t((c + 1) * 32), r1);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      ptx::st_cluster_v4(dst + uint32_t(c * 128 + q * 16), r0[4 * q], r0[4 * q + 1], r0[4 * q + 2], r0[4 * q + 3]);
    ptx::tmem_ld_wait(r1);
    if (c + 2 < BN / 32) ptx::tmem_ld_32x32b_x32(t_row + uint32_t((c + 2) * 32), r0);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      ptx::st_cluster_v4(dst + uint32_t((c + 1) * 128 + q * 16), r1[4 * q], r1[4 * q + 1], r1[4 * q + 2],
                         r1[4 * q + 3]);
  }
}

// The launch: grid.x = tiles * S, cluster dims (S, 1, 1), S in {1, 2, 4, 8}
// and S <= a.kb_total; a.splits == 1 and a.kb_per_split == a.kb_total (the
// tile walk of decode_unit_tm), a.units == tiles.
template <class T, int BN, int STAGES, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    umma_cluster_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ Args a) {
  using L = LayoutCluster<BN, STAGES>;
  using E = Elem<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = ptx::smem_addr(smem);
  const int warp = int(threadIdx.x >> 5);
  const int lane = int(threadIdx.x & 31);
  const uint32_t S = ptx::cluster_nctarank();
  const uint32_t rank = ptx::cluster_ctarank();
  const uint32_t R = uint32_t(BM) / S;  // tile rows each CTA reduces
  // The host launches S in {1, 2, 4, 8} with S <= kb_total; any other cluster
  // shape skips the exchange (every owner index stays below S) and reports.
  const bool shape_ok = (S & (S - 1u)) == 0u && S <= uint32_t(kMaxClusterSplits) && S <= uint32_t(a.kb_total);

  const uint32_t bar0 = sbase + L::BAR_OFF;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  const uint32_t tfull_bar = bar0 + 8u * (2 * STAGES);
  const uint32_t recv_bar = bar0 + 8u * (2 * STAGES + 1);
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);

  // This CTA's tile and k-block slice: the even split [r*kb/S, (r+1)*kb/S),
  // never empty for S <= kb_total.
  Unit u = decode_unit_tm<BM, BN>(a, (long long)ptx::cluster_id_x());
  {
    const uint32_t kb = uint32_t(a.kb_total);
    const uint32_t kb0 = rank * kb / S, kb1 = (rank + 1) * kb / S;
    u.kb0 = int(kb0);
    u.nkb = int(kb1 - kb0);
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      ptx::mbar_init(empty_bar(s), 1);
    }
    ptx::mbar_init(tfull_bar, 1);
    ptx::mbar_init(recv_bar, uint32_t(BM));  // S senders x R rows, one arrive per row
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&tmA);
    ptx::prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_addr(tmem_slot), L::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  ptx::cluster_arrive();  // this CTA's barriers exist; waited on before the first remote access
  // Programmatic dependent launch, as in umma_gemm_kernel: no global access
  // before the previous grid on the stream has completed.
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (one lane)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t filled = 0, fill_parity = 0;
      const int za = a.a_batched ? u.b : 0, zb = a.b_batched ? u.b : 0;
      for (int i = 0; i < u.nkb; ++i) {
        if (!ptx::mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, a.status, kStatusTimeoutProducer,
                                    a.wait_limit_ns))
          break;
        const int k0 = (u.kb0 + i) * BK;
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
      // Every copy this CTA issued has landed before shared memory is released.
      for (int s = 0; s < STAGES; ++s)
        if (filled & (1u << s))
          if (!ptx::mbar_wait_teardown(full_bar(s), (fill_parity >> s) & 1u, a.wait_limit_ns) && a.status)
            atomicOr(a.status, kStatusTimeoutDrain);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (one lane)
    constexpr uint32_t idesc = ptx::umma_idesc_f16(Elem<T>::kBf16, A_MN, B_MN, BM, BN);
    constexpr uint32_t a_lbo = A_MN ? 8192u : 16u, b_lbo = B_MN ? 8192u : 16u;
    constexpr uint32_t a_kstep = A_MN ? 2048u : 32u, b_kstep = B_MN ? 2048u : 32u;
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
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
          ptx::umma_f16(tmem_base, ad, bd, idesc, (i > 0 || ks > 0) ? 1u : 0u);
        }
        ptx::umma_commit(empty_bar(stage));
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) ptx::umma_commit(tfull_bar);  // the partial tile is complete
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const uint32_t row_in_tile = uint32_t(quarter * 32 + lane);
    bool ok = true;
    if (lane == 0)
      ok = ptx::mbar_wait_bounded(tfull_bar, 0, abort_flag, a.status, kStatusTimeoutEpilogue, a.wait_limit_ns);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    ptx::cluster_wait();  // every CTA of the cluster has its barriers
    if (!shape_ok && threadIdx.x == 64 && a.status) atomicOr(a.status, kStatusTimeoutEpilogue);
    if (ok && shape_ok) {
      ptx::tc_fence_after();
      // Row -> (owner CTA, row in its slot `rank`).
      const uint32_t owner = row_in_tile / R;
      const uint32_t slot_row = rank * R + (row_in_tile - owner * R);
      const uint32_t dst = ptx::map_to_rank(sbase + uint32_t(L::RECV_OFF) + slot_row * uint32_t(L::RSTRIDE), owner);
      send_row<BN>(tmem_base + (uint32_t(quarter * 32) << 16), dst);
      ptx::mbar_arrive_cluster(ptx::map_to_rank(recv_bar, owner));
    }
    // This CTA's rows: slots 0..S-1 of the receive buffer, summed in order.
    if (shape_ok && ptx::mbar_wait_bounded_cluster(recv_bar, 0, abort_flag, a.status, kStatusTimeoutEpilogue,
                                                   a.wait_limit_ns)) {
      constexpr uint32_t C4 = BN / 4;  // 4-column groups per row
      const uint32_t items = R * C4;
      const uint8_t* recv = smem + L::RECV_OFF;
      T* cb = static_cast<T*>(a.C) + (long long)u.b * a.stride_c;
      for (uint32_t i = threadIdx.x - 64u; i < items; i += 128u) {
        const int rl = int(i / C4), c4 = int(i % C4);
        const int row = u.m0 + int(rank * R) + rl;
        const int col = u.n0 + 4 * c4;
        if (row >= a.M || col >= a.N) continue;
        float4 acc = *reinterpret_cast<const float4*>(recv + rl * L::RSTRIDE + c4 * 16);  // slot 0
        for (uint32_t s = 1; s < S; ++s) {
          const float4 v = *reinterpret_cast<const float4*>(recv + (int(s * R) + rl) * L::RSTRIDE + c4 * 16);
          acc.x += v.x;
          acc.y += v.y;
          acc.z += v.z;
          acc.w += v.w;
        }
        float v[4] = {a.alpha * acc.x, a.alpha * acc.y, a.alpha * acc.z, a.alpha * acc.w};
        T* c = cb + (long long)row * a.ldc + col;
        const int nc = min(4, a.N - col);
        if (a.beta != 0.f)
          for (int j = 0; j < nc; ++j) v[j] += a.beta * E::to_f32(c[j]);
        if (nc == 4 && a.c_vec4) {
          uint2 w;
          w.x = E::pack(v[0], v[1]);
          w.y = E::pack(v[2], v[3]);
          *reinterpret_cast<uint2*>(c) = w;
        } else {
          for (int j = 0; j < nc; ++j) c[j] = E::from_f32(v[j]);
        }
      }
    }
  }

  // ------------------------------------------------ teardown
  if (warp < 2) ptx::cluster_wait();  // the epilogue warps completed this phase before their remote stores
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
  ptx::cluster_sync();  // no CTA leaves while another may still store into its shared memory
}

}  // namespace aegis::umma
