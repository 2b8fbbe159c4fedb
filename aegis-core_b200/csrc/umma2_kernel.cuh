#pragma once
// The tcgen05 GEMM on CTA pairs (cta_group::2): one 256 x BN output tile per
// pair of SMs.
//
// A cluster of two CTAs shares each tile: CTA r loads rows [m0 + 128r, +128)
// of A and columns [n0 + r*BN/2, +BN/2) of B into its own shared memory (plain
// TMA, no multicast; the transaction bytes of both CTAs complete on the
// leader's "full" barrier), the leader (rank 0) issues
// tcgen05.mma.cta_group::2 with M = 256, N = BN, which reads both CTAs' tiles
// and writes each CTA's 128 rows of the accumulator into that CTA's TMEM,
// and commits to the barrier at the same offset in both CTAs (tcgen05.commit
// .multicast::cluster: "stage free" to both producers, "accumulator ready" to
// both epilogues). Each CTA's epilogue writes its 128 rows and releases the
// accumulator with a remote arrive on the leader's "empty" barrier.
//
// Per SM and k-block this moves 32 KB instead of the 48 KB of the one-CTA
// 128 x 256 tile for the same tensor work, so six stages fit and the L2->SM
// traffic per FLOP drops by a third.
//
// Start and end are guarded by cluster barriers (no remote arrive before the
// peer's barriers exist, no CTA leaves while its peer may still touch its
// memory). Every mbarrier wait is bounded as in the one-CTA kernel; at
// teardown each CTA waits (bounded) until the copies it issued have landed.
#include "umma_kernel.cuh"

namespace aegis::umma {

inline constexpr int BM_PAIR = 256;

template <int BN, int STAGES>
struct LayoutPair {
  static constexpr int A_BYTES = 128 * BK * 2;       // this CTA's 128 rows of A
  static constexpr int B_BYTES = (BN / 2) * BK * 2;  // this CTA's BN/2 columns of B
  static constexpr int STAGE_TX = A_BYTES + B_BYTES;
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = STAGES * A_BYTES;
  static constexpr int BAR_OFF = STAGES * (A_BYTES + B_BYTES);
  static constexpr int NBARS = 2 * STAGES + 5;  // full[S], empty[S], tfull[2], tempty[2], drain
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int SCHED_OFF = (MISC_OFF + 16 + 15) / 16 * 16;  // tile schedule (tile_sched.cuh)
  static constexpr int BYTES = SCHED_OFF + SchedSmem::BYTES;
  static constexpr int ALLOC = BYTES + 1024;
  static constexpr int TMEM_COLS = 2 * BN;
  static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "tiles must stay 1024-byte aligned");
  static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation is a power of two");
};

template <int BN>
__device__ __forceinline__ Unit decode_unit_pair(const Args& a, long long u) {
  return decode_unit_tm<BM_PAIR, BN>(a, u);
}

template <class T, int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    umma2_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ Args a) {
  using L = LayoutPair<BN, STAGES>;
  constexpr int BNH = BN / 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = ptx::smem_addr(smem);
  const int warp = int(threadIdx.x >> 5);
  const int lane = int(threadIdx.x & 31);
  const uint32_t rank = ptx::cluster_ctarank();  // 0: the pair leader
  const long long first_unit = blockIdx.x >> 1;  // one cluster per unit; later units come from the schedule

  const uint32_t bar0 = sbase + L::BAR_OFF;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int acc) { return bar0 + 8u * (2 * STAGES + acc); };
  auto tempty_bar = [&](int acc) { return bar0 + 8u * (2 * STAGES + 2 + acc); };
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);
  const Sched sched{sbase + L::SCHED_OFF, abort_flag, a.status, a.wait_limit_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      ptx::mbar_init(full_bar(s), 1);   // the leader's producer arrives; both CTAs' bytes complete it
      ptx::mbar_init(empty_bar(s), 1);  // the leader's multicast commit
    }
    for (int acc = 0; acc < 2; ++acc) {
      ptx::mbar_init(tfull_bar(acc), 1);     // the leader's multicast commit
      ptx::mbar_init(tempty_bar(acc), 256);  // every epilogue thread of both CTAs (leader's copy is used)
    }
    ptx::mbar_init(drain_bar, 1);
    // Schedule slots are released on the leader's barrier by the leader's MMA
    // lane and epilogue warps (1 + 4) and the peer's producer and epilogue
    // warps (1 + 4); the peer's copy of the barrier goes unused.
    sched.init(10);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&tmA);
    ptx::prefetch_tensormap(&tmB);
    // This CTA's half of the first unit's first k-blocks into L2 while the
    // previous grid ends (unsplit walks only, as in umma_gemm_kernel).
    const Unit u = decode_unit_pair<BN>(a, first_unit);
    if (a.splits == 1)
      prefetch_first_blocks<A_MN, B_MN, 128, BNH>(&tmA, &tmB, a.M, a.N, a.K, u.m0 + 128 * int(rank),
                                                u.n0 + BNH * int(rank),
                                                u.rev ? u.kb0 + u.nkb - min(u.nkb, STAGES) : u.kb0,
                                                min(u.nkb, STAGES),
                                                a.a_batched ? u.b : 0, a.b_batched ? u.b : 0);
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(ptx::smem_addr(tmem_slot), L::TMEM_COLS);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  ptx::cluster_sync();  // both CTAs' barriers exist before any remote arrive or copy
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: the prologue above (barriers, TMEM,
  // descriptor prefetch) may overlap the previous grid on the stream; no
  // thread touches global memory before that grid has completed, and the
  // next grid may launch (its CTAs start as SMs free up).
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    // One lane runs the whole loop: a warp-wide shuffle or __syncwarp per
    // k-block measured ~100 cycles of the ~512 a k-block's MMAs take.
    int stage = 0;
    uint32_t phase = 0, filled = 0, fill_parity = 0;
    bool ok = true;
    if (lane == 0) {
      SchedOwner owner;  // used by the leader only
      int seq = 0;       // the peer's position in the schedule
      for (long long unit = first_unit; ok && unit >= 0;) {
        if (rank == 0 && a.steal) owner.request(sched);  // the next unit, answered while this one loads
        const Unit u = decode_unit_pair<BN>(a, unit);
        const int za = a.a_batched ? u.b : 0, zb = a.b_batched ? u.b : 0;
        const int my_m = u.m0 + 128 * int(rank), my_n = u.n0 + BNH * int(rank);
        for (int i = 0; i < u.nkb; ++i) {
          ok = ptx::mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, a.status, kStatusTimeoutProducer,
                                      a.wait_limit_ns);
          if (!ok) break;
          const int k0 = unit_kb(u, i) * BK;
          if (rank == 0) ptx::mbar_arrive_expect_tx(full_bar(stage), 2 * L::STAGE_TX);
          const uint32_t fb = ptx::map_to_rank(full_bar(stage), 0);  // the leader's barrier
          const uint32_t sa = sbase + L::A_OFF + stage * L::A_BYTES;
          const uint32_t sb = sbase + L::B_OFF + stage * L::B_BYTES;
          if constexpr (A_MN) {
#pragma unroll
            for (int j = 0; j < 2; ++j) ptx::tma_load_3d_pair(sa + j * 8192, &tmA, fb, my_m + 64 * j, k0, za);
          } else {
            ptx::tma_load_3d_pair(sa, &tmA, fb, k0, my_m, za);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BNH / 64; ++j) ptx::tma_load_3d_pair(sb + j * 8192, &tmB, fb, my_n + 64 * j, k0, zb);
          } else {
            ptx::tma_load_3d_pair(sb, &tmB, fb, k0, my_n, zb);
          }
          filled |= 1u << stage;
          fill_parity = (fill_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        ok = rank == 0 ? owner.publish_next(sched, 2, true, &unit, kStatusTimeoutProducer)
                       : sched_take(sched, seq, true, &unit, kStatusTimeoutProducer);
      }
      // Teardown: every copy this CTA issued (and a schedule request still in
      // flight) has landed. The leader sees its barrier complete; the peer sees
      // the stage released by the leader's MMA (which waited for the bytes).
      // Immediate on the normal path.
      owner.drain(sched);
      for (int s = 0; s < STAGES; ++s)
        if (filled & (1u << s)) {
          const uint32_t par = (fill_parity >> s) & 1u;
          const bool done = rank == 0 ? ptx::mbar_wait_teardown(full_bar(s), par, a.wait_limit_ns)
                                      : ptx::mbar_wait_teardown(empty_bar(s), par, a.wait_limit_ns);
          if (!done && a.status) atomicOr(a.status, kStatusTimeoutDrain);
        }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (leader only)
    if (rank == 0) {
      constexpr uint32_t idesc = ptx::umma_idesc_f16(Elem<T>::kBf16, A_MN, B_MN, BM_PAIR, BN);
      constexpr uint32_t a_lbo = A_MN ? 8192u : 16u, b_lbo = B_MN ? 8192u : 16u;
      constexpr uint32_t a_kstep = A_MN ? 2048u : 32u, b_kstep = B_MN ? 2048u : 32u;
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      if (lane == 0) {  // one lane issues everything (see the producer)
        int seq = 0;
        for (long long unit = first_unit; ok && unit >= 0;) {
          const Unit u = decode_unit_pair<BN>(a, unit);
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
              ptx::umma_f16_pair(d_tmem, ad, bd, idesc, (i > 0 || ks > 0) ? 1u : 0u);
            }
            ptx::umma_commit_pair(empty_bar(stage), 0x3);  // both CTAs' stage is free
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          ptx::umma_commit_pair(tfull_bar(acc), 0x3);  // both halves of the accumulator ready
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1u;
          ok = sched_take(sched, seq, false, &unit, kStatusTimeoutMma);
        }
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2..5, both CTAs)
    const int quarter = warp & 3;
    const int row_in_tile = 128 * int(rank) + quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    int seq = 0;
    for (long long unit = first_unit; ok && unit >= 0;) {
      const Unit u = decode_unit_pair<BN>(a, unit);
      if (lane == 0)
        ok = ptx::mbar_wait_bounded(tfull_bar(acc), acc_phase, abort_flag, a.status, kStatusTimeoutEpilogue,
                                    a.wait_limit_ns);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      ptx::tc_fence_after();
      const int row = u.m0 + row_in_tile;
      const uint32_t t_row = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
      drain_rows<T, EPI, BN>(a, u, row, t_row);
      ptx::tc_fence_before();
      ptx::mbar_arrive_cluster(ptx::map_to_rank(tempty_bar(acc), 0));  // this half of the accumulator is free
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
      if constexpr (EPI == kEpiPeers) push_warp_rows<T, BN>(a, u, u.m0 + 128 * int(rank) + quarter * 32, lane);
      long long next = -1;
      if (lane == 0) ok = sched_take(sched, seq, rank != 0, &next, kStatusTimeoutEpilogue);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      unit = __shfl_sync(0xffffffffu, next, 0);
    }
    if constexpr (EPI == kEpiPeers) __threadfence_system();
  }

  // ------------------------------------------------ teardown
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1 && lane == 0) {
    if (rank == 0) ptx::umma_commit_pair(drain_bar, 0x3);  // every MMA of the pair has finished
    if (!ptx::mbar_wait_teardown(drain_bar, 0, a.wait_limit_ns) && a.status) atomicOr(a.status, kStatusTimeoutDrain);
  }
  __syncwarp();
  ptx::tc_fence_before();
  ptx::cluster_sync();  // neither CTA leaves while its peer may still touch its memory
  ptx::tc_fence_after();
  if (warp == 1) ptx::tmem_dealloc_pair(tmem_base, L::TMEM_COLS);
}

}  // namespace aegis::umma
