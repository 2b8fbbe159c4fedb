#pragma once
// In-order dynamic tile schedule for the persistent umma kernels, on
// Blackwell cluster launch control (CLC).
//
// The grid has one cluster per unit (tile x split), so every unit has a
// cluster that would run it. The clusters that fit start; each runs its own
// unit (cluster index), then asks the hardware to cancel a cluster that has
// not started yet and runs that cluster's unit instead, until a request
// fails. Clusters start and are cancelled in launch order, so the units in
// flight stay a contiguous run of the raster: the tiles running at the same
// time share A and B stripes in L2. (A static round-robin lets CTAs drift
// apart over a long run; at 16384^3 that doubled the DRAM reads.)
//
// One lane (the producer of the pair leader, or of the lone CTA) owns the
// requests: it issues the request for the next unit while it loads the
// current one, and publishes each answer (the unit, or -1 = done) through a
// kSchedDepth-deep ring of shared-memory slots to every other role: the MMA
// lane, the epilogue warps, and in a pair the peer CTA's producer and
// epilogue warps (the leader writes the peer's slot with st.shared::cluster
// and arrives on the peer's barrier; consumers release slots on the leader's
// "empty" barrier). Every wait is bounded like the kernels' other waits.
#include <cstdint>

#include "common.cuh"
#include "ptx.cuh"

namespace aegis::umma {

inline constexpr int kSchedDepth = 4;

// Shared-memory block of the schedule (16-byte aligned): CLC response,
// unit slots, and the clc / full[D] / empty[D] mbarriers.
struct SchedSmem {
  static constexpr int RESP = 0;                             // 16 B
  static constexpr int SLOTS = 16;                           // int64 each
  static constexpr int BARS = SLOTS + 8 * kSchedDepth;       // clc, full[D], empty[D]
  static constexpr int BYTES = BARS + 8 * (1 + 2 * kSchedDepth);
};

struct Sched {
  uint32_t base;  // this CTA's SchedSmem block
  volatile int* abort;
  unsigned* status;
  long long limit_ns;

  __device__ uint32_t resp() const { return base + SchedSmem::RESP; }
  __device__ uint32_t slot(int i) const { return base + SchedSmem::SLOTS + 8u * uint32_t(i); }
  __device__ uint32_t clc_bar() const { return base + SchedSmem::BARS; }
  __device__ uint32_t full_bar(int i) const { return base + SchedSmem::BARS + 8u * uint32_t(1 + i); }
  __device__ uint32_t empty_bar(int i) const {
    return base + SchedSmem::BARS + 8u * uint32_t(1 + kSchedDepth + i);
  }

  // One thread, before the CTA's first barrier sync. `consumers` = arrivals
  // that free a slot (every role that reads it).
  __device__ void init(uint32_t consumers) const {
    ptx::mbar_init(clc_bar(), 1);
    for (int i = 0; i < kSchedDepth; ++i) {
      ptx::mbar_init(full_bar(i), 1);
      ptx::mbar_init(empty_bar(i), consumers);
    }
  }
};

// State of the lane that owns the requests.
struct SchedOwner {
  int seq = 0;            // slots published
  uint32_t clc_phase = 0;
  bool pending = false;   // a request is in flight
  bool exhausted = false; // a request failed: none may follow

  // Request the next unit (no-op once exhausted or while one is pending).
  __device__ void request(const Sched& s) {
    if (exhausted || pending) return;
    ptx::mbar_arrive_expect_tx(s.clc_bar(), 16);
    ptx::clc_try_cancel(s.resp(), s.clc_bar());
    pending = true;
  }

  // The answer to the pending request (-1 when none was pending or it
  // failed), published to every consumer; `peer` also writes CTA rank 1 of a
  // pair. False if a wait ran out (the abort flag is then set).
  __device__ bool publish_next(const Sched& s, int ctas_per_cluster, bool peer, long long* next, unsigned bit) {
    long long nxt = -1;
    if (pending) {
      if (!ptx::mbar_wait_bounded(s.clc_bar(), clc_phase, s.abort, s.status, bit, s.limit_ns)) return false;
      clc_phase ^= 1u;
      pending = false;
      const int x = ptx::clc_first_ctaid_x(s.resp());
      if (x < 0)
        exhausted = true;
      else
        nxt = x / ctas_per_cluster;
    }
    const int i = seq % kSchedDepth;
    const uint32_t par = uint32_t(seq / kSchedDepth) & 1u;
    if (!ptx::mbar_wait_bounded_cluster(s.empty_bar(i), par ^ 1u, s.abort, s.status, bit, s.limit_ns)) return false;
    ptx::st_shared_s64(s.slot(i), nxt);
    if (peer) {
      ptx::st_cluster_s64(ptx::map_to_rank(s.slot(i), 1), nxt);
      ptx::mbar_arrive_cluster(ptx::map_to_rank(s.full_bar(i), 1));
    }
    ptx::mbar_arrive(s.full_bar(i));
    ++seq;
    *next = nxt;
    return true;
  }

  // Teardown: a request still in flight lands before shared memory is
  // released (bounded; ignores the abort flag).
  __device__ void drain(const Sched& s) {
    if (pending && !ptx::mbar_wait_teardown(s.clc_bar(), clc_phase, s.limit_ns) && s.status)
      atomicOr(s.status, kStatusTimeoutDrain);
    pending = false;
  }
};

// A consumer's next unit (slot `seq`); releases the slot on the owner's
// barrier (in cluster CTA 0; `remote` when that is another CTA).
__device__ __forceinline__ bool sched_take(const Sched& s, int& seq, bool remote, long long* unit, unsigned bit) {
  const int i = seq % kSchedDepth;
  const uint32_t par = uint32_t(seq / kSchedDepth) & 1u;
  if (!ptx::mbar_wait_bounded_cluster(s.full_bar(i), par, s.abort, s.status, bit, s.limit_ns)) return false;
  *unit = ptx::ld_shared_s64(s.slot(i));
  if (remote)
    ptx::mbar_arrive_cluster(ptx::map_to_rank(s.empty_bar(i), 0));
  else
    ptx::mbar_arrive(s.empty_bar(i));
  ++seq;
  return true;
}

}  // namespace aegis::umma
