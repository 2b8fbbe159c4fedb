#pragma once
// Runtime device limits. Every launch-sizing decision (split-K S, grid size,
// smem opt-in) reads these, never a constant tuned on one device
// (reference src/hw/device.h:23-95: DeviceLimits, current/physical,
// ScopedSimulation, once_per_device, configure_smem).
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <string>

namespace aegis::hw {

inline constexpr int kMaxCachedDevices = 64;

struct DeviceLimits {
  int device = -1;
  std::string name;
  int arch = 0;  // major*10 + minor (B200: 100)
  int sm_count = 0;
  size_t smem_per_sm = 0;
  size_t smem_per_block = 0;
  size_t smem_per_block_optin = 0;
  int regs_per_sm = 0;
  int regs_per_block = 0;
  int max_threads_per_sm = 0;
  int max_threads_per_block = 0;
  size_t l2_bytes = 0;
  size_t global_mem_bytes = 0;
  bool unified = false;
  bool simulated = false;
};

cudaError_t query(int dev, DeviceLimits* out);
// The current device's limits (cached), or the thread's simulated profile.
const DeviceLimits* current();
// The real current device, ignoring any simulation.
const DeviceLimits* physical();

// While alive, current() on this thread returns `sim` (sizing decisions only;
// launches still run on the real device). Used by CPU-side sizing tests.
class ScopedSimulation {
 public:
  explicit ScopedSimulation(const DeviceLimits& sim);
  ~ScopedSimulation();
  ScopedSimulation(const ScopedSimulation&) = delete;
  ScopedSimulation& operator=(const ScopedSimulation&) = delete;

 private:
  DeviceLimits sim_;
  const DeviceLimits* prev_;
};

struct PerDevice {
  std::atomic<int> state[kMaxCachedDevices] = {};  // 0: not yet; else result + 1
};

// Runs fn() once per device (on the current device) and returns its result
// on every later call there. fn must be idempotent (a race may run it twice).
template <class Fn>
cudaError_t once_per_device(PerDevice& once, Fn&& fn) {
  int dev = 0;
  if (const cudaError_t e = cudaGetDevice(&dev); e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxCachedDevices) return fn();
  const int s = once.state[dev].load(std::memory_order_acquire);
  if (s != 0) return cudaError_t(s - 1);
  const cudaError_t e = fn();
  once.state[dev].store(int(e) + 1, std::memory_order_release);
  return e;
}

template <class Kern>
cudaError_t configure_smem(PerDevice& once, Kern* kernel, size_t bytes) {
  return once_per_device(once, [&] {
    const DeviceLimits* d = physical();
    if (d && bytes > d->smem_per_block_optin) return cudaErrorInvalidValue;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
  });
}

}  // namespace aegis::hw
