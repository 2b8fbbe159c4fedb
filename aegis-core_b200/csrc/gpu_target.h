#pragma once
// What the launch planners know about a GPU, and the one piece of per-device
// kernel set-up they need (the dynamic shared-memory opt-in).
//
// The planners size grids, split counts and tile slots from the device the
// call runs on: 148 SMs and 232,448 bytes of opt-in shared memory on a B200,
// nothing hard-coded. A CPU test can ask "what would the planner do on a
// device with S SMs" by installing a modelled target for the duration of a
// scope (PlanOn); launches are never made while one is installed.
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>

namespace aegis::gpu {

// Devices with an ordinal below this have cached targets and per-device
// set-up bits; the library refuses higher ordinals where it keeps per-device
// state.
inline constexpr int kMaxDevices = 64;

struct Target {
  int ordinal = -1;            // CUDA ordinal; -1 for a modelled device
  int cc = 0;                  // compute capability as major*10 + minor (B200: 100)
  int sms = 0;                 // streaming multiprocessors
  size_t smem_optin = 0;       // largest dynamic shared memory one CTA may opt into
  int regs_per_cta = 0;        // 32-bit registers one CTA may hold
  int threads_per_cta = 0;     // largest CTA
  bool modelled = false;       // installed by PlanOn, not queried from hardware
};

// The target sizing decisions use on this thread: the modelled one inside a
// PlanOn scope, else the current device. Null if the device cannot be queried.
const Target* planning_target();

// The current CUDA device, queried once per ordinal and cached; never a
// modelled target. Null if the query fails.
const Target* this_device();

// Installs `t` as this thread's planning target until the scope ends. Scopes
// nest; the innermost wins.
class PlanOn {
 public:
  explicit PlanOn(const Target& t);
  ~PlanOn();
  PlanOn(const PlanOn&) = delete;
  PlanOn& operator=(const PlanOn&) = delete;

 private:
  Target t_;
  const Target* outer_;
};

// One per kernel instantiation (a function-local static at the launch site):
// raises the kernel's dynamic shared-memory limit to `bytes` on each device
// the first time it launches there. A race may set the attribute twice, which
// is harmless.
class SmemOptIn {
 public:
  cudaError_t ensure(const void* kernel, size_t bytes);

 private:
  std::atomic<uint64_t> done_{0};  // bit d: device d is set up
};

}  // namespace aegis::gpu
