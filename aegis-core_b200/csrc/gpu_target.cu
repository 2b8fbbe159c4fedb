// Device targets for the launch planners (see gpu_target.h).
#include "gpu_target.h"

#include <mutex>

namespace aegis::gpu {
namespace {

thread_local const Target* t_model = nullptr;

// Ordinal -> target. `ready` is published after the slot is written, so the
// fast path is one acquire load; the mutex only serialises first queries.
struct Table {
  std::mutex fill;
  std::atomic<int8_t> ready[kMaxDevices] = {};  // 0 unknown, 1 valid, -1 query failed
  Target slot[kMaxDevices];
};

Table& table() {
  static Table t;
  return t;
}

// Individual attribute queries: cudaGetDeviceProperties fills ~100 fields and
// can take milliseconds; the planners need six.
cudaError_t query(int ordinal, Target* out) {
  Target t;
  t.ordinal = ordinal;
  int major = 0, minor = 0, optin = 0;
  const struct {
    cudaDeviceAttr attr;
    int* dst;
  } q[] = {
      {cudaDevAttrComputeCapabilityMajor, &major},
      {cudaDevAttrComputeCapabilityMinor, &minor},
      {cudaDevAttrMultiProcessorCount, &t.sms},
      {cudaDevAttrMaxSharedMemoryPerBlockOptin, &optin},
      {cudaDevAttrMaxRegistersPerBlock, &t.regs_per_cta},
      {cudaDevAttrMaxThreadsPerBlock, &t.threads_per_cta},
  };
  for (const auto& e : q)
    if (const cudaError_t err = cudaDeviceGetAttribute(e.dst, e.attr, ordinal); err != cudaSuccess) return err;
  t.cc = major * 10 + minor;
  t.smem_optin = size_t(optin);
  *out = t;
  return cudaSuccess;
}

}  // namespace

const Target* this_device() {
  int ordinal = 0;
  if (cudaGetDevice(&ordinal) != cudaSuccess || ordinal < 0 || ordinal >= kMaxDevices) {
    cudaGetLastError();
    return nullptr;
  }
  Table& tb = table();
  int8_t r = tb.ready[ordinal].load(std::memory_order_acquire);
  if (r == 0) {
    std::lock_guard<std::mutex> lock(tb.fill);
    r = tb.ready[ordinal].load(std::memory_order_relaxed);
    if (r == 0) {
      const bool ok = query(ordinal, &tb.slot[ordinal]) == cudaSuccess;
      if (!ok) cudaGetLastError();
      r = ok ? 1 : -1;
      tb.ready[ordinal].store(r, std::memory_order_release);
    }
  }
  return r == 1 ? &tb.slot[ordinal] : nullptr;
}

const Target* planning_target() { return t_model ? t_model : this_device(); }

PlanOn::PlanOn(const Target& t) : t_(t), outer_(t_model) {
  t_.modelled = true;
  t_.ordinal = -1;
  t_model = &t_;
}

PlanOn::~PlanOn() { t_model = outer_; }

cudaError_t SmemOptIn::ensure(const void* kernel, size_t bytes) {
  int ordinal = 0;
  if (const cudaError_t e = cudaGetDevice(&ordinal); e != cudaSuccess) return e;
  const uint64_t bit = ordinal >= 0 && ordinal < kMaxDevices ? uint64_t(1) << ordinal : 0;
  if (bit && (done_.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  const Target* t = this_device();
  if (t && bytes > t->smem_optin) return cudaErrorInvalidValue;
  if (const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
      e != cudaSuccess)
    return e;
  if (bit) done_.fetch_or(bit, std::memory_order_release);
  return cudaSuccess;
}

}  // namespace aegis::gpu
