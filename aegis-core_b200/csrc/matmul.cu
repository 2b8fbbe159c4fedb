// aegis::matmul dispatch (see include/aegis/matmul.h). Mirrors the
// reference's src/matmul.cu:386-467 (validate -> empty -> alpha == 0 ->
// choose -> KernelEntry::run) without a vendor-library path: every choice is
// one of this library's kernels.
#include <cmath>
#include <mutex>
#include <string>
#include <unordered_map>

#include "aegis/gemm.h"
#include "aegis/matmul.h"
#include "device.h"
#include "kernels.h"

// One generated table per arch; a missing file means no tuned winners yet.
#if __has_include("aegis/winners/sm_100a.h")
#include "aegis/winners/sm_100a.h"
#endif

namespace aegis {
namespace {

std::span<const detail::Winner> winners_for(int arch) {
  switch (arch) {
#ifdef AEGIS_WINNERS_SM100
    case 100: return kWinners_sm100a;
#endif
    default: return {};
  }
}

thread_local std::string t_last_error;

cudaError_t fail(cudaError_t e, const std::string& what) {
  t_last_error = what + ": " + cudaGetErrorString(e);
  return e;
}

int current_arch() {
  const hw::DeviceLimits* d = hw::current();
  return d ? d->arch : 0;
}

const gemm::KernelEntry* find_cached(const detail::Winner& w) {
  static std::mutex mu;
  static std::unordered_map<const detail::Winner*, const gemm::KernelEntry*> cache;
  std::lock_guard<std::mutex> lock(mu);
  const auto it = cache.find(&w);
  if (it != cache.end()) return it->second;
  return cache[&w] = gemm::find(w.impl);
}

const gemm::KernelEntry* by_name(const char* name) {
  const gemm::KernelEntry* e = gemm::find(name);
  return e;
}

}  // namespace

namespace detail {

const gemm::KernelEntry* rule_for(const gemm::GemmParams& p, const gemm::DeviceCaps& caps) {
  if (p.M <= 16) {
    // Decode. M <= 2: the CUDA-core weight stream (gemv_256x256_ksm) measured
    // fastest at M = 1 on every BASELINE decode shape. From M = 4 the FP32 FMA
    // work (M per weight element) makes the tensor-core stream (ummav) faster;
    // it takes row-major operands the TMA path can address, the CUDA-core GEMV
    // everything else.
    if (p.M <= 2) return by_name("gemv_256x256_ksm");
    if (caps.arch == 100 && ummav_takes(p)) return by_name("ummav_128x16x64_s6x2");
    if (p.M <= 8) return by_name("gemv_128x256_ksm");
    return by_name("gemv_64x256_ksm");
  }
  if (gemm::tma_compatible(p) && caps.arch == 100) {
    // CTA pairs (256 x 256 tiles) measured fastest from 4096^2 up; a single
    // CTA's 128-row tile wastes less when M or N is small.
    if (p.N <= 128) return by_name("umma_128x128x64_s6_ksm");
    if (p.M <= 128) return by_name("umma_128x256x64_s4_ksm");
    return by_name("umma_256x256x64_s7_c2_ksm");
  }
  return by_name("simt_64x64x16");
}

Choice choose(std::span<const Winner> table, const gemm::GemmParams& p, const gemm::DeviceCaps& caps,
              std::string* why) {
  Choice c;
  const Winner* best = nullptr;
  const gemm::KernelEntry* best_kernel = nullptr;
  double best_dist = INFINITY;
  for (const Winner& w : table) {
    if (w.N != p.N || w.K != p.K) continue;
    const gemm::KernelEntry* e = find_cached(w);
    std::string reason;
    if (!e || !gemm::supported(*e, caps, why ? &reason : nullptr)) {
      ++c.filtered;
      if (why) *why += std::string(why->empty() ? "" : "; ") + w.impl + ": " + (e ? reason : "not in this build");
      continue;
    }
    const double d = w.M == p.M ? -1.0 : std::abs(std::log2(double(w.M)) - std::log2(double(p.M)));
    if (!best || d < best_dist || (d == best_dist && w.M > best->M)) {
      best = &w;
      best_dist = d;
      best_kernel = e;
    }
  }
  if (best) {
    c.kind = Choice::Kind::Aegis;
    c.winner = best;
    c.kernel = best_kernel;
  } else {
    c.kind = Choice::Kind::Rule;
    c.kernel = rule_for(p, caps);
  }
  return c;
}

std::span<const Winner> winners_table() { return winners_for(current_arch()); }

}  // namespace detail

cudaError_t matmul(const gemm::GemmParams& p, cudaStream_t stream) {
  if (const cudaError_t e = gemm::validate(p); e != cudaSuccess) return fail(e, "aegis::matmul: invalid GEMM parameters");
  if (gemm::is_empty(p)) return cudaSuccess;
  if (p.alpha == 0.f) {  // BLAS: A*B does not contribute
    const cudaError_t e = scale_c(p, stream);
    return e == cudaSuccess ? e : fail(e, "aegis::matmul: scale C (alpha == 0)");
  }
  const gemm::DeviceCaps caps = gemm::current_caps();
  const detail::Choice c = detail::choose(winners_for(caps.arch), p, caps);
  if (!c.kernel || !c.kernel->run) return fail(cudaErrorNotSupported, "aegis::matmul: no kernel for this problem");
  const cudaError_t e = c.kernel->run(p, stream);
  return e == cudaSuccess ? e : fail(e, std::string("launch ") + c.kernel->name);
}

cudaError_t matmul(const void* A, const void* B, void* C, int M, int N, int K, cudaStream_t stream) {
  return matmul(gemm::row_major_params(A, B, C, M, N, K), stream);
}

const char* matmul_last_error() { return t_last_error.c_str(); }

const char* matmul_choice(const gemm::GemmParams& p) {
  const gemm::DeviceCaps caps = gemm::current_caps();
  const detail::Choice c = detail::choose(winners_for(caps.arch), p, caps);
  return c.kernel ? c.kernel->name : "none";
}

const char* matmul_choice(int M, int N, int K) {
  // Aligned placeholder pointers: the choice depends on shape and alignment only.
  static const char dummy[16] alignas(16) = {};
  return matmul_choice(gemm::row_major_params(dummy, dummy, const_cast<char*>(dummy), M, N, K));
}

}  // namespace aegis
