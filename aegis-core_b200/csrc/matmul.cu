// aegis::matmul dispatch (see include/aegis/matmul.h). Mirrors the
// reference's src/matmul.cu:386-467 (validate -> empty -> alpha == 0 ->
// choose -> KernelEntry::run) without a vendor-library path: every choice is
// one of this library's kernels.
#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>
#include <unordered_map>

#include "aegis/gemm.h"
#include "aegis/matmul.h"
#include "common.cuh"
#include "gpu_target.h"
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
  const gpu::Target* d = gpu::planning_target();
  return d ? d->cc : 0;
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
  // The rule for shapes with no tuned row for their (N, K), from the B200
  // tuner runs of the BASELINE shapes (aegis-core_b200/tune/runs/):
  const bool tma = gemm::tma_compatible(p) && caps.arch == 100;
  if (p.M <= 16) {
    // Decode. M <= 2: the CUDA-core weight stream (the gemv configs within 3%
    // of each other and of the best at M = 1). M <= 8: the tensor-core
    // stream ummav (fastest at M = 4). M <= 16: split-K on 128 x 128 tiles
    // (fastest at M = 16 on all three decode shapes; ummav 1.09-1.30x
    // slower). Operands the TMA path cannot address: the CUDA-core GEMV.
    if (p.M <= 2) return by_name("gemv_256x256_ksm");
    if (p.M <= 8) {
      if (caps.arch == 100 && ummav_takes(p)) return by_name("ummav_128x16x64_s6x2");
      return by_name("gemv_128x256_ksm");
    }
    return tma ? by_name("umma_128x128x64_s6_ksm") : by_name("gemv_64x256_ksm");
  }
  if (!tma) return by_name("simt_64x64x16");
  if (p.N <= 128) return by_name("umma_128x128x64_s6_ksm");
  if (p.M <= 128) return by_name("umma_128x256x64_s4_ksm");
  // Larger problems, by tile count on the device's SMs:
  //  - one wave of 128 x 64 tiles and a short K (512^3, 1024^3): the small
  //    tiles (CTA pairs 1.3-2.1x slower there);
  //  - fewer than 12 tiles of 256 x 256 and a long K (256^2 and 512^2 x
  //    65536): split-K on 128 x 128 tiles;
  //  - otherwise CTA pairs with split-K (1024^2 x 65536, 2048^3 and up).
  const gpu::Target* d = gpu::planning_target();
  const long long sms = d && d->sms > 0 ? d->sms : 148;
  const long long batch = std::max(1, p.batch);
  const long long t64 = (long long)ceil_div(p.M, 128) * ceil_div(p.N, 64) * batch;
  const long long t256 = (long long)ceil_div(p.M, 256) * ceil_div(p.N, 256) * batch;
  if (t64 <= sms && p.K <= 4096) return by_name("umma_128x64x64_s8_ksm");
  if (t256 < 12 && p.K > 4096) return by_name("umma_128x128x64_s6_ksm");
  return by_name("umma_256x256x64_s7_c2_ksm");
}

Choice choose(std::span<const Winner> table, const gemm::GemmParams& p, const gemm::DeviceCaps& caps,
              std::string* why) {
  Choice c;
  const Winner* best = nullptr;
  const gemm::KernelEntry* best_kernel = nullptr;
  double best_dist = INFINITY;
  // Rows of the call's operand type first; the other type's rows only when
  // (N, K) has no usable row of this one.
  for (const bool same_type : {true, false}) {
    for (const Winner& w : table) {
      if (w.N != p.N || w.K != p.K || (w.dtype == p.dtype) != same_type) continue;
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
    if (best) break;
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

cudaError_t matmul(const __half* A, const __half* B, __half* C, int M, int N, int K, cudaStream_t stream) {
  return matmul(gemm::row_major_params(A, B, C, M, N, K, gemm::DType::F16), stream);
}

cudaError_t matmul(const __nv_bfloat16* A, const __nv_bfloat16* B, __nv_bfloat16* C, int M, int N, int K,
                   cudaStream_t stream) {
  return matmul(gemm::row_major_params(A, B, C, M, N, K, gemm::DType::BF16), stream);
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
