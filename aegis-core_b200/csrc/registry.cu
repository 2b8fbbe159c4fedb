// The kernel registry: one entry per launchable configuration of every
// family, with its requirements; plus validate(GemmParams) shared by every
// run(). Mirrors the reference's src/gemm/registry.cu:13-119.
#include <algorithm>
#include <cstdio>
#include <string>
#include <deque>
#include <vector>

#include "aegis/gemm.h"
#include "gpu_target.h"
#include "kernels.h"

namespace aegis {
cudaError_t simt_attrs(cudaFuncAttributes* attrs);
}

namespace aegis::gemm {

cudaError_t validate(const GemmParams& p) {
  if (p.M < 0 || p.N < 0 || p.K < 0 || p.batch < 0) return cudaErrorInvalidValue;
  if (p.M > kMaxDim || p.N > kMaxDim || p.K > kMaxDim) return cudaErrorInvalidValue;
  if (is_empty(p)) return cudaSuccess;  // nothing read or written
  if (!p.A || !p.B || !p.C) return cudaErrorInvalidValue;
  if (p.dtype != DType::F16 && p.dtype != DType::BF16) return cudaErrorInvalidValue;
  const bool ar = p.layout_a == Layout::RowMajor, br = p.layout_b == Layout::RowMajor;
  if ((!ar && p.layout_a != Layout::ColMajor) || (!br && p.layout_b != Layout::ColMajor)) return cudaErrorInvalidValue;
  if (p.lda < (ar ? p.K : p.M) || p.ldb < (br ? p.N : p.K) || p.ldc < p.N) return cudaErrorInvalidValue;
  if (p.batch > 1) {
    // A and B may be shared by every batch (stride 0); C batches must not overlap.
    if (p.stride_a < 0 || p.stride_b < 0) return cudaErrorInvalidValue;
    if (p.stride_c < (long long)(p.M - 1) * p.ldc + p.N) return cudaErrorInvalidValue;
  }
  return cudaSuccess;
}

bool tma_compatible(const GemmParams& p) {
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (!al16(p.A) || !al16(p.B)) return false;
  if (p.lda % 8 != 0 || p.ldb % 8 != 0) return false;
  if (p.batch > 1) {
    if (p.stride_a % 8 != 0 || p.stride_b % 8 != 0) return false;
  }
  // TMA dims and strides: < 2^32 elements per dim, strides < 2^40 bytes.
  const long long lim = 1ll << 38;
  if (p.lda >= lim || p.ldb >= lim || p.stride_a >= lim || p.stride_b >= lim) return false;
  return true;
}

namespace {

std::string umma_name(const UmmaConfig& c) {
  return "umma_" + std::to_string(c.BM) + "x" + std::to_string(c.BN) + "x" + std::to_string(c.BK) + "_s" +
         std::to_string(c.STAGES) + (c.CTAS == 2 ? "_c2" : "") + (c.SPLITK ? "_ksm" : "") + (c.KWAVE ? "_kw" : "");
}
std::string umma_config(const UmmaConfig& c) {
  return std::string("{\"family\":\"umma\",\"bm\":") + std::to_string(c.BM) + ",\"bn\":" + std::to_string(c.BN) +
         ",\"bk\":" + std::to_string(c.BK) + ",\"stages\":" + std::to_string(c.STAGES) +
         ",\"cta_group\":" + std::to_string(c.CTAS) + ",\"splitk\":" + (c.SPLITK ? "\"sm\"" : "1") +
         ",\"k_walk\":" + (c.KWAVE ? "\"by_wave\"" : "\"forward\"") + "}";
}
std::string gemv_name(const GemvConfig& c) {
  return "gemv_" + std::to_string(c.BN) + "x" + std::to_string(c.THREADS) + "_ksm";
}
std::string gemv_config(const GemvConfig& c) {
  return std::string("{\"family\":\"gemv\",\"bn\":") + std::to_string(c.BN) + ",\"threads\":" +
         std::to_string(c.THREADS) + ",\"vec_bytes\":16,\"splitk\":\"sm\"}";
}

// Names and configs are built once and kept for the process (KernelEntry holds
// const char*).
std::deque<std::string>& strings() {  // deque: push_back keeps earlier elements in place
  static std::deque<std::string> s;
  return s;
}
const char* keep(std::string s) {
  strings().push_back(std::move(s));
  return strings().back().c_str();
}

template <int I>
cudaError_t umma_run_i(const GemmParams& p, cudaStream_t s) { return umma_run(I, p, s); }
template <int I>
cudaError_t umma_attrs_i(cudaFuncAttributes* a) { return umma_attrs(I, a); }
template <int I>
cudaError_t umma_launch_i(const void* A, const void* B, void* C, int M, int N, int K, cudaStream_t s) {
  return umma_run(I, row_major_params(A, B, C, M, N, K), s);
}
template <int I>
cudaError_t gemv_run_i(const GemmParams& p, cudaStream_t s) { return gemv_run(I, p, s); }
template <int I>
cudaError_t gemv_attrs_i(cudaFuncAttributes* a) { return gemv_attrs(I, a); }
template <int I>
cudaError_t gemv_launch_i(const void* A, const void* B, void* C, int M, int N, int K, cudaStream_t s) {
  return gemv_run(I, row_major_params(A, B, C, M, N, K), s);
}
cudaError_t simt_launch_rm(const void* A, const void* B, void* C, int M, int N, int K, cudaStream_t s) {
  return simt_run(row_major_params(A, B, C, M, N, K), s);
}

constexpr int kNumUmma = int(sizeof(UMMA_CONFIGS) / sizeof(UMMA_CONFIGS[0]));
constexpr int kNumGemv = int(sizeof(GEMV_CONFIGS) / sizeof(GEMV_CONFIGS[0]));
static_assert(kNumUmma == 9 && kNumGemv == 4, "registry tables below list every config row");

const std::vector<KernelEntry>& umma_vec() {
  static const std::vector<KernelEntry> v = [] {
    const RunFn runs[] = {&umma_run_i<0>, &umma_run_i<1>, &umma_run_i<2>, &umma_run_i<3>, &umma_run_i<4>,
                          &umma_run_i<5>, &umma_run_i<6>, &umma_run_i<7>, &umma_run_i<8>};
    const AttrsFn attrs[] = {&umma_attrs_i<0>, &umma_attrs_i<1>, &umma_attrs_i<2>, &umma_attrs_i<3>, &umma_attrs_i<4>,
                             &umma_attrs_i<5>, &umma_attrs_i<6>, &umma_attrs_i<7>, &umma_attrs_i<8>};
    const LaunchFn launches[] = {&umma_launch_i<0>, &umma_launch_i<1>, &umma_launch_i<2>, &umma_launch_i<3>,
                                 &umma_launch_i<4>, &umma_launch_i<5>, &umma_launch_i<6>, &umma_launch_i<7>,
                                 &umma_launch_i<8>};
    std::vector<KernelEntry> out;
    for (int i = 0; i < kNumUmma; ++i) {
      const UmmaConfig& c = UMMA_CONFIGS[i];
      KernelReq req;
      req.min_arch = 100;
      req.tma = true;
      req.tcgen05 = true;
      req.smem_bytes = umma_smem_bytes(i);
      req.threads = 192;
      out.push_back({keep(umma_name(c)), keep(umma_config(c)), launches[i], attrs[i], runs[i], 0, req});
    }
    return out;
  }();
  return v;
}

const std::vector<KernelEntry>& gemv_vec() {
  static const std::vector<KernelEntry> v = [] {
    const RunFn runs[] = {&gemv_run_i<0>, &gemv_run_i<1>, &gemv_run_i<2>, &gemv_run_i<3>};
    const AttrsFn attrs[] = {&gemv_attrs_i<0>, &gemv_attrs_i<1>, &gemv_attrs_i<2>, &gemv_attrs_i<3>};
    const LaunchFn launches[] = {&gemv_launch_i<0>, &gemv_launch_i<1>, &gemv_launch_i<2>, &gemv_launch_i<3>};
    std::vector<KernelEntry> out;
    for (int i = 0; i < kNumGemv; ++i) {
      const GemvConfig& c = GEMV_CONFIGS[i];
      KernelReq req;
      req.min_arch = 100;
      req.smem_bytes = 32 << 10;
      req.threads = c.THREADS;
      out.push_back({keep(gemv_name(c)), keep(gemv_config(c)), launches[i], attrs[i], runs[i], 16, req});
    }
    return out;
  }();
  return v;
}

template <int I>
cudaError_t ummav_run_i(const GemmParams& p, cudaStream_t s) { return ummav_run(I, p, s); }
template <int I>
cudaError_t ummav_attrs_i(cudaFuncAttributes* a) { return ummav_attrs(I, a); }
template <int I>
cudaError_t ummav_launch_i(const void* A, const void* B, void* C, int M, int N, int K, cudaStream_t s) {
  return ummav_run(I, row_major_params(A, B, C, M, N, K), s);
}

const std::vector<KernelEntry>& ummav_vec() {
  static const std::vector<KernelEntry> v = [] {
    static_assert(sizeof(UMMAV_CONFIGS) / sizeof(UMMAV_CONFIGS[0]) == 2, "ummav table below lists every row");
    const RunFn runs[] = {&ummav_run_i<0>, &ummav_run_i<1>};
    const AttrsFn attrs[] = {&ummav_attrs_i<0>, &ummav_attrs_i<1>};
    const LaunchFn launches[] = {&ummav_launch_i<0>, &ummav_launch_i<1>};
    std::vector<KernelEntry> out;
    for (int i = 0; i < 2; ++i) {
      const UmmavConfig& c = UMMAV_CONFIGS[i];
      KernelReq req;
      req.min_arch = 100;
      req.tma = true;
      req.tcgen05 = true;
      req.smem_bytes = ummav_smem_bytes(i);
      req.threads = 192;
      const std::string name = "ummav_128x16x64_s" + std::to_string(c.STAGES) +
                               (c.CTAS_PER_SM > 1 ? "x" + std::to_string(c.CTAS_PER_SM) : std::string());
      const std::string cfg = std::string("{\"family\":\"ummav\",\"bm\":128,\"bn\":16,\"bk\":64,\"stages\":") +
                              std::to_string(c.STAGES) + ",\"cta_group\":1,\"ctas_per_sm\":" +
                              std::to_string(c.CTAS_PER_SM) + ",\"split\":\"stream-k\"}";
      out.push_back({keep(name), keep(cfg), launches[i], attrs[i], runs[i], 16, req});
    }
    return out;
  }();
  return v;
}

const std::vector<KernelEntry>& simt_vec() {
  static const std::vector<KernelEntry> v = [] {
    KernelReq req;
    req.min_arch = 100;
    req.smem_bytes = 2 * 16 * 68 * 4;
    req.threads = 256;
    return std::vector<KernelEntry>{{"simt_64x64x16", "{\"family\":\"simt\",\"bm\":64,\"bn\":64,\"bk\":16}",
                                     &simt_launch_rm, &simt_attrs, &simt_run, 0, req}};
  }();
  return v;
}

}  // namespace

std::span<const KernelEntry> umma_entries() { return umma_vec(); }
std::span<const KernelEntry> gemv_entries() { return gemv_vec(); }
std::span<const KernelEntry> simt_entries() { return simt_vec(); }
std::span<const KernelEntry> ummav_entries() { return ummav_vec(); }

std::span<const KernelEntry> registry() {
  static const std::vector<KernelEntry> all = [] {
    std::vector<KernelEntry> v;
    for (auto fam : {umma_entries(), gemv_entries(), ummav_entries(), simt_entries()})
      v.insert(v.end(), fam.begin(), fam.end());
    // Registers (and static smem) from the compiled binary where a device answers.
    for (KernelEntry& e : v) {
      cudaFuncAttributes a{};
      if (e.attrs && e.attrs(&a) == cudaSuccess) {
        e.req.regs = a.numRegs;
        e.req.smem_bytes = std::max(e.req.smem_bytes, size_t(a.sharedSizeBytes));
      } else {
        cudaGetLastError();
      }
    }
    return v;
  }();
  return all;
}

const KernelEntry* find(std::string_view name) {
  for (const KernelEntry& e : registry())
    if (name == e.name) return &e;
  return nullptr;
}

DeviceCaps current_caps() {
  DeviceCaps c;
  const gpu::Target* d = gpu::planning_target();
  if (!d) return c;
  c.arch = d->cc;
  c.smem_per_block_optin = d->smem_optin;
  c.regs_per_block = d->regs_per_cta;
  c.max_threads_per_block = d->threads_per_cta;
  return c;
}

bool supported(const KernelEntry& e, const DeviceCaps& c, std::string* why) {
  auto no = [&](std::string w) {
    if (why) *why = std::move(w);
    return false;
  };
  const KernelReq& r = e.req;
  // This library ships sm_100a code only (tcgen05 and TMA included).
  if (c.arch != 100) return no("needs sm_100 (B200), device is sm_" + std::to_string(c.arch));
  if (r.smem_bytes > c.smem_per_block_optin)
    return no("needs " + std::to_string(r.smem_bytes) + " B smem per block, device allows " +
              std::to_string(c.smem_per_block_optin));
  if (r.threads > c.max_threads_per_block)
    return no("needs " + std::to_string(r.threads) + " threads per block, device allows " +
              std::to_string(c.max_threads_per_block));
  if (r.regs > 0 && (long long)r.regs * r.threads > c.regs_per_block)
    return no("needs " + std::to_string(r.regs * r.threads) + " registers per block, device has " +
              std::to_string(c.regs_per_block));
  return true;
}

bool launch_plan(const char* impl, const GemmParams& p, LaunchPlan* out) {
  const std::string_view name = impl;
  const auto um = umma_entries();
  for (size_t i = 0; i < um.size(); ++i)
    if (name == um[i].name) return *out = umma_plan(int(i), p), true;
  const auto gv = gemv_entries();
  for (size_t i = 0; i < gv.size(); ++i)
    if (name == gv[i].name) return *out = gemv_plan(int(i), p), true;
  const auto uv = ummav_entries();
  for (size_t i = 0; i < uv.size(); ++i)
    if (name == uv[i].name) return *out = ummav_plan(int(i), p), true;
  return false;
}

int split_count(const char* impl, const GemmParams& p) {
  LaunchPlan l;
  return launch_plan(impl, p, &l) ? l.splits : 0;
}

}  // namespace aegis::gemm
