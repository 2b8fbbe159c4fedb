#pragma once
// Host-side launch of one umma kernel instantiation, selected at run time by
// (BN, layouts, epilogue). Instantiated once per element type in
// umma_f16.cu / umma_bf16.cu so the two compile in parallel.
#include <cuda.h>

#include "aegis/gemm.h"
#include "gpu_target.h"
#include "umma2_kernel.cuh"

namespace aegis::umma {

struct LaunchKey {
  int BN, STAGES;
  bool a_mn, b_mn;
  int epi;
  bool pair = false;  // cta_group::2 kernel, clusters of two CTAs
};

template <class T, int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
cudaError_t launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const Args& a, int grid,
                       cudaStream_t stream) {
  auto* kern = &umma_gemm_kernel<T, BN, STAGES, A_MN, B_MN, EPI>;
  static gpu::SmemOptIn optin;
  constexpr size_t smem = size_t(Layout<BN, STAGES>::alloc_for(EPI));
  if (const cudaError_t e = optin.ensure(reinterpret_cast<const void*>(kern), smem); e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // the kernel waits (griddepcontrol.wait)
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, a);
}

template <class T, int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
cudaError_t launch_one_pair(const CUtensorMap& ta, const CUtensorMap& tb, const Args& a, int grid,
                            cudaStream_t stream) {
  auto* kern = &umma2_gemm_kernel<T, BN, STAGES, A_MN, B_MN, EPI>;
  static gpu::SmemOptIn optin;
  constexpr size_t smem = size_t(LayoutPair<BN, STAGES>::ALLOC);
  if (const cudaError_t e = optin.ensure(reinterpret_cast<const void*>(kern), smem); e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // the kernel waits (griddepcontrol.wait)
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, a);
}

template <class T, int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
cudaError_t attrs_one(cudaFuncAttributes* attrs) {
  const cudaError_t e = cudaFuncGetAttributes(attrs, &umma_gemm_kernel<T, BN, STAGES, A_MN, B_MN, EPI>);
  if (e == cudaSuccess) attrs->sharedSizeBytes += Layout<BN, STAGES>::alloc_for(EPI);
  return e;
}

template <class T, int BN, int STAGES, int EPI, bool PAIR>
cudaError_t launch_layouts(const LaunchKey& k, const CUtensorMap& ta, const CUtensorMap& tb, const Args& a,
                           int grid, cudaStream_t s) {
#define AEGIS_UMMA_LAUNCH(AM, BMJ)                                                        \
  [&] {                                                                                   \
    if constexpr (PAIR) return launch_one_pair<T, BN, STAGES, AM, BMJ, EPI>(ta, tb, a, grid, s); \
    else return launch_one<T, BN, STAGES, AM, BMJ, EPI>(ta, tb, a, grid, s);              \
  }()
  if (!k.a_mn && k.b_mn) return AEGIS_UMMA_LAUNCH(false, true);
  if constexpr (EPI != kEpiPeers) {
    if (!k.a_mn && !k.b_mn) return AEGIS_UMMA_LAUNCH(false, false);
    if (k.a_mn && k.b_mn) return AEGIS_UMMA_LAUNCH(true, true);
    return AEGIS_UMMA_LAUNCH(true, false);
  }
#undef AEGIS_UMMA_LAUNCH
  return cudaErrorNotSupported;
}

template <class T, int BN, int STAGES, bool PAIR>
cudaError_t launch_epi(const LaunchKey& k, const CUtensorMap& ta, const CUtensorMap& tb, const Args& a, int grid,
                       cudaStream_t s) {
  switch (k.epi) {
    case kEpiStore: return launch_layouts<T, BN, STAGES, kEpiStore, PAIR>(k, ta, tb, a, grid, s);
    case kEpiPartial: return launch_layouts<T, BN, STAGES, kEpiPartial, PAIR>(k, ta, tb, a, grid, s);
    case kEpiPeers:
      if constexpr (BN == 256) return launch_layouts<T, BN, STAGES, kEpiPeers, PAIR>(k, ta, tb, a, grid, s);
      return cudaErrorNotSupported;
    default: return cudaErrorInvalidValue;
  }
}

// The instantiations the registry lists (gemm::UMMA_CONFIGS): one CTA (256, 4),
// (128, 6) and (64, 8); CTA pairs (256, gemm::kUmmaPairStages).
template <class T>
cudaError_t launch_family(const LaunchKey& k, const CUtensorMap& ta, const CUtensorMap& tb, const Args& a,
                          int grid, cudaStream_t s) {
  if (k.pair) {
    constexpr int PS = gemm::kUmmaPairStages;
    if (k.BN == 256 && k.STAGES == PS) return launch_epi<T, 256, PS, true>(k, ta, tb, a, grid, s);
    return cudaErrorNotSupported;
  }
  if (k.BN == 256 && k.STAGES == 4) return launch_epi<T, 256, 4, false>(k, ta, tb, a, grid, s);
  if (k.BN == 128 && k.STAGES == 6) return launch_epi<T, 128, 6, false>(k, ta, tb, a, grid, s);
  if (k.BN == 64 && k.STAGES == 8) return launch_epi<T, 64, 8, false>(k, ta, tb, a, grid, s);
  return cudaErrorNotSupported;
}

template <class T>
cudaError_t attrs_family(int BN, int STAGES, bool pair, cudaFuncAttributes* attrs) {
  constexpr int PS = gemm::kUmmaPairStages;
  if (pair && BN == 256 && STAGES == PS) {
    const cudaError_t e = cudaFuncGetAttributes(attrs, &umma2_gemm_kernel<T, 256, PS, false, true, kEpiStore>);
    if (e == cudaSuccess) attrs->sharedSizeBytes += LayoutPair<256, PS>::ALLOC;
    return e;
  }
  if (BN == 256 && STAGES == 4) return attrs_one<T, 256, 4, false, true, kEpiStore>(attrs);
  if (BN == 128 && STAGES == 6) return attrs_one<T, 128, 6, false, true, kEpiStore>(attrs);
  if (BN == 64 && STAGES == 8) return attrs_one<T, 64, 8, false, true, kEpiStore>(attrs);
  return cudaErrorNotSupported;
}

// Explicit instantiations live in umma_f16.cu and umma_bf16.cu.
extern template cudaError_t launch_family<__half>(const LaunchKey&, const CUtensorMap&, const CUtensorMap&,
                                                  const Args&, int, cudaStream_t);
extern template cudaError_t launch_family<__nv_bfloat16>(const LaunchKey&, const CUtensorMap&, const CUtensorMap&,
                                                         const Args&, int, cudaStream_t);
extern template cudaError_t attrs_family<__half>(int, int, bool, cudaFuncAttributes*);
extern template cudaError_t attrs_family<__nv_bfloat16>(int, int, bool, cudaFuncAttributes*);

}  // namespace aegis::umma
