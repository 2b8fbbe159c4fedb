// umma kernel instantiations for bf16 operands (see umma_launch.cuh).
#include "umma_launch.cuh"

namespace aegis::umma {
template cudaError_t launch_family<__nv_bfloat16>(const LaunchKey&, const CUtensorMap&, const CUtensorMap&,
                                                  const Args&, int, cudaStream_t);
template cudaError_t attrs_family<__nv_bfloat16>(int, int, bool, cudaFuncAttributes*);
}  // namespace aegis::umma
