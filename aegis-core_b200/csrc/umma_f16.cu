// umma kernel instantiations for f16 operands (see umma_launch.cuh).
#include "umma_launch.cuh"

namespace aegis::umma {
template cudaError_t launch_family<__half>(const LaunchKey&, const CUtensorMap&, const CUtensorMap&, const Args&,
                                           int, cudaStream_t);
template cudaError_t attrs_family<__half>(int, int, bool, cudaFuncAttributes*);
}  // namespace aegis::umma
