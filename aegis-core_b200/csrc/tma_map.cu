// TMA tensor-map encoding (see tma_map.h).
#include "tma_map.h"

#include <cudaTypedefs.h>
#include <cuda_runtime.h>

namespace aegis {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      p = nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

}  // namespace

bool encode_map(CUtensorMap* map, gemm::DType dt, const void* base, long long inner, long long outer, long long ld,
                long long batch, long long bstride, int box_outer) {
  auto fn = encode_fn();
  if (!fn) return false;
  if (batch <= 1) {
    batch = 1;
    bstride = ((outer * ld + 7) / 8) * 8;  // unused coordinate; any legal stride
  }
  cuuint64_t dims[3] = {cuuint64_t(inner), cuuint64_t(outer), cuuint64_t(batch)};
  cuuint64_t strides[2] = {cuuint64_t(ld) * 2, cuuint64_t(bstride) * 2};
  cuuint32_t box[3] = {64, cuuint32_t(box_outer), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType t =
      dt == gemm::DType::BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(map, t, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace aegis
