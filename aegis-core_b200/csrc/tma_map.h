#pragma once
// TMA tensor-map encoding for 16-bit operands (cuTensorMapEncodeTiled through
// the runtime's driver entry point, so the library needs no libcuda link).
#include <cuda.h>

#include "aegis/gemm.h"

namespace aegis {

// A 3-D (inner, outer, batch) 16-bit tensor with 128-byte-swizzled boxes of
// {64, box_outer, 1}; ld and batch stride in elements. batch <= 1: the batch
// coordinate is unused. False if the driver refuses the geometry.
bool encode_map(CUtensorMap* map, gemm::DType dt, const void* base, long long inner, long long outer, long long ld,
                long long batch, long long bstride, int box_outer);

}  // namespace aegis
