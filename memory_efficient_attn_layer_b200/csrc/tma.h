// Host-side construction of TMA tensor maps (cuTensorMapEncodeTiled), resolved
// through the runtime's driver entry point so the library needs no -lcuda.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace mea {

// Encodes a 2-D tiled tensor map.
//   inner      : elements along the contiguous dimension
//   outer      : rows
//   row_bytes  : bytes between consecutive rows (multiple of 16)
//   box_inner / box_outer : box extent in elements / rows
// Returns 0 on success, a CUresult otherwise.
int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle,
                 CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);

// Swizzle mode for a row of `row_bytes` bytes in shared memory (32, 64 or 128).
inline CUtensorMapSwizzle swizzle_for(uint32_t row_bytes) {
  return row_bytes >= 128 ? CU_TENSOR_MAP_SWIZZLE_128B
         : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                           : CU_TENSOR_MAP_SWIZZLE_32B;
}

}  // namespace mea
