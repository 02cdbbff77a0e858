// Host-side launch helpers shared by the breccia_b200 translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace brc {

// Multiprocessor count of the current device (cached per device).
int sm_count();
// cudaGetLastError() after a launch: BRC_OK, or BRC_ERR_CUDA with the error
// recorded for brc_last_cuda_error().
int check_launch();
// Map a CUDA runtime status to BRC_OK / BRC_ERR_CUDA, recording failures.
int check_cuda(cudaError_t e);
// 2-D tensor map over a row-major [outer, inner] array of `dtype` elements
// (`row_bytes` apart), box [box_outer, box_inner], no swizzle; through the
// driver's cuTensorMapEncodeTiled. BRC_OK or BRC_ERR_CUDA.
int encode_tmap_2d(CUtensorMap* m, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                   uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer);

}  // namespace brc
