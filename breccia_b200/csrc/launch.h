// Host-side launch helpers shared by the breccia_b200 translation units.
#pragma once

#include <cstdint>
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

// Pieces of the per-tensor FP8 cast that the fused cast-GEMM
// (brc_cast_gemm_pertensor_fp8) runs around its kernel; cast.cu.
// Scale into *scale_out: from the amax history (`from_history`, the scale of
// brc_cast_pertensor_fp8_delayed), else from the amax of x[0, n), reduced
// into *amax_ws (zeroed by the caller): the scale of brc_cast_pertensor_fp8.
int pertensor_fp8_scale(const void* x, int x_dtype, int64_t n, int fmt, const float* history,
                        int history_len, int margin, bool from_history, uint32_t* amax_ws,
                        float* scale_out, cudaStream_t st);
// Codes of x[0, n) with the scale at *scale (one pass); the amax of those
// elements is folded into *amax_ws.
int pertensor_fp8_encode(const void* x, int x_dtype, int64_t n, int fmt, const float* scale,
                         uint8_t* codes, uint32_t* amax_ws, cudaStream_t st);
// History ring update with the amax in *amax_ws.
int pertensor_fp8_history_push(float* history, int history_len, const uint32_t* amax_ws,
                               cudaStream_t st);

}  // namespace brc
