// Host-side launch helpers shared by the breccia_b200 translation units.
#pragma once

#include <cuda_runtime.h>

namespace brc {

// Multiprocessor count of the current device (cached per device).
int sm_count();
// cudaGetLastError() after a launch: BRC_OK, or BRC_ERR_CUDA with the error
// recorded for brc_last_cuda_error().
int check_launch();
// Map a CUDA runtime status to BRC_OK / BRC_ERR_CUDA, recording failures.
int check_cuda(cudaError_t e);

}  // namespace brc
