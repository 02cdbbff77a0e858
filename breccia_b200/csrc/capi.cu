// Library-wide C ABI helpers: status strings, error bookkeeping, version.
#include <atomic>

#include "breccia_b200.h"
#include "launch.h"

namespace brc {

namespace {
thread_local int g_last_cuda_error = 0;
constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];
}  // namespace

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  int n = g_sm_count[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

int check_cuda(cudaError_t e) {
  if (e == cudaSuccess) return BRC_OK;
  g_last_cuda_error = (int)e;
  return BRC_ERR_CUDA;
}

int check_launch() { return check_cuda(cudaGetLastError()); }

}  // namespace brc

extern "C" {

const char* brc_status_string(int status) {
  switch (status) {
    case BRC_OK: return "ok";
    case BRC_ERR_NULL: return "a required pointer is NULL";
    case BRC_ERR_SHAPE: return "inconsistent sizes";
    case BRC_ERR_ALIGN: return "pointer not 16-byte aligned";
    case BRC_ERR_DTYPE: return "unknown dtype or format";
    case BRC_ERR_UNSUPPORTED: return "unsupported configuration";
    case BRC_ERR_CUDA: return "CUDA error";
    case BRC_ERR_TIMEOUT: return "device-side wait timed out";
    case BRC_ERR_RANGE: return "size exceeds a documented limit";
    default: return "unknown status";
  }
}

int brc_last_cuda_error(void) { return brc::g_last_cuda_error; }

int brc_version(void) { return 100; }

}  // extern "C"

// ---------------------------------------------------------------- self-test
// Device division used by the casts (Markstein refinement of RN(1/s)) next to
// IEEE division, so tests can compare them on arbitrary inputs.
#include "common.cuh"

namespace {
__global__ void k_selftest_division(const float* x, const float* s, int64_t n, float* q_fast,
                                    float* q_ieee) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float r = __frcp_rn(s[i]);
    q_fast[i] = brc::div_by(x[i], s[i], r);
    q_ieee[i] = __fdiv_rn(x[i], s[i]);
  }
}
}  // namespace

extern "C" int brc_selftest_division(const float* x, const float* s, int64_t n, float* q_fast,
                                     float* q_ieee, void* stream) {
  if (!x || !s || !q_fast || !q_ieee) return BRC_ERR_NULL;
  if (n <= 0) return n == 0 ? BRC_OK : BRC_ERR_SHAPE;
  k_selftest_division<<<brc::sm_count() * 4, 256, 0, (cudaStream_t)stream>>>(x, s, n, q_fast,
                                                                              q_ieee);
  return brc::check_launch();
}
