// INT4 weight-only skinny GEMM (decode-shaped: M <= 16 activation rows).
//
//   out[m, n] = sum_g s[n, g] * sum_{k in g} A[m, k] * (q[n, k] - zp[n, g])
//
// A is bfloat16 (M, K); the weight is the packed INT4 cast of W^T (N, K)
// (two codes per byte, element 2i in the low nibble) with fp16 / fp32 scales
// and zero points per 128-element group. The value (q - zp) is an integer in
// [-15, 15], exact in bfloat16, so each group's inner sum runs on the tensor
// cores (mma.sync m16n8k16, bf16 x bf16 -> fp32) with the weight as the
// 16-row "A" operand and the activations as the 8-column "B" operand (one
// n8 tile for M <= 8, two for M <= 16); the group scale is applied to the
// fp32 partial. This equals the reference's dequantize-then-float32-matmul
// (src/breccia/kernels/reference/matmul.py:123-133 on
// src/breccia/kernels/reference/cast.py:574-586) up to float32 rounding order.
//
// The MMA is fed bf16 (128 + code) (one byte permute per pair of codes) and
// the offset is removed per group in float32:
//   sum_k A_k (q_k - zp) = sum_k A_k (128 + q_k) - (128 + zp) * sum_k A_k,
// with sum_k A_k over the group precomputed per activation row.
//
// Inside a 128-element group the reduction order is permuted. Thread t reads
// bytes 16t..16t+15 of each of its two rows' 64-byte group (word i = bytes
// 16t+4i..+3, elements 32t+8i .. 32t+8i+7, one low and one high nibble per
// byte). For word i, k-tile 2i takes the low nibbles: column slots 2t, 2t+1
// hold elements 32t+8i+{0,2}, slots 2t+8, 2t+9 hold 32t+8i+{4,6}; k-tile
// 2i+1 takes the high nibbles (+1). The activations are stored in shared
// memory with each 8-element chunk reordered to [0,2,4,6,1,3,5,7], so every
// B fragment is one 8-byte load.
//
// The kernel is bound by HBM reads of the packed weight, so what matters is
// the number of bytes in flight. One CTA per SM, 16 warps; each warp owns a
// 16-row block of the weight and streams it through its own ring of TMA
// stages in shared memory (16 rows x 64*sg bytes = sg groups per stage), while the activations sit in shared memory (only the M real rows;
// the MMA's unused activation columns are zero registers). Every mbarrier
// wait is bounded: on a timeout the warp records the status bit, waits for
// its own copies in flight and stops.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <mutex>

#include "breccia_b200.h"
#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"

namespace brc {

uint32_t* gemm_status_ptr();  // device address of the GEMM status word (gemm_sm100.cu)

namespace int4gemm {

using namespace sm100;

constexpr int kWarps = 16;
constexpr int kThreads = 32 * kWarps;
constexpr int G = 128;                // group size handled by this kernel
constexpr int GROUP_BYTES = 16 * 64;  // 16 rows x one group of packed codes
constexpr int kSmemLimit = 227 * 1024;

struct Params {
  const __nv_bfloat16* a;  // (M, K)
  const uint8_t* w;        // tiles: ((n/16) * (K/128) + g) * 1024 + (n%16) * 64 + (k%128)/2
  const float* sc;         // tile scales: ((n/16) * (K/128) + g) * 16 + n%16
  const float* zp;         // tile zero points (asymmetric) or null
  void* out;               // (M, N)
  int M, N, K;
  int kc;                  // K elements of A resident in shared memory per chunk
  int stages;              // bulk-copy stages per warp
  int sg;                  // groups per stage
  uint32_t* status;
};

// bytes of one group in a stage: 1 KB of codes + 16 fp32 scales + 16 fp32 zero points
constexpr int SLOT_BYTES = GROUP_BYTES + 64 + 64;

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two 4-bit codes (bytes 2j and 2j+1 of x, one code per byte) as the bf16
// pair (128 + code): bf16 0x43cc is 128 + cc for cc < 128, so one byte
// permute against the constant 0x43 builds both halves.
template <int J>
__device__ __forceinline__ uint32_t code_pair(uint32_t x) {
  constexpr uint32_t sel = (2 * J) | (4 << 4) | ((2 * J + 1) << 8) | (4 << 12);
  return prmt(x, 0x43434343u, sel);
}



// Shared memory: [A chunk: M rows x (kc + 8) bf16][warp rings: kWarps x stages x sg KB]
// [mbarriers: kWarps x stages][abort flags: kWarps]
__host__ __device__ inline int a_row_elems(int kc) { return kc + 8; }
// activations (M rows) + per-(row, group) sums (16 rows x kc/128 floats)
__host__ __device__ inline size_t a_area_bytes(int M, int kc) {
  return ((size_t)M * a_row_elems(kc) * 2 + (size_t)16 * (kc / 128) * 4 + 1023) & ~size_t(1023);
}
__host__ __device__ inline size_t smem_bytes(int M, int kc, int stages, int sg) {
  const size_t a = a_area_bytes(M, kc);
  return a + (size_t)kWarps * stages * sg * SLOT_BYTES + (size_t)kWarps * stages * 8 + kWarps * 4;
}

template <int MT, int MODE, int OUT>  // MODE 0: unsigned sym, 1: signed sym, 2: asym
__global__ void __launch_bounds__(kThreads, 1) k_int4_skinny(const Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, t = lane & 3;
  const int S = p.stages;
  const int SG = p.sg;
  const int stage_bytes = SG * SLOT_BYTES;  // [codes SG KB][scales SG*64][zero points SG*64]
  const int arow = a_row_elems(p.kc);
  const size_t a_bytes = a_area_bytes(p.M, p.kc);
  __nv_bfloat16* As = reinterpret_cast<__nv_bfloat16*>(smem);
  float* SA = reinterpret_cast<float*>(smem + (size_t)p.M * arow * 2);  // [16][kc/128]
  uint8_t* ring = smem + a_bytes + (size_t)warp * S * stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a_bytes + (size_t)kWarps * S * stage_bytes) +
                   warp * S;
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(
      smem + a_bytes + (size_t)kWarps * S * stage_bytes + (size_t)kWarps * S * 8) + warp;

  const int n_rb = p.N / 16;
  const int rb = blockIdx.x + gridDim.x * warp;  // this warp's 16-row block
  const bool active = rb < n_rb;
  const int n0 = rb * 16;
  const int groups = p.K / G;
  const int nstages_total = groups / SG;  // stage loads over the whole K
  const int nchunks = p.K / p.kc;
  const int gpc = p.kc / G;  // groups per chunk

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    *abort_flag = 0u;
    fence_mbar_init();
  }
  __syncwarp();

  // bulk-copy stage q (groups q*SG .. q*SG+SG-1: contiguous codes, scales and
  // zero points of this warp's row block) into its ring slot
  const int64_t tile0 = (int64_t)rb * groups;
  int issue_slot = 0;  // ring slot the next issue fills (lane 0)
  auto issue = [&](int q) {
    const int s = issue_slot;
    if (++issue_slot == S) issue_slot = 0;
    uint8_t* dst = ring + s * stage_bytes;
    const int64_t t = tile0 + (int64_t)q * SG;
    const uint32_t bytes = SG * (GROUP_BYTES + 64) + (MODE == 2 ? SG * 64 : 0);
    mbar_arrive_expect_tx(&bars[s], bytes);
    bulk_load(dst, p.w + t * GROUP_BYTES, SG * GROUP_BYTES, &bars[s]);
    bulk_load(dst + SG * GROUP_BYTES, p.sc + t * 16, SG * 64, &bars[s]);
    if constexpr (MODE == 2) bulk_load(dst + SG * (GROUP_BYTES + 64), p.zp + t * 16, SG * 64, &bars[s]);
  };
  int issued = 0;
  if (active && lane == 0)
    for (; issued < S && issued < nstages_total; ++issued) issue(issued);

  float tot[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) tot[mt][i] = 0.f;

  // activation rows this thread reads as the MMA B operand (zeros beyond M)
  const bool brow_ok0 = gid < p.M, brow_ok1 = 8 + gid < p.M;
  bool ok = true;
  int slot = 0, gin = 0;  // ring slot of the current stage, group within the stage
  uint32_t phase = 0;     // parity of the slot's current fill

  for (int c = 0; c < nchunks; ++c) {
    // stage the activations' chunk c (all warps): each 8-element chunk is
    // stored reordered to [0,2,4,6,1,3,5,7]; then the per-(row, group) sums
    const int vec_per_row = p.kc / 8;
    for (int i = threadIdx.x; i < p.M * vec_per_row; i += blockDim.x) {
      const int m = i / vec_per_row, v = i - m * vec_per_row;
      const uint4 w = ldg16(p.a + (int64_t)m * p.K + (int64_t)c * p.kc + v * 8);
      const uint4 o = make_uint4(prmt(w.x, w.y, 0x5410), prmt(w.z, w.w, 0x5410),
                                 prmt(w.x, w.y, 0x7632), prmt(w.z, w.w, 0x7632));
      *reinterpret_cast<uint4*>(As + (int64_t)m * arow + v * 8) = o;
    }
    __syncthreads();
    // one warp per (row, group): 4 elements per lane, then a shuffle tree
    for (int task = warp; task < 16 * gpc; task += kWarps) {
      const int m = task / gpc, g = task - m * gpc;
      float sum = 0.f;
      if (m < p.M) {
        const uint2 v = *reinterpret_cast<const uint2*>(As + (int64_t)m * arow + g * G + 4 * lane);
        sum = (__uint_as_float(v.x << 16) + __uint_as_float(v.x & 0xFFFF0000u)) +
              (__uint_as_float(v.y << 16) + __uint_as_float(v.y & 0xFFFF0000u));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
      }
      if (lane == 0) SA[m * gpc + g] = sum;
    }
    __syncthreads();
    if (active && ok) {
      for (int gg = 0; gg < gpc; ++gg) {
        // running counters (no divisions): ring slot, its phase parity, and
        // the group's index inside its stage
        const int s = slot;
        const int gs = gin;
        if (gs == 0 && !mbar_wait(&bars[s], phase, abort_flag, p.status, 1u)) {
          ok = false;
          break;
        }
        const uint8_t* stg = ring + s * stage_bytes;
        const uint4 w0 = *reinterpret_cast<const uint4*>(stg + gs * GROUP_BYTES + gid * 64 + 16 * t);
        const uint4 w1 =
            *reinterpret_cast<const uint4*>(stg + gs * GROUP_BYTES + (gid + 8) * 64 + 16 * t);
        const float* ssc = reinterpret_cast<const float*>(stg + SG * GROUP_BYTES) + gs * 16;
        const float s0 = ssc[gid], s1 = ssc[gid + 8];
        float off0, off1;  // value of the bf16 operand's offset for each row
        if constexpr (MODE == 2) {
          const float* szp = reinterpret_cast<const float*>(stg + SG * (GROUP_BYTES + 64)) + gs * 16;
          off0 = 128.f + szp[gid];
          off1 = 128.f + szp[gid + 8];
        } else {
          off0 = off1 = MODE == 1 ? 136.f : 128.f;
        }
        if (++gin == SG) {
          gin = 0;
          __syncwarp();
          if (lane == 0 && issued < nstages_total) issue(issued++);  // refill the slot just read
          if (++slot == S) {
            slot = 0;
            phase ^= 1u;
          }
        }
        const uint32_t r0[4] = {w0.x, w0.y, w0.z, w0.w};
        const uint32_t r1[4] = {w1.x, w1.y, w1.z, w1.w};
        float acc[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[mt][i] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t a0 = r0[i], a1 = r1[i];
          if constexpr (MODE == 1) {
            a0 ^= 0x88888888u;
            a1 ^= 0x88888888u;
          }
          const uint32_t x0 = a0 & 0x0F0F0F0Fu, y0 = (a0 >> 4) & 0x0F0F0F0Fu;
          const uint32_t x1 = a1 & 0x0F0F0F0Fu, y1 = (a1 >> 4) & 0x0F0F0F0Fu;
#pragma unroll
          for (int h = 0; h < 2; ++h) {  // k-tile 2i (low nibbles), 2i+1 (high nibbles)
            const uint32_t u0 = h ? y0 : x0, u1 = h ? y1 : x1;
            const uint32_t af[4] = {code_pair<0>(u0), code_pair<0>(u1), code_pair<1>(u0),
                                    code_pair<1>(u1)};
            const int kk = gg * G + (4 * t + i) * 8 + 4 * h;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              uint2 b = make_uint2(0u, 0u);
              if (mt == 0 ? brow_ok0 : brow_ok1)
                b = *reinterpret_cast<const uint2*>(As + (int64_t)(mt * 8 + gid) * arow + kk);
              mma_bf16(acc[mt], af, b.x, b.y);
            }
          }
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const float sa0 = SA[(mt * 8 + 2 * t) * gpc + gg];
          const float sa1 = SA[(mt * 8 + 2 * t + 1) * gpc + gg];
          tot[mt][0] = __fmaf_rn(s0, __fmaf_rn(-off0, sa0, acc[mt][0]), tot[mt][0]);
          tot[mt][1] = __fmaf_rn(s0, __fmaf_rn(-off0, sa1, acc[mt][1]), tot[mt][1]);
          tot[mt][2] = __fmaf_rn(s1, __fmaf_rn(-off1, sa0, acc[mt][2]), tot[mt][2]);
          tot[mt][3] = __fmaf_rn(s1, __fmaf_rn(-off1, sa1, acc[mt][3]), tot[mt][3]);
        }
      }
    }
    __syncthreads();  // the next chunk overwrites the activations
  }

  if (active && !ok && lane == 0) {
    // wait (bounded) for this warp's copies still in flight before exiting
    const int first = issued > S ? issued - S : 0;
    for (int q = first; q < issued; ++q) {
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(&bars[q % S], (uint32_t)((q / S) & 1)) &&
             globaltimer() - t0 < kWaitLimitNs) {
      }
    }
  }
  if (!active || !ok) return;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = mt * 8 + 2 * t + (i & 1);
      const int n = n0 + gid + (i >> 1) * 8;
      if (m < p.M) {
        const int64_t o = (int64_t)m * p.N + n;
        if constexpr (OUT == BRC_DTYPE_F32) static_cast<float*>(p.out)[o] = tot[mt][i];
        else if constexpr (OUT == BRC_DTYPE_BF16)
          static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(tot[mt][i]);
        else static_cast<__half*>(p.out)[o] = __float2half_rn(tot[mt][i]);
      }
    }
  }
}

// ------------------------------------------------------------------ host
template <int MT, int MODE, int OUT>
int launch(const Params& p, size_t smem, cudaStream_t st) {
  auto kern = k_int4_skinny<MT, MODE, OUT>;
  // the opt-in shared-memory size is set once per device (to the maximum)
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BRC_ERR_CUDA;
  if (!configured[dev]) {
    int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemLimit));
    if (rc) return rc;
    configured[dev] = true;
  }
  const int n_rb = p.N / 16;
  int grid = sm_count();
  const int need = (n_rb + kWarps - 1) / kWarps;
  if (need > grid) grid = need;
  kern<<<grid, kThreads, smem, st>>>(p);
  return check_launch();
}

template <int MT, int MODE>
int launch_out(int out_dtype, const Params& p, size_t smem, cudaStream_t st) {
  if (out_dtype == BRC_DTYPE_F32) return launch<MT, MODE, BRC_DTYPE_F32>(p, smem, st);
  if (out_dtype == BRC_DTYPE_BF16) return launch<MT, MODE, BRC_DTYPE_BF16>(p, smem, st);
  return launch<MT, MODE, BRC_DTYPE_F16>(p, smem, st);
}

template <int MT>
int launch_mode(int mode, int out_dtype, const Params& p, size_t smem, cudaStream_t st) {
  if (mode == 0) return launch_out<MT, 0>(out_dtype, p, smem, st);
  if (mode == 1) return launch_out<MT, 1>(out_dtype, p, smem, st);
  return launch_out<MT, 2>(out_dtype, p, smem, st);
}

}  // namespace int4gemm
}  // namespace brc

extern "C" int brc_gemm_int4(const void* a_bf16, int M, int K, const uint8_t* w_tiles, int N,
                             int is_signed, int symmetric, const float* scale_tiles,
                             const float* zp_tiles, void* d, int d_dtype, void* stream) {
  using namespace brc::int4gemm;
  if (!a_bf16 || !w_tiles || !scale_tiles || !d) return BRC_ERR_NULL;
  if (!symmetric && !zp_tiles) return BRC_ERR_NULL;
  if (M <= 0 || N <= 0 || K <= 0) return (M == 0 || N == 0) ? BRC_OK : BRC_ERR_SHAPE;
  if (d_dtype != BRC_DTYPE_F32 && d_dtype != BRC_DTYPE_BF16 && d_dtype != BRC_DTYPE_F16)
    return BRC_ERR_DTYPE;
  if (M > 16 || K % 1024 || N % 16 || (!symmetric && is_signed)) return BRC_ERR_UNSUPPORTED;
  if (((uintptr_t)a_bf16 | (uintptr_t)w_tiles | (uintptr_t)scale_tiles |
       (uintptr_t)(zp_tiles ? zp_tiles : scale_tiles)) & 15)
    return BRC_ERR_ALIGN;
  // Activations chunk: the largest multiple of 1024 dividing K that leaves
  // room for 2 stages per warp; then as many groups per stage (up to 4) and
  // stages (up to 16) as fit.
  int kc = K;
  while (kc > 1024 && (smem_bytes(M, kc, 2, 1) > (size_t)kSmemLimit || K % kc)) kc -= 1024;
  if (smem_bytes(M, kc, 2, 1) > (size_t)kSmemLimit || K % kc) return BRC_ERR_UNSUPPORTED;
  int sg = 4;
  while (sg > 1 && smem_bytes(M, kc, 2, sg) > (size_t)kSmemLimit) sg /= 2;
  int stages = 2;
  while (stages < 16 && smem_bytes(M, kc, stages + 1, sg) <= (size_t)kSmemLimit) ++stages;
  Params p{};
  p.a = static_cast<const __nv_bfloat16*>(a_bf16);
  p.w = w_tiles;
  p.sc = scale_tiles;
  p.zp = zp_tiles;
  p.out = d;
  p.M = M;
  p.N = N;
  p.K = K;
  p.kc = kc;
  p.stages = stages;
  p.sg = sg;
  p.status = brc::gemm_status_ptr();
  const size_t smem = smem_bytes(M, kc, stages, sg);
  const int mode = symmetric ? (is_signed ? 1 : 0) : 2;
  cudaStream_t st = (cudaStream_t)stream;
  return M <= 8 ? launch_mode<1>(mode, d_dtype, p, smem, st)
                : launch_mode<2>(mode, d_dtype, p, smem, st);
}
