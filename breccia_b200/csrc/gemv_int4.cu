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
// Inside a 128-element group the reduction order is permuted so that each
// thread's weight fragment comes from the 16 contiguous bytes it loads and its
// activation fragment is 4 consecutive bf16: k-tile j, MMA column slot
// 2t+e (e in {0,1}) holds k = 32t + 8(j/2) + 4(j%2) + e, slot 2t+8+e holds
// k = 32t + 8(j/2) + 4(j%2) + 2 + e (t = lane % 4).
//
// The kernel is HBM-bound on the packed weight: one CTA per SM, 16 warps,
// each warp owning interleaved 16-row blocks of the weight; the activations
// stream through shared memory in K chunks shared by the CTA's warps.

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "breccia_b200.h"
#include "common.cuh"
#include "launch.h"

namespace brc {
namespace int4gemm {

constexpr int kWarps = 16;
constexpr int kThreads = 32 * kWarps;
constexpr int KC = 1024;       // K elements per shared-memory chunk
constexpr int PAD = 8;         // bf16 elements of row padding
constexpr int ROW = KC + PAD;  // shared row stride (elements)
constexpr int G = 128;         // group size handled by this kernel

struct Params {
  const __nv_bfloat16* a;  // (M, K)
  const uint8_t* w;        // (N, K/2)
  const void* scales;      // (N, K/G)
  const void* zp;          // (N, K/G) or null
  void* out;               // (M, N)
  int M, N, K;
  int scale_f16;
};

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Pair of codes (low, high nibble of byte b of x/y) as bf16x2 128 + code.
template <int B>
__device__ __forceinline__ uint32_t nib_pair(uint32_t x, uint32_t y) {
  constexpr uint32_t sel = B | ((8 | B) << 4) | ((4 + B) << 8) | ((8 | (4 + B)) << 12);
  return prmt(x, y, sel) | 0x43004300u;
}

__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&a),
                             *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ float load_sc(const void* p, int64_t i, int f16) {
  return f16 ? __half2float(static_cast<const __half*>(p)[i]) : static_cast<const float*>(p)[i];
}

// bf16x2 (128 + zp, 128 + zp) for a zero point held as fp16/fp32 (an
// integer in [0, 15]); signed symmetric codes use 136 after flipping bit 3.
__device__ __forceinline__ uint32_t offset_pair(float zp_plus) {
  const __nv_bfloat16 h = __float2bfloat16_rn(zp_plus);
  const uint32_t u = *reinterpret_cast<const uint16_t*>(&h);
  return u | (u << 16);
}

template <int MT, int MODE, int OUT>  // MODE 0: unsigned sym, 1: signed sym, 2: asym
__global__ void __launch_bounds__(kThreads, 1) k_int4_skinny(const Params p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* As = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [2][8*MT][ROW]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, t = lane & 3;
  const int rows_a = 8 * MT;
  const int n_rb = p.N / 16;
  const int rb = blockIdx.x + gridDim.x * warp;  // this warp's 16-row block
  const bool active = rb < n_rb;
  const int n0 = rb * 16;
  const int kpb = p.K / 2;  // bytes per weight row
  const int groups = p.K / G;

  // zero the activation rows beyond M once (both buffers)
  for (int i = threadIdx.x; i < 2 * rows_a * ROW; i += blockDim.x) {
    const int r = (i / ROW) % rows_a;
    if (r >= p.M) As[i] = __float2bfloat16_rn(0.f);
  }

  auto load_chunk = [&](int chunk, int buf) {
    // rows m < M, KC elements from k = chunk*KC, 16 bytes per cp.async
    const int vec_per_row = KC / 8;
    for (int i = threadIdx.x; i < p.M * vec_per_row; i += blockDim.x) {
      const int m = i / vec_per_row, v = i - m * vec_per_row;
      const __nv_bfloat16* src = p.a + (int64_t)m * p.K + (int64_t)chunk * KC + v * 8;
      __nv_bfloat16* dst = As + ((int64_t)buf * rows_a + m) * ROW + v * 8;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                       (uint32_t)__cvta_generic_to_shared(dst)),
                   "l"(src)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  float tot[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) tot[mt][i] = 0.f;

  const int nchunks = p.K / KC;
  const int ngroups = p.K / G;
  load_chunk(0, 0);
  const uint8_t* wrow0 = p.w + (int64_t)(n0 + gid) * kpb + 16 * t;
  const uint8_t* wrow1 = wrow0 + (int64_t)8 * kpb;
  const int64_t srow0 = (int64_t)(n0 + gid) * groups, srow1 = srow0 + 8 * (int64_t)groups;

  // Prefetch ring: the weight bytes, scales and zero points of the next
  // PF groups are in flight while the current group is computed (the loop is
  // latency-bound otherwise: one 32-byte load per thread per group).
  constexpr int PF = 4;
  static_assert((KC / G) % PF == 0, "ring must divide the groups of a chunk");
  uint4 rw0[PF], rw1[PF];
  float rs0[PF], rs1[PF], rz0[PF], rz1[PF];
  auto fetch = [&](int grp, int slot_ignored, uint4& a, uint4& b, float& s0, float& s1,
                   float& z0, float& z1) {
    (void)slot_ignored;
    if (active && grp < ngroups) {
      a = ldg16(wrow0 + (int64_t)grp * 64);
      b = ldg16(wrow1 + (int64_t)grp * 64);
      s0 = load_sc(p.scales, srow0 + grp, p.scale_f16);
      s1 = load_sc(p.scales, srow1 + grp, p.scale_f16);
      if constexpr (MODE == 2) {
        z0 = load_sc(p.zp, srow0 + grp, p.scale_f16);
        z1 = load_sc(p.zp, srow1 + grp, p.scale_f16);
      }
    }
  };
#pragma unroll
  for (int i = 0; i < PF; ++i) fetch(i, i, rw0[i], rw1[i], rs0[i], rs1[i], rz0[i], rz1[i]);

  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    if (c + 1 < nchunks) {
      load_chunk(c + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    if (active) {
      const __nv_bfloat16* Ab = As + (int64_t)buf * rows_a * ROW;
#pragma unroll
      for (int gg = 0; gg < KC / G; ++gg) {
        constexpr int kSlots = PF;
        const int slot = gg % kSlots;
        const int grp = c * (KC / G) + gg;
        const uint4 w0 = rw0[slot], w1 = rw1[slot];
        const float s0 = rs0[slot], s1 = rs1[slot];
        uint32_t off0, off1;
        if constexpr (MODE == 2) {
          off0 = offset_pair(128.f + rz0[slot]);
          off1 = offset_pair(128.f + rz1[slot]);
        } else {
          off0 = off1 = offset_pair(MODE == 1 ? 136.f : 128.f);
        }
        fetch(grp + PF, slot, rw0[slot], rw1[slot], rs0[slot], rs1[slot], rz0[slot], rz1[slot]);
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
          for (int h = 0; h < 2; ++h) {  // k-tile j = 2i + h
            uint32_t af[4];
            if (h == 0) {
              af[0] = bf2_sub(nib_pair<0>(x0, y0), off0);
              af[1] = bf2_sub(nib_pair<0>(x1, y1), off1);
              af[2] = bf2_sub(nib_pair<1>(x0, y0), off0);
              af[3] = bf2_sub(nib_pair<1>(x1, y1), off1);
            } else {
              af[0] = bf2_sub(nib_pair<2>(x0, y0), off0);
              af[1] = bf2_sub(nib_pair<2>(x1, y1), off1);
              af[2] = bf2_sub(nib_pair<3>(x0, y0), off0);
              af[3] = bf2_sub(nib_pair<3>(x1, y1), off1);
            }
            const int kk = gg * G + 32 * t + 8 * i + 4 * h;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              const uint2 b = *reinterpret_cast<const uint2*>(Ab + (int64_t)(mt * 8 + gid) * ROW + kk);
              mma_bf16(acc[mt], af, b.x, b.y);
            }
          }
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          tot[mt][0] = __fmaf_rn(s0, acc[mt][0], tot[mt][0]);
          tot[mt][1] = __fmaf_rn(s0, acc[mt][1], tot[mt][1]);
          tot[mt][2] = __fmaf_rn(s1, acc[mt][2], tot[mt][2]);
          tot[mt][3] = __fmaf_rn(s1, acc[mt][3], tot[mt][3]);
        }
      }
    }
    __syncthreads();
  }

  if (!active) return;
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

template <int MT, int MODE, int OUT>
int launch(const Params& p, cudaStream_t st) {
  auto kern = k_int4_skinny<MT, MODE, OUT>;
  const int smem = 2 * 8 * MT * ROW * 2;
  if (smem > 48 * 1024) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return BRC_ERR_CUDA;
    if (!configured[dev]) {
      int rc = check_cuda(
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      if (rc) return rc;
      configured[dev] = true;
    }
  }
  const int n_rb = p.N / 16;
  int grid = sm_count();
  const int need = (n_rb + kWarps - 1) / kWarps;
  if (need > grid) grid = need;
  kern<<<grid, kThreads, smem, st>>>(p);
  return check_launch();
}

template <int MT, int MODE>
int launch_out(int out_dtype, const Params& p, cudaStream_t st) {
  if (out_dtype == BRC_DTYPE_F32) return launch<MT, MODE, BRC_DTYPE_F32>(p, st);
  if (out_dtype == BRC_DTYPE_BF16) return launch<MT, MODE, BRC_DTYPE_BF16>(p, st);
  return launch<MT, MODE, BRC_DTYPE_F16>(p, st);
}

template <int MT>
int launch_mode(int mode, int out_dtype, const Params& p, cudaStream_t st) {
  if (mode == 0) return launch_out<MT, 0>(out_dtype, p, st);
  if (mode == 1) return launch_out<MT, 1>(out_dtype, p, st);
  return launch_out<MT, 2>(out_dtype, p, st);
}

}  // namespace int4gemm
}  // namespace brc

extern "C" int brc_gemm_int4(const void* a_bf16, int M, int K, const uint8_t* w_packed, int N,
                             int group, int is_signed, int symmetric, int scale_dtype,
                             const void* scales, const void* zero_points, void* d, int d_dtype,
                             void* stream) {
  using namespace brc::int4gemm;
  if (!a_bf16 || !w_packed || !scales || !d) return BRC_ERR_NULL;
  if (!symmetric && !zero_points) return BRC_ERR_NULL;
  if (M <= 0 || N <= 0 || K <= 0) return (M == 0 || N == 0) ? BRC_OK : BRC_ERR_SHAPE;
  if (d_dtype != BRC_DTYPE_F32 && d_dtype != BRC_DTYPE_BF16 && d_dtype != BRC_DTYPE_F16)
    return BRC_ERR_DTYPE;
  if (scale_dtype != BRC_SCALE_F16 && scale_dtype != BRC_SCALE_F32) return BRC_ERR_DTYPE;
  if (M > 16 || group != G || K % KC || N % 16 || (!symmetric && is_signed))
    return BRC_ERR_UNSUPPORTED;
  if (((uintptr_t)a_bf16 | (uintptr_t)w_packed) & 15) return BRC_ERR_ALIGN;
  Params p{};
  p.a = static_cast<const __nv_bfloat16*>(a_bf16);
  p.w = w_packed;
  p.scales = scales;
  p.zp = zero_points;
  p.out = d;
  p.M = M;
  p.N = N;
  p.K = K;
  p.scale_f16 = scale_dtype == BRC_SCALE_F16;
  const int mode = symmetric ? (is_signed ? 1 : 0) : 2;
  cudaStream_t st = (cudaStream_t)stream;
  return M <= 8 ? launch_mode<1>(mode, d_dtype, p, st) : launch_mode<2>(mode, d_dtype, p, st);
}
