// Layout kernels for breccia's own matmul orientation.
//
// breccia's matmul(a, b) takes b as (K, N) with its scale blocks along the
// last axis, N (src/breccia/kernels/reference/matmul.py:123-133 multiplies the
// dequantized operands; cast.py blocks the last axis). The tensor-core GEMMs
// consume both operands K-major, (rows, K). These kernels move a (K, N)
// operand into the (N, K) orientation on the way:
//
//   k_dequant_t    decode(code) * scale of a block-scaled (rows, cols) tensor
//                  (any recipe: per-tensor FP8, block FP8, MXFP8, NVFP4, INT4),
//                  written transposed as (cols, rows) float32 / bf16 / f16.
//                  The products are the reference's float32 dequantize
//                  (cast.py:376-586), then rounded once to the output type.
//   k_transpose_u8 (rows, cols) bytes -> (cols, rows): per-tensor FP8 codes do
//                  not depend on orientation, so they move as plain bytes.
//
// Both stage 128 x 128 tiles of codes through shared memory as transposed
// bytes: a thread loads 16 consecutive codes of each of 4 source rows
// (16-byte loads, 128 contiguous bytes per row per warp), transposes the 4 x 4
// byte blocks in registers and stores whole 32-bit words; destination rows are
// written in 16-byte pieces, so global traffic stays coalesced in both
// orientations.

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "breccia_b200.h"
#include "common.cuh"
#include "launch.h"

namespace brc {
namespace {

constexpr int kThreads = 256;

struct DqtArgs {
  const uint8_t* codes;
  const void* scales;
  const void* zp;
  void* out;
  int64_t rows, cols;
  int block;           // scale run along cols
  int64_t scale_cols;  // cols / block
  int is_signed;
  int scale_f16;
};

// Up to 32 CTAs per SM: measured on B200 against 8, the transposing
// dequantize (8192 x 28672) ran 286 -> 259 us (MXFP8), 266 -> 241 us (NVFP4)
// and the byte transpose 161 -> 147 us.
int grid_tiles(int64_t tiles) {
  const int64_t cap = (int64_t)sm_count() * 32;
  return (int)(tiles < cap ? (tiles < 1 ? 1 : tiles) : cap);
}

__device__ __forceinline__ float e8m0_value(uint32_t e) {
  // 2^(e - 127) in float32, as the reference's float32 power gives it:
  // e = 0 is the subnormal 2^-127, e = 255 overflows to +inf.
  if (e == 255u) return __uint_as_float(0x7F800000u);
  if (e == 0u) return __uint_as_float(0x00400000u);
  return __uint_as_float(e << 23);
}

template <int OUT>
__device__ __forceinline__ void store8(void* out, int64_t e0, const float* v) {
  if constexpr (OUT == BRC_DTYPE_F32) {
    float* o = static_cast<float*>(out) + e0;
    stg16(o, make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                        __float_as_uint(v[3])));
    stg16(o + 4, make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]),
                            __float_as_uint(v[6]), __float_as_uint(v[7])));
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (OUT == BRC_DTYPE_BF16) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    stg16(static_cast<char*>(out) + e0 * 2, make_uint4(w[0], w[1], w[2], w[3]));
  }
}

// (rows, cols) bytes -> (cols, rows); rows % 16 == 0, cols % 16 == 0.
// 128 x 128 tiles: every input row segment read and every output row segment
// written is 128 contiguous bytes. Thread (a, b) loads rows 4a..4a+3 of the
// 16-byte column group b and transposes each 4 x 4 byte block in registers
// (byte permutes), so shared memory sees whole 32-bit words: word a of output
// row R (input rows 4a..4a+3 of column R) sits at a ^ 4 * (R / 16), which puts
// a warp's 32 stores and each quarter-warp's 16-byte reads in distinct banks.
constexpr int kTT = 128;
__global__ void __launch_bounds__(kThreads) k_transpose_u8(const uint8_t* __restrict__ in,
                                                          int64_t rows, int64_t cols,
                                                          uint8_t* __restrict__ out) {
  __shared__ __align__(16) uint32_t tile[kTT][kTT / 4];
  const int64_t tiles_r = (rows + kTT - 1) / kTT;
  const int64_t tiles_c = (cols + kTT - 1) / kTT;
  const int a = threadIdx.x >> 3, b = threadIdx.x & 7;  // load: 4-row group, column group
  for (int64_t t = blockIdx.x; t < tiles_r * tiles_c; t += gridDim.x) {
    const int64_t r0 = (t / tiles_c) * kTT, c0 = (t % tiles_c) * kTT;
    uint4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t r = r0 + 4 * a + k, c = c0 + 16 * b;
      v[k] = (r < rows && c < cols) ? ldg16(in + r * cols + c) : make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads();  // the previous tile's readers are done with `tile`
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t x0 = (&v[0].x)[j], x1 = (&v[1].x)[j], x2 = (&v[2].x)[j],
                     x3 = (&v[3].x)[j];
      const uint32_t t0 = prmt(x0, x1, 0x5140u), t1 = prmt(x0, x1, 0x7362u);
      const uint32_t t2 = prmt(x2, x3, 0x5140u), t3 = prmt(x2, x3, 0x7362u);
      const uint32_t o[4] = {prmt(t0, t2, 0x5410u), prmt(t0, t2, 0x7632u),
                             prmt(t1, t3, 0x5410u), prmt(t1, t3, 0x7632u)};
#pragma unroll
      for (int m = 0; m < 4; ++m) tile[16 * b + 4 * j + m][a ^ (b << 2)] = o[m];
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int R = 32 * q + (threadIdx.x >> 3), sg = threadIdx.x & 7;
      const int64_t oc = c0 + R, orow = r0 + 16 * sg;
      if (oc < cols && orow < rows) {
        const uint4 w = *reinterpret_cast<const uint4*>(&tile[R][(sg ^ (R >> 4)) * 4]);
        stg16(out + oc * rows + orow, w);
      }
    }
  }
}

// KIND: BRC_STE_BLOCK_FP8, BRC_STE_MXFP8, BRC_STE_NVFP4, BRC_STE_INT4 or
// BRC_KIND_PERTENSOR_FP8. rows % 8 == 0, cols % 16 == 0, block % 16 == 0,
// cols % block == 0. One 128 x 128 tile of codes per iteration: the codes are
// transposed as bytes (as in k_transpose_u8), the tile's scales (and zero
// points) are decoded once into a table of [column block][row], and each
// thread then decodes 8 codes of one output row (8 consecutive source rows of
// one source column) with their 8 scales and stores 8 output values.
constexpr int kDqtMaxCb = kTT / 16 + 1;  // column blocks a tile can touch
template <int KIND, int FMT, int OUT>
__global__ void __launch_bounds__(kThreads) k_dequant_t(DqtArgs a) {
  constexpr bool kTable = KIND != BRC_KIND_PERTENSOR_FP8;
  constexpr bool kZp = KIND == BRC_STE_INT4;
  __shared__ __align__(16) uint32_t ctile[kTT][kTT / 4];
  __shared__ __align__(16) float sc[kTable ? kDqtMaxCb : 1][kTT];
  __shared__ __align__(16) float zpt[kZp ? kDqtMaxCb : 1][kTT];
  const int64_t tiles_r = (a.rows + kTT - 1) / kTT;
  const int64_t tiles_c = (a.cols + kTT - 1) / kTT;
  const int la = threadIdx.x >> 3, lb = threadIdx.x & 7;  // load: 4-row group, column group
  float pt_scale = 0.f;
  if constexpr (!kTable) pt_scale = *static_cast<const float*>(a.scales);
  for (int64_t t = blockIdx.x; t < tiles_r * tiles_c; t += gridDim.x) {
    const int64_t r0 = (t / tiles_c) * kTT, c0 = (t % tiles_c) * kTT;
    uint4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t r = r0 + 4 * la + k, c = c0 + 16 * lb;
      v[k] = (r < a.rows && c < a.cols) ? ldg16(a.codes + r * a.cols + c)
                                        : make_uint4(0u, 0u, 0u, 0u);
    }
    const int64_t cb0 = c0 / a.block;
    const int ncb = kTable ? (int)((min(c0 + kTT, a.cols) - 1) / a.block - cb0 + 1) : 0;
    // Table entries of this thread (one tile row, every (kThreads / kTT)-th
    // column block): their raw scale / zero-point bits are loaded here, beside
    // the codes, so the two global loads overlap; decoded after the barrier.
    constexpr int kPer = (kDqtMaxCb + kThreads / kTT - 1) / (kThreads / kTT);
    const int r = threadIdx.x & (kTT - 1);
    uint32_t sraw[kTable ? kPer : 1], zraw[kZp ? kPer : 1];
    if constexpr (kTable) {
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int cbi = threadIdx.x / kTT + u * (kThreads / kTT);
        sraw[u] = 0u;
        if constexpr (kZp) zraw[u] = 0u;
        if (cbi < ncb && r0 + r < a.rows) {
          const int64_t si = (r0 + r) * a.scale_cols + cb0 + cbi;
          if constexpr (KIND == BRC_STE_BLOCK_FP8) {
            sraw[u] = __float_as_uint(static_cast<const float*>(a.scales)[si]);
          } else if constexpr (KIND == BRC_STE_MXFP8 || KIND == BRC_STE_NVFP4) {
            sraw[u] = static_cast<const uint8_t*>(a.scales)[si];
          } else if (a.scale_f16) {
            sraw[u] = __half_as_ushort(static_cast<const __half*>(a.scales)[si]);
            if constexpr (kZp)
              if (a.zp) zraw[u] = __half_as_ushort(static_cast<const __half*>(a.zp)[si]);
          } else {
            sraw[u] = __float_as_uint(static_cast<const float*>(a.scales)[si]);
            if constexpr (kZp)
              if (a.zp) zraw[u] = __float_as_uint(static_cast<const float*>(a.zp)[si]);
          }
        }
      }
    }
    __syncthreads();  // the previous tile's readers are done with the shared tables
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t x0 = (&v[0].x)[j], x1 = (&v[1].x)[j], x2 = (&v[2].x)[j],
                     x3 = (&v[3].x)[j];
      const uint32_t t0 = prmt(x0, x1, 0x5140u), t1 = prmt(x0, x1, 0x7362u);
      const uint32_t t2 = prmt(x2, x3, 0x5140u), t3 = prmt(x2, x3, 0x7362u);
      const uint32_t o[4] = {prmt(t0, t2, 0x5410u), prmt(t0, t2, 0x7632u),
                             prmt(t1, t3, 0x5410u), prmt(t1, t3, 0x7632u)};
#pragma unroll
      for (int m = 0; m < 4; ++m) ctile[16 * lb + 4 * j + m][la ^ (lb << 2)] = o[m];
    }
    if constexpr (kTable) {
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int cbi = threadIdx.x / kTT + u * (kThreads / kTT);
        if (cbi < ncb) {
          float scale, zp = 0.f;
          if constexpr (KIND == BRC_STE_BLOCK_FP8) {
            scale = __uint_as_float(sraw[u]);
          } else if constexpr (KIND == BRC_STE_MXFP8) {
            scale = e8m0_value(sraw[u]);
          } else if constexpr (KIND == BRC_STE_NVFP4) {
            scale = dec_e4m3(sraw[u]);
          } else if (a.scale_f16) {
            scale = __half2float(__ushort_as_half((unsigned short)sraw[u]));
            if constexpr (kZp) zp = __half2float(__ushort_as_half((unsigned short)zraw[u]));
          } else {
            scale = __uint_as_float(sraw[u]);
            if constexpr (kZp) zp = __uint_as_float(zraw[u]);
          }
          sc[cbi][r] = scale;
          if constexpr (kZp) zpt[cbi][r] = zp;
        }
      }
    }
    __syncthreads();
#pragma unroll 2
    for (int q = 0; q < 8; ++q) {
      const int R = 16 * q + (threadIdx.x >> 4), sg = threadIdx.x & 15;  // output row, 8-row segment
      const int64_t c = c0 + R, orow = r0 + 8 * sg;
      if (c >= a.cols || orow >= a.rows) continue;
      const uint2 w = *reinterpret_cast<const uint2*>(&ctile[R][(2 * sg) ^ ((R >> 4) << 2)]);
      float s8[8], z8[8];
      if constexpr (kTable) {
        const int cbi = (int)(c / a.block - cb0);
        const float4 sa = *reinterpret_cast<const float4*>(&sc[cbi][8 * sg]);
        const float4 sb = *reinterpret_cast<const float4*>(&sc[cbi][8 * sg + 4]);
        s8[0] = sa.x; s8[1] = sa.y; s8[2] = sa.z; s8[3] = sa.w;
        s8[4] = sb.x; s8[5] = sb.y; s8[6] = sb.z; s8[7] = sb.w;
        if constexpr (kZp) {
          const float4 za = *reinterpret_cast<const float4*>(&zpt[cbi][8 * sg]);
          const float4 zb = *reinterpret_cast<const float4*>(&zpt[cbi][8 * sg + 4]);
          z8[0] = za.x; z8[1] = za.y; z8[2] = za.z; z8[3] = za.w;
          z8[4] = zb.x; z8[5] = zb.y; z8[6] = zb.z; z8[7] = zb.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) s8[i] = pt_scale;
      }
      float d8[8], o8[8];
      if constexpr (KIND == BRC_STE_INT4) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t lo = ((i < 4 ? w.x : w.y) >> (8 * (i & 3))) & 0xFu;
          d8[i] = (a.is_signed && lo >= 8) ? (float)((int)lo - 16) : (float)lo;
          if (a.zp) d8[i] = __fsub_rn(d8[i], z8[i]);
        }
      } else {
        // code pairs through the exact hardware conversions to f16
        const uint32_t pr[4] = {w.x, w.x >> 16, w.y, w.y >> 16};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if constexpr (KIND == BRC_STE_NVFP4)
            f16x2_to_f32(e2m1_bytes_to_f16x2(pr[k]), d8[2 * k], d8[2 * k + 1]);
          else
            f16x2_to_f32(fp8x2_to_f16x2<FMT>(pr[k]), d8[2 * k], d8[2 * k + 1]);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) o8[i] = __fmul_rn(d8[i], s8[i]);
      store8<OUT>(a.out, c * a.rows + orow, o8);
    }
  }
}

template <int KIND, int FMT>
int launch_dqt(const DqtArgs& a, int out_dtype, cudaStream_t st) {
  const int64_t tiles = ((a.rows + kTT - 1) / kTT) * ((a.cols + kTT - 1) / kTT);
  const int grid = grid_tiles(tiles);
  if (out_dtype == BRC_DTYPE_F32)
    k_dequant_t<KIND, FMT, BRC_DTYPE_F32><<<grid, kThreads, 0, st>>>(a);
  else if (out_dtype == BRC_DTYPE_BF16)
    k_dequant_t<KIND, FMT, BRC_DTYPE_BF16><<<grid, kThreads, 0, st>>>(a);
  else
    k_dequant_t<KIND, FMT, BRC_DTYPE_F16><<<grid, kThreads, 0, st>>>(a);
  return check_launch();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace brc

using namespace brc;

extern "C" {

int brc_dequant_transposed(const uint8_t* codes, int64_t rows, int64_t cols, int kind, int fmt,
                           int block, int is_signed, int scale_dtype, const void* scales,
                           const void* zero_points, void* out, int out_dtype, void* stream) {
  if (rows < 0 || cols < 0) return BRC_ERR_SHAPE;
  if ((!codes || !scales || !out) && rows * cols > 0) return BRC_ERR_NULL;
  if (out_dtype != BRC_DTYPE_F32 && out_dtype != BRC_DTYPE_BF16 && out_dtype != BRC_DTYPE_F16)
    return BRC_ERR_DTYPE;
  if (fmt != BRC_FP8_E4M3 && fmt != BRC_FP8_E5M2) return BRC_ERR_DTYPE;
  if (kind == BRC_STE_MXFP8) block = 32;
  if (kind == BRC_STE_NVFP4) block = 16;
  if (kind == BRC_KIND_PERTENSOR_FP8) block = 16;
  if (kind < 0 || kind > BRC_KIND_PERTENSOR_FP8) return BRC_ERR_UNSUPPORTED;
  if (block <= 0 || block % 16 || cols % block || cols % 16 || rows % 8) return BRC_ERR_SHAPE;
  if (kind == BRC_STE_INT4 && scale_dtype != BRC_SCALE_F16 && scale_dtype != BRC_SCALE_F32)
    return BRC_ERR_DTYPE;
  if (rows * cols == 0) return BRC_OK;
  if (!aligned16(codes) || !aligned16(out)) return BRC_ERR_ALIGN;
  DqtArgs a{};
  a.codes = codes;
  a.scales = scales;
  a.zp = zero_points;
  a.out = out;
  a.rows = rows;
  a.cols = cols;
  a.block = block;
  a.scale_cols = cols / block;
  a.is_signed = is_signed ? 1 : 0;
  a.scale_f16 = scale_dtype == BRC_SCALE_F16;
  cudaStream_t st = (cudaStream_t)stream;
  const bool e4 = fmt == BRC_FP8_E4M3;
  switch (kind) {
    case BRC_STE_BLOCK_FP8:
      return e4 ? launch_dqt<BRC_STE_BLOCK_FP8, BRC_FP8_E4M3>(a, out_dtype, st)
                : launch_dqt<BRC_STE_BLOCK_FP8, BRC_FP8_E5M2>(a, out_dtype, st);
    case BRC_STE_MXFP8:
      return e4 ? launch_dqt<BRC_STE_MXFP8, BRC_FP8_E4M3>(a, out_dtype, st)
                : launch_dqt<BRC_STE_MXFP8, BRC_FP8_E5M2>(a, out_dtype, st);
    case BRC_STE_NVFP4:
      return launch_dqt<BRC_STE_NVFP4, BRC_FP8_E4M3>(a, out_dtype, st);
    case BRC_STE_INT4:
      return launch_dqt<BRC_STE_INT4, BRC_FP8_E4M3>(a, out_dtype, st);
    default:
      return e4 ? launch_dqt<BRC_KIND_PERTENSOR_FP8, BRC_FP8_E4M3>(a, out_dtype, st)
                : launch_dqt<BRC_KIND_PERTENSOR_FP8, BRC_FP8_E5M2>(a, out_dtype, st);
  }
}

int brc_transpose_u8(const uint8_t* in, int64_t rows, int64_t cols, uint8_t* out, void* stream) {
  if (rows < 0 || cols < 0 || rows % 16 || cols % 16) return BRC_ERR_SHAPE;
  if ((!in || !out) && rows * cols > 0) return BRC_ERR_NULL;
  if (rows * cols == 0) return BRC_OK;
  if (!aligned16(in) || !aligned16(out)) return BRC_ERR_ALIGN;
  const int64_t tiles = ((rows + kTT - 1) / kTT) * ((cols + kTT - 1) / kTT);
  k_transpose_u8<<<grid_tiles(tiles), kThreads, 0, (cudaStream_t)stream>>>(in, rows, cols, out);
  return check_launch();
}

}  // extern "C"
