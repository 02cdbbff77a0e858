// Stored 4-bit data and GEMM operands rebuilt from stored tensors.
//
// breccia's on-disk nibble order (src/breccia/_formats.py:227-260,
// pack_nibbles / unpack_nibbles) puts element 2i in the HIGH nibble of byte
// i; the tensor cores read element 2i from the LOW nibble. The kernels here
// convert between one-code-per-byte data (the reference's ScaledTensor.data)
// and both packed orders, and rebuild, from stored codes and scales alone,
// the side operands the cast writes for the tensor-core GEMMs: the tcgen05
// scale-factor atoms (MXFP8 E8M0 / NVFP4 E4M3 scales) and the INT4
// skinny-GEMM tiles. Rebuilt operands equal the cast's byte for byte, so a
// tensor loaded from a file (or produced by another implementation) takes the
// same GEMM path as one cast here. All of this is byte movement: each kernel
// reads and writes every byte once, with 16-byte vector accesses where the
// layout allows.

#include <cuda_fp16.h>

#include "breccia_b200.h"
#include "common.cuh"
#include "launch.h"

namespace brc {
namespace bridge {

constexpr int kThreads = 256;

__host__ inline int grid_for(int64_t items) {
  int64_t g = (items + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (g > cap) g = cap;
  return g < 1 ? 1 : (int)g;
}

// Four packed bytes in breccia's order from eight codes (one per byte, low
// nibble): lo4 holds codes 0..3, hi4 codes 4..7.
__device__ __forceinline__ uint32_t pack_hi_word(uint32_t lo4, uint32_t hi4) {
  const uint32_t a = lo4 & 0x0F0F0F0Fu, b = hi4 & 0x0F0F0F0Fu;
  const uint32_t x = prmt(a, b, 0x6420u);  // codes 0, 2, 4, 6
  const uint32_t y = prmt(a, b, 0x7531u);  // codes 1, 3, 5, 7
  return (x << 4) | y;                     // the first code of each pair in the high nibble
}
// The same in the tensor-core order (the first code of each pair in the low nibble).
__device__ __forceinline__ uint32_t pack_lo_word(uint32_t lo4, uint32_t hi4) {
  const uint32_t a = lo4 & 0x0F0F0F0Fu, b = hi4 & 0x0F0F0F0Fu;
  const uint32_t x = prmt(a, b, 0x6420u);
  const uint32_t y = prmt(a, b, 0x7531u);
  return x | (y << 4);
}

// 16 codes -> 8 packed bytes per thread step (HI: breccia order, else tensor-core order).
template <bool HI>
__global__ void __launch_bounds__(kThreads) k_pack(const uint8_t* __restrict__ codes, int64_t n,
                                                    uint8_t* __restrict__ out) {
  const int64_t nv = n / 16;
  for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < nv;
       i += (int64_t)gridDim.x * kThreads) {
    const uint4 c = *reinterpret_cast<const uint4*>(codes + 16 * i);
    const uint32_t w0 = HI ? pack_hi_word(c.x, c.y) : pack_lo_word(c.x, c.y);
    const uint32_t w1 = HI ? pack_hi_word(c.z, c.w) : pack_lo_word(c.z, c.w);
    *reinterpret_cast<uint2*>(out + 8 * i) = make_uint2(w0, w1);
  }
  // tail (n % 16, even): one packed byte per thread
  const int64_t done = nv * 16;
  for (int64_t j = done / 2 + blockIdx.x * (int64_t)kThreads + threadIdx.x; j < n / 2;
       j += (int64_t)gridDim.x * kThreads) {
    const uint32_t e0 = codes[2 * j] & 0xFu, e1 = codes[2 * j + 1] & 0xFu;
    out[j] = (uint8_t)(HI ? (e0 << 4) | e1 : e0 | (e1 << 4));
  }
}

// 8 packed bytes (high-first) -> 16 codes and/or 8 bytes in the tensor-core
// order per thread step, so that a warp's loads (256 bytes), code stores
// (512 bytes) and packed stores (256 bytes) are each one contiguous run; eight
// steps' loads are in flight per thread (the kernel waits on memory: with
// four, ncu put 46 cycles of long-scoreboard stall on every issued
// instruction). packed and packed_lo are 16-byte aligned on this path.
__device__ __forceinline__ void unpack8_hi(const uint2 p, uint4& c, uint2& l) {
  const uint32_t pw[2] = {p.x, p.y};
  uint32_t cw[4], lw[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t hi = (pw[h] >> 4) & 0x0F0F0F0Fu;  // elements 0, 2, 4, 6
    const uint32_t lo = pw[h] & 0x0F0F0F0Fu;         // elements 1, 3, 5, 7
    cw[2 * h] = prmt(hi, lo, 0x5140u);               // 0, 1, 2, 3
    cw[2 * h + 1] = prmt(hi, lo, 0x7362u);           // 4, 5, 6, 7
    lw[h] = hi | (lo << 4);
  }
  c = make_uint4(cw[0], cw[1], cw[2], cw[3]);
  l = make_uint2(lw[0], lw[1]);
}

__global__ void __launch_bounds__(kThreads) k_unpack_hi(const uint8_t* __restrict__ packed,
                                                        int64_t n, uint8_t* __restrict__ codes,
                                                        uint8_t* __restrict__ packed_lo) {
  constexpr int U = 8;
  const int64_t nv = n / 16;
  const int64_t stride = (int64_t)gridDim.x * kThreads;
  auto emit = [&](int64_t i, const uint2 p) {
    uint4 c;
    uint2 l;
    unpack8_hi(p, c, l);
    if (codes) *reinterpret_cast<uint4*>(codes + 16 * i) = c;
    if (packed_lo) *reinterpret_cast<uint2*>(packed_lo + 8 * i) = l;
  };
  int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x;
  for (; i + (U - 1) * stride < nv; i += U * stride) {
    uint2 p[U];
#pragma unroll
    for (int u = 0; u < U; ++u) p[u] = *reinterpret_cast<const uint2*>(packed + 8 * (i + u * stride));
#pragma unroll
    for (int u = 0; u < U; ++u) emit(i + u * stride, p[u]);
  }
  for (; i < nv; i += stride) emit(i, *reinterpret_cast<const uint2*>(packed + 8 * i));
  const int64_t done = nv * 16;
  for (int64_t j = done / 2 + blockIdx.x * (int64_t)kThreads + threadIdx.x; j < n / 2;
       j += stride) {
    const uint32_t b = packed[j];
    if (codes) {
      codes[2 * j] = (uint8_t)(b >> 4);
      codes[2 * j + 1] = (uint8_t)(b & 0xFu);
    }
    if (packed_lo) packed_lo[j] = (uint8_t)((b >> 4) | ((b & 0xFu) << 4));
  }
}

// tcgen05 scale-factor atoms: every output byte, padding (rows past `rows`,
// columns past `cols`) written as zero. Byte b of atom (R, C) holds scale
// (128 R + 32 ((b % 16) / 4) + b / 16, 4 C + b % 4).
__global__ void __launch_bounds__(kThreads) k_scale_atoms(const uint8_t* __restrict__ scales,
                                                          int64_t rows, int64_t cols,
                                                          int64_t col_tiles,
                                                          uint8_t* __restrict__ atoms,
                                                          int64_t total_words, bool whole) {
  // whole: a word's 4 scales are one aligned 32-bit load (cols % 4 == 0 and
  // a 4-byte aligned base)
  for (int64_t wi = blockIdx.x * (int64_t)kThreads + threadIdx.x; wi < total_words;
       wi += (int64_t)gridDim.x * kThreads) {
    // one 32-bit word = 4 consecutive columns of one row; atom indices fit
    // 32 bits (the host checks), so the division is a 32-bit one
    const int64_t byte0 = 4 * wi;
    const uint32_t atom = (uint32_t)(byte0 >> 9);
    const uint32_t in_atom = (uint32_t)(byte0 & 511);
    const uint32_t R = atom / (uint32_t)col_tiles, C = atom - R * (uint32_t)col_tiles;
    const int64_t row = 128 * (int64_t)R + 32 * ((in_atom & 15u) >> 2) + (in_atom >> 4);
    uint32_t w = 0;
    if (row < rows) {
      const uint8_t* src = scales + row * cols + 4 * (int64_t)C;
      if (whole) {
        w = *reinterpret_cast<const uint32_t*>(src);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (4 * (int64_t)C + k < cols) w |= (uint32_t)src[k] << (8 * k);
      }
    }
    *reinterpret_cast<uint32_t*>(atoms + byte0) = w;
  }
}

// INT4 skinny-GEMM tiles (group 128, rows % 16 == 0) from stored codes, one
// thread per two 8-element runs: tile (r / 16) * groups + g, row r % 16 at
// 64 * (r % 16), byte 4j + i = element 8j + i | element 8j + i + 4 << 4; the
// first thread of each (row, group) also writes the float32 scale and
// 128 + zero point at tile * 16 + 2 * (r % 8) + (r % 16) / 8.
template <bool F16>
__global__ void __launch_bounds__(kThreads) k_int4_tiles(
    const uint8_t* __restrict__ codes, int64_t rows, int64_t cols, const void* __restrict__ scales,
    const void* __restrict__ zp, uint8_t* __restrict__ tiles, float* __restrict__ scale_tiles,
    float* __restrict__ zp_tiles) {
  const int64_t groups = cols / 128;
  const int64_t pairs = rows * groups * 8;  // pairs of 8-element runs (< 2^32: the host checks)
  const uint32_t per_row = (uint32_t)(groups * 8);
  for (int64_t t = blockIdx.x * (int64_t)kThreads + threadIdx.x; t < pairs;
       t += (int64_t)gridDim.x * kThreads) {
    const uint32_t t32 = (uint32_t)t;
    const int64_t row = t32 / per_row;
    const uint32_t rem = t32 - (uint32_t)row * per_row;
    const int64_t g = rem >> 3;
    const int j = 2 * (int)(rem & 7);  // first run of the pair
    const uint4 c = *reinterpret_cast<const uint4*>(codes + row * cols + 128 * g + 8 * j);
    const int64_t tile = (row >> 4) * groups + g;
    *reinterpret_cast<uint2*>(tiles + tile * 1024 + (row & 15) * 64 + 4 * j) =
        make_uint2((c.x & 0x0F0F0F0Fu) | ((c.y & 0x0F0F0F0Fu) << 4),
                   (c.z & 0x0F0F0F0Fu) | ((c.w & 0x0F0F0F0Fu) << 4));
    if (j == 0) {
      const int64_t q = tile * 16 + (row & 7) * 2 + ((row >> 3) & 1);
      const int64_t si = row * groups + g;
      const float s = F16 ? __half2float(static_cast<const __half*>(scales)[si])
                          : static_cast<const float*>(scales)[si];
      scale_tiles[q] = s;
      if (zp_tiles) {
        const float z = F16 ? __half2float(static_cast<const __half*>(zp)[si])
                            : static_cast<const float*>(zp)[si];
        zp_tiles[q] = __fadd_rn(128.f, z);
      }
    }
  }
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace bridge
}  // namespace brc

using namespace brc;
using namespace brc::bridge;

extern "C" {

int brc_pack_nibbles_hi(const uint8_t* codes, int64_t n, uint8_t* packed, void* stream) {
  if (n < 0 || n % 2) return BRC_ERR_SHAPE;
  if (n == 0) return BRC_OK;
  if (!codes || !packed) return BRC_ERR_NULL;
  if (!al16(codes) || (reinterpret_cast<uintptr_t>(packed) & 7u)) return BRC_ERR_ALIGN;
  k_pack<true><<<grid_for(n / 16 + 1), kThreads, 0, (cudaStream_t)stream>>>(codes, n, packed);
  return check_launch();
}

int brc_pack_codes_lo(const uint8_t* codes, int64_t n, uint8_t* packed_lo, void* stream) {
  if (n < 0 || n % 2) return BRC_ERR_SHAPE;
  if (n == 0) return BRC_OK;
  if (!codes || !packed_lo) return BRC_ERR_NULL;
  if (!al16(codes) || (reinterpret_cast<uintptr_t>(packed_lo) & 7u)) return BRC_ERR_ALIGN;
  k_pack<false><<<grid_for(n / 16 + 1), kThreads, 0, (cudaStream_t)stream>>>(codes, n,
                                                                              packed_lo);
  return check_launch();
}

int brc_unpack_nibbles_hi(const uint8_t* packed, int64_t n, uint8_t* codes, uint8_t* packed_lo,
                          void* stream) {
  if (n < 0 || n % 2) return BRC_ERR_SHAPE;
  if (n == 0) return BRC_OK;
  if (!packed || (!codes && !packed_lo)) return BRC_ERR_NULL;
  if (!al16(packed) || (codes && !al16(codes)) || (packed_lo && !al16(packed_lo)))
    return BRC_ERR_ALIGN;
  k_unpack_hi<<<grid_for(n / 128 + 1), kThreads, 0, (cudaStream_t)stream>>>(packed, n, codes,
                                                                            packed_lo);
  return check_launch();
}

int brc_scale_atoms(const uint8_t* scales, int64_t rows, int64_t scale_cols, uint8_t* atoms,
                    void* stream) {
  if (rows < 0 || scale_cols < 0) return BRC_ERR_SHAPE;
  if (rows == 0 || scale_cols == 0) return BRC_OK;
  if (!scales || !atoms) return BRC_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(atoms) & 3u) return BRC_ERR_ALIGN;
  const int64_t col_tiles = (scale_cols + 3) / 4;
  const int64_t total_words = ((rows + 127) / 128) * col_tiles * 128;
  if (total_words / 128 > 0xFFFFFFFFll) return BRC_ERR_RANGE;
  const bool whole = scale_cols % 4 == 0 && (reinterpret_cast<uintptr_t>(scales) & 3u) == 0;
  k_scale_atoms<<<grid_for(total_words), kThreads, 0, (cudaStream_t)stream>>>(
      scales, rows, scale_cols, col_tiles, atoms, total_words, whole);
  return check_launch();
}

int brc_int4_tiles(const uint8_t* codes, int64_t rows, int64_t cols, const void* scales,
                   const void* zero_points, int scale_dtype, uint8_t* tiles, float* scale_tiles,
                   float* zp_tiles, void* stream) {
  if (rows < 0 || cols < 0) return BRC_ERR_SHAPE;
  if (rows % 16 || cols % 128) return BRC_ERR_UNSUPPORTED;
  if (rows == 0 || cols == 0) return BRC_OK;
  if (!codes || !scales || !tiles || !scale_tiles) return BRC_ERR_NULL;
  if ((zero_points == nullptr) != (zp_tiles == nullptr)) return BRC_ERR_NULL;
  if (scale_dtype != BRC_SCALE_F16 && scale_dtype != BRC_SCALE_F32) return BRC_ERR_DTYPE;
  if (!al16(codes) || !al16(tiles)) return BRC_ERR_ALIGN;
  const int64_t pairs = rows * (cols / 128) * 8;
  if (pairs > 0xFFFFFFFFll) return BRC_ERR_RANGE;
  cudaStream_t st = (cudaStream_t)stream;
  if (scale_dtype == BRC_SCALE_F16)
    k_int4_tiles<true><<<grid_for(pairs), kThreads, 0, st>>>(codes, rows, cols, scales,
                                                            zero_points, tiles, scale_tiles,
                                                            zp_tiles);
  else
    k_int4_tiles<false><<<grid_for(pairs), kThreads, 0, st>>>(codes, rows, cols, scales,
                                                             zero_points, tiles, scale_tiles,
                                                             zp_tiles);
  return check_launch();
}

}  // extern "C"
