// Cast / dequantize / requantize kernels for every breccia recipe (sm_100a).
//
// All row-local recipes (Float8BlockScaling 1 x block_k, MXFP8, NVFP4, INT4)
// share one kernel shape. Because blocks run along the last axis and the
// row length is a multiple of the block, a row-major (rows, cols) tensor is
// a flat sequence of contiguous blocks, and the row-major scale tensor is
// indexed by the flat block number. Each warp processes "tiles" of
// 32 / LPB blocks; LPB adjacent lanes share one block, each lane owning
// B / LPB contiguous elements loaded as 16-byte vectors. The block statistic
// (abs-max, or min and max) is reduced with xor-shuffles over those lanes.
// Grids are sized to the SM count and loop over tiles.
//
// HBM traffic per element is the input read plus the code write; the kernels
// keep the per-element instruction count low enough (~10-14 ops) that a
// 2-byte input stays bandwidth-bound.

#include <cmath>
#include <mutex>

#include "common.cuh"
#include "e8m0_thresholds.h"
#include "launch.h"
#include "sm100.cuh"

namespace brc {

uint32_t* gemm_status_ptr();  // device address of the status word (gemm_sm100.cu)

__device__ const uint32_t g_e8m0_thr[kE8m0Binades] = {BRC_E8M0_THRESHOLDS};

// n / d for n < 2^32 with a precomputed 33-bit multiplier (Granlund and
// Montgomery, "Division by invariant integers using multiplication", 1994).
struct FastDiv {
  uint32_t d, mul, shift;
};
static FastDiv make_fastdiv(uint32_t d) {
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  FastDiv f;
  f.d = d;
  f.shift = l;
  f.mul = (uint32_t)((((1ull << 32) * ((1ull << l) - d)) / d) + 1);
  return f;
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
  return (uint32_t)(((uint64_t)__umulhi(n, f.mul) + n) >> f.shift);
}

// Byte offset of scale (row, col) in the tcgen05 block-scale layout.
__device__ __forceinline__ uint32_t sf_mma_offset(uint32_t row, uint32_t col,
                                                  uint32_t col_tiles) {
  return ((row >> 7) * col_tiles + (col >> 2)) * 512u + (row & 31u) * 16u +
         ((row >> 5) & 3u) * 4u + (col & 3u);
}

// --------------------------------------------------------------- helpers
template <int NW>
__device__ __forceinline__ void store_words(uint8_t* p, const uint32_t* w) {
  if constexpr (NW == 1) {
    *reinterpret_cast<uint32_t*>(p) = w[0];
  } else if constexpr (NW == 2) {
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
  } else {
#pragma unroll
    for (int i = 0; i < NW; i += 4)
      stg16(p + 4 * i, make_uint4(w[i], w[i + 1], w[i + 2], w[i + 3]));
  }
}

// Pack unpacked FP4/INT4 code words (one code per byte, 4 per word) two per
// byte, element 2i in the low nibble.
template <int NW>
__device__ __forceinline__ void store_packed(uint8_t* p, const uint32_t* w) {
  uint32_t out[NW / 2];
#pragma unroll
  for (int i = 0; i < NW / 2; ++i) {
    const uint32_t a = w[2 * i] | (w[2 * i] >> 4);
    const uint32_t b = w[2 * i + 1] | (w[2 * i + 1] >> 4);
    out[i] = prmt(a, b, 0x6420);
  }
  store_words<NW / 2>(p, out);
}

template <int DT>
__device__ __forceinline__ void vec_minmax(const uint4 v, float& mn, float& mx) {
  float f[In<DT>::kVec];
  unpack<DT>(v, f);
#pragma unroll
  for (int i = 0; i < In<DT>::kVec; ++i) {
    mn = fmin_nan(mn, f[i]);
    mx = fmax_nan(mx, f[i]);
  }
}

template <int DT>
constexpr int elem_bytes() { return DT == BRC_DTYPE_F32 ? 4 : 2; }

// Power of two 2^k as a float32 for k in [-149, 127] (exact).
__device__ __forceinline__ float exp2i(int k) {
  if (k >= -126) return __uint_as_float((uint32_t)(k + 127) << 23);
  return __uint_as_float(1u << (k + 149));
}

// --------------------------------------------------------------- modes
enum Mode { kBlockFp8 = 0, kMxfp8 = 1, kNvfp4 = 2, kInt4Sym = 3, kInt4Asym = 4 };

struct BlockCastArgs {
  const void* x;
  uint8_t* codes;       // one code per element, or null (nvfp4/int4)
  uint8_t* packed;      // two per byte, or null
  void* scales;
  void* zp;
  uint8_t* scales_mma;  // tcgen05 layout, or null
  int64_t n_blocks;
  FastDiv blocks_per_row;
  uint32_t sf_col_tiles;
  int is_signed;
  int scale_f16;
  // INT4, group 128, rows % 16 == 0: the skinny-GEMM layout (16-row x 128
  // element tiles of packed codes, fp32 scales / zero points per tile row)
  uint8_t* packed_tiles;
  float* scale_tiles;
  float* zp_tiles;
  // cast_ste: float32 x + (dequantize(cast(x)) - x), one per element; no
  // codes or scales are written
  float* ste_out;
};

template <int E>
struct LaneVals {
  float f[E];
};

// cast_ste output for one lane: each code's dequantized value y (decode x
// the stored scale; asymmetric INT4 (q - zp) x scale, as cast.py:574-586) and
// x + (y - x) in float32, as the reference's x + (y - x).detach() evaluates it.
// The values go straight to this lane's slot of the warp's shared-memory
// stage (16 bytes at a time), so no register array holds them.
template <int MODE, int FMT, int NW>
__device__ __forceinline__ void ste_values(const BlockCastArgs& a, const float* f,
                                           const uint32_t* w, float dqs, float dqz, float* o) {
#pragma unroll
  for (int j = 0; j < NW; ++j) {
    float q[4], d[4];
    if constexpr (MODE == kBlockFp8 || MODE == kMxfp8) {
      // hardware pair conversions (exact; a NaN code's sign and payload do
      // not reach the result: the float32 arithmetic below returns the
      // canonical NaN for any NaN operand)
      f16x2_to_f32(fp8x2_to_f16x2<FMT>(w[j]), d[0], d[1]);
      f16x2_to_f32(fp8x2_to_f16x2<FMT>(w[j] >> 16), d[2], d[3]);
    } else if constexpr (MODE == kNvfp4) {
      f16x2_to_f32(e2m1_bytes_to_f16x2(w[j]), d[0], d[1]);
      f16x2_to_f32(e2m1_bytes_to_f16x2(w[j] >> 16), d[2], d[3]);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t lo = (w[j] >> (8 * i)) & 0xFu;
        d[i] = (MODE == kInt4Sym && a.is_signed && lo >= 8) ? (float)((int)lo - 16) : (float)lo;
        if constexpr (MODE == kInt4Asym) d[i] = __fsub_rn(d[i], dqz);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float x = f[4 * j + i];
      q[i] = __fadd_rn(x, __fsub_rn(__fmul_rn(d[i], dqs), x));
    }
    *reinterpret_cast<float4*>(o + 4 * j) = make_float4(q[0], q[1], q[2], q[3]);
  }
}

// The warp's cast_ste values go out through a per-warp shared-memory
// transpose: lane l has written its E consecutive values (elements l * E ..
// l * E + E of the warp's tile, which is contiguous in memory) to row l of
// `stage` (32 rows of E + 4 floats); stores of 16 bytes per lane at lane
// stride E * 4 bytes would each touch 32 separate lines, while after the
// transpose every warp store writes 512 contiguous bytes. Every lane of the
// warp calls this; elements past the tensor's end are not stored.
template <int E>
__device__ __forceinline__ void ste_warp_store(const BlockCastArgs& a, int64_t tile_e0,
                                               int64_t n_elems, const float* stage) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
#pragma unroll
  for (int q = 0; q < E / 4; ++q) {
    const int e = q * 128 + 4 * lane;  // element of the warp's tile
    if (tile_e0 + e < n_elems) {
      const float4 v = *reinterpret_cast<const float4*>(stage + (e / E) * (E + 4) + e % E);
      stg16(a.ste_out + tile_e0 + e, make_uint4(__float_as_uint(v.x), __float_as_uint(v.y),
                                                __float_as_uint(v.z), __float_as_uint(v.w)));
    }
  }
  __syncwarp();  // the stage is rewritten by the next tile
}

// Encode one lane's E values given the block's scale; writes codes/packed
// (or, STE, the cast_ste values with the stored scale dqs and zero point dqz).
template <int MODE, int FMT, int E, bool STE = false>
__device__ __forceinline__ void encode_lane(const BlockCastArgs& a, int64_t e0, const float* f,
                                            float s, float zp, bool fast, int64_t tile_off,
                                            float dqs = 0.f, float dqz = 0.f,
                                            float* ste = nullptr) {
  constexpr int NW = E / 4;
  uint32_t w[NW];
  if constexpr (MODE == kBlockFp8 || MODE == kMxfp8) {
    if (fast) {
      if constexpr (MODE == kMxfp8) {
        // s holds the exact power-of-two reciprocal of the E8M0 scale.
#pragma unroll
        for (int j = 0; j < NW; ++j)
          w[j] = enc4_fp8<FMT>(__fmul_rn(f[4 * j], s), __fmul_rn(f[4 * j + 1], s),
                               __fmul_rn(f[4 * j + 2], s), __fmul_rn(f[4 * j + 3], s));
      } else {
        const float r = __frcp_rn(s);
#pragma unroll
        for (int j = 0; j < NW; ++j)
          w[j] = enc4_div<enc4p_fp8<FMT>>(f + 4 * j, s, r);
      }
    } else {
#pragma unroll
      for (int j = 0; j < NW; ++j) {
        uint32_t c = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) c |= enc1_fp8<FMT>(div_ieee(f[4 * j + i], s)) << (8 * i);
        w[j] = c;
      }
    }
    if constexpr (STE) {
      ste_values<MODE, FMT, NW>(a, f, w, dqs, dqz, ste);
      return;
    }
    store_words<NW>(a.codes + e0, w);
  } else if constexpr (MODE == kNvfp4) {
    if (fast) {
      const float r = __frcp_rn(s);
#pragma unroll
      for (int j = 0; j < NW; ++j)
        w[j] = enc4_div<enc4p_e2m1>(f + 4 * j, s, r);
    } else {
#pragma unroll
      for (int j = 0; j < NW; ++j) {
        uint32_t c = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) c |= enc1_e2m1(div_ieee(f[4 * j + i], s)) << (8 * i);
        w[j] = c;
      }
    }
    if constexpr (STE) {
      ste_values<MODE, FMT, NW>(a, f, w, dqs, dqz, ste);
      return;
    }
    if (a.codes) store_words<NW>(a.codes + e0, w);
    if (a.packed) store_packed<NW>(a.packed + e0 / 2, w);
  } else {
    // INT4: np.round(np.clip(v, lo, hi)) with half-to-even rounding via the
    // 1.5 * 2^23 addition; the low nibble of the sum's bits is the code.
    const float lo = (MODE == kInt4Sym && a.is_signed) ? -8.f : 0.f;
    const float hi = (MODE == kInt4Sym && a.is_signed) ? 7.f : 15.f;
    if (fast) {
      const float r = __frcp_rn(s);
#pragma unroll
      for (int j = 0; j < NW; ++j) {
        uint32_t c = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float q = div_by(f[4 * j + i], s, r);
          if constexpr (MODE == kInt4Asym) q = __fadd_rn(q, zp);
          // np.round(np.clip(q, lo, hi)) with half-to-even rounding via
          // 1.5 * 2^23; NaN inputs clip to lo with fminf/fmaxf, but a block
          // holding a NaN has a NaN statistic and takes the slow path
          const float v = fminf(fmaxf(q, lo), hi);
          c |= (__float_as_uint(__fadd_rn(v, 12582912.f)) & 0xFu) << (8 * i);
        }
        w[j] = c;
      }
    } else {
      for (int j = 0; j < NW; ++j) {
        uint32_t c = 0;
        for (int i = 0; i < 4; ++i) {
          float q = div_ieee(f[4 * j + i], s);
          if constexpr (MODE == kInt4Asym) q = __fadd_rn(q, zp);
          uint32_t code = 0u;  // NumPy's float->uint8 conversion of NaN gives 0
          if (!isnan(q)) {
            const float v = fminf(fmaxf(q, lo), hi);
            code = __float_as_uint(__fadd_rn(v, 12582912.f)) & 0xFu;
          }
          c |= code << (8 * i);
        }
        w[j] = c;
      }
    }
    if constexpr (STE) {
      ste_values<MODE, FMT, NW>(a, f, w, dqs, dqz, ste);
      return;
    }
    if (a.codes) store_words<NW>(a.codes + e0, w);
    if (a.packed) store_packed<NW>(a.packed + e0 / 2, w);
    if (a.packed_tiles) {
      // skinny-GEMM tile order: in each run of 8 elements, byte j holds
      // element j (low nibble) and element j + 4 (high nibble)
      static_assert(NW % 2 == 0, "tile packing works on 8-element runs");
      uint32_t t[NW / 2];
#pragma unroll
      for (int i = 0; i < NW / 2; ++i) t[i] = w[2 * i] | (w[2 * i + 1] << 4);
      store_words<NW / 2>(a.packed_tiles + tile_off, t);
    }
  }
}

template <int DT, int MODE, int FMT, int B, int LPB, bool STE = false>
__global__ void __launch_bounds__(256) k_block_cast(BlockCastArgs a) {
  constexpr int V = In<DT>::kVec;
  constexpr int E = B / LPB;
  constexpr int NV = E / V;
  constexpr int BPW = 32 / LPB;
  static_assert(E % V == 0 && E % 8 == 0, "lane chunk must be whole vectors");
  const int lane = threadIdx.x & 31;
  const int part = lane % LPB;
  const int64_t n_warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t n_tiles = (a.n_blocks + BPW - 1) / BPW;
  int64_t tile = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  // The next tile's vectors are loaded before the current tile is encoded, so
  // each lane keeps two tiles of loads in flight.
  uint4 vn[NV];
  auto load_tile = [&](int64_t tl, uint4* dst) {
    const int64_t b = tl * BPW + lane / LPB;
    if (tl < n_tiles && b < a.n_blocks) {
      const char* src = static_cast<const char*>(a.x) + (b * B + (int64_t)part * E) * elem_bytes<DT>();
#pragma unroll
      for (int i = 0; i < NV; ++i) dst[i] = ldg16(src + 16 * i);
    }
  };
  // cast_ste: per-warp transpose area for coalesced float32 stores (8 warps)
  __shared__ __align__(16) float ste_stage[STE ? 8 * 32 * (E + 4) : 4];
  float* my_stage = ste_stage + (STE ? (threadIdx.x >> 5) * 32 * (E + 4) : 0);
  float* my_row = my_stage + (STE ? lane * (E + 4) : 0);
  load_tile(tile, vn);
  for (; tile < n_tiles; tile += n_warps) {
    const int64_t blk = tile * BPW + lane / LPB;
    const bool valid = blk < a.n_blocks;
    const int64_t e0 = blk * B + (int64_t)part * E;
    uint4 v[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = vn[i];
    load_tile(tile + n_warps, vn);
    float st0, st1;  // abs-max, or (min, max) for asymmetric INT4
    if constexpr (MODE == kInt4Asym) {
      st0 = __int_as_float(0x7F800000);
      st1 = -__int_as_float(0x7F800000);
    } else {
      st0 = 0.f;
      st1 = 0.f;
    }
    if (valid) {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        if constexpr (MODE == kInt4Asym) vec_minmax<DT>(v[i], st0, st1);
        else st0 = fmax_nan(st0, vec_absmax<DT>(v[i]));
      }
    }
#pragma unroll
    for (int o = 1; o < LPB; o <<= 1) {
      if constexpr (MODE == kInt4Asym) {
        st0 = fmin_nan(st0, __shfl_xor_sync(0xFFFFFFFFu, st0, o));
        st1 = fmax_nan(st1, __shfl_xor_sync(0xFFFFFFFFu, st1, o));
      } else {
        st0 = fmax_nan(st0, __shfl_xor_sync(0xFFFFFFFFu, st0, o));
      }
    }
    if (!valid && !STE) continue;
    if (valid) {
    float f[E];
#pragma unroll
    for (int i = 0; i < NV; ++i) unpack<DT>(v[i], f + i * V);

    float s, zp = 0.f;
    float dqs = 0.f, dqz = 0.f;  // stored scale / zero point (what dequantize uses)
    bool fast;
    if constexpr (MODE == kBlockFp8) {
      constexpr float kMax = FMT == BRC_FP8_E4M3 ? 448.f : 57344.f;
      s = div_const(fmax_nan(st0, 1e-10f), kMax, FMT == BRC_FP8_E4M3 ? kRcp448 : kRcp57344);
      if (!STE && part == 0) static_cast<float*>(a.scales)[blk] = canon_nan(s);
      dqs = s;
      fast = isfinite(s);
    } else if constexpr (MODE == kMxfp8) {
      constexpr float kMax = FMT == BRC_FP8_E4M3 ? 448.f : 57344.f;
      const float am = fmax_nan(st0, 1e-10f);
      const uint32_t e =
          e8m0_code(div_const(am, kMax, FMT == BRC_FP8_E4M3 ? kRcp448 : kRcp57344), g_e8m0_thr);
      dqs = e == 255 ? __int_as_float(0x7F800000) : exp2i((int)e - 127);
      if (!STE && part == 0) {
        static_cast<uint8_t*>(a.scales)[blk] = (uint8_t)e;
        if (a.scales_mma) {
          const uint32_t row = fdiv((uint32_t)blk, a.blocks_per_row);
          const uint32_t col = (uint32_t)blk - row * a.blocks_per_row.d;
          a.scales_mma[sf_mma_offset(row, col, a.sf_col_tiles)] = (uint8_t)e;
        }
      }
      fast = isfinite(am);
      // fast: multiply by 2^(127-e) (exact); slow: IEEE divide by 2^(e-127).
      s = fast ? exp2i(127 - (int)e)
               : (e == 255 ? __int_as_float(0x7F800000) : exp2i((int)e - 127));
    } else if constexpr (MODE == kNvfp4) {
      const float am = fmax_nan(st0, 1e-10f);
      const uint32_t sc = enc1_e4m3(div_const(am, 6.f, kRcp6));
      float actual = dec_e4m3(sc);
      dqs = actual;
      if (!(actual > 0.f)) actual = 0x1p-9f;  // np.where(actual > 0, actual, 2^-9)
      if (!STE && part == 0) {
        static_cast<uint8_t*>(a.scales)[blk] = (uint8_t)sc;
        if (a.scales_mma) {
          const uint32_t row = fdiv((uint32_t)blk, a.blocks_per_row);
          const uint32_t col = (uint32_t)blk - row * a.blocks_per_row.d;
          a.scales_mma[sf_mma_offset(row, col, a.sf_col_tiles)] = (uint8_t)sc;
        }
      }
      s = actual;
      fast = isfinite(am);
    } else if constexpr (MODE == kInt4Sym) {
      s = a.is_signed ? div_const(fmax_nan(st0, 1e-10f), 7.f, kRcp7)
                      : div_const(fmax_nan(st0, 1e-10f), 15.f, kRcp15);
      dqs = a.scale_f16 ? __half2float(__float2half_rn(s)) : s;
      if (!STE && part == 0) {
        if (a.scale_f16) static_cast<__half*>(a.scales)[blk] = to_half_canon(s);
        else static_cast<float*>(a.scales)[blk] = canon_nan(s);
      }
      fast = isfinite(s);
    } else {
      const float range = fmax_nan(__fsub_rn(st1, st0), 1e-10f);
      s = div_const(range, 15.f, kRcp15);
      const float zf = rintf(__fdiv_rn(-st0, s));
      // np.clip keeps the operand (including -0.0 and NaN) when it is in range
      zp = zf < 0.f ? 0.f : (zf > 15.f ? 15.f : zf);
      dqs = a.scale_f16 ? __half2float(__float2half_rn(s)) : s;
      dqz = a.scale_f16 ? __half2float(__float2half_rn(zp)) : zp;
      if (!STE && part == 0) {
        if (a.scale_f16) {
          static_cast<__half*>(a.scales)[blk] = to_half_canon(s);
          static_cast<__half*>(a.zp)[blk] = to_half_canon(zp);
        } else {
          static_cast<float*>(a.scales)[blk] = canon_nan(s);
          static_cast<float*>(a.zp)[blk] = canon_nan(zp);
        }
      }
      fast = isfinite(s) && isfinite(zp);
    }
    int64_t tile_off = 0;
    if constexpr (!STE && (MODE == kInt4Sym || MODE == kInt4Asym)) {
      if (a.packed_tiles) {
        // tile (row / 16, group) of 16 rows x 64 bytes; per tile 16 fp32
        // scales (the stored value) and, asymmetric, 16 fp32 values 128 + the
        // stored zero point, tile row r at 2 * (r % 8) + r / 8, so that one
        // 8-byte load gives an MMA thread its rows r and r + 8
        const uint32_t row = fdiv((uint32_t)blk, a.blocks_per_row);
        const uint32_t g = (uint32_t)blk - row * a.blocks_per_row.d;
        const int64_t tile = (int64_t)(row >> 4) * a.blocks_per_row.d + g;
        tile_off = tile * 1024 + (row & 15) * 64 + (part * E) / 2;
        if (part == 0) {
          const int64_t q = tile * 16 + (row & 7) * 2 + ((row >> 3) & 1);
          const float sv = a.scale_f16 ? __half2float(to_half_canon(s)) : canon_nan(s);
          a.scale_tiles[q] = sv;
          if constexpr (MODE == kInt4Asym) {
            const float zv = a.scale_f16 ? __half2float(to_half_canon(zp)) : canon_nan(zp);
            a.zp_tiles[q] = __fadd_rn(128.f, zv);
          }
        }
      }
    }
    encode_lane<MODE, FMT, E, STE>(a, e0, f, s, zp, fast, tile_off, dqs, dqz, my_row);
    }  // valid
    if constexpr (STE) ste_warp_store<E>(a, tile * BPW * B, a.n_blocks * B, my_stage);
  }
}

// Generic fallback: one thread per block, any block size, scalar loads.
template <int DT>
__device__ __forceinline__ float load1(const void* x, int64_t i) {
  if constexpr (DT == BRC_DTYPE_F32) return static_cast<const float*>(x)[i];
  else if constexpr (DT == BRC_DTYPE_BF16)
    return __uint_as_float((uint32_t)static_cast<const uint16_t*>(x)[i] << 16);
  else return __half2float(static_cast<const __half*>(x)[i]);
}

template <int DT, int MODE, int FMT>
__global__ void __launch_bounds__(256) k_block_cast_generic(BlockCastArgs a, int B) {
  for (int64_t blk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; blk < a.n_blocks;
       blk += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e0 = blk * B;
    float amax = 0.f, mn = __int_as_float(0x7F800000), mx = -__int_as_float(0x7F800000);
    for (int i = 0; i < B; ++i) {
      const float v = load1<DT>(a.x, e0 + i);
      amax = fmax_nan(amax, fabsf(v));
      mn = fmin_nan(mn, v);
      mx = fmax_nan(mx, v);
    }
    float s, zp = 0.f;
    if constexpr (MODE == kBlockFp8) {
      constexpr float kMax = FMT == BRC_FP8_E4M3 ? 448.f : 57344.f;
      s = __fdiv_rn(fmax_nan(amax, 1e-10f), kMax);
      static_cast<float*>(a.scales)[blk] = canon_nan(s);
      for (int i = 0; i < B; ++i)
        a.codes[e0 + i] = (uint8_t)enc1_fp8<FMT>(div_ieee(load1<DT>(a.x, e0 + i), s));
    } else if constexpr (MODE == kInt4Sym || MODE == kInt4Asym) {
      if constexpr (MODE == kInt4Sym) {
        s = __fdiv_rn(fmax_nan(amax, 1e-10f), a.is_signed ? 7.f : 15.f);
      } else {
        s = __fdiv_rn(fmax_nan(__fsub_rn(mx, mn), 1e-10f), 15.f);
        const float zf = rintf(__fdiv_rn(-mn, s));
        zp = zf < 0.f ? 0.f : (zf > 15.f ? 15.f : zf);
      }
      if (a.scale_f16) static_cast<__half*>(a.scales)[blk] = to_half_canon(s);
      else static_cast<float*>(a.scales)[blk] = canon_nan(s);
      if constexpr (MODE == kInt4Asym) {
        if (a.scale_f16) static_cast<__half*>(a.zp)[blk] = to_half_canon(zp);
        else static_cast<float*>(a.zp)[blk] = canon_nan(zp);
      }
      const float lo = (MODE == kInt4Sym && a.is_signed) ? -8.f : 0.f;
      const float hi = (MODE == kInt4Sym && a.is_signed) ? 7.f : 15.f;
      for (int i = 0; i < B; ++i) {
        float q = div_ieee(load1<DT>(a.x, e0 + i), s);
        if constexpr (MODE == kInt4Asym) q = __fadd_rn(q, zp);
        const uint32_t code =
            isnan(q) ? 0u : (__float_as_uint(__fadd_rn(fminf(fmaxf(q, lo), hi), 12582912.f)) & 0xFu);
        if (a.codes) a.codes[e0 + i] = (uint8_t)code;
        if (a.packed) {
          // only reached with even B: element pairs never straddle blocks
          uint8_t* p = a.packed + (e0 + i) / 2;
          if (((e0 + i) & 1) == 0) *p = (uint8_t)code;
          else *p = (uint8_t)(*p | (code << 4));
        }
      }
    }
  }
}

// --------------------------------------------------------------- per-tensor
template <int DT>
__global__ void __launch_bounds__(256) k_amax(const void* __restrict__ x, int64_t n,
                                              uint32_t* amax_bits) {
  constexpr int V = In<DT>::kVec;
  const int64_t nvec = n / V;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  float m = 0.f;
  const char* base = static_cast<const char*>(x);
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < nvec; i += 4 * stride) {
    const uint4 v0 = ldg16(base + 16 * i);
    const uint4 v1 = ldg16(base + 16 * (i + stride));
    const uint4 v2 = ldg16(base + 16 * (i + 2 * stride));
    const uint4 v3 = ldg16(base + 16 * (i + 3 * stride));
    m = fmax_nan(m, fmax_nan(fmax_nan(vec_absmax<DT>(v0), vec_absmax<DT>(v1)),
                             fmax_nan(vec_absmax<DT>(v2), vec_absmax<DT>(v3))));
  }
  for (; i < nvec; i += stride) m = fmax_nan(m, vec_absmax<DT>(ldg16(base + 16 * i)));
  for (int64_t t = nvec * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += stride)
    m = fmax_nan(m, fabsf(load1<DT>(x, t)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmax_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) m = fmax_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (threadIdx.x == 0 && __float_as_uint(m) != 0u) atomicMax(amax_bits, __float_as_uint(m));
  }
}

__global__ void k_amax_reset(uint32_t* amax_bits) { *amax_bits = 0u; }

// scale = float32(max(float64(amax), 1e-10) / fmt_max), as
// src/breccia/kernels/reference/cast.py:368-370 computes it in float64.
// For amax >= 1e-10 this equals float32 division (double rounding through
// float64 is innocuous for division); below the floor it is the constant
// float32(1e-10 / fmt_max) computed on the host.
__device__ __forceinline__ float pertensor_scale(uint32_t bits, float fmt_max, float floor_scale) {
  const float amax = __uint_as_float(bits);
  if (isnan(amax)) return amax;
  if ((double)amax < 1e-10) return floor_scale;
  return __fdiv_rn(amax, fmt_max);
}

// cast_ste value of one element: x + (dequantize(code) - x) in float32.
template <int FMT>
__device__ __forceinline__ float ste1(float x, uint32_t code, float scale) {
  return __fadd_rn(x, __fsub_rn(__fmul_rn(dec_fp8<FMT>(code), scale), x));
}

template <int DT, int FMT, bool STE = false>
__global__ void __launch_bounds__(256) k_pertensor_apply(const void* __restrict__ x, int64_t n,
                                                         const uint32_t* amax_bits,
                                                         float floor_scale, uint8_t* codes,
                                                         float* scale_out, float* ste_out) {
  constexpr int V = In<DT>::kVec;
  constexpr float kMax = FMT == BRC_FP8_E4M3 ? 448.f : 57344.f;
  const float s = pertensor_scale(*amax_bits, kMax, floor_scale);
  if (!STE && blockIdx.x == 0 && threadIdx.x == 0) *scale_out = canon_nan(s);
  const bool fast = isfinite(s);
  const float r = __frcp_rn(s);
  const int64_t nvec = n / V;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const char* base = static_cast<const char*>(x);
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (fast) {
    // Vectors are visited from the end of the tensor backwards: the amax
    // pass that ran just before read it front to back, so its tail is still
    // in L2 and is consumed first. Input lines are read here for the last
    // time and the codes are not read back by this kernel, so both carry an
    // evict-first policy and leave the cached tail in place.
    const uint64_t pol = l2_evict_first_policy();
    auto encode_store = [&](const uint4 v, int64_t vi) {
      float f0[V];
      unpack<DT>(v, f0);
      uint32_t w0[V / 4];
#pragma unroll
      for (int j = 0; j < V / 4; ++j)
        w0[j] = enc4_fp8<FMT>(div_by(f0[4 * j], s, r), div_by(f0[4 * j + 1], s, r),
                              div_by(f0[4 * j + 2], s, r), div_by(f0[4 * j + 3], s, r));
      if constexpr (STE) {
#pragma unroll
        for (int j = 0; j < V / 4; ++j) {
          // the fast path's codes are finite: decode them by the hardware pair
          // conversions (exact), then ste1's arithmetic
          float o[4], d[4];
          f16x2_to_f32(fp8x2_to_f16x2<FMT>(w0[j]), d[0], d[1]);
          f16x2_to_f32(fp8x2_to_f16x2<FMT>(w0[j] >> 16), d[2], d[3]);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            o[q] = __fadd_rn(f0[4 * j + q], __fsub_rn(__fmul_rn(d[q], s), f0[4 * j + q]));
          stg16(ste_out + vi * V + 4 * j, make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]),
                                                      __float_as_uint(o[2]), __float_as_uint(o[3])));
        }
      } else if constexpr (V == 8) {
        stg8_last_use(codes + vi * V, w0[0], w0[1], pol);
      } else {
        *reinterpret_cast<uint32_t*>(codes + vi * V) = w0[0];
      }
    };
    // four 16-byte vectors in flight per thread per iteration
    for (; i + 3 * stride < nvec; i += 4 * stride) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = ldg16_last_use(base + 16 * (nvec - 1 - (i + u * stride)), pol);
#pragma unroll
      for (int u = 0; u < 4; ++u) encode_store(v[u], nvec - 1 - (i + u * stride));
    }
    for (; i < nvec; i += stride)
      encode_store(ldg16_last_use(base + 16 * (nvec - 1 - i), pol), nvec - 1 - i);
  } else {
    for (; i < nvec; i += stride) {
      float f0[V];
      unpack<DT>(ldg16(base + 16 * i), f0);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const uint32_t c = enc1_fp8<FMT>(div_ieee(f0[j], s));
        if constexpr (STE) ste_out[i * V + j] = ste1<FMT>(f0[j], c, s);
        else codes[i * V + j] = (uint8_t)c;
      }
    }
  }
  for (int64_t t = nvec * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += stride) {
    const float xv = load1<DT>(x, t);
    const uint32_t c = enc1_fp8<FMT>(div_ieee(xv, s));
    if constexpr (STE) ste_out[t] = ste1<FMT>(xv, c, s);
    else codes[t] = (uint8_t)c;
  }
}

// --------------------------------------------------------------- 2-D tiles
// One CTA per (block_m x block_k) tile; the tile's vectors stay in registers
// between the amax pass and the encode pass. VPR > 0 fixes the vectors per
// tile row at compile time (block_k = 128), so a vector's row and column are
// a shift and a mask rather than a runtime division.
template <int DT, int FMT, int MAXV, int VPR>
__global__ void __launch_bounds__(256) k_block2d_cast(const void* __restrict__ x, int64_t cols,
                                                      int bm, int bk, uint8_t* codes,
                                                      float* scales) {
  constexpr int V = In<DT>::kVec;
  constexpr float kMax = FMT == BRC_FP8_E4M3 ? 448.f : 57344.f;
  const int vec_per_row = VPR > 0 ? VPR : bk / V;
  const int nvec = bm * vec_per_row;
  const int64_t r0 = (int64_t)blockIdx.y * bm, c0 = (int64_t)blockIdx.x * bk;
  // vector idx = threadIdx.x + k * 256 sits at tile row idx / vpr, column
  // (idx % vpr) * V; with a compile-time vpr dividing 256 the column is fixed
  // per thread and the row advances by 256 / vpr per k.
  auto offset = [&](int k) -> int64_t {
    const int idx = threadIdx.x + k * 256;
    const int rr = idx / vec_per_row, cc = (idx % vec_per_row) * V;
    return (r0 + rr) * cols + c0 + cc;
  };
  const char* xb = static_cast<const char*>(x);
  uint4 v[MAXV];
  float m = 0.f;
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    if (threadIdx.x + k * 256 < nvec) {
      v[k] = ldg16(xb + offset(k) * elem_bytes<DT>());
      m = fmax_nan(m, vec_absmax<DT>(v[k]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmax_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  __shared__ float red[8];
  __shared__ float s_sh;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t = fmax_nan(t, red[w]);
    const float s = __fdiv_rn(fmax_nan(t, 1e-10f), kMax);
    s_sh = s;
    scales[(int64_t)blockIdx.y * gridDim.x + blockIdx.x] = canon_nan(s);
  }
  __syncthreads();
  const float s = s_sh;
  const float r = __frcp_rn(s);
  if (isfinite(s)) {
#pragma unroll
    for (int k = 0; k < MAXV; ++k) {
      if (threadIdx.x + k * 256 < nvec) {
        float f[V];
        unpack<DT>(v[k], f);
        uint32_t w[V / 4];
#pragma unroll
        for (int j = 0; j < V / 4; ++j)
          w[j] = enc4_div<enc4p_fp8<FMT>>(f + 4 * j, s, r);
        store_words<V / 4>(codes + offset(k), w);
      }
    }
  } else {
    for (int k = 0; k < MAXV; ++k) {
      if (threadIdx.x + k * 256 < nvec) {
        float f[V];
        unpack<DT>(v[k], f);
        uint32_t w[V / 4];
        for (int j = 0; j < V / 4; ++j) {
          uint32_t c = 0;
          for (int i = 0; i < 4; ++i) c |= enc1_fp8<FMT>(div_ieee(f[4 * j + i], s)) << (8 * i);
          w[j] = c;
        }
        store_words<V / 4>(codes + offset(k), w);
      }
    }
  }
}

// Persistent, TMA-fed form for 128-wide tiles: each (bm x 128) tile arrives
// in one 2-D tensor copy into a ring of shared-memory stages; the threads copy
// it into registers, the stage is refilled at once, and the tile's amax
// reduction and encode run from registers while the next tiles stream in.
// Every wait is bounded; a timeout is decided for the whole CTA through
// __syncthreads_or, the status word records it and the CTA stops after
// waiting for its own copies in flight.
constexpr int kB2dThreads = 512;

template <int DT, int FMT, int NV>  // NV = 16-byte vectors per thread per tile (bm <= 128)
__global__ void __launch_bounds__(kB2dThreads, 1)
    k_block2d_cast_tma(const __grid_constant__ CUtensorMap tm, int64_t rows, int64_t cols, int bm,
                       int stages, uint8_t* codes, float* scales, uint32_t* status) {
  using namespace sm100;
  constexpr int V = In<DT>::kVec;
  constexpr int VPR = 128 / V;  // vectors per tile row
  constexpr float kMax = FMT == BRC_FP8_E4M3 ? 448.f : 57344.f;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tile_bytes = bm * 128 * elem_bytes<DT>();
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)stages * tile_bytes);
  // per-warp maxima, two sets used by alternate tiles
  float* red = reinterpret_cast<float*>(full + stages);
  volatile uint32_t* abort_flag =
      reinterpret_cast<volatile uint32_t*>(red + 2 * (kB2dThreads / 32));
  const int64_t tiles_c = cols / 128;
  const int64_t ntiles = tiles_c * (rows / bm);
  const int nvec = bm * VPR;
  const int64_t my_tiles =
      ntiles > (int64_t)blockIdx.x ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    *abort_flag = 0u;
    fence_mbar_init();
  }
  __syncthreads();
  int64_t issued = 0;  // thread 0: tiles whose copy has been issued
  auto issue = [&]() {
    const int64_t t = blockIdx.x + issued * gridDim.x;
    const int s = (int)(issued % stages);
    mbar_arrive_expect_tx(&full[s], (uint32_t)tile_bytes);
    tma_load_2d(smem + (size_t)s * tile_bytes, &tm, (int32_t)((t % tiles_c) * 128),
                (int32_t)((t / tiles_c) * bm), &full[s]);
    ++issued;
  };
  if (threadIdx.x == 0)
    while (issued < stages && issued < my_tiles) issue();

  bool aborted = false;
  for (int64_t j = 0; j < my_tiles; ++j) {
    const int s = (int)(j % stages);
    const bool ok = mbar_wait(&full[s], (uint32_t)((j / stages) & 1), abort_flag, status, 1u);
    uint4 v[NV];
    float m = 0.f;
    if (ok) {
      const uint8_t* tile = smem + (size_t)s * tile_bytes;
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int idx = threadIdx.x + k * kB2dThreads;
        if (idx < nvec) {
          v[k] = *reinterpret_cast<const uint4*>(tile + (size_t)idx * 16);
          m = fmax_nan(m, vec_absmax<DT>(v[k]));
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmax_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    float* red_j = red + (j & 1) * (kB2dThreads / 32);
    if ((threadIdx.x & 31) == 0) red_j[threadIdx.x >> 5] = m;
    if (__syncthreads_or(!ok)) {  // also: every thread has read stage s
      aborted = true;
      break;
    }
    const int64_t t = blockIdx.x + j * gridDim.x;
    if (threadIdx.x == 0 && issued < my_tiles && !*abort_flag) issue();
    // Every thread reduces the per-warp maxima itself (the max is
    // order-independent, NaN included), so no second barrier waits on one
    // thread. A set is rewritten two tiles later, after a barrier that every
    // thread reaches only once it has read the set.
    float a = red_j[0];
#pragma unroll
    for (int w = 1; w < kB2dThreads / 32; ++w) a = fmax_nan(a, red_j[w]);
    const float sc = __fdiv_rn(fmax_nan(a, 1e-10f), kMax);
    if (threadIdx.x == 0) scales[t] = canon_nan(sc);
    const float r = __frcp_rn(sc);
    uint8_t* cbase = codes + (t / tiles_c) * bm * cols + (t % tiles_c) * 128;
    if (isfinite(sc)) {
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const int idx = threadIdx.x + k * kB2dThreads;
        if (idx < nvec) {
          float f[V];
          unpack<DT>(v[k], f);
          uint32_t w[V / 4];
#pragma unroll
          for (int q = 0; q < V / 4; ++q)
            w[q] = enc4_div<enc4p_fp8<FMT>>(f + 4 * q, sc, r);
          store_words<V / 4>(cbase + (int64_t)(idx / VPR) * cols + (idx % VPR) * V, w);
        }
      }
    } else {
      for (int k = 0; k < NV; ++k) {
        const int idx = threadIdx.x + k * kB2dThreads;
        if (idx < nvec) {
          float f[V];
          unpack<DT>(v[k], f);
          uint32_t w[V / 4];
          for (int q = 0; q < V / 4; ++q) {
            uint32_t c = 0;
            for (int i = 0; i < 4; ++i) c |= enc1_fp8<FMT>(div_ieee(f[4 * q + i], sc)) << (8 * i);
            w[q] = c;
          }
          store_words<V / 4>(cbase + (int64_t)(idx / VPR) * cols + (idx % VPR) * V, w);
        }
      }
    }
  }
  if (aborted && threadIdx.x == 0) {
    // wait (bounded) for the copies still in flight before the CTA exits
    for (int64_t q = issued > stages ? issued - stages : 0; q < issued; ++q) {
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(&full[q % stages], (uint32_t)((q / stages) & 1)) &&
             globaltimer() - t0 < kWaitLimitNs) {
      }
    }
  }
}

// --------------------------------------------------------------- dequantize
// 16 codes per lane-iteration; out = decode(code) * scale.
enum DqMode { kDqFp8 = 0, kDqMx = 1, kDqNv = 2, kDqInt4 = 3 };

struct DequantArgs {
  const uint8_t* codes;
  const void* scales;
  const void* zp;
  void* out;
  int64_t n;           // elements
  int64_t cols;
  int block_k;         // scale run along the last axis (must be a multiple of 16)
  int block_m;         // rows per scale (2-D block FP8), else 1
  int64_t scale_cols;  // cols / block_k
  int per_tensor;
  int is_signed;
  int scale_f16;
};

template <int OUT>
__device__ __forceinline__ void store_out16(void* out, int64_t e0, const float* v) {
  if constexpr (OUT == BRC_DTYPE_F32) {
    float* o = static_cast<float*>(out) + e0;
#pragma unroll
    for (int i = 0; i < 16; i += 4)
      stg16(o + i, make_uint4(__float_as_uint(v[i]), __float_as_uint(v[i + 1]),
                              __float_as_uint(v[i + 2]), __float_as_uint(v[i + 3])));
  } else {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if constexpr (OUT == BRC_DTYPE_BF16) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    char* o = static_cast<char*>(out) + e0 * 2;
    stg16(o, make_uint4(w[0], w[1], w[2], w[3]));
    stg16(o + 16, make_uint4(w[4], w[5], w[6], w[7]));
  }
}

__device__ __forceinline__ uint32_t ldg4(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ void stg8(void* p, uint32_t a, uint32_t b) {
  asm volatile("st.global.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}

// 16 codes (one 16-byte word group) -> 16 decoded float32 values.
template <int DQ, int FMT>
__device__ __forceinline__ void decode4(uint32_t w, float (&v)[4], int is_signed, bool has_zp,
                                        float zp) {
  if constexpr (DQ == kDqFp8 || DQ == kDqMx) {
    f16x2_to_f32(fp8x2_to_f16x2<FMT>(w), v[0], v[1]);
    f16x2_to_f32(fp8x2_to_f16x2<FMT>(w >> 16), v[2], v[3]);
  } else if constexpr (DQ == kDqNv) {
    f16x2_to_f32(e2m1_bytes_to_f16x2(w), v[0], v[1]);
    f16x2_to_f32(e2m1_bytes_to_f16x2(w >> 16), v[2], v[3]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = (w >> (8 * i)) & 0xFu;
      float d = (is_signed && lo >= 8) ? (float)((int)lo - 16) : (float)lo;
      if (has_zp) d = __fsub_rn(d, zp);
      v[i] = d;
    }
  }
}
template <int DQ, int FMT>
__device__ __forceinline__ void decode16(const uint32_t (&w)[4], float (&v)[16], int is_signed,
                                         bool has_zp, float zp) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float q[4];
    decode4<DQ, FMT>(w[j], q, is_signed, has_zp, zp);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[4 * j + i] = q[i];
  }
}

// Scale (and zero point) of the 16-code chunk `c`.
template <int DQ>
__device__ __forceinline__ float chunk_scale(const DequantArgs& a, uint32_t c, const FastDiv& cpr,
                                             const FastDiv& bm, const FastDiv& cpb, float& zp,
                                             bool& has_zp) {
  const uint32_t row = fdiv(c, cpr);
  const uint32_t cin = c - row * cpr.d;  // chunk within the row
  const int64_t si = (int64_t)fdiv(row, bm) * a.scale_cols + fdiv(cin, cpb);
  if constexpr (DQ == kDqFp8) {
    return static_cast<const float*>(a.scales)[si];
  } else if constexpr (DQ == kDqMx) {
    const uint32_t e = static_cast<const uint8_t*>(a.scales)[si];
    return e == 255 ? __int_as_float(0x7F800000) : exp2i((int)e - 127);
  } else if constexpr (DQ == kDqNv) {
    return dec_e4m3(static_cast<const uint8_t*>(a.scales)[si]);
  } else {
    has_zp = a.zp != nullptr;
    if (a.scale_f16) {
      if (has_zp) zp = __half2float(static_cast<const __half*>(a.zp)[si]);
      return __half2float(static_cast<const __half*>(a.scales)[si]);
    }
    if (has_zp) zp = static_cast<const float*>(a.zp)[si];
    return static_cast<const float*>(a.scales)[si];
  }
}

// A warp walks spans of 512 codes; in each, lane t takes codes 4t..4t+3 of
// every 128-code quarter, so each warp-wide 4-byte load reads 128
// contiguous bytes and each store writes 512 (float32) or 256 (bf16/f16)
// contiguous bytes. The chunk's row and scale index come from 32-bit
// multiply-shift divisions (chunks per row, block height, chunks per block).
template <int DQ, int FMT, int OUT>
__global__ void __launch_bounds__(256) k_dequant(DequantArgs a, FastDiv cpr, FastDiv bm,
                                                 FastDiv cpb) {
  const uint32_t ngroups = (uint32_t)(a.n / 4);  // 4-code groups (n % 16 == 0)
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t nwarps = gridDim.x * (blockDim.x >> 5);
  float pscale = 0.f;
  if constexpr (DQ == kDqFp8) {
    if (a.per_tensor) pscale = *static_cast<const float*>(a.scales);
  }
  for (uint32_t span = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
       (uint64_t)span * 128 < ngroups; span += nwarps) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t g = span * 128 + 32 * j + lane;
      w[j] = g < ngroups ? ldg4(a.codes + (int64_t)g * 4) : 0u;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t g = span * 128 + 32 * j + lane;
      if (g >= ngroups) break;
      float zp = 0.f;
      bool has_zp = false;
      float scale = pscale;
      if (!(DQ == kDqFp8 && a.per_tensor)) scale = chunk_scale<DQ>(a, g >> 2, cpr, bm, cpb, zp, has_zp);
      float v[4];
      decode4<DQ, FMT>(w[j], v, a.is_signed, has_zp, zp);
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(v[i], scale);
      if constexpr (OUT == BRC_DTYPE_F32) {
        stg16(static_cast<float*>(a.out) + (int64_t)g * 4,
              make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                         __float_as_uint(v[3])));
      } else {
        uint32_t h0, h1;
        if constexpr (OUT == BRC_DTYPE_BF16) {
          const __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0], v[1]);
          const __nv_bfloat162 p1 = __floats2bfloat162_rn(v[2], v[3]);
          h0 = *reinterpret_cast<const uint32_t*>(&p0);
          h1 = *reinterpret_cast<const uint32_t*>(&p1);
        } else {
          const __half2 p0 = __floats2half2_rn(v[0], v[1]);
          const __half2 p1 = __floats2half2_rn(v[2], v[3]);
          h0 = *reinterpret_cast<const uint32_t*>(&p0);
          h1 = *reinterpret_cast<const uint32_t*>(&p1);
        }
        stg8(static_cast<char*>(a.out) + (int64_t)g * 8, h0, h1);
      }
    }
  }
}

// Tensors of 2^31 chunks (2^35 elements) or more: 64-bit indices.
template <int DQ, int FMT, int OUT>
__global__ void __launch_bounds__(256) k_dequant_wide(DequantArgs a) {
  const int64_t nchunks = a.n / 16;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < nchunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e0 = c * 16;
    const uint4 cv = ldg16(a.codes + e0);
    float scale = 0.f, zp = 0.f;
    bool has_zp = false;
    if (a.per_tensor) {
      scale = *static_cast<const float*>(a.scales);
    } else {
      const int64_t row = e0 / a.cols, col = e0 - row * a.cols;
      const int64_t si = (row / a.block_m) * a.scale_cols + col / a.block_k;
      if constexpr (DQ == kDqFp8) scale = static_cast<const float*>(a.scales)[si];
      else if constexpr (DQ == kDqMx) {
        const uint32_t e = static_cast<const uint8_t*>(a.scales)[si];
        scale = e == 255 ? __int_as_float(0x7F800000) : exp2i((int)e - 127);
      } else if constexpr (DQ == kDqNv) {
        scale = dec_e4m3(static_cast<const uint8_t*>(a.scales)[si]);
      } else {
        if (a.scale_f16) {
          scale = __half2float(static_cast<const __half*>(a.scales)[si]);
          if (a.zp) zp = __half2float(static_cast<const __half*>(a.zp)[si]);
        } else {
          scale = static_cast<const float*>(a.scales)[si];
          if (a.zp) zp = static_cast<const float*>(a.zp)[si];
        }
        has_zp = a.zp != nullptr;
      }
    }
    const uint32_t w[4] = {cv.x, cv.y, cv.z, cv.w};
    float v[16];
    decode16<DQ, FMT>(w, v, a.is_signed, has_zp, zp);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __fmul_rn(v[i], scale);
    store_out16<OUT>(a.out, e0, v);
  }
}

// --------------------------------------------------------------- requantize
// NVFP4 (unpacked codes + E4M3 scales) -> MXFP8, one lane per 32-element
// MXFP8 block. Every dequantized value e2m1 * e4m3 has at most 6 significant
// bits and lies in [2^-10, 2688], so it is exact in float16: codes are
// converted two at a time by the hardware (cvt e2m1x2 -> f16x2), multiplied by
// the f16 scale and reduced in packed form, and widened to float32 only for
// the E4M3 encode. The result equals cast(dequantize(st), MXFP8BlockScaling(fmt)).
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t pair_byte) {
  uint32_t d;
  asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
      : "=r"(d)
      : "r"(pair_byte));
  return d;
}
__device__ __forceinline__ uint32_t e4m3_to_f16x2_bcast(uint32_t code) {
  uint32_t d;
  const uint16_t two = (uint16_t)(code | (code << 8));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(two));
  return d;
}
__device__ __forceinline__ uint32_t h2mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t h2min(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// 2^k in both halves of an f16x2 (k in [-14, 15], a normal f16).
__device__ __forceinline__ uint32_t f16x2_pow2(int k) {
  const uint32_t h = (uint32_t)(k + 15) << 10;
  return h | (h << 16);
}

// Four MXFP8 codes of four f16 values (h0 = elements 0, 1; h1 = elements 2, 3)
// that are scaled by m1 * m2 (powers of two) before encoding. The f16 values
// are exact products, and so are their scaled values wherever these reach the
// format's first midpoint (see k_requant_nv_to_mx). As the float32 encoders
// do with float32 bits, the code is read off the scaled f16 bits: E4M3 scales
// carry an extra 2^-8 that puts E4M3's smallest normal (2^-6) on f16's
// (2^-14), E5M2's smallest normal is f16's; clamp to the format maximum
// (np.clip; an f16 overflow to inf clamps too), add half-1 below the code bits
// and truncate (ties toward zero). A zero magnitude drops its sign.
template <int FMT>
__device__ __forceinline__ uint32_t enc4_fp8_from_f16x2(uint32_t h0, uint32_t h1, uint32_t m1,
                                                        uint32_t m2, bool two_steps) {
  constexpr uint32_t kMaxH = FMT == BRC_FP8_E4M3 ? 0x3F003F00u    // 448 * 2^-8 = 1.75
                                                 : 0x7B007B00u;   // 57344
  constexpr uint32_t kRnd = FMT == BRC_FP8_E4M3 ? 0x003F003Fu : 0x007F007Fu;
  constexpr int kDrop = FMT == BRC_FP8_E4M3 ? 7 : 8;  // f16 mantissa bits below the code
  uint32_t v0 = h2mul(h0 & 0x7FFF7FFFu, m1), v1 = h2mul(h1 & 0x7FFF7FFFu, m1);
  if (two_steps) {
    v0 = h2mul(v0, m2);
    v1 = h2mul(v1, m2);
  }
  v0 = h2min(v0, kMaxH);
  v1 = h2min(v1, kMaxH);
  const uint32_t c0 = ((v0 + kRnd) >> kDrop) & 0x007F007Fu;  // codes in bytes 0 and 2
  const uint32_t c1 = ((v1 + kRnd) >> kDrop) & 0x007F007Fu;
  const uint32_t w = prmt(c0, c1, 0x6420u);
  const uint32_t neg = prmt(h0, h1, 0xFDB9u);  // sign of each f16 replicated into its byte
  return apply_sign8(w, neg);
}

// One thread per 32-element block. The next block's 34 input bytes are loaded
// before the current block is encoded, so two blocks' loads are in flight per
// thread (4 CTAs of 256 threads per SM: about 70 KB per SM).
template <int FMT>
__global__ void __launch_bounds__(256, 4) k_requant_nv_to_mx(const uint8_t* __restrict__ codes,
                                                             const uint8_t* __restrict__ scales,
                                                             int64_t n_blocks, FastDiv bpr,
                                                             uint32_t sf_col_tiles, uint8_t* out,
                                                             uint8_t* out_scales,
                                                             uint8_t* out_mma) {
  constexpr float kMax = FMT == BRC_FP8_E4M3 ? 448.f : 57344.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t blk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint4 n0 = make_uint4(0u, 0u, 0u, 0u), n1 = n0;
  uint8_t ns0 = 0, ns1 = 0;
  if (blk < n_blocks) {
    n0 = ldg16(codes + blk * 32);
    n1 = ldg16(codes + blk * 32 + 16);
    ns0 = scales[2 * blk];
    ns1 = scales[2 * blk + 1];
  }
  for (; blk < n_blocks; blk += stride) {
    const uint4 c0 = n0, c1 = n1;
    const uint32_t hs0 = e4m3_to_f16x2_bcast(ns0);
    const uint32_t hs1 = e4m3_to_f16x2_bcast(ns1);
    if (blk + stride < n_blocks) {
      const int64_t nxt = blk + stride;
      n0 = ldg16(codes + nxt * 32);
      n1 = ldg16(codes + nxt * 32 + 16);
      ns0 = scales[2 * nxt];
      ns1 = scales[2 * nxt + 1];
    }
    const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    uint32_t h[16];  // f16x2 values (element 2i low, 2i+1 high)
    uint32_t amax2 = 0u;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // codes are one per byte: byte (b0 | b1 << 4) holds the pair, low nibble first
      const uint32_t lo = (w[i] & 0x0Fu) | ((w[i] >> 4) & 0xF0u);
      const uint32_t hi = ((w[i] >> 16) & 0x0Fu) | ((w[i] >> 20) & 0xF0u);
      const uint32_t sc = i < 4 ? hs0 : hs1;
      h[2 * i] = h2mul(e2m1x2_to_f16x2(lo), sc);
      h[2 * i + 1] = h2mul(e2m1x2_to_f16x2(hi), sc);
      amax2 = f16x2_max_nan(amax2, f16x2_max_nan(h[2 * i] & 0x7FFF7FFFu, h[2 * i + 1] & 0x7FFF7FFFu));
    }
    const __half2 am2 = *reinterpret_cast<const __half2*>(&amax2);
    float am = fmax_nan(__low2float(am2), __high2float(am2));
    am = fmax_nan(am, 1e-10f);
    const uint32_t e = e8m0_code(__fdiv_rn(am, kMax), g_e8m0_thr);
    out_scales[blk] = (uint8_t)e;
    if (out_mma) {
      const uint32_t row = fdiv((uint32_t)blk, bpr);
      out_mma[sf_mma_offset(row, (uint32_t)blk - row * bpr.d, sf_col_tiles)] = (uint8_t)e;
    }
    uint32_t o[8];
    if (isfinite(am)) {
      // Exactness of the f16 route. Each product y = decode(code) * decode(scale)
      // has at most 6 significant bits and is 0 or lies in [2^-10, 2688], so the
      // f16 h[] hold y exactly. The scaled value y * 2^(127 - e) (* 2^-8 for
      // E4M3) is exact wherever it is at least the format's first midpoint (f16
      // subnormals step by 2^-24, which 6 bits from 2^-18 up never need), and
      // below that midpoint the code is 0 however it rounds. 2^k is applied in
      // at most two steps of f16 powers of two (E4M3: k in [-11, 11]; E5M2: k in
      // [0, 26]); a value that overflows f16 lies above the format maximum and
      // clamps to it, as np.clip does.
      // (a block whose products are all 0 has am at the 1e-10 floor and a larger
      // k; its codes are 0 under any finite multiplier, so k is capped at 30)
      const int k = min(127 - (int)e - (FMT == BRC_FP8_E4M3 ? 8 : 0), 30);
      const int k1 = k > 15 ? 15 : k;
      const uint32_t m1 = f16x2_pow2(k1), m2 = f16x2_pow2(k - k1);
      const bool two = k != k1;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        o[j] = enc4_fp8_from_f16x2<FMT>(h[2 * j], h[2 * j + 1], m1, m2, two);
    } else {
      float f[32];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const __half2 v = *reinterpret_cast<const __half2*>(&h[i]);
        f[2 * i] = __low2float(v);
        f[2 * i + 1] = __high2float(v);
      }
      const float act = e == 255 ? __int_as_float(0x7F800000) : exp2i((int)e - 127);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t c = 0;
        for (int i = 0; i < 4; ++i) c |= enc1_fp8<FMT>(div_ieee(f[4 * j + i], act)) << (8 * i);
        o[j] = c;
      }
    }
    stg16(out + blk * 32, make_uint4(o[0], o[1], o[2], o[3]));
    stg16(out + blk * 32 + 16, make_uint4(o[4], o[5], o[6], o[7]));
  }
}

}  // namespace brc

// ========================================================================
// Host side: argument checks, launch configuration, C ABI.
// ========================================================================
using namespace brc;

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool valid_dtype(int dt) { return dt == BRC_DTYPE_F32 || dt == BRC_DTYPE_BF16 || dt == BRC_DTYPE_F16; }
bool valid_fmt(int f) { return f == BRC_FP8_E4M3 || f == BRC_FP8_E5M2; }
bool valid_out(int dt) { return valid_dtype(dt); }

// Grid of a grid-stride kernel: one CTA per `per_cta` work items, at most
// `per_sm` CTAs per SM. Measured on B200: 8 suits most casts; the per-tensor
// cast_ste apply and the INT4 casts ran 7-8% faster at 32 and dequantize
// 10-14% faster, while the other casts ran 3-14% slower there (and slower
// still at one resident wave) and requantize did not change.
int grid_for(int64_t work_items, int per_cta, int per_sm = 8) {
  const int64_t want = (work_items + per_cta - 1) / per_cta;
  const int64_t cap = (int64_t)sm_count() * per_sm;
  return (int)(want < 1 ? 1 : (want > cap ? cap : want));
}

// Dispatch helpers: map runtime enums onto template instances.
template <template <int, int> class F, typename... Args>
int dispatch_dt_fmt(int dt, int fmt, Args... args) {
  if (dt == BRC_DTYPE_F32)
    return fmt == BRC_FP8_E4M3 ? F<BRC_DTYPE_F32, BRC_FP8_E4M3>::run(args...)
                               : F<BRC_DTYPE_F32, BRC_FP8_E5M2>::run(args...);
  if (dt == BRC_DTYPE_BF16)
    return fmt == BRC_FP8_E4M3 ? F<BRC_DTYPE_BF16, BRC_FP8_E4M3>::run(args...)
                               : F<BRC_DTYPE_BF16, BRC_FP8_E5M2>::run(args...);
  return fmt == BRC_FP8_E4M3 ? F<BRC_DTYPE_F16, BRC_FP8_E4M3>::run(args...)
                             : F<BRC_DTYPE_F16, BRC_FP8_E5M2>::run(args...);
}

// Launch the vectorised block kernel for block size B with LPB lanes per
// block, choosing LPB so each lane owns 64 bytes (32 halves / 16 floats), or
// the whole block when it is smaller. The per-block work (statistic, scale,
// scale stores) then runs on as few lanes as possible.
template <int DT, int MODE, int FMT, int B, bool STE = false>
int launch_block_b(const BlockCastArgs& a, cudaStream_t st) {
  constexpr int V = In<DT>::kVec;
  constexpr int E0 = (DT == BRC_DTYPE_F32) ? 16 : 32;  // 64 bytes per lane
  constexpr int E = B < E0 ? B : E0;
  constexpr int LPB = B / E;
  static_assert(E % V == 0 && LPB >= 1 && LPB <= 32, "bad lane split");
  const int64_t tiles = (a.n_blocks + (32 / LPB) - 1) / (32 / LPB);
  constexpr int kPerSm = (MODE == kInt4Sym || MODE == kInt4Asym) ? 32 : 8;
  const int grid = grid_for(tiles, 8, kPerSm);
  k_block_cast<DT, MODE, FMT, B, LPB, STE><<<grid, 256, 0, st>>>(a);
  return check_launch();
}

template <int DT, int MODE, int FMT, bool STE = false>
int launch_block(const BlockCastArgs& a, int B, cudaStream_t st) {
  switch (B) {
    case 16: return launch_block_b<DT, MODE, FMT, 16, STE>(a, st);
    case 32: return launch_block_b<DT, MODE, FMT, 32, STE>(a, st);
    case 64: return launch_block_b<DT, MODE, FMT, 64, STE>(a, st);
    case 128: return launch_block_b<DT, MODE, FMT, 128, STE>(a, st);
    case 256: return launch_block_b<DT, MODE, FMT, 256, STE>(a, st);
    default: break;
  }
  if (!STE && (MODE == kBlockFp8 || MODE == kInt4Sym || MODE == kInt4Asym)) {
    if (a.packed && (B & 1)) return BRC_ERR_UNSUPPORTED;
    k_block_cast_generic<DT, MODE, FMT>
        <<<grid_for(a.n_blocks, 256), 256, 0, st>>>(a, B);
    return check_launch();
  }
  return BRC_ERR_UNSUPPORTED;
}

template <int MODE, int FMT, bool STE = false>
int launch_block_any_dt(int dt, const BlockCastArgs& a, int B, cudaStream_t st) {
  if (dt == BRC_DTYPE_F32) return launch_block<BRC_DTYPE_F32, MODE, FMT, STE>(a, B, st);
  if (dt == BRC_DTYPE_BF16) return launch_block<BRC_DTYPE_BF16, MODE, FMT, STE>(a, B, st);
  return launch_block<BRC_DTYPE_F16, MODE, FMT, STE>(a, B, st);
}

// Empty inputs are valid no-ops (their data pointers may be NULL).
bool empty_input(int64_t rows, int64_t cols, int B) {
  return rows >= 0 && cols >= 0 && B > 0 && cols % B == 0 && rows * cols == 0;
}

int common_checks(const void* x, int dt, int64_t rows, int64_t cols, int B) {
  if (empty_input(rows, cols, B)) return valid_dtype(dt) ? BRC_OK : BRC_ERR_DTYPE;
  if (!x) return BRC_ERR_NULL;
  if (!valid_dtype(dt)) return BRC_ERR_DTYPE;
  if (rows < 0 || cols < 0 || B <= 0) return BRC_ERR_SHAPE;
  if (cols % B != 0) return BRC_ERR_SHAPE;
  if (!aligned16(x)) return BRC_ERR_ALIGN;
  return BRC_OK;
}

BlockCastArgs make_args(const void* x, int64_t rows, int64_t cols, int B) {
  BlockCastArgs a{};
  a.x = x;
  a.n_blocks = rows * (cols / B);
  const int64_t bpr = cols / B;
  a.blocks_per_row = make_fastdiv((uint32_t)(bpr > 0 ? bpr : 1));
  a.sf_col_tiles = (uint32_t)((bpr + 3) / 4);
  return a;
}

}  // namespace

extern "C" {

int brc_amax_reset(uint32_t* amax_bits, void* stream) {
  if (!amax_bits) return BRC_ERR_NULL;
  k_amax_reset<<<1, 1, 0, (cudaStream_t)stream>>>(amax_bits);
  return check_launch();
}

int brc_amax_accumulate(const void* x, int x_dtype, int64_t n, uint32_t* amax_bits,
                        void* stream) {
  if (!amax_bits || (!x && n > 0)) return BRC_ERR_NULL;
  if (!valid_dtype(x_dtype)) return BRC_ERR_DTYPE;
  if (n < 0) return BRC_ERR_SHAPE;
  if (n == 0) return BRC_OK;
  if (!aligned16(x)) return BRC_ERR_ALIGN;
  const int V = x_dtype == BRC_DTYPE_F32 ? 4 : 8;
  cudaStream_t st = (cudaStream_t)stream;
  auto kern = x_dtype == BRC_DTYPE_F32    ? k_amax<BRC_DTYPE_F32>
              : x_dtype == BRC_DTYPE_BF16 ? k_amax<BRC_DTYPE_BF16>
                                          : k_amax<BRC_DTYPE_F16>;
  kern<<<grid_for(n / V + 1, 256 * 4), 256, 0, st>>>(x, n, amax_bits);
  return check_launch();
}

}  // extern "C"
namespace {
template <int DT, int FMT>
struct PerTensorApply {
  static int run(const void* x, int64_t n, const uint32_t* amax_bits, uint8_t* codes,
                 float* scale_out, cudaStream_t st) {
    const double fmax = FMT == BRC_FP8_E4M3 ? 448.0 : 57344.0;
    const float floor_scale = (float)(1e-10 / fmax);
    const int V = In<DT>::kVec;
    const int grid = grid_for(n / V + 1, 256 * 4);
    k_pertensor_apply<DT, FMT><<<grid, 256, 0, st>>>(x, n, amax_bits, floor_scale, codes,
                                                     scale_out, nullptr);
    return check_launch();
  }
};
}  // namespace
extern "C" {

int brc_cast_pertensor_fp8_apply(const void* x, int x_dtype, int64_t n, int fmt,
                                 const uint32_t* amax_bits, uint8_t* codes, float* scale_out,
                                 void* stream) {
  if (!amax_bits || !scale_out || ((!x || !codes) && n > 0)) return BRC_ERR_NULL;
  if (!valid_dtype(x_dtype) || !valid_fmt(fmt)) return BRC_ERR_DTYPE;
  if (n < 0) return BRC_ERR_SHAPE;
  if (n > 0 && (!aligned16(x) || !aligned16(codes))) return BRC_ERR_ALIGN;
  return dispatch_dt_fmt<PerTensorApply>(x_dtype, fmt, x, n, amax_bits, codes, scale_out,
                                         (cudaStream_t)stream);
}

int brc_cast_pertensor_fp8(const void* x, int x_dtype, int64_t n, int fmt, uint8_t* codes,
                           float* scale_out, uint32_t* workspace, void* stream) {
  if (!workspace) return BRC_ERR_NULL;
  if (!valid_dtype(x_dtype) || !valid_fmt(fmt)) return BRC_ERR_DTYPE;
  int rc = brc_amax_reset(workspace, stream);
  if (rc) return rc;
  rc = brc_amax_accumulate(x, x_dtype, n, workspace, stream);
  if (rc) return rc;
  return brc_cast_pertensor_fp8_apply(x, x_dtype, n, fmt, workspace, codes, scale_out, stream);
}

int brc_cast_block_fp8(const void* x, int x_dtype, int64_t rows, int64_t cols, int block_k,
                       int fmt, uint8_t* codes, float* scales, void* stream) {
  int rc = common_checks(x, x_dtype, rows, cols, block_k);
  if (rc) return rc;
  if (!valid_fmt(fmt)) return BRC_ERR_DTYPE;
  if (empty_input(rows, cols, block_k)) return BRC_OK;
  if (!codes || !scales) return BRC_ERR_NULL;
  if (!aligned16(codes)) return BRC_ERR_ALIGN;
  BlockCastArgs a = make_args(x, rows, cols, block_k);
  a.codes = codes;
  a.scales = scales;
  cudaStream_t st = (cudaStream_t)stream;
  return fmt == BRC_FP8_E4M3 ? launch_block_any_dt<kBlockFp8, BRC_FP8_E4M3>(x_dtype, a, block_k, st)
                             : launch_block_any_dt<kBlockFp8, BRC_FP8_E5M2>(x_dtype, a, block_k, st);
}

}  // extern "C"
namespace {
template <int DT, int FMT>
struct Block2d {
  static int run(const void* x, int64_t rows, int64_t cols, int bm, int bk, uint8_t* codes,
                 float* scales, cudaStream_t st) {
    constexpr int V = In<DT>::kVec;
    if (bk % V) return BRC_ERR_UNSUPPORTED;
    const int64_t nvec = (int64_t)bm * (bk / V);
    if (nvec > 256 * 16) return BRC_ERR_UNSUPPORTED;
    if (bk == 128 && bm <= 128 && (cols * elem_bytes<DT>()) % 16 == 0 &&
        (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
      // persistent TMA-fed form
      constexpr int NV = (128 * (128 / V) + kB2dThreads - 1) / kB2dThreads;
      auto kern = k_block2d_cast_tma<DT, FMT, NV>;
      static std::once_flag once[64];
      int dev = 0;
      if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BRC_ERR_CUDA;
      constexpr int kSmemMax = 227 * 1024;
      std::call_once(once[dev], [&] {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
      });
      const int tile_bytes = bm * 128 * elem_bytes<DT>();
      const int extra = 16 * 8 + 2 * (kB2dThreads / 32) * 4 + 16;
      int stages = (kSmemMax - extra) / tile_bytes;
      if (stages > 6) stages = 6;
      if (stages >= 2) {
        CUtensorMap tm;
        const CUtensorMapDataType dt = DT == BRC_DTYPE_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                       : DT == BRC_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        int rc = encode_tmap_2d(&tm, dt, x, (uint64_t)cols, (uint64_t)rows,
                                (uint64_t)cols * elem_bytes<DT>(), 128, (uint32_t)bm);
        if (rc) return rc;
        const int64_t ntiles = (cols / 128) * (rows / bm);
        const int grid = (int)(ntiles < sm_count() ? ntiles : sm_count());
        const size_t smem = (size_t)stages * tile_bytes + extra;
        kern<<<grid, kB2dThreads, smem, st>>>(tm, rows, cols, bm, stages, codes, scales,
                                               gemm_status_ptr());
        return check_launch();
      }
    }
    dim3 grid((unsigned)(cols / bk), (unsigned)(rows / bm));
    constexpr int kVpr128 = 128 / V;  // vectors per row of a 128-wide tile
    if (bk == 128) {
      if (nvec <= 256 * (V == 4 ? 16 : 8))
        k_block2d_cast<DT, FMT, (V == 4 ? 16 : 8), kVpr128>
            <<<grid, 256, 0, st>>>(x, cols, bm, bk, codes, scales);
      else
        k_block2d_cast<DT, FMT, 16, kVpr128><<<grid, 256, 0, st>>>(x, cols, bm, bk, codes, scales);
    } else {
      k_block2d_cast<DT, FMT, 16, 0><<<grid, 256, 0, st>>>(x, cols, bm, bk, codes, scales);
    }
    return check_launch();
  }
};
}  // namespace
extern "C" {

int brc_cast_block_fp8_2d(const void* x, int x_dtype, int64_t rows, int64_t cols, int block_m,
                          int block_k, int fmt, uint8_t* codes, float* scales, void* stream) {
  int rc = common_checks(x, x_dtype, rows, cols, block_k);
  if (rc) return rc;
  if (!valid_fmt(fmt)) return BRC_ERR_DTYPE;
  if (block_m <= 0 || rows % block_m) return BRC_ERR_SHAPE;
  if (empty_input(rows, cols, block_k)) return BRC_OK;
  if (!codes || !scales) return BRC_ERR_NULL;
  if (!aligned16(codes)) return BRC_ERR_ALIGN;
  if (rows / block_m > 65535 || cols / block_k > INT32_MAX) return BRC_ERR_RANGE;
  return dispatch_dt_fmt<Block2d>(x_dtype, fmt, x, rows, cols, block_m, block_k, codes, scales,
                                  (cudaStream_t)stream);
}

int brc_cast_mxfp8(const void* x, int x_dtype, int64_t rows, int64_t cols, int fmt,
                   uint8_t* codes, uint8_t* scales, uint8_t* scales_mma, void* stream) {
  int rc = common_checks(x, x_dtype, rows, cols, 32);
  if (rc) return rc;
  if (!valid_fmt(fmt)) return BRC_ERR_DTYPE;
  if (empty_input(rows, cols, 32)) return BRC_OK;
  if (!codes || !scales) return BRC_ERR_NULL;
  if (!aligned16(codes)) return BRC_ERR_ALIGN;
  if (rows * (cols / 32) >= (1ll << 31)) return BRC_ERR_RANGE;
  BlockCastArgs a = make_args(x, rows, cols, 32);
  a.codes = codes;
  a.scales = scales;
  a.scales_mma = scales_mma;
  cudaStream_t st = (cudaStream_t)stream;
  return fmt == BRC_FP8_E4M3 ? launch_block_any_dt<kMxfp8, BRC_FP8_E4M3>(x_dtype, a, 32, st)
                             : launch_block_any_dt<kMxfp8, BRC_FP8_E5M2>(x_dtype, a, 32, st);
}

int brc_cast_nvfp4(const void* x, int x_dtype, int64_t rows, int64_t cols, uint8_t* codes,
                   uint8_t* packed, uint8_t* scales, uint8_t* scales_mma, void* stream) {
  int rc = common_checks(x, x_dtype, rows, cols, 16);
  if (rc) return rc;
  if (empty_input(rows, cols, 16)) return BRC_OK;
  if (!scales || (!codes && !packed)) return BRC_ERR_NULL;
  if ((codes && !aligned16(codes)) || (packed && !aligned16(packed))) return BRC_ERR_ALIGN;
  if (rows * (cols / 16) >= (1ll << 31)) return BRC_ERR_RANGE;
  BlockCastArgs a = make_args(x, rows, cols, 16);
  a.codes = codes;
  a.packed = packed;
  a.scales = scales;
  a.scales_mma = scales_mma;
  return launch_block_any_dt<kNvfp4, 0>(x_dtype, a, 16, (cudaStream_t)stream);
}

int brc_cast_int4(const void* x, int x_dtype, int64_t rows, int64_t cols, int group,
                  int is_signed, int symmetric, int scale_dtype, uint8_t* codes,
                  uint8_t* packed, void* scales, void* zero_points, uint8_t* packed_tiles,
                  float* scale_tiles, float* zp_tiles, void* stream) {
  int rc = common_checks(x, x_dtype, rows, cols, group);
  if (rc) return rc;
  if (!symmetric && is_signed) return BRC_ERR_UNSUPPORTED;
  if (scale_dtype != BRC_SCALE_F16 && scale_dtype != BRC_SCALE_F32) return BRC_ERR_DTYPE;
  if (empty_input(rows, cols, group)) return BRC_OK;
  if (!scales || (!codes && !packed)) return BRC_ERR_NULL;
  if (!symmetric && !zero_points) return BRC_ERR_NULL;
  if ((codes && !aligned16(codes)) || (packed && !aligned16(packed))) return BRC_ERR_ALIGN;
  if (packed_tiles) {
    if (group != 128 || rows % 16 || !scale_tiles || (!symmetric && !zp_tiles))
      return BRC_ERR_UNSUPPORTED;
    if (!aligned16(packed_tiles)) return BRC_ERR_ALIGN;
  }
  BlockCastArgs a = make_args(x, rows, cols, group);
  a.codes = codes;
  a.packed = packed;
  a.scales = scales;
  a.zp = zero_points;
  a.packed_tiles = packed_tiles;
  a.scale_tiles = scale_tiles;
  a.zp_tiles = zp_tiles;
  a.is_signed = is_signed ? 1 : 0;
  a.scale_f16 = scale_dtype == BRC_SCALE_F16;
  cudaStream_t st = (cudaStream_t)stream;
  return symmetric ? launch_block_any_dt<kInt4Sym, 0>(x_dtype, a, group, st)
                   : launch_block_any_dt<kInt4Asym, 0>(x_dtype, a, group, st);
}

// ---------------------------------------------------------------- cast_ste
}  // extern "C"
namespace {
template <int DT, int FMT>
struct PerTensorSte {
  static int run(const void* x, int64_t n, const uint32_t* amax_bits, float* out,
                 cudaStream_t st) {
    const double fmax = FMT == BRC_FP8_E4M3 ? 448.0 : 57344.0;
    const float floor_scale = (float)(1e-10 / fmax);
    const int grid = grid_for(n / In<DT>::kVec + 1, 256 * 4, 32);
    k_pertensor_apply<DT, FMT, true>
        <<<grid, 256, 0, st>>>(x, n, amax_bits, floor_scale, nullptr, nullptr, out);
    return check_launch();
  }
};
}  // namespace
extern "C" {

int brc_cast_ste_pertensor_fp8(const void* x, int x_dtype, int64_t n, int fmt,
                               uint32_t* amax_word, float* out, void* stream) {
  if (!amax_word || ((!x || !out) && n > 0)) return BRC_ERR_NULL;
  if (!valid_dtype(x_dtype) || !valid_fmt(fmt)) return BRC_ERR_DTYPE;
  if (n < 0) return BRC_ERR_SHAPE;
  if (n == 0) return BRC_OK;
  if (!aligned16(x) || !aligned16(out)) return BRC_ERR_ALIGN;
  int rc = brc_amax_reset(amax_word, stream);
  if (rc) return rc;
  if ((rc = brc_amax_accumulate(x, x_dtype, n, amax_word, stream))) return rc;
  return dispatch_dt_fmt<PerTensorSte>(x_dtype, fmt, x, n, amax_word, out, (cudaStream_t)stream);
}

int brc_cast_ste_block(const void* x, int x_dtype, int64_t rows, int64_t cols, int kind,
                       int block, int fmt, int is_signed, int symmetric, int scale_dtype,
                       float* out, void* stream) {
  int rc = common_checks(x, x_dtype, rows, cols, block);
  if (rc) return rc;
  if (kind == BRC_STE_MXFP8 && block != 32) return BRC_ERR_UNSUPPORTED;
  if (kind == BRC_STE_NVFP4 && block != 16) return BRC_ERR_UNSUPPORTED;
  if ((kind == BRC_STE_BLOCK_FP8 || kind == BRC_STE_MXFP8) && !valid_fmt(fmt)) return BRC_ERR_DTYPE;
  if (kind == BRC_STE_INT4 && !symmetric && is_signed) return BRC_ERR_UNSUPPORTED;
  if (kind == BRC_STE_INT4 && scale_dtype != BRC_SCALE_F16 && scale_dtype != BRC_SCALE_F32)
    return BRC_ERR_DTYPE;
  if (kind < BRC_STE_BLOCK_FP8 || kind > BRC_STE_INT4) return BRC_ERR_UNSUPPORTED;
  if (empty_input(rows, cols, block)) return BRC_OK;
  if (!out) return BRC_ERR_NULL;
  if (!aligned16(out)) return BRC_ERR_ALIGN;
  BlockCastArgs a = make_args(x, rows, cols, block);
  a.ste_out = out;
  a.is_signed = is_signed ? 1 : 0;
  a.scale_f16 = scale_dtype == BRC_SCALE_F16;
  cudaStream_t st = (cudaStream_t)stream;
  const bool e4 = fmt == BRC_FP8_E4M3;
  switch (kind) {
    case BRC_STE_BLOCK_FP8:
      return e4 ? launch_block_any_dt<kBlockFp8, BRC_FP8_E4M3, true>(x_dtype, a, block, st)
                : launch_block_any_dt<kBlockFp8, BRC_FP8_E5M2, true>(x_dtype, a, block, st);
    case BRC_STE_MXFP8:
      return e4 ? launch_block_any_dt<kMxfp8, BRC_FP8_E4M3, true>(x_dtype, a, block, st)
                : launch_block_any_dt<kMxfp8, BRC_FP8_E5M2, true>(x_dtype, a, block, st);
    case BRC_STE_NVFP4:
      return launch_block_any_dt<kNvfp4, 0, true>(x_dtype, a, block, st);
    default:
      return symmetric ? launch_block_any_dt<kInt4Sym, 0, true>(x_dtype, a, block, st)
                       : launch_block_any_dt<kInt4Asym, 0, true>(x_dtype, a, block, st);
  }
}

// ---------------------------------------------------------------- dequant
}  // extern "C"
namespace {
template <int DQ, int FMT>
int launch_dequant(const DequantArgs& a, int out_dtype, cudaStream_t st) {
  const int grid = grid_for(a.n / 16 + 1, 256 * 2, 32);
  const int64_t cpr = a.cols / 16, cpb = a.block_k / 16;
  if (a.n / 4 >= (1ll << 31) || cpr >= (1ll << 31)) {
    if (out_dtype == BRC_DTYPE_F32) k_dequant_wide<DQ, FMT, BRC_DTYPE_F32><<<grid, 256, 0, st>>>(a);
    else if (out_dtype == BRC_DTYPE_BF16)
      k_dequant_wide<DQ, FMT, BRC_DTYPE_BF16><<<grid, 256, 0, st>>>(a);
    else k_dequant_wide<DQ, FMT, BRC_DTYPE_F16><<<grid, 256, 0, st>>>(a);
    return check_launch();
  }
  const FastDiv fcpr = make_fastdiv((uint32_t)cpr), fbm = make_fastdiv((uint32_t)a.block_m),
                fcpb = make_fastdiv((uint32_t)cpb);
  if (out_dtype == BRC_DTYPE_F32)
    k_dequant<DQ, FMT, BRC_DTYPE_F32><<<grid, 256, 0, st>>>(a, fcpr, fbm, fcpb);
  else if (out_dtype == BRC_DTYPE_BF16)
    k_dequant<DQ, FMT, BRC_DTYPE_BF16><<<grid, 256, 0, st>>>(a, fcpr, fbm, fcpb);
  else k_dequant<DQ, FMT, BRC_DTYPE_F16><<<grid, 256, 0, st>>>(a, fcpr, fbm, fcpb);
  return check_launch();
}

int dq_checks(const uint8_t* codes, const void* scales, void* out, int64_t n, int out_dtype) {
  if ((!codes || !out || !scales) && n > 0) return BRC_ERR_NULL;
  if (!valid_out(out_dtype)) return BRC_ERR_DTYPE;
  if (n < 0 || n % 16) return BRC_ERR_SHAPE;
  if (n > 0 && (!aligned16(codes) || !aligned16(out))) return BRC_ERR_ALIGN;
  return BRC_OK;
}
}  // namespace
extern "C" {

int brc_dequant_pertensor_fp8(const uint8_t* codes, int64_t n, int fmt, const float* scale,
                              void* out, int out_dtype, void* stream) {
  int rc = dq_checks(codes, scale, out, n, out_dtype);
  if (rc) return rc;
  if (!valid_fmt(fmt)) return BRC_ERR_DTYPE;
  if (n == 0) return BRC_OK;
  DequantArgs a{};
  a.codes = codes;
  a.scales = scale;
  a.out = out;
  a.n = n;
  a.cols = n;
  a.block_k = 16;
  a.block_m = 1;
  a.per_tensor = 1;
  cudaStream_t st = (cudaStream_t)stream;
  return fmt == BRC_FP8_E4M3 ? launch_dequant<kDqFp8, BRC_FP8_E4M3>(a, out_dtype, st)
                             : launch_dequant<kDqFp8, BRC_FP8_E5M2>(a, out_dtype, st);
}

int brc_dequant_block_fp8(const uint8_t* codes, int64_t rows, int64_t cols, int block_m,
                          int block_k, int fmt, const float* scales, void* out, int out_dtype,
                          void* stream) {
  const int64_t n = rows * cols;
  int rc = dq_checks(codes, scales, out, n, out_dtype);
  if (rc) return rc;
  if (!valid_fmt(fmt)) return BRC_ERR_DTYPE;
  if (block_k <= 0 || block_m <= 0 || cols % block_k || rows % block_m) return BRC_ERR_SHAPE;
  if (block_k % 16) return BRC_ERR_UNSUPPORTED;
  if (n == 0) return BRC_OK;
  DequantArgs a{};
  a.codes = codes;
  a.scales = scales;
  a.out = out;
  a.n = n;
  a.cols = cols;
  a.block_k = block_k;
  a.block_m = block_m;
  a.scale_cols = cols / block_k;
  cudaStream_t st = (cudaStream_t)stream;
  return fmt == BRC_FP8_E4M3 ? launch_dequant<kDqFp8, BRC_FP8_E4M3>(a, out_dtype, st)
                             : launch_dequant<kDqFp8, BRC_FP8_E5M2>(a, out_dtype, st);
}

int brc_dequant_mxfp8(const uint8_t* codes, int64_t rows, int64_t cols, int fmt,
                      const uint8_t* scales, void* out, int out_dtype, void* stream) {
  const int64_t n = rows * cols;
  int rc = dq_checks(codes, scales, out, n, out_dtype);
  if (rc) return rc;
  if (!valid_fmt(fmt)) return BRC_ERR_DTYPE;
  if (cols % 32) return BRC_ERR_SHAPE;
  if (n == 0) return BRC_OK;
  DequantArgs a{};
  a.codes = codes;
  a.scales = scales;
  a.out = out;
  a.n = n;
  a.cols = cols;
  a.block_k = 32;
  a.block_m = 1;
  a.scale_cols = cols / 32;
  cudaStream_t st = (cudaStream_t)stream;
  return fmt == BRC_FP8_E4M3 ? launch_dequant<kDqMx, BRC_FP8_E4M3>(a, out_dtype, st)
                             : launch_dequant<kDqMx, BRC_FP8_E5M2>(a, out_dtype, st);
}

int brc_dequant_nvfp4(const uint8_t* codes, int64_t rows, int64_t cols, const uint8_t* scales,
                      void* out, int out_dtype, void* stream) {
  const int64_t n = rows * cols;
  int rc = dq_checks(codes, scales, out, n, out_dtype);
  if (rc) return rc;
  if (cols % 16) return BRC_ERR_SHAPE;
  if (n == 0) return BRC_OK;
  DequantArgs a{};
  a.codes = codes;
  a.scales = scales;
  a.out = out;
  a.n = n;
  a.cols = cols;
  a.block_k = 16;
  a.block_m = 1;
  a.scale_cols = cols / 16;
  return launch_dequant<kDqNv, 0>(a, out_dtype, (cudaStream_t)stream);
}

int brc_dequant_int4(const uint8_t* codes, int64_t rows, int64_t cols, int group, int is_signed,
                     int scale_dtype, const void* scales, const void* zero_points, void* out,
                     int out_dtype, void* stream) {
  const int64_t n = rows * cols;
  int rc = dq_checks(codes, scales, out, n, out_dtype);
  if (rc) return rc;
  if (group <= 0 || cols % group) return BRC_ERR_SHAPE;
  if (group % 16) return BRC_ERR_UNSUPPORTED;
  if (scale_dtype != BRC_SCALE_F16 && scale_dtype != BRC_SCALE_F32) return BRC_ERR_DTYPE;
  if (n == 0) return BRC_OK;
  DequantArgs a{};
  a.codes = codes;
  a.scales = scales;
  a.zp = zero_points;
  a.out = out;
  a.n = n;
  a.cols = cols;
  a.block_k = group;
  a.block_m = 1;
  a.scale_cols = cols / group;
  a.is_signed = is_signed ? 1 : 0;
  a.scale_f16 = scale_dtype == BRC_SCALE_F16;
  return launch_dequant<kDqInt4, 0>(a, out_dtype, (cudaStream_t)stream);
}

int brc_requant_nvfp4_to_mxfp8(const uint8_t* codes, const uint8_t* scales, int64_t rows,
                               int64_t cols, int fmt, uint8_t* codes_out, uint8_t* scales_out,
                               uint8_t* scales_mma_out, void* stream) {
  if (!codes || !scales || !codes_out || !scales_out) return BRC_ERR_NULL;
  if (!valid_fmt(fmt)) return BRC_ERR_DTYPE;
  if (rows < 0 || cols < 0 || cols % 32) return BRC_ERR_SHAPE;
  if (!aligned16(codes) || !aligned16(codes_out)) return BRC_ERR_ALIGN;
  const int64_t n_blocks = rows * (cols / 32);
  if (n_blocks >= (1ll << 31)) return BRC_ERR_RANGE;
  if (n_blocks == 0) return BRC_OK;
  const int64_t bpr = cols / 32;
  const FastDiv f = make_fastdiv((uint32_t)bpr);
  const uint32_t tiles = (uint32_t)((bpr + 3) / 4);
  const int grid = grid_for(n_blocks, 256);
  cudaStream_t st = (cudaStream_t)stream;
  if (fmt == BRC_FP8_E4M3)
    k_requant_nv_to_mx<BRC_FP8_E4M3><<<grid, 256, 0, st>>>(codes, scales, n_blocks, f, tiles,
                                                            codes_out, scales_out, scales_mma_out);
  else
    k_requant_nv_to_mx<BRC_FP8_E5M2><<<grid, 256, 0, st>>>(codes, scales, n_blocks, f, tiles,
                                                            codes_out, scales_out, scales_mma_out);
  return check_launch();
}

}  // extern "C"

// ========================================================================
// Per-tensor FP8 cast for callers that cannot allocate device memory.
//
// Some callers have no allocator to hand: a host runtime that only receives
// pre-allocated input and output buffers, a custom-op slot with no workspace
// argument, or code running where cudaMalloc is not allowed (it would block
// or break an enclosing memory pool's accounting). brc_cast_pertensor_fp8
// needs a caller-provided workspace word for the global amax; this variant
// keeps that scratch in a fixed device array inside the library instead.
//
// Scratch: kNoAllocMaxChunks partial maxima (one per kNoAllocChunk-element
// chunk of the input) plus one final amax word, 65,792 bytes, in a
// file-scope __device__ array that every GPU loading the library holds until
// exit. Each call writes every slot it later reads (the chunk partials, then
// the final word), so nothing has to be cleared between calls. All calls on a
// device share the array: calls whose kernels overlap on that GPU (different
// streams, or different host threads) race and must be serialised by the
// caller.
// ========================================================================
namespace brc {
namespace noalloc {

constexpr int64_t kChunk = 32768;
constexpr int64_t kMaxChunks = 16384;
constexpr int64_t kMaxElems = kChunk * kMaxChunks;  // 536,870,912 elements
constexpr int64_t kFinal = kMaxChunks;              // index of the final amax word

static __device__ __align__(256) uint32_t g_scratch[kMaxChunks + 64];

// One CTA per chunk: abs-max of elements [chunk * kChunk, min(n, ...)).
template <int DT>
__global__ void __launch_bounds__(256) k_chunk_amax(const void* __restrict__ x, int64_t n,
                                                     uint32_t* partials) {
  constexpr int V = In<DT>::kVec;
  const int64_t lo = (int64_t)blockIdx.x * kChunk;
  const int64_t hi = lo + kChunk < n ? lo + kChunk : n;
  float m = 0.f;
  if (((hi - lo) % V) == 0) {
    const char* base = static_cast<const char*>(x) + lo * elem_bytes<DT>();
    for (int64_t v = threadIdx.x; v < (hi - lo) / V; v += blockDim.x)
      m = fmax_nan(m, vec_absmax<DT>(ldg16(base + 16 * v)));
  } else {
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x)
      m = fmax_nan(m, fabsf(load1<DT>(x, i)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmax_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t = fmax_nan(t, red[w]);
    partials[blockIdx.x] = __float_as_uint(t);
  }
}

// One CTA: final = max(partials[0..count)), 0 when count == 0.
__global__ void __launch_bounds__(1024) k_reduce_partials(const uint32_t* partials, int count,
                                                          uint32_t* final_word) {
  uint32_t m = 0u;
  for (int i = threadIdx.x; i < count; i += blockDim.x) m = max(m, partials[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  __shared__ uint32_t red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = max(m, red[w]);
    *final_word = max(m, red[0]);
  }
}

}  // namespace noalloc
}  // namespace brc

#include <mutex>

namespace {
// Device address of the scratch array, looked up once per device with that
// device current. In host code `g_scratch` names a host-side shadow, not the
// device array, so kernels must be given this address. The address is cached
// for the life of the process; a device reset after the first call would
// leave it stale, which the header documents as unsupported.
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
uint32_t* g_noalloc_ptr[kNoAllocMaxDevices] = {};

int noalloc_scratch(uint32_t** out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev));
  if (rc) return rc;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return BRC_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    uint32_t* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(reinterpret_cast<void**>(&p), brc::noalloc::g_scratch));
    if (rc) return rc;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return BRC_OK;
}

template <int DT, int FMT>
struct NoAllocCast {
  static int run(const void* x, int64_t n, uint8_t* codes, float* scale_out, uint32_t* scratch,
                 cudaStream_t st) {
    using namespace brc::noalloc;
    const int chunks = (int)((n + kChunk - 1) / kChunk);
    if (chunks > 0) {
      k_chunk_amax<DT><<<chunks, 256, 0, st>>>(x, n, scratch);
      int rc = check_launch();
      if (rc) return rc;
    }
    k_reduce_partials<<<1, 1024, 0, st>>>(scratch, chunks, scratch + kFinal);
    int rc = check_launch();
    if (rc) return rc;
    return PerTensorApply<DT, FMT>::run(x, n, scratch + kFinal, codes, scale_out, st);
  }
};
}  // namespace

extern "C" int brc_cast_pertensor_fp8_noalloc(const void* x, int x_dtype, int64_t n, int fmt,
                                              uint8_t* codes, float* scale_out, void* stream) {
  if (!scale_out || ((!x || !codes) && n > 0)) return BRC_ERR_NULL;
  if (!valid_dtype(x_dtype) || !valid_fmt(fmt)) return BRC_ERR_DTYPE;
  if (n < 0) return BRC_ERR_SHAPE;
  if (n > brc::noalloc::kMaxElems) return BRC_ERR_RANGE;
  if (n > 0 && (!aligned16(x) || !aligned16(codes))) return BRC_ERR_ALIGN;
  uint32_t* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return dispatch_dt_fmt<NoAllocCast>(x_dtype, fmt, x, n, codes, scale_out, scratch,
                                      (cudaStream_t)stream);
}

// ========================================================================
// DelayedScaling with an amax history (extension; the reference's cast
// ignores the recipe's amax_history_len / margin: recipes.py:43-77,
// cast.py:364-373). The history is a caller-owned float32 ring on the
// device, most recent first. A cast that uses it takes its dequantization
// scale from the history before reading the tensor,
//   s = float32(max(max(history), 1e-10) / fmt_max) * 2^margin  (float32),
// so it is ONE pass: each element is read once, encoded with s (the same
// clip-then-encode and IEEE division as the current-amax cast) while the
// tensor's own amax is reduced, and that amax is pushed into the ring
// afterwards. A cast without history (the caller's first) is the current-
// amax cast of the reference, bit for bit, and records its amax.
// ========================================================================
namespace brc {
namespace delayed {

template <int FMT>
__global__ void k_history_scale(const float* __restrict__ hist, int len, float margin_pow2,
                                float floor_scale, float* scale_out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  constexpr float kMax = FMT == BRC_FP8_E4M3 ? 448.f : 57344.f;
  float m = 0.f;
  for (int i = 0; i < len; ++i) m = fmax_nan(m, fabsf(hist[i]));
  const float s = __fmul_rn(pertensor_scale(__float_as_uint(m), kMax, floor_scale), margin_pow2);
  *scale_out = canon_nan(s);
}

// Encode with a scale known before the pass; reduce the tensor's amax on the
// way (NaN propagates; the float bits of a non-negative value or NaN order
// as integers, so atomicMax on the bits is the float maximum).
template <int DT, int FMT>
__global__ void __launch_bounds__(256) k_delayed_apply(const void* __restrict__ x, int64_t n,
                                                       const float* scale_in, uint8_t* codes,
                                                       uint32_t* amax_bits) {
  constexpr int V = In<DT>::kVec;
  const float s = *scale_in;
  const bool fast = isfinite(s) && s > 0.f;
  const float r = __frcp_rn(s);
  const int64_t nvec = n / V;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const char* base = static_cast<const char*>(x);
  float m = 0.f;
  auto encode_store = [&](const uint4 v, int64_t vi) {
    const float vmax = vec_absmax<DT>(v);
    m = fmax_nan(m, vmax);
    float f0[V];
    unpack<DT>(v, f0);
    uint32_t w0[V / 4];
    // The scale is finite while the tensor may hold NaN (the current-amax
    // cast never meets this: a NaN makes its scale NaN). The fast encoder
    // clamps with fminf, which maps NaN to the maximum code, so a vector
    // holding a NaN takes the per-element path (NaN -> the NaN code).
    if (fast && !isnan(vmax)) {
#pragma unroll
      for (int j = 0; j < V / 4; ++j)
        w0[j] = enc4_fp8<FMT>(div_by(f0[4 * j], s, r), div_by(f0[4 * j + 1], s, r),
                              div_by(f0[4 * j + 2], s, r), div_by(f0[4 * j + 3], s, r));
    } else {
#pragma unroll
      for (int j = 0; j < V / 4; ++j) {
        uint32_t c = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) c |= enc1_fp8<FMT>(div_ieee(f0[4 * j + i], s)) << (8 * i);
        w0[j] = c;
      }
    }
    if constexpr (V == 8) {
      *reinterpret_cast<uint2*>(codes + vi * V) = make_uint2(w0[0], w0[1]);
    } else {
      *reinterpret_cast<uint32_t*>(codes + vi * V) = w0[0];
    }
  };
  // Four 16-byte vectors per iteration; the next iteration's four are loaded
  // before this iteration's are encoded, so loads stay in flight while the
  // thread computes.
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint4 nv[4];
  if (i + 3 * stride < nvec) {
#pragma unroll
    for (int u = 0; u < 4; ++u) nv[u] = ldg16(base + 16 * (i + u * stride));
  }
  for (; i + 3 * stride < nvec; i += 4 * stride) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = nv[u];
    if (i + 7 * stride < nvec) {
#pragma unroll
      for (int u = 0; u < 4; ++u) nv[u] = ldg16(base + 16 * (i + (4 + u) * stride));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) encode_store(v[u], i + u * stride);
  }
  for (; i < nvec; i += stride) encode_store(ldg16(base + 16 * i), i);
  for (int64_t t = nvec * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += stride) {
    const float xv = load1<DT>(x, t);
    m = fmax_nan(m, fabsf(xv));
    codes[t] = (uint8_t)enc1_fp8<FMT>(div_ieee(xv, s));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmax_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) m = fmax_nan(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (threadIdx.x == 0 && __float_as_uint(m) != 0u) atomicMax(amax_bits, __float_as_uint(m));
  }
}

// Ring update: the entries move one place back and the new amax goes first.
__global__ void k_history_push(float* hist, int len, const uint32_t* amax_bits) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  for (int i = len - 1; i > 0; --i) hist[i] = hist[i - 1];
  hist[0] = canon_nan(__uint_as_float(*amax_bits));
}

}  // namespace delayed
}  // namespace brc

namespace {
template <int DT, int FMT>
struct DelayedCast {
  static int run(const void* x, int64_t n, float* hist, int len, int margin, uint8_t* codes,
                 float* scale_out, uint32_t* ws, cudaStream_t st) {
    using namespace brc::delayed;
    const double fmax = FMT == BRC_FP8_E4M3 ? 448.0 : 57344.0;
    const float floor_scale = (float)(1e-10 / fmax);
    k_history_scale<FMT><<<1, 32, 0, st>>>(hist, len, std::ldexp(1.0f, margin), floor_scale,
                                           scale_out);
    int rc = check_launch();
    if (rc) return rc;
    if ((rc = brc_amax_reset(ws, st))) return rc;
    if (n > 0) {
      const int V = In<DT>::kVec;
      k_delayed_apply<DT, FMT><<<grid_for(n / V + 1, 256 * 4), 256, 0, st>>>(x, n, scale_out,
                                                                          codes, ws);
      if ((rc = check_launch())) return rc;
    }
    k_history_push<<<1, 32, 0, st>>>(hist, len, ws);
    return check_launch();
  }
};
}  // namespace

namespace {
template <int DT, int FMT>
struct PrefixEncode {
  static int run(const void* x, int64_t n, const float* scale, uint8_t* codes, uint32_t* amax_ws,
                 cudaStream_t st) {
    const int V = In<DT>::kVec;
    brc::delayed::k_delayed_apply<DT, FMT>
        <<<grid_for(n / V + 1, 256 * 4), 256, 0, st>>>(x, n, scale, codes, amax_ws);
    return check_launch();
  }
};
}  // namespace

namespace brc {
int pertensor_fp8_scale(const void* x, int x_dtype, int64_t n, int fmt, const float* history,
                        int history_len, int margin, bool from_history, uint32_t* amax_ws,
                        float* scale_out, cudaStream_t st) {
  const double fmax = fmt == BRC_FP8_E4M3 ? 448.0 : 57344.0;
  const float floor_scale = (float)(1e-10 / fmax);
  if (!from_history) {
    // the current-amax scale: one amax pass, then the same float32 scale as
    // the apply kernel (a history of one entry holding the amax, margin 0)
    int rc = brc_amax_accumulate(x, x_dtype, n, amax_ws, st);
    if (rc) return rc;
    history = reinterpret_cast<const float*>(amax_ws);
    history_len = 1;
    margin = 0;
  }
  if (fmt == BRC_FP8_E4M3)
    delayed::k_history_scale<BRC_FP8_E4M3><<<1, 32, 0, st>>>(
        history, history_len, std::ldexp(1.0f, margin), floor_scale, scale_out);
  else
    delayed::k_history_scale<BRC_FP8_E5M2><<<1, 32, 0, st>>>(
        history, history_len, std::ldexp(1.0f, margin), floor_scale, scale_out);
  return check_launch();
}

int pertensor_fp8_encode(const void* x, int x_dtype, int64_t n, int fmt, const float* scale,
                         uint8_t* codes, uint32_t* amax_ws, cudaStream_t st) {
  if (n <= 0) return BRC_OK;
  return dispatch_dt_fmt<PrefixEncode>(x_dtype, fmt, x, n, scale, codes, amax_ws, st);
}

int pertensor_fp8_history_push(float* history, int history_len, const uint32_t* amax_ws,
                               cudaStream_t st) {
  delayed::k_history_push<<<1, 32, 0, st>>>(history, history_len, amax_ws);
  return check_launch();
}
}  // namespace brc

extern "C" int brc_cast_pertensor_fp8_delayed(const void* x, int x_dtype, int64_t n, int fmt,
                                              float* history, int history_len, int margin,
                                              int use_history, uint8_t* codes, float* scale_out,
                                              uint32_t* workspace, void* stream) {
  if (!history || !scale_out || !workspace || ((!x || !codes) && n > 0)) return BRC_ERR_NULL;
  if (!valid_dtype(x_dtype) || !valid_fmt(fmt)) return BRC_ERR_DTYPE;
  if (n < 0 || history_len < 1) return BRC_ERR_SHAPE;
  if (margin < -126 || margin > 127) return BRC_ERR_RANGE;
  if (n > 0 && (!aligned16(x) || !aligned16(codes))) return BRC_ERR_ALIGN;
  cudaStream_t st = (cudaStream_t)stream;
  if (!use_history) {
    // no history yet: the reference's current-amax cast, then record its amax
    int rc = brc_cast_pertensor_fp8(x, x_dtype, n, fmt, codes, scale_out, workspace, stream);
    if (rc) return rc;
    brc::delayed::k_history_push<<<1, 32, 0, st>>>(history, history_len, workspace);
    return check_launch();
  }
  return dispatch_dt_fmt<DelayedCast>(x_dtype, fmt, x, n, history, history_len, margin, codes,
                                      scale_out, workspace, st);
}
