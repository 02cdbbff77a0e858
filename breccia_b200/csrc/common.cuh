// Shared device numerics for the breccia_b200 kernels (sm_100a).
//
// Every encoder here reproduces the reference NumPy path bit for bit
// (jvoltci/breccia v0.1.3):
//   * FP8/FP4 encode = argmin |LUT - v| with the first (lowest) code winning
//     ties (src/breccia/_formats.py:117-174). For magnitudes that is
//     round-to-nearest with ties toward zero, saturating (np.clip) to the
//     format maximum; a value whose magnitude rounds to 0 gets code 0, never
//     the negative-zero code.
//   * Every scaled value is the IEEE float32 quotient x / scale
//     (src/breccia/kernels/reference/cast.py:371,398,438,488,532,557).
//
// Build WITHOUT --use_fast_math: the code relies on IEEE rounding of fmul,
// fadd, fma and on the directed-rounding intrinsics below.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "breccia_b200.h"

namespace brc {

// ------------------------------------------------------------ input types
// Inputs are float32, bfloat16 or float16 (BRC_DTYPE_*). A "vector" is 16
// bytes: 4 floats or 8 halves.
template <int DT> struct In;
template <> struct In<BRC_DTYPE_F32> { static constexpr int kVec = 4; };
template <> struct In<BRC_DTYPE_BF16> { static constexpr int kVec = 8; };
template <> struct In<BRC_DTYPE_F16> { static constexpr int kVec = 8; };

// Unpack one 16-byte vector into floats (exact conversions).
template <int DT>
__device__ __forceinline__ void unpack(const uint4 v, float* f);

template <>
__device__ __forceinline__ void unpack<BRC_DTYPE_F32>(const uint4 v, float* f) {
  f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
}

template <>
__device__ __forceinline__ void unpack<BRC_DTYPE_BF16>(const uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <>
__device__ __forceinline__ void unpack<BRC_DTYPE_F16>(const uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    const float2 g = __half22float2(h);
    f[2 * i] = g.x;
    f[2 * i + 1] = g.y;
  }
}

// ------------------------------------------------------------ reductions
// NaN-propagating max (np.max semantics): max.NaN returns NaN if either
// operand is NaN.
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ float fmin_nan(float a, float b) {
  float d;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// Abs-max of one 16-byte vector, NaN-propagating. bf16/f16 vectors are
// reduced pairwise in packed form before widening.
template <int DT>
__device__ __forceinline__ float vec_absmax(const uint4 v);

template <>
__device__ __forceinline__ float vec_absmax<BRC_DTYPE_F32>(const uint4 v) {
  return fmax_nan(fmax_nan(fabsf(__uint_as_float(v.x)), fabsf(__uint_as_float(v.y))),
                  fmax_nan(fabsf(__uint_as_float(v.z)), fabsf(__uint_as_float(v.w))));
}

__device__ __forceinline__ uint32_t bf16x2_max_nan(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t f16x2_max_nan(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

template <>
__device__ __forceinline__ float vec_absmax<BRC_DTYPE_BF16>(const uint4 v) {
  const uint32_t m = bf16x2_max_nan(bf16x2_max_nan(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu),
                                    bf16x2_max_nan(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu));
  return fmax_nan(__uint_as_float(m << 16), __uint_as_float(m & 0xFFFF0000u));
}

template <>
__device__ __forceinline__ float vec_absmax<BRC_DTYPE_F16>(const uint4 v) {
  const uint32_t m = f16x2_max_nan(f16x2_max_nan(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu),
                                   f16x2_max_nan(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu));
  const __half2 h = *reinterpret_cast<const __half2*>(&m);
  const float2 g = __half22float2(h);
  return fmax_nan(g.x, g.y);
}

// ------------------------------------------------------------ division
// Correctly rounded x / s from r = RN(1/s): one FMA residual and one FMA
// correction (Markstein, "Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990). Valid for
// finite non-zero s and results in the normal float range; callers route
// non-finite scales through div_ieee. Checked against IEEE division by
// tests/test_kernels_gpu.py.
__device__ __forceinline__ float div_by(float x, float s, float r) {
  const float q = __fmul_rn(x, r);
  const float e = __fmaf_rn(-q, s, x);
  return __fmaf_rn(e, r, q);
}
__device__ __forceinline__ float div_ieee(float x, float s) { return __fdiv_rn(x, s); }
// Four quotients f[i] / s in two packed pairs (mul.rn.f32x2 and fma.rn.f32x2
// round each element exactly as the scalar instructions do): the same three
// roundings per element as div_by, in half the FMA-pipe instructions.
__device__ __forceinline__ void div4(const float* f, float s, float r, float* q) {
  const float2 r2 = make_float2(r, r), ns2 = make_float2(-s, -s);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float2 x = make_float2(f[2 * h], f[2 * h + 1]);
    const float2 t = __fmul2_rn(x, r2);
    const float2 e = __ffma2_rn(t, ns2, x);  // x - t*s, one rounding
    const float2 y = __ffma2_rn(e, r2, t);
    q[2 * h] = y.x;
    q[2 * h + 1] = y.y;
  }
}

// IEEE x / d for a constant d with rd = RN(1/d): Markstein's step for finite
// x (the callers' x are amax values floored at 1e-10, so the quotient is a
// normal float), the division itself for inf and NaN.
constexpr float kRcp448 = 0x1.24924ap-9f;    // RN(1/448), bits 0x3B124925
constexpr float kRcp57344 = 0x1.24924ap-16f; // RN(1/57344), bits 0x37924925
constexpr float kRcp6 = 0x1.555556p-3f;      // RN(1/6), bits 0x3E2AAAAB
constexpr float kRcp7 = 0x1.24924ap-3f;      // RN(1/7), bits 0x3E124925
constexpr float kRcp15 = 0x1.111112p-4f;     // RN(1/15), bits 0x3D888889
__device__ __forceinline__ float div_const(float x, float d, float rd) {
  return isfinite(x) ? div_by(x, d, rd) : __fdiv_rn(x, d);
}

// ------------------------------------------------------------ FP8 / FP4 encode
// Magnitude encoders. The float is first scaled by a power of two that puts
// the format's smallest normal at float32's smallest normal (2^-126), with
// rounding toward +inf. Above that boundary the scaling is exact; below it
// the product is a float32 subnormal whose bits are the format's subnormal
// mantissa followed by the dropped bits, and rounding up keeps every value
// that lies above a midpoint above it. Adding (half - 1) to the bit pattern
// and truncating then rounds to nearest with ties toward zero, with the
// mantissa carry stepping into the exponent. The result is returned in the
// top byte of a word (so four codes pack with byte permutes).
//
// Callers clamp |v| to the format maximum first (np.clip).

// E4M3: 3 mantissa bits; smallest normal 2^-6 -> factor 2^-120; code in bits
// [20,28) of the scaled pattern.
__device__ __forceinline__ uint32_t e4m3_mag_hi(float mag_clamped) {
  const float t = __fmul_ru(mag_clamped, 0x1p-120f);
  return (__float_as_uint(t) << 4) + 0x007FFFF0u;  // top byte = code
}
// E5M2: 2 mantissa bits; smallest normal 2^-14 -> factor 2^-112; code in bits
// [21,29).
__device__ __forceinline__ uint32_t e5m2_mag_hi(float mag_clamped) {
  const float t = __fmul_ru(mag_clamped, 0x1p-112f);
  return (__float_as_uint(t) << 3) + 0x007FFFF8u;
}
// E2M1: 1 mantissa bit; smallest normal 1 -> factor 2^-126; code in bits
// [22,26).
__device__ __forceinline__ uint32_t e2m1_mag_hi(float mag_clamped) {
  const float t = __fmul_ru(mag_clamped, 0x1p-126f);
  return (__float_as_uint(t) << 2) + 0x007FFFFCu;
}

// Pack the top bytes of four words into one word (byte i <- word i).
__device__ __forceinline__ uint32_t pack_top_bytes(uint32_t a, uint32_t b, uint32_t c,
                                                   uint32_t d) {
  const uint32_t ab = __byte_perm(a, b, 0x0073);  // [a.b3, b.b3, a.b0, a.b0]
  const uint32_t cd = __byte_perm(c, d, 0x0073);
  return __byte_perm(ab, cd, 0x5410);
}
// PTX prmt in its default mode: a selector nibble with bit 3 set replicates
// the sign bit of the selected byte into the whole result byte.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
// 0xFF in byte i where value i is negative.
__device__ __forceinline__ uint32_t sign_bytes(float a, float b, float c, float d) {
  const uint32_t ab = prmt(__float_as_uint(a), __float_as_uint(b), 0x00FB);
  const uint32_t cd = prmt(__float_as_uint(c), __float_as_uint(d), 0x00FB);
  return prmt(ab, cd, 0x5410);
}

// Four FP8 codes (magnitudes < 0x80 in w) plus signs; a zero magnitude keeps
// code 0 whatever the sign.
__device__ __forceinline__ uint32_t apply_sign8(uint32_t w, uint32_t neg) {
  const uint32_t nz = w + 0x7F7F7F7Fu;  // bit 7 of a byte set iff byte != 0
  return w | (neg & nz & 0x80808080u);
}
// Four FP4 codes, one per byte (magnitudes < 8), plus signs in bit 3.
__device__ __forceinline__ uint32_t apply_sign4(uint32_t w, uint32_t neg) {
  const uint32_t nz = w + 0x07070707u;  // bit 3 of a byte set iff byte != 0
  return w | (neg & nz & 0x08080808u);
}

// Encode four already-divided values to E4M3 / E5M2 / E2M1 codes, one byte
// each. Values must not be NaN (callers route NaN blocks elsewhere).
__device__ __forceinline__ uint32_t enc4_e4m3(float a, float b, float c, float d) {
  const uint32_t w = pack_top_bytes(e4m3_mag_hi(fminf(fabsf(a), 448.f)),
                                    e4m3_mag_hi(fminf(fabsf(b), 448.f)),
                                    e4m3_mag_hi(fminf(fabsf(c), 448.f)),
                                    e4m3_mag_hi(fminf(fabsf(d), 448.f)));
  return apply_sign8(w, sign_bytes(a, b, c, d));
}
__device__ __forceinline__ uint32_t enc4_e5m2(float a, float b, float c, float d) {
  const uint32_t w = pack_top_bytes(e5m2_mag_hi(fminf(fabsf(a), 57344.f)),
                                    e5m2_mag_hi(fminf(fabsf(b), 57344.f)),
                                    e5m2_mag_hi(fminf(fabsf(c), 57344.f)),
                                    e5m2_mag_hi(fminf(fabsf(d), 57344.f)));
  return apply_sign8(w, sign_bytes(a, b, c, d));
}
__device__ __forceinline__ uint32_t enc4_e2m1(float a, float b, float c, float d) {
  const uint32_t w = pack_top_bytes(e2m1_mag_hi(fminf(fabsf(a), 6.f)),
                                    e2m1_mag_hi(fminf(fabsf(b), 6.f)),
                                    e2m1_mag_hi(fminf(fabsf(c), 6.f)),
                                    e2m1_mag_hi(fminf(fabsf(d), 6.f)));
  return apply_sign4(w, sign_bytes(a, b, c, d));
}

// Packed forms of the encoders above (same codes): the round-up scaling of the
// *_mag_hi encoders two values per packed multiply (mul.ru.f32x2), then the
// same bit step. They halve the FMA-pipe work of instruction-bound casts
// (NVFP4, the 2-D block cast); an HBM-bound pass (the per-tensor encode)
// measured 5% slower with them, so the scalar forms remain: SHIFT and the (half - 1)
// addend are the encoders' (4 / 0x007FFFF0 E4M3, 3 / 0x007FFFF8 E5M2,
// 2 / 0x007FFFFC E2M1).
template <int SHIFT, uint32_t ADD>
__device__ __forceinline__ uint32_t enc4_mag(float ma, float mb, float mc, float md,
                                             float factor) {
  const float2 f2 = make_float2(factor, factor);
  const float2 t01 = __fmul2_ru(make_float2(ma, mb), f2);
  const float2 t23 = __fmul2_ru(make_float2(mc, md), f2);
  return pack_top_bytes((__float_as_uint(t01.x) << SHIFT) + ADD,
                        (__float_as_uint(t01.y) << SHIFT) + ADD,
                        (__float_as_uint(t23.x) << SHIFT) + ADD,
                        (__float_as_uint(t23.y) << SHIFT) + ADD);
}
__device__ __forceinline__ uint32_t enc4p_e4m3(float a, float b, float c, float d) {
  const uint32_t w = enc4_mag<4, 0x007FFFF0u>(fminf(fabsf(a), 448.f), fminf(fabsf(b), 448.f),
                                             fminf(fabsf(c), 448.f), fminf(fabsf(d), 448.f),
                                             0x1p-120f);
  return apply_sign8(w, sign_bytes(a, b, c, d));
}
__device__ __forceinline__ uint32_t enc4p_e5m2(float a, float b, float c, float d) {
  const uint32_t w = enc4_mag<3, 0x007FFFF8u>(fminf(fabsf(a), 57344.f), fminf(fabsf(b), 57344.f),
                                             fminf(fabsf(c), 57344.f), fminf(fabsf(d), 57344.f),
                                             0x1p-112f);
  return apply_sign8(w, sign_bytes(a, b, c, d));
}
__device__ __forceinline__ uint32_t enc4p_e2m1(float a, float b, float c, float d) {
  const uint32_t w = enc4_mag<2, 0x007FFFFCu>(fminf(fabsf(a), 6.f), fminf(fabsf(b), 6.f),
                                             fminf(fabsf(c), 6.f), fminf(fabsf(d), 6.f),
                                             0x1p-126f);
  return apply_sign4(w, sign_bytes(a, b, c, d));
}

template <int FMT>
__device__ __forceinline__ uint32_t enc4_fp8(float a, float b, float c, float d) {
  if constexpr (FMT == BRC_FP8_E4M3) return enc4_e4m3(a, b, c, d);
  else return enc4_e5m2(a, b, c, d);
}
template <int FMT>
__device__ __forceinline__ uint32_t enc4p_fp8(float a, float b, float c, float d) {
  if constexpr (FMT == BRC_FP8_E4M3) return enc4p_e4m3(a, b, c, d);
  else return enc4p_e5m2(a, b, c, d);
}
// Encode f[0..3] / s (r = RN(1/s)) with one of the four-value encoders:
// quotients and scaling both in packed pairs.
template <uint32_t (*ENC)(float, float, float, float)>
__device__ __forceinline__ uint32_t enc4_div(const float* f, float s, float r) {
  float q[4];
  div4(f, s, r, q);
  return ENC(q[0], q[1], q[2], q[3]);
}

// Single-value encoders with full NaN / inf handling (scale paths and the
// non-finite slow path). NaN -> 0x7F (E4M3), 0x7D (E5M2), 0 (E2M1): the
// reference overwrites NaN positions after the LUT search.
__device__ __forceinline__ uint32_t enc1_e4m3(float v) {
  if (isnan(v)) return 0x7Fu;
  const uint32_t m = e4m3_mag_hi(fminf(fabsf(v), 448.f)) >> 24;
  return (m && signbit(v)) ? (m | 0x80u) : m;
}
__device__ __forceinline__ uint32_t enc1_e5m2(float v) {
  if (isnan(v)) return 0x7Du;
  const uint32_t m = e5m2_mag_hi(fminf(fabsf(v), 57344.f)) >> 24;
  return (m && signbit(v)) ? (m | 0x80u) : m;
}
__device__ __forceinline__ uint32_t enc1_e2m1(float v) {
  if (isnan(v)) return 0u;
  const uint32_t m = e2m1_mag_hi(fminf(fabsf(v), 6.f)) >> 24;
  return (m && signbit(v)) ? (m | 0x8u) : m;
}
template <int FMT>
__device__ __forceinline__ uint32_t enc1_fp8(float v) {
  if constexpr (FMT == BRC_FP8_E4M3) return enc1_e4m3(v);
  else return enc1_e5m2(v);
}

// ------------------------------------------------------------ decode
// Exact decoders (src/breccia/_formats.py:41-99 tables, computed from bits).
__device__ __forceinline__ float dec_e4m3(uint32_t c) {
  const uint32_t e = (c >> 3) & 0xF, m = c & 7;
  float v;
  if (e == 15 && m == 7) return __uint_as_float(0x7FC00000u);  // unsigned NaN, as the LUT
  if (e == 0) v = (float)m * 0x1p-9f;
  else v = __uint_as_float(((e + 120u) << 23) | (m << 20));
  return (c & 0x80) ? -v : v;
}
__device__ __forceinline__ float dec_e5m2(uint32_t c) {
  const uint32_t e = (c >> 2) & 0x1F, m = c & 3;
  float v;
  if (e == 31 && m) return __uint_as_float(0x7FC00000u);  // unsigned NaN, as the LUT
  if (e == 31) v = __uint_as_float(0x7F800000u);
  else if (e == 0) v = (float)m * 0x1p-16f;
  else v = __uint_as_float(((e + 112u) << 23) | (m << 21));
  return (c & 0x80) ? -v : v;
}
__device__ __forceinline__ float dec_e2m1(uint32_t c) {
  const uint32_t e = (c >> 1) & 3, m = c & 1;
  const float v = (e == 0) ? (m ? 0.5f : 0.f) : __uint_as_float(((e + 126u) << 23) | (m << 22));
  return (c & 0x8) ? -v : v;
}
template <int FMT>
__device__ __forceinline__ float dec_fp8(uint32_t c) {
  if constexpr (FMT == BRC_FP8_E4M3) return dec_e4m3(c);
  else return dec_e5m2(c);
}

// FP8 pairs to f16 pairs by the hardware conversion: every E4M3 / E5M2 value
// (subnormals, infinities and NaN included) is exact in float16 and again in
// float32, so a float32 product of the decoded value rounds exactly once, as
// the reference's decode-then-multiply does. Byte i of the pair lands in half i.
template <int FMT>
__device__ __forceinline__ uint32_t fp8x2_to_f16x2(uint32_t two) {
  uint32_t d;
  const uint16_t b = (uint16_t)two;
  if constexpr (FMT == BRC_FP8_E4M3) asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(b));
  else asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(d) : "h"(b));
  return d;
}
// Two E2M1 codes (one per byte, low nibbles) to f16 pairs, exactly.
__device__ __forceinline__ uint32_t e2m1_bytes_to_f16x2(uint32_t two) {
  uint32_t d;
  const uint32_t pair = (two & 0x0Fu) | ((two >> 4) & 0xF0u);
  asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
      : "=r"(d)
      : "r"(pair));
  return d;
}
__device__ __forceinline__ void f16x2_to_f32(uint32_t h, float& lo, float& hi) {
  const __half2 v = *reinterpret_cast<const __half2*>(&h);
  lo = __low2float(v);
  hi = __high2float(v);
}

// ------------------------------------------------------------ E8M0
// E8M0 exponent of a float32 scale exactly as numpy computes
// round(log2(max(s, 1e-10f))) + 127 clipped to [0, 255]
// (src/breccia/kernels/reference/_utils.py:40-50). numpy's float32 log2
// rounds to the next exponent at a mantissa that differs per binade by a few
// ulps from sqrt(2); `thr[k + 33]` holds that mantissa for binade k in
// [-33, 127] (generated from numpy by gen_e8m0_thresholds.py).
constexpr int kE8m0Binades = 161;

__device__ __forceinline__ uint32_t e8m0_code(float s, const uint32_t* thr) {
  if (!(s == s)) return 0u;        // NaN: numpy's float->int32 gives INT_MIN -> clip 0
  if (isinf(s)) return 0u;         // +inf: same conversion
  const uint32_t b = __float_as_uint(s);
  const int k = (int)((b >> 23) & 0xFF) - 127;
  if (k < -33) return 94u;         // s < 2^-33 (incl. the 1e-10 floor) -> 94
  const uint32_t m = b & 0x7FFFFFu;
  return (uint32_t)(127 + k) + (m >= thr[k + 33] ? 1u : 0u);
}

// ------------------------------------------------------------ NaN payloads
// GPU arithmetic returns the canonical NaN 0x7FFFFFFF; NumPy propagates the
// input's quiet NaN, which for NaN values created by NumPy or torch is
// 0x7FC00000 (float16: 0x7E00). Stored scales and zero points use those.
__device__ __forceinline__ float canon_nan(float v) {
  return isnan(v) ? __uint_as_float(0x7FC00000u) : v;
}
__device__ __forceinline__ __half to_half_canon(float v) {
  return isnan(v) ? __ushort_as_half((unsigned short)0x7E00u) : __float2half_rn(v);
}

// ------------------------------------------------------------ misc
__device__ __forceinline__ uint4 ldg16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// L2 policy that makes lines the first candidates for eviction: for data a
// kernel touches for the last time, so that it does not displace lines that
// are about to be read again.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint4 ldg16_last_use(const void* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ void stg8_last_use(void* p, uint32_t a, uint32_t b, uint64_t pol) {
  asm volatile("st.global.L1::no_allocate.L2::cache_hint.v2.u32 [%0], {%1,%2}, %3;" ::"l"(p),
               "r"(a), "r"(b), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void stg16(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

}  // namespace brc
