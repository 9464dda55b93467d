// MXFP8 quantization arithmetic shared by the standalone quantizer and the
// GEMV that quantizes its activations on the fly (bit-identical results):
// per 32 values, the UE8M0 code of ceil(log2(amax / 448)) and E4M3 values
// rounded to nearest even with saturation (quantize_fp8.py:23-39).
#pragma once

#include "common.cuh"

namespace mambo {

// Exact MXFP8 block exponent from the float bits of amax (amax >= 0).
// Returns the UE8M0 scale code, 0xFF for a non-finite amax.
__device__ __forceinline__ uint32_t mxfp8_scale_code(float amax) {
  const uint32_t bits = __float_as_uint(amax);
  const uint32_t biased = bits >> 23;  // sign is 0
  if (bits == 0) return 127u;          // amax == 0 -> e = 0
  if (biased == 0xFF) return 0xFFu;    // Inf / NaN
  if (biased == 0) return 0u;          // subnormal amax -> e clamps to -127
  // amax = 1.m * 2^(biased-127); 448 = 1.75 * 2^8.
  int e = (int)biased - 127 - ((bits & 0x7FFFFFu) <= 0x600000u ? 8 : 7);
  e = max(-127, min(127, e));
  return (uint32_t)(e + 127);
}

// Two floats -> two E4M3 bytes (lo in bits 0..7), round-to-nearest-even, saturating.
__device__ __forceinline__ uint32_t cvt_e4m3x2_rn(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// The largest magnitude of a 32-value group held by 4 consecutive lanes (8
// values each; the quad must be converged), the same in all four lanes. The
// magnitudes' bit patterns are compared as unsigned integers: for numbers
// that is their order, and every NaN orders above infinity, so a NaN anywhere
// in the group reaches every lane (and gives the group the scale code 0xFF).
__device__ __forceinline__ float quad_absmax(const float (&v)[8]) {
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = max(m, __float_as_uint(v[i]) & 0x7FFFFFFFu);
  m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
  m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
  return __uint_as_float(m);
}

// One 32-value group held by 4 consecutive lanes (8 values each; the quad
// must be converged): returns the group's scale code and this lane's 8 E4M3
// bytes (value i in byte i % 4 of word i / 4), round-to-nearest-even.
__device__ __forceinline__ uint32_t mxfp8_quad_rne(const float (&v)[8], uint2& out) {
  const uint32_t code = mxfp8_scale_code(quad_absmax(v));
  // 2^-e with e = code - 127 (code 0xFF: scale by 2^-127, values become 0 / NaN / +-448).
  const float inv = e8m0_to_float(code == 0xFFu ? 0u : 254u - code);
  uint32_t packed[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t lo = cvt_e4m3x2_rn(v[4 * h] * inv, v[4 * h + 1] * inv);
    const uint32_t hi = cvt_e4m3x2_rn(v[4 * h + 2] * inv, v[4 * h + 3] * inv);
    packed[h] = lo | (hi << 16);
  }
  out = make_uint2(packed[0], packed[1]);
  return code;
}

// Per half: the larger magnitude of a and b, NaN if either is NaN (sign bits unspecified).
__device__ __forceinline__ uint32_t absmax_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// One 32-value group of bf16 held by 4 consecutive lanes (c: this lane's 8
// values, the even one of each pair in the low half; the quad must be
// converged): returns the group's scale code and this lane's 8 E4M3 bytes, as
// mxfp8_quad_rne on the widened values.
__device__ __forceinline__ uint32_t mxfp8_quad_bf16_rne(const uint4& c, uint2& q) {
  uint32_t a = absmax_bf16x2(absmax_bf16x2(c.x, c.y), absmax_bf16x2(c.z, c.w));
  a = absmax_bf16x2(a, __shfl_xor_sync(0xFFFFFFFFu, a, 1));
  a = absmax_bf16x2(a, __shfl_xor_sync(0xFFFFFFFFu, a, 2));
  const uint32_t mb = max(a & 0x7FFFu, (a >> 16) & 0x7FFFu);
  const uint32_t code = mxfp8_scale_code(__uint_as_float(mb << 16));
  const float inv = e8m0_to_float(code == 0xFFu ? 0u : 254u - code);
  const uint32_t w4[4] = {c.x, c.y, c.z, c.w};
  uint32_t b[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float lo, hi;
    mul2(lo, hi, __uint_as_float(w4[j] << 16), __uint_as_float(w4[j] & 0xFFFF0000u), inv, inv);
    b[j] = cvt_e4m3x2_rn(lo, hi);
  }
  q = make_uint2(prmt(b[0], b[1], 0x5410u), prmt(b[2], b[3], 0x5410u));
  return code;
}

// One 32-value group of bf16 held by one lane (c[i]: values 8i .. 8i+7, two
// per word, the even one in the low half): returns the scale code and the
// 32 E4M3 bytes (q[i]: those of c[i], as mxfp8_quad_rne packs them). The same
// results as mxfp8_quad_rne on the widened values: the largest magnitude comes
// from a bf16x2 maximum of absolute values that propagates NaN (the magnitude
// is one of the inputs, exactly), and each product is one round-to-nearest
// FP32 multiply, two per packed instruction.
__device__ __forceinline__ uint32_t mxfp8_group32_bf16_rne(const uint4 (&c)[4], uint2 (&q)[4]) {
  uint32_t m4[4];  // a tree of maxima: a short dependency chain
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t a = absmax_bf16x2(c[i].x, c[i].y), b = absmax_bf16x2(c[i].z, c[i].w);
    m4[i] = absmax_bf16x2(a, b);
  }
  const uint32_t mx = absmax_bf16x2(absmax_bf16x2(m4[0], m4[1]), absmax_bf16x2(m4[2], m4[3]));
  const uint32_t mb = max(mx & 0x7FFFu, (mx >> 16) & 0x7FFFu);  // the result's sign bits are not used
  const uint32_t code = mxfp8_scale_code(__uint_as_float(mb << 16));
  const float inv = e8m0_to_float(code == 0xFFu ? 0u : 254u - code);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w4[4] = {c[i].x, c[i].y, c[i].z, c[i].w};
    uint32_t b[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float lo, hi;
      mul2(lo, hi, __uint_as_float(w4[j] << 16), __uint_as_float(w4[j] & 0xFFFF0000u), inv, inv);
      b[j] = cvt_e4m3x2_rn(lo, hi);
    }
    q[i] = make_uint2(prmt(b[0], b[1], 0x5410u), prmt(b[2], b[3], 0x5410u));
  }
  return code;
}

}  // namespace mambo
