// Deterministic fp32 arithmetic of the routing and activation-quantization steps.
//
// Every function here is a fixed sequence of IEEE-754 binary32 operations with
// round-to-nearest-even (the __f*_rn intrinsics, so no contraction or fast-math
// rewrite applies), plus exact bit manipulations. The CPU oracle evaluates the
// same sequences with C99 float arithmetic and fmaf, so scores, routing keys,
// top-k ids, routing weights and MX scale/code bytes match it bit for bit.
//
// Reference numerics followed:
//  * routing keys, ties and NaN rules: deepseek_v41/sm103/moe/src/gate_topk.cuh:129-145
//    (order-preserving u32 key of score + bias, -0 ranked as +0) and
//    glm5_3/sm103/primitives/ptx_tc.py:393-402 (NaN ranks as -inf);
//    the lowest expert id wins a tie (gate_topk.cuh:211-290, routing.py:32-70).
//  * weights: gate_topk.cuh:187-198 (score / (sum + eps) or the guarded sum, then
//    the routed scale); glm5_3/sm103/moe/routing.py:3-11 (sigmoid + bias, renorm).
//  * MX quantization: deepseek_v41/sm103/moe/src/route_quant.cuh:1-15 and
//    gemm1.cu:905-1000 (block-32 amax, times fp32(1/448), E8M0 rounded up,
//    multiply by the exact inverse power of two, e4m3 RN satfinite); the same
//    rule with E2M1 codes (largest magnitude 6, fp32(1/6)) for the MXFP4 terms
//    of the activations.
// The sigmoid and sqrt(softplus) use this file's own exp and log (Cody-Waite
// reduction + Taylor polynomial; atanh series) instead of the reference's
// tanh.approx / libm / approximate-reciprocal sequences, whose bits no CPU code
// can reproduce; everything else is the reference's rule.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include <cuda_bf16.h>

namespace mm {

// exp(x): x = n ln2 + r with n = rint(x log2e) and r by a two-constant
// Cody-Waite reduction, e^r by the degree-7 Taylor polynomial in Horner form,
// then an exact scaling by 2^n (two steps outside the normal exponent range).
__device__ __forceinline__ float det_exp(float x) {
  if (x != x) return x;
  if (x > 0x1.62e430p+6f) return __int_as_float(0x7f800000);
  if (x < -0x1.a00000p+6f) return 0.0f;  // below -104: under half the least subnormal
  const float kLog2e = 0x1.715476p+0f;
  const float kMagic = 0x1.8p+23f;  // adding 1.5 * 2^23 rounds to an integer
  const float kLn2Hi = 0x1.62e400p-1f;
  const float kLn2Lo = 0x1.7f7d1cp-20f;
  const float t = __fmaf_rn(x, kLog2e, kMagic);
  const float n = __fsub_rn(t, kMagic);
  float r = __fmaf_rn(-n, kLn2Hi, x);
  r = __fmaf_rn(-n, kLn2Lo, r);
  float p = 0x1.a01a02p-13f;  // 1/5040
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);  // 1/720
  p = __fmaf_rn(p, r, 0x1.111112p-7f);   // 1/120
  p = __fmaf_rn(p, r, 0x1.555556p-5f);   // 1/24
  p = __fmaf_rn(p, r, 0x1.555556p-3f);   // 1/6
  p = __fmaf_rn(p, r, 0x1.000000p-1f);   // 1/2
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = static_cast<int>(n);
  if (ni > 127) return __fmul_rn(__fmul_rn(p, __int_as_float((ni - 1 + 127) << 23)), 2.0f);
  if (ni < -126)
    return __fmul_rn(__fmul_rn(p, __int_as_float((ni + 100 + 127) << 23)),
                     __int_as_float((-100 + 127) << 23));
  return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

__device__ __forceinline__ float det_sigmoid(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, det_exp(-x)));
}

// log(u) for finite u >= 1: u = m 2^k with m in [sqrt(1/2), sqrt(2)), log u =
// k ln2 + 2 atanh(f / (2 + f)), f = m - 1 (exact), atanh(s) = s (1 + z/3 +
// z^2/5 + z^3/7 + z^4/9 + z^5/11), z = s^2 (|s| <= 0.172: the next term is
// below fp32 resolution); ln2 split in two constants as in det_exp.
__device__ __forceinline__ float det_log(float u) {
  const uint32_t bits = __float_as_uint(u);
  int k = static_cast<int>((bits >> 23) & 0xffu) - 127;
  float m = __uint_as_float((bits & 0x7fffffu) | 0x3f800000u);
  if (m > 0x1.6a09e6p+0f) {
    m = __fmul_rn(m, 0.5f);
    k += 1;
  }
  const float f = __fsub_rn(m, 1.0f);
  const float s = __fdiv_rn(f, __fadd_rn(2.0f, f));
  const float z = __fmul_rn(s, s);
  float q = 0x1.745d18p-4f;              // 1/11
  q = __fmaf_rn(q, z, 0x1.c71c72p-4f);   // 1/9
  q = __fmaf_rn(q, z, 0x1.24924ap-3f);   // 1/7
  q = __fmaf_rn(q, z, 0x1.99999ap-3f);   // 1/5
  q = __fmaf_rn(q, z, 0x1.555556p-2f);   // 1/3
  q = __fmaf_rn(q, z, 1.0f);
  const float lm = __fmul_rn(__fadd_rn(s, s), q);
  const float kf = static_cast<float>(k);
  return __fmaf_rn(kf, 0x1.62e400p-1f, __fmaf_rn(kf, 0x1.7f7d1cp-20f, lm));
}

// log1p(y) for y >= 0 (Goldberg's form): u = 1 + y; y when u == 1, else
// log(u) * (y / (u - 1)), which cancels the rounding of 1 + y.
__device__ __forceinline__ float det_log1p(float y) {
  const float u = __fadd_rn(1.0f, y);
  if (u == 1.0f) return y;
  return __fmul_rn(det_log(u), __fdiv_rn(y, __fsub_rn(u, 1.0f)));
}

// sqrt(softplus(x)), the DeepSeek-V4.1 router score (gate_topk.cuh:99-104):
// softplus(x) = x above 20, else log1p(exp(x)); the square root is IEEE.
__device__ __forceinline__ float det_sqrtsoftplus(float x) {
  if (x != x) return x;
  const float sp = x > 20.0f ? x : det_log1p(det_exp(x));
  return __fsqrt_rn(sp);
}

// Order-preserving key of v (larger key = better candidate); -0 ranks as +0
// and NaN ranks below every number (key 0).
__device__ __forceinline__ uint32_t routing_key(float v) {
  if (v != v) return 0u;
  const uint32_t bits = __float_as_uint(__fadd_rn(v, 0.0f));
  return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}

// ---- MXFP8 (E4M3 codes + E8M0 block scale) ------------------------------------
// E8M0 code of a block whose absolute maximum is `amax`: the exponent of
// amax * fp32(1/448), rounded up when the mantissa is non-zero.
__device__ __forceinline__ uint32_t mx_scale_code(float amax) {
  const float numerator = amax == 0.0f ? 448.0f : amax;
  const uint32_t bits = __float_as_uint(__fmul_rn(numerator, 0x1.24924ap-9f));
  const uint32_t exponent = (bits >> 23) & 0xffu;
  const uint32_t mantissa = bits & 0x7fffffu;
  uint32_t code = exponent;
  if (mantissa != 0u && exponent != 254u) {
    if (exponent != 0u) code = exponent + 1u;
    else if (mantissa > 0x400000u) code = 1u;
  }
  if (exponent == 255u) code = 255u;
  return code;
}
// E8M0 code of an MXFP4 block (E2M1 codes, largest magnitude 6): the exponent of
// amax * fp32(1/6), rounded up when the mantissa is non-zero (a zero block gets
// scale 1), so amax / scale never exceeds 6 by more than the rounding of 1/6.
__device__ __forceinline__ uint32_t mx4_scale_code(float amax) {
  const float numerator = amax == 0.0f ? 6.0f : amax;
  const uint32_t bits = __float_as_uint(__fmul_rn(numerator, 0x1.555556p-3f));
  const uint32_t exponent = (bits >> 23) & 0xffu;
  const uint32_t mantissa = bits & 0x7fffffu;
  uint32_t code = exponent;
  if (mantissa != 0u && exponent != 254u) {
    if (exponent != 0u) code = exponent + 1u;
    else if (mantissa > 0x400000u) code = 1u;
  }
  if (exponent == 255u) code = 255u;
  return code;
}
// 2^(127 - code): the exact multiplier that maps the block into E4M3 range.
__device__ __forceinline__ float mx_inverse(uint32_t code) {
  return code == 254u ? __uint_as_float(0x400000u) : __uint_as_float((254u - code) << 23);
}
// 2^(code - 127).
__device__ __forceinline__ float mx_scale_value(uint32_t code) {
  return code == 0u ? __uint_as_float(0x400000u) : __uint_as_float(code << 23);
}
// Two floats -> two E4M3 codes (RN, saturating to +-448); lo in the low byte.
__device__ __forceinline__ uint16_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float e4m3_value(uint8_t code) {
  // exact decode of an E4M3 (fn) byte
  const uint32_t s = code >> 7, e = (code >> 3) & 15u, m = code & 7u;
  float v;
  if (e == 0u) v = static_cast<float>(m) * 0x1p-9f;
  else if (e == 15u && m == 7u) v = __uint_as_float(0x7fc00000u);
  else v = __uint_as_float(((e + 120u) << 23) | (m << 20));
  return s ? -v : v;
}

// NVFP4 block scale of a 16-element block with absolute maximum amax under
// the global scale gs: the E4M3 byte of gs * (amax * fp32(1/6)), RN, saturating
// to 448 (the reference's rule, glm5_3/sm103/primitives/ptx_tc.py:320-337,
// written with IEEE operations where the reference uses approximate ones).
__device__ __forceinline__ uint32_t nv4_scale_code(float amax, float gs) {
  const float s = __fmul_rn(gs, __fmul_rn(amax, 0x1.555556p-3f));
  return static_cast<uint32_t>(e4m3x2(s, 0.0f) & 0xffu);
}
// The multiplier mapping a block onto E2M1: gs / sf (IEEE), 0 for a zero scale.
__device__ __forceinline__ float nv4_multiplier(float sf, float gs) {
  return sf == 0.0f ? 0.0f : __fdiv_rn(gs, sf);
}

// Two floats -> one byte of two E2M1 codes (RN, saturating to +-6); lo in bits 0-3.
__device__ __forceinline__ uint32_t e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tcvt.u32.u8 %0, t;\n\t}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r & 0xffu;
}
// exact value of an E2M1 code (bits 0-3): the hardware conversion of the code,
// as the low nibble of an e2m1x2 byte, to the low half of an f16x2 (every E2M1
// value, 0 0.5 1 1.5 2 3 4 6 and their negatives, is exact in f16)
__device__ __forceinline__ float e2m1_value(uint32_t code) {
  uint32_t h2;
  asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(h2) : "r"(code & 15u));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xffffu)));
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
__device__ __forceinline__ uint16_t float_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

}  // namespace mm
