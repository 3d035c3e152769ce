// Per-token e4m3 quantisation arithmetic shared by the standalone quantiser
// (fp8_quant.cu) and the FFN kernel that requantises its intermediate
// (ffn_fused.cu).  It follows _quantize_activation_torch
// (src/vflash/native/h3_fp8_linear.py:18-31) and the Triton _rows_fp8 kernel
// (src/vflash/native/h3_fp8_activation.py:13-28) bit for bit:
//   amax  = max |x| over the row (fp32)
//   scale = amax > 0 ? max(amax / 448, FLT_MIN) : 1      (IEEE division)
//   code  = e4m3_rn(clamp(x / scale, -448, 448))         (correctly rounded quotient)
#pragma once

#include <cfloat>

#include "common.cuh"

namespace vfb {

__device__ __forceinline__ float row_scale(float amax, bool nan) {
  if (nan || !(amax > 0.0f)) return 1.0f;
  return fmaxf(__fdiv_rn(amax, 448.0f), FLT_MIN);
}

// Correctly rounded x / scale for a finite, normal scale (the row scale is
// >= FLT_MIN by construction) given recip = RN(1 / scale).  Markstein's
// theorem (P. Markstein, "Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990): when recip is
// the correctly rounded reciprocal and q = RN(x * recip) is within one ulp
// of x / scale, the remainder x - q * scale is exact under FMA and
// RN(q + remainder * recip) is the correctly rounded quotient.  Quotients
// small enough to lose precision to fp32 underflow lie far below half the
// smallest e4m3 subnormal, so their codes (signed zero) are unaffected.
// The remainder is formed negated, q * scale - x (exact, the negation of
// x - q * scale), so the correction -rem_neg * recip + q keeps the sign of a
// zero quotient: -0 / scale = -0 without a separate sign copy.
__device__ __forceinline__ float div_rn_by_scale(float x, float scale, float recip) {
  const float q = x * recip;
  const float rem_neg = fmaf(q, scale, -x);
  return fmaf(-rem_neg, recip, q);
}

// Whether a row may use div_rn_by_scale.  Its remainder is inf - inf for an
// infinite x, and a row holds an infinity only when its scale is inf (amax =
// inf) or 1 (a NaN in the row makes amax NaN, and the reference clamps the
// row's +-inf to +-448).  Such rows take the IEEE division, which for a scale
// of 1 is x itself; a row of finite values gets the same bits either way.
__device__ __forceinline__ bool markstein_ok(float scale) { return isfinite(scale) && scale != 1.0f; }

// Quotient used for the codes: exact division routine for non-finite scales.
__device__ __forceinline__ float quotient(float x, float scale, float recip, bool fast) {
  return fast ? div_rn_by_scale(x, scale, recip) : __fdiv_rn(x, scale);
}

// The clamp to [-448, 448] of the reference is the saturation of
// cvt.rn.satfinite.e4m3x2 (finite values beyond 448 and infinities become
// +-448, NaN stays NaN), so no separate clamp is applied.

// Codes of 8 bf16 values (one 16-byte vector) for a finite scale.
__device__ __forceinline__ uint2 quantize8(const uint4 &v, float scale, float recip) {
  const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&v);
  uint16_t q[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f = __bfloat1622float2(h[j]);
    q[j] = pack_e4m3x2(div_rn_by_scale(f.x, scale, recip), div_rn_by_scale(f.y, scale, recip));
  }
  return make_uint2(static_cast<uint32_t>(q[0]) | (static_cast<uint32_t>(q[1]) << 16),
                    static_cast<uint32_t>(q[2]) | (static_cast<uint32_t>(q[3]) << 16));
}

// Same for a non-finite scale (a row containing +-inf): IEEE division.
static __device__ __noinline__ uint2 quantize8_ieee(uint4 v, float scale) {
  const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&v);
  uint16_t q[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f = __bfloat1622float2(h[j]);
    q[j] = pack_e4m3x2(__fdiv_rn(f.x, scale), __fdiv_rn(f.y, scale));
  }
  return make_uint2(static_cast<uint32_t>(q[0]) | (static_cast<uint32_t>(q[1]) << 16),
                    static_cast<uint32_t>(q[2]) | (static_cast<uint32_t>(q[3]) << 16));
}

// Row maximum on the bf16 bit patterns: with the sign cleared, |x| orders
// like the unsigned bits, and every NaN pattern (0x7f81..0x7fff) orders above
// +inf (0x7f80).  One packed 16-bit max per two values gives both the row's
// amax (the largest non-NaN magnitude when the maximum is <= 0x7f80) and its
// NaN flag (maximum > 0x7f80); the amax value is the bf16 with those bits.
constexpr uint32_t kBf16Inf = 0x7f80u;

__device__ __forceinline__ uint32_t abs_bits_max8(const uint4 &v, uint32_t acc) {
  acc = __vmaxu2(acc, v.x & 0x7fff7fffu);
  acc = __vmaxu2(acc, v.y & 0x7fff7fffu);
  acc = __vmaxu2(acc, v.z & 0x7fff7fffu);
  acc = __vmaxu2(acc, v.w & 0x7fff7fffu);
  return acc;
}

// Row scale from the row maximum kept as bf16 bit patterns with the sign
// cleared (abs_bits_max8): patterns above +inf mean the row holds a NaN.
__device__ __forceinline__ float row_scale_from_bits(uint32_t bits) {
  return row_scale(__uint_as_float(bits << 16), bits > kBf16Inf);
}

}  // namespace vfb
