// The NVFP4 quantisation of one 16-element group, shared by the standalone
// quantiser (nvfp4.cu) and the block-scaled GEMM's quantising epilogue
// (nvfp4_gemm.cu), so both produce the same codes and scales bit for bit.
//
// Recipe (FlashInfer 0.6.18's default, non-TE-exact nvfp4_quantize, restated
// from its published quantization_utils.cuh:294-380; the reference calls it
// at src/vflash/native/h3_nvfp4_linear.py:102):
//   amax   = max |x|
//   sf     = e4m3_rn_satfinite(gsf * (amax * rcp(6)))
//   scale  = amax != 0 ? rcp(float(sf) * rcp(gsf)) : 0
//   code_i = e2m1_rn_satfinite(x_i * scale)        (element 2i in the low nibble)
// with rcp = rcp.approx.ftz.f32 and the multiplies flushing subnormals, as the
// reference's fast-math build does.  Scales go to the 128x4 layout: for row m
// and 16-element group k, byte
//   (m/128)*(kt*512) + (k/4)*512 + (m%32)*16 + ((m%128)/32)*4 + k%4,
// kt = ceil(K/64).
#pragma once

#include "common.cuh"

namespace vfb {

// Multiplication with subnormal inputs and results flushed to zero.
__device__ __forceinline__ float mul_ftz(float a, float b) {
  float r;
  asm("mul.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ uint32_t e4m3_byte(float x) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(x));
  return r & 0xFFu;
}

// Exact decode of a non-negative finite e4m3 byte.
__device__ __forceinline__ float e4m3_value(uint32_t byte) {
  const uint32_t e = (byte >> 3) & 0xF, m = byte & 0x7;
  if (e == 0) return static_cast<float>(m) * 0.001953125f;  // m * 2^-9
  return __uint_as_float(((e + 120u) << 23) | (m << 20));
}

__device__ __forceinline__ int64_t sf_offset(int64_t m, int64_t k, int64_t ktiles) {
  return (m >> 7) * (ktiles * 512) + (k >> 2) * 512 + (m & 31) * 16 + ((m & 127) >> 5) * 4 + (k & 3);
}

// The per-tensor constants of the recipe: rcp(6) and rcp(global scale).
struct Nvfp4Consts {
  float gsf, rcp6, rcp_gsf;
};

__device__ __forceinline__ Nvfp4Consts nvfp4_consts(float gsf) {
  return Nvfp4Consts{gsf, rcp_approx_ftz(6.0f), rcp_approx_ftz(gsf)};
}

// One group of 16 values (v[0..15]): returns the scale byte and the eight
// code bytes in `packed` (element 2i in the low nibble of byte i).
__device__ __forceinline__ uint32_t nvfp4_group(const float *v, const Nvfp4Consts &c, uint2 &packed) {
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
  const float sf_value = mul_ftz(c.gsf, mul_ftz(amax, c.rcp6));
  const uint32_t sf_byte = e4m3_byte(sf_value);
  // amax != 0 compared after flushing a subnormal amax to zero
  const float scale =
      mul_ftz(amax, 1.0f) != 0.0f ? rcp_approx_ftz(mul_ftz(e4m3_value(sf_byte), c.rcp_gsf)) : 0.0f;
  float lo[8], hi[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    lo[j] = mul_ftz(v[j], scale);
    hi[j] = mul_ftz(v[8 + j], scale);
  }
  packed = make_uint2(pack_e2m1x8(lo), pack_e2m1x8(hi));
  return sf_byte;
}

}  // namespace vfb
