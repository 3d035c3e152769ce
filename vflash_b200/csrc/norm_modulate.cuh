// RMSNorm + AdaLN modulate of the block's hidden state, the prologue of the
// FP8 (fp8_quant.cu) and NVFP4 (nvfp4.cu) activation quantisers, so both
// produce the same bf16 values bit for bit:
//   rstd = 1 / sqrt(mean(x^2) + eps)    (fp32 sum of squares, mean and eps in
//                                        fp32 IEEE, the root in fp64, rounded)
//   n    = bf16((x * rstd) * w)          (_rms_norm, src/vflash/native/
//                                        h3_native_denoiser.py:231-243)
//   out  = bf16(bf16(n * bf16(1 + scale)) + shift)
//                                       (strict_modulate_kernel,
//                                        h3_fused_ops.py:52-122)
// with scale and shift rows chosen by token = row % tokens.
#pragma once

#include "common.cuh"

namespace vfb {

// Sum of v over the TPR threads of a row (TPR a multiple of 32); `red` holds
// rows_per_block x warps_per_row floats.  Every thread of the block calls it.
__device__ __forceinline__ float block_row_sum(float v, uint32_t *red_u32, int r_local, int t,
                                               int warps_per_row) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  if (warps_per_row > 1) {
    float *row_red = reinterpret_cast<float *>(red_u32) + r_local * warps_per_row;
    if ((t & 31) == 0) row_red[t / 32] = v;
    __syncthreads();
    v = 0.0f;
    for (int w = 0; w < warps_per_row; ++w) v += row_red[w];
    __syncthreads();  // the buffer is reused by the reduction that follows
  }
  return v;
}

// Sum of squares of eight packed bf16 values, accumulated into ss.
__device__ __forceinline__ float sum_squares8(const uint4 &v, float ss) {
  const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    ss = fmaf(f.x, f.x, ss);
    ss = fmaf(f.y, f.y, ss);
  }
  return ss;
}

__device__ __forceinline__ float rms_rstd(float ss, int64_t K, float eps) {
  const float mean_eps = __fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps);
  return static_cast<float>(1.0 / sqrt(static_cast<double>(mean_eps)));
}

// Norm and modulate of eight packed bf16 values (w: the norm weight, or all
// ones; sc / sh: the token's scale and shift), packed bf16 out.
__device__ __forceinline__ uint4 norm_modulate8(const uint4 &x, float rstd, const uint4 &w, const uint4 &sc,
                                                const uint4 &sh) {
  const __nv_bfloat162 *hx = reinterpret_cast<const __nv_bfloat162 *>(&x);
  const __nv_bfloat162 *hw = reinterpret_cast<const __nv_bfloat162 *>(&w);
  const __nv_bfloat162 *hs = reinterpret_cast<const __nv_bfloat162 *>(&sc);
  const __nv_bfloat162 *hb = reinterpret_cast<const __nv_bfloat162 *>(&sh);
  uint32_t out[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 fx = __bfloat1622float2(hx[j]);
    const float2 fw = __bfloat1622float2(hw[j]);
    const float2 fs = __bfloat1622float2(hs[j]);
    const float2 fb = __bfloat1622float2(hb[j]);
    const float n0 = bf16r((fx.x * rstd) * fw.x);
    const float n1 = bf16r((fx.y * rstd) * fw.y);
    const float m0 = bf16r(n0 * bf16r(1.0f + fs.x)) + fb.x;
    const float m1 = bf16r(n1 * bf16r(1.0f + fs.y)) + fb.y;
    out[j] = pack_bf16x2(m0, m1);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

}  // namespace vfb
