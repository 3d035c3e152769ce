// NVFP4 (e2m1 with one ue4m3 scale per 16 elements) activation quantiser for
// sm_100a.
//
// Replaces FlashInfer nvfp4_quantize(x, global_scale, sfLayout=128x4,
// do_shuffle=False) as called by NVFP4Execution.linear
// (src/vflash/native/h3_nvfp4_linear.py:102).  The arithmetic of a 16-element
// group (FlashInfer's recipe, bit for bit) is nvfp4_group() in
// nvfp4_quant.cuh, which the GEMM's quantising epilogue shares.  Scales are
// written in the 128x4 layout for rows up to ceil128(M) and groups up to
// 4*ceil(K/64); the padding entries are written as 0.  One thread handles one
// 16-element group (two 16-byte loads, one 8-byte store of codes, one scale
// byte).
//
// The block-scaled GEMM that consumes these codes is in nvfp4_gemm.cu.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "nvfp4_quant.cuh"
#include "norm_modulate.cuh"

namespace vfb {
namespace {

// ---------------------------------------------------------------------------
// quantiser
// ---------------------------------------------------------------------------
template <bool FP16>
__device__ __forceinline__ float to_f32(uint16_t bits) {
  if (FP16) return __half2float(__ushort_as_half(bits));
  return __uint_as_float(static_cast<uint32_t>(bits) << 16);
}

template <bool FP16, bool VEC>
__global__ void __launch_bounds__(256) nvfp4_quant_kernel(const uint16_t *__restrict__ x, int64_t M,
                                                          int64_t K, int64_t ldx,
                                                          const float *__restrict__ gsf_ptr,
                                                          uint8_t *__restrict__ codes,
                                                          uint8_t *__restrict__ sf, int64_t rows_pad,
                                                          int64_t groups_pad) {
  grid_launch_dependents();  // the GEMM reading this output may be scheduled now
  const Nvfp4Consts consts = nvfp4_consts(__ldg(gsf_ptr));
  const int64_t groups = K / 16;
  const int64_t ktiles = groups_pad / 4;
  const int64_t total = rows_pad * groups_pad;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / groups_pad;
    const int64_t k = i - m * groups_pad;
    uint32_t sf_byte = 0;
    if (m < M && k < groups) {
      float v[16];
      const uint16_t *src = x + m * ldx + k * 16;
      if (VEC) {
        const uint4 a = __ldg(reinterpret_cast<const uint4 *>(src));
        const uint4 b = __ldg(reinterpret_cast<const uint4 *>(src) + 1);
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[2 * j] = to_f32<FP16>(static_cast<uint16_t>(w[j] & 0xFFFF));
          v[2 * j + 1] = to_f32<FP16>(static_cast<uint16_t>(w[j] >> 16));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = to_f32<FP16>(src[j]);
      }
      uint2 packed;
      sf_byte = nvfp4_group(v, consts, packed);
      *reinterpret_cast<uint2 *>(codes + m * (K / 2) + k * 8) = packed;
    }
    sf[sf_offset(m, k, ktiles)] = static_cast<uint8_t>(sf_byte);
  }
}

// ---------------------------------------------------------------------------
// RMSNorm + AdaLN modulate + NVFP4 quantisation in one pass (the pre-GEMM
// fusion of the block's norm and modulate into the NVFP4 activation
// quantiser): the bf16 values of norm_modulate8 (norm_modulate.cuh, the same
// arithmetic as the FP8 prologue) are quantised group by group with
// nvfp4_group, so the codes and scales equal vfb_nvfp4_quant_rows of the
// modulated bf16 tensor.  One group of TPR threads owns a row: each thread
// keeps kNormGroups groups of 16 values (two 16-byte vectors each) in
// registers across the row's sum-of-squares reduction.  K % 64 == 0; rows
// past M up to ceil128(M) get zero scales.
// ---------------------------------------------------------------------------
constexpr int kNormGroups = 2;          // 16-element groups per thread (measured: 2 beats 4 and 8)
constexpr int kNormBlockThreads = 128;

__global__ void __launch_bounds__(512) nvfp4_norm_modulate_quant_kernel(
    const __nv_bfloat16 *__restrict__ x, int64_t M, int64_t K, int64_t ldx,
    const __nv_bfloat16 *__restrict__ norm_w, float eps, const __nv_bfloat16 *__restrict__ mod_scale,
    int64_t scale_ts, const __nv_bfloat16 *__restrict__ mod_shift, int64_t shift_ts, int64_t tokens,
    const float *__restrict__ gsf_ptr, uint8_t *__restrict__ codes, uint8_t *__restrict__ sf, int64_t rows_pad,
    int tpr) {
  grid_launch_dependents();  // the GEMM reading this output may be scheduled now
  extern __shared__ uint32_t red[];
  const int rows_per_block = blockDim.x / tpr;
  const int r_local = threadIdx.x / tpr;
  const int t = threadIdx.x % tpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_block + r_local;
  const int warps_per_row = tpr / 32;
  const int64_t groups = K / 16;
  const int64_t ktiles = groups / 4;
  const bool live = row < M;

  uint4 v[2 * kNormGroups];
  float ss = 0.0f;
  if (live) {
    const uint4 *src = reinterpret_cast<const uint4 *>(x + row * ldx);
#pragma unroll
    for (int i = 0; i < kNormGroups; ++i) {
      const int64_t g = static_cast<int64_t>(i) * tpr + t;
      const bool in = g < groups;
      v[2 * i] = in ? __ldcs(src + 2 * g) : make_uint4(0, 0, 0, 0);
      v[2 * i + 1] = in ? __ldcs(src + 2 * g + 1) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < 2 * kNormGroups; ++i) ss = sum_squares8(v[i], ss);
  }
  ss = block_row_sum(ss, red, r_local, t, warps_per_row);  // block-uniform call
  if (row >= rows_pad) return;
  if (!live) {
#pragma unroll
    for (int i = 0; i < kNormGroups; ++i) {
      const int64_t g = static_cast<int64_t>(i) * tpr + t;
      if (g < groups) sf[sf_offset(row, g, ktiles)] = 0;
    }
    return;
  }
  const Nvfp4Consts consts = nvfp4_consts(__ldg(gsf_ptr));
  const float rstd = rms_rstd(ss, K, eps);
  const int64_t token = row % tokens;
  const uint4 *wq = reinterpret_cast<const uint4 *>(norm_w);
  const uint4 *scq = reinterpret_cast<const uint4 *>(mod_scale + token * scale_ts);
  const uint4 *shq = reinterpret_cast<const uint4 *>(mod_shift + token * shift_ts);
  const uint4 ones = make_uint4(0x3f803f80u, 0x3f803f80u, 0x3f803f80u, 0x3f803f80u);
#pragma unroll
  for (int i = 0; i < kNormGroups; ++i) {
    const int64_t g = static_cast<int64_t>(i) * tpr + t;
    if (g >= groups) continue;
    float f[16];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t c = 2 * g + h;
      const uint4 y = norm_modulate8(v[2 * i + h], rstd, norm_w != nullptr ? __ldg(wq + c) : ones,
                                     __ldg(scq + c), __ldg(shq + c));
      const __nv_bfloat162 *hy = reinterpret_cast<const __nv_bfloat162 *>(&y);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fy = __bfloat1622float2(hy[j]);
        f[8 * h + 2 * j] = fy.x;
        f[8 * h + 2 * j + 1] = fy.y;
      }
    }
    uint2 packed;
    const uint32_t sf_byte = nvfp4_group(f, consts, packed);
    *reinterpret_cast<uint2 *>(codes + row * (K / 2) + g * 8) = packed;
    sf[sf_offset(row, g, ktiles)] = static_cast<uint8_t>(sf_byte);
  }
}

bool a16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace
}  // namespace vfb

extern "C" int vfb_nvfp4_quant_rows(const void *x, int32_t dtype, int64_t M, int64_t K, int64_t ldx,
                                    const float *global_scale, void *codes, void *sf, void *stream) {
  using namespace vfb;
  if (M < 0 || K <= 0 || K % 16 || ldx < K || (dtype != 0 && dtype != 1))
    return set_error(VFB_EINVAL,
                     "vfb_nvfp4_quant_rows: need K %% 16 == 0, ldx >= K, dtype 0 (bf16) or 1 (fp16)");
  if (M == 0) return VFB_OK;
  if (x == nullptr || global_scale == nullptr || codes == nullptr || sf == nullptr)
    return set_error(VFB_EINVAL, "vfb_nvfp4_quant_rows: NULL pointer");
  if (reinterpret_cast<uintptr_t>(codes) % 8)
    return set_error(VFB_EINVAL, "vfb_nvfp4_quant_rows: codes must be 8-byte aligned");
  int sms = 0;
  int rc = check_device(&sms);
  if (rc != VFB_OK) return rc;
  const int64_t rows_pad = (M + 127) / 128 * 128;
  const int64_t groups_pad = (K / 16 + 3) / 4 * 4;
  const int64_t total = rows_pad * groups_pad;
  int64_t blocks = (total + 255) / 256;
  if (blocks > (int64_t)sms * 32) blocks = (int64_t)sms * 32;
  const bool vec = a16(x) && ldx % 8 == 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto *xi = static_cast<const uint16_t *>(x);
  auto *c = static_cast<uint8_t *>(codes);
  auto *f = static_cast<uint8_t *>(sf);
  const unsigned g = static_cast<unsigned>(blocks);
  if (dtype == 0) {
    if (vec) nvfp4_quant_kernel<false, true><<<g, 256, 0, s>>>(xi, M, K, ldx, global_scale, c, f, rows_pad, groups_pad);
    else nvfp4_quant_kernel<false, false><<<g, 256, 0, s>>>(xi, M, K, ldx, global_scale, c, f, rows_pad, groups_pad);
  } else {
    if (vec) nvfp4_quant_kernel<true, true><<<g, 256, 0, s>>>(xi, M, K, ldx, global_scale, c, f, rows_pad, groups_pad);
    else nvfp4_quant_kernel<true, false><<<g, 256, 0, s>>>(xi, M, K, ldx, global_scale, c, f, rows_pad, groups_pad);
  }
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return set_error(VFB_ECUDA, "vfb_nvfp4_quant_rows launch: %s", cudaGetErrorString(err));
  return VFB_OK;
}

extern "C" int vfb_nvfp4_norm_modulate_quant(const void *x, int64_t M, int64_t K, int64_t ldx,
                                             const void *norm_weight, float eps, const void *scale,
                                             int64_t scale_token_stride, const void *shift,
                                             int64_t shift_token_stride, int64_t tokens,
                                             const float *global_scale, void *codes, void *sf, void *stream) {
  using namespace vfb;
  if (M < 0 || K < 64 || K > 32768 || K % 64 || ldx < K || tokens <= 0 || scale_token_stride < 0 ||
      shift_token_stride < 0 || !(eps >= 0.0f))
    return set_error(VFB_EINVAL,
                     "vfb_nvfp4_norm_modulate_quant: need 64 <= K <= 32768, K %% 64 == 0, ldx >= K, "
                     "tokens > 0, strides >= 0, eps >= 0");
  if (M == 0) return VFB_OK;
  if (!x || !scale || !shift || !global_scale || !codes || !sf)
    return set_error(VFB_EINVAL, "vfb_nvfp4_norm_modulate_quant: NULL pointer");
  if (!a16(x) || ldx % 8 || (norm_weight && !a16(norm_weight)) || !a16(scale) || !a16(shift) ||
      scale_token_stride % 8 || shift_token_stride % 8 || reinterpret_cast<uintptr_t>(codes) % 8)
    return set_error(VFB_EINVAL,
                     "vfb_nvfp4_norm_modulate_quant: rows of x, weight, scale and shift must be 16-byte "
                     "aligned (strides %% 8 == 0) and codes 8-byte aligned");
  int rc = check_device(nullptr);
  if (rc != VFB_OK) return rc;
  const int64_t groups = K / 16;
  int tpr = static_cast<int>((groups + kNormGroups - 1) / kNormGroups);
  tpr = (tpr + 31) / 32 * 32;
  const int rows_per_block = tpr >= kNormBlockThreads ? 1 : kNormBlockThreads / tpr;
  const int threads = tpr * rows_per_block;
  const int64_t rows_pad = (M + 127) / 128 * 128;
  const int64_t blocks = (rows_pad + rows_per_block - 1) / rows_per_block;
  const size_t smem = static_cast<size_t>(rows_per_block) * (tpr / 32) * sizeof(uint32_t);
  nvfp4_norm_modulate_quant_kernel<<<static_cast<unsigned>(blocks), threads, smem,
                                     static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16 *>(x), M, K, ldx, static_cast<const __nv_bfloat16 *>(norm_weight), eps,
      static_cast<const __nv_bfloat16 *>(scale), scale_token_stride, static_cast<const __nv_bfloat16 *>(shift),
      shift_token_stride, tokens, global_scale, static_cast<uint8_t *>(codes), static_cast<uint8_t *>(sf), rows_pad,
      tpr);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return set_error(VFB_ECUDA, "vfb_nvfp4_norm_modulate_quant launch: %s", cudaGetErrorString(err));
  return VFB_OK;
}
