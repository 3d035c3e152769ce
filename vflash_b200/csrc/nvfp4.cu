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
