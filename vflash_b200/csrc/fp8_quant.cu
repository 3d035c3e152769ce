// Per-token dynamic e4m3 activation quantisation (HBM-bound).
//
// Arithmetic follows _quantize_activation_torch
// (src/vflash/native/h3_fp8_linear.py:18-31) and the Triton _rows_fp8 kernel
// (src/vflash/native/h3_fp8_activation.py:13-28) bit for bit:
//   amax  = max |x| over the row (fp32)
//   scale = amax > 0 ? max(amax / 448, FLT_MIN) : 1      (IEEE division)
//   code  = e4m3_rn(clamp(x / scale, -448, 448))         (correctly rounded
//           quotient: reciprocal per row + one FMA correction per element)
// Rows are padded to the caller's M_pad (16 in the reference) with code 0 and
// scale 1.  A NaN anywhere in a row makes amax NaN as in torch, so the row's
// scale is 1 and NaN inputs stay NaN codes.
//
// Layout: one group of TPR threads (a multiple of 32) owns one row and keeps
// the whole row in registers as packed bf16 (8 x 16-byte loads per thread, so
// K <= 32768 needs at most 512 threads); the row maximum is taken on the bf16
// bit patterns (packed 16-bit max), reduced with redux.sync and, across the
// row's warps, through shared memory.  Each byte of
// x is read once and each code written once: 3 bytes of traffic per element.
#include <cfloat>

#include "common.cuh"
#include "quant.cuh"
#include "norm_modulate.cuh"

namespace vfb {
namespace {

constexpr int kVecPerThread = 8;     // 16-byte vectors (8 bf16) per thread: 128 bytes in flight
constexpr int kBlockThreads = 128;   // measured best with 8 vectors per thread (K = 4096 and 16384)
constexpr int kScalarThreads = 256;  // unaligned rows: one block per row
constexpr int kNormVecPerThread = 8; // the RMSNorm + modulate prologue: 16-byte vectors per thread

// Vector path: x rows 16-byte aligned, K % 8 == 0.
// amax_in != NULL: use these row maxima instead of reducing (a row split over
//   several ranks quantised with the full row's scale);
// amax_out != NULL: only write the row maxima (NaN for a row with a NaN).
__global__ void __launch_bounds__(512) fp8_quant_rows_vec(
    const __nv_bfloat16 *__restrict__ x, int64_t M, int64_t K, int64_t ldx,
    uint8_t *__restrict__ codes, float *__restrict__ scales, int64_t M_pad, int tpr,
    const float *__restrict__ amax_in, float *__restrict__ amax_out) {
  grid_launch_dependents();  // the GEMM reading this output may be scheduled now
  extern __shared__ uint32_t red[];  // [rows per block][warps per row] maxima (bit patterns)
  const int rows_per_block = blockDim.x / tpr;
  const int r_local = threadIdx.x / tpr;
  const int t = threadIdx.x % tpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_block + r_local;
  const int warps_per_row = tpr / 32;
  const int64_t nvec = K / 8;

  uint4 v[kVecPerThread];
  float amax = 0.0f;
  bool nan = false;
  const bool live = row < M;
  uint32_t bits = 0;
  if (live) {
    const uint4 *src = reinterpret_cast<const uint4 *>(x + row * ldx);
#pragma unroll
    for (int i = 0; i < kVecPerThread; ++i) {
      const int64_t c = static_cast<int64_t>(i) * tpr + t;
      v[i] = c < nvec ? __ldcs(src + c) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < kVecPerThread; ++i) bits = abs_bits_max8(v[i], bits);
  }
  if (amax_in == nullptr) {  // block-uniform
    uint32_t m = __reduce_max_sync(0xffffffffu, max(bits & 0xffffu, bits >> 16));
    if (warps_per_row > 1) {
      uint32_t *row_red = red + r_local * warps_per_row;
      if ((t & 31) == 0) row_red[t / 32] = m;
      __syncthreads();
      m = 0;
      for (int w = 0; w < warps_per_row; ++w) m = max(m, row_red[w]);
    }
    nan = m > kBf16Inf;
    amax = __uint_as_float(m << 16);
  } else {
    amax = live ? amax_in[row] : 0.0f;
    nan = amax != amax;
  }
  if (amax_out != nullptr) {
    if (live && t == 0) amax_out[row] = nan ? __int_as_float(0x7fc00000) : amax;
    return;
  }
  if (row >= M_pad) return;
  const float scale = live ? row_scale(amax, nan) : 1.0f;
  const bool fast = markstein_ok(scale);
  const float recip = fast ? __frcp_rn(scale) : 0.0f;
  uint2 *dst = reinterpret_cast<uint2 *>(codes + row * K);
#pragma unroll
  for (int i = 0; i < kVecPerThread; ++i) {
    const int64_t c = static_cast<int64_t>(i) * tpr + t;
    if (c >= nvec) continue;
    uint2 out = make_uint2(0, 0);
    if (live) out = fast ? quantize8(v[i], scale, recip) : quantize8_ieee(v[i], scale);
    dst[c] = out;
  }
  if (t == 0) scales[row] = scale;
}

// Generic path (any K, any alignment): one block per row, two passes over
// the row (the second from cache).
__global__ void __launch_bounds__(kScalarThreads) fp8_quant_rows_scalar(
    const __nv_bfloat16 *__restrict__ x, int64_t M, int64_t K, int64_t ldx,
    uint8_t *__restrict__ codes, float *__restrict__ scales, int64_t M_pad,
    const float *__restrict__ amax_in, float *__restrict__ amax_out) {
  grid_launch_dependents();  // the GEMM reading this output may be scheduled now
  __shared__ float red[kScalarThreads / 32 * 2];
  const int64_t row = blockIdx.x;
  const bool live = row < M;
  float amax = 0.0f;
  float any_nan = 0.0f;
  if (amax_in == nullptr) {  // block-uniform
    bool nan = false;
    if (live) {
      for (int64_t c = threadIdx.x; c < K; c += blockDim.x) {
        float f = __bfloat162float(x[row * ldx + c]);
        nan |= f != f;
        amax = fmaxf(amax, fabsf(f));
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    nan = __any_sync(0xffffffffu, nan);
    const int warps = blockDim.x / 32;
    if ((threadIdx.x & 31) == 0) {
      red[threadIdx.x / 32] = amax;
      red[warps + threadIdx.x / 32] = nan ? 1.0f : 0.0f;
    }
    __syncthreads();
    amax = 0.0f;
    for (int w = 0; w < warps; ++w) {
      amax = fmaxf(amax, red[w]);
      any_nan = fmaxf(any_nan, red[warps + w]);
    }
  } else {
    amax = live ? amax_in[row] : 0.0f;
    any_nan = amax != amax ? 1.0f : 0.0f;
  }
  if (amax_out != nullptr) {
    if (live && threadIdx.x == 0) amax_out[row] = any_nan != 0.0f ? __int_as_float(0x7fc00000) : amax;
    return;
  }
  const float scale = live ? row_scale(amax, any_nan != 0.0f) : 1.0f;
  const bool fast = markstein_ok(scale);
  const float recip = fast ? __frcp_rn(scale) : 0.0f;
  for (int64_t c = threadIdx.x; c < K; c += blockDim.x) {
    uint8_t q = 0;
    if (live) {
      float f = __bfloat162float(x[row * ldx + c]);
      q = static_cast<uint8_t>(pack_e4m3x2(quotient(f, scale, recip, fast), 0.0f) & 0xFF);
    }
    codes[row * K + c] = q;
  }
  if (threadIdx.x == 0) scales[row] = scale;
}

// ---------------------------------------------------------------------------
// RMSNorm + AdaLN modulate + per-token e4m3 quantisation in one pass.
//
// For each token row x (bf16, K values), as the reference block computes it
// before its QKV and FFN-input projections (src/vflash/native/
// h3_native_denoiser.py:534-541 and 561-568):
//   rstd = rsqrt(mean(x^2) + eps)                 fp32 (torch's fused rms_norm:
//                                                 fp32 upcast, mean, rsqrt)
//   n    = bf16((x * rstd) * w)                   one rounding (fp32 products)
//   m    = bf16(bf16(n * bf16(1 + scale)) + shift) strict-BF16 modulate
//                                                 (h3_fused_ops.py:52-122)
//   codes, row scale = the per-token quantisation of m (as above)
// scale / shift are [tokens, K] rows selected by row % tokens.  The sum of
// squares is accumulated in fp32 in this kernel's order and the reciprocal
// square root is correctly rounded (computed in fp64), so rstd can differ
// from another implementation's by an ulp of fp32; n, m and the codes then
// differ from it only where that ulp crosses a bf16 rounding boundary.
// x stays in registers between the two row reductions (sum of squares, then
// max |m|): 2 bytes read per element of x, scale and shift each, 1 written.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512) fp8_norm_modulate_quant_vec(
    const __nv_bfloat16 *__restrict__ x, int64_t M, int64_t K, int64_t ldx,
    const __nv_bfloat16 *__restrict__ norm_w, float eps, const __nv_bfloat16 *__restrict__ mod_scale,
    int64_t scale_ts, const __nv_bfloat16 *__restrict__ mod_shift, int64_t shift_ts, int64_t tokens,
    uint8_t *__restrict__ codes, float *__restrict__ scales, int64_t M_pad, int tpr) {
  grid_launch_dependents();  // the GEMM reading this output may be scheduled now
  extern __shared__ uint32_t red[];
  const int rows_per_block = blockDim.x / tpr;
  const int r_local = threadIdx.x / tpr;
  const int t = threadIdx.x % tpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_block + r_local;
  const int warps_per_row = tpr / 32;
  const int64_t nvec = K / 8;
  const bool live = row < M;

  uint4 v[kNormVecPerThread];
  float ss = 0.0f;
  if (live) {
    const uint4 *src = reinterpret_cast<const uint4 *>(x + row * ldx);
#pragma unroll
    for (int i = 0; i < kNormVecPerThread; ++i) {
      const int64_t c = static_cast<int64_t>(i) * tpr + t;
      v[i] = c < nvec ? __ldcs(src + c) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < kNormVecPerThread; ++i) ss = sum_squares8(v[i], ss);
  }
  ss = block_row_sum(ss, red, r_local, t, warps_per_row);  // block-uniform call
  uint32_t bits = 0;
  if (live) {
    const float rstd = rms_rstd(ss, K, eps);
    const int64_t token = row % tokens;
    const uint4 *wq = reinterpret_cast<const uint4 *>(norm_w);
    const uint4 *scq = reinterpret_cast<const uint4 *>(mod_scale + token * scale_ts);
    const uint4 *shq = reinterpret_cast<const uint4 *>(mod_shift + token * shift_ts);
#pragma unroll
    for (int i = 0; i < kNormVecPerThread; ++i) {
      const int64_t c = static_cast<int64_t>(i) * tpr + t;
      if (c >= nvec) continue;
      const uint4 wv = norm_w != nullptr ? __ldg(wq + c) : make_uint4(0x3f803f80u, 0x3f803f80u,
                                                                       0x3f803f80u, 0x3f803f80u);
      v[i] = norm_modulate8(v[i], rstd, wv, __ldg(scq + c), __ldg(shq + c));
      bits = abs_bits_max8(v[i], bits);
    }
  }
  uint32_t m = __reduce_max_sync(0xffffffffu, max(bits & 0xffffu, bits >> 16));
  if (warps_per_row > 1) {
    uint32_t *row_red = red + r_local * warps_per_row;
    if ((t & 31) == 0) row_red[t / 32] = m;
    __syncthreads();
    m = 0;
    for (int w = 0; w < warps_per_row; ++w) m = max(m, row_red[w]);
  }
  if (row >= M_pad) return;
  const float amax = __uint_as_float(m << 16);
  const float scale = live ? row_scale(amax, m > kBf16Inf) : 1.0f;
  const bool fast = markstein_ok(scale);
  const float recip = fast ? __frcp_rn(scale) : 0.0f;
  uint2 *dst = reinterpret_cast<uint2 *>(codes + row * K);
#pragma unroll
  for (int i = 0; i < kNormVecPerThread; ++i) {
    const int64_t c = static_cast<int64_t>(i) * tpr + t;
    if (c >= nvec) continue;
    uint2 q = make_uint2(0, 0);
    if (live) q = fast ? quantize8(v[i], scale, recip) : quantize8_ieee(v[i], scale);
    dst[c] = q;
  }
  if (t == 0) scales[row] = scale;
}

int launch_quant(const char *what, const void *x, int64_t M, int64_t K, int64_t ldx, void *codes,
                 float *scales, int64_t M_pad, const float *amax_in, float *amax_out,
                 cudaStream_t s) {
  if (M < 0 || K < 1 || K > 32768 || ldx < K || M_pad < M)
    return set_error(VFB_EINVAL,
                     "%s: need M >= 0, 1 <= K <= 32768, ldx >= K, M_pad >= M "
                     "(M=%lld K=%lld ldx=%lld M_pad=%lld)",
                     what, (long long)M, (long long)K, (long long)ldx, (long long)M_pad);
  if (M_pad == 0) return VFB_OK;
  if (M > 0 && x == nullptr) return set_error(VFB_EINVAL, "%s: NULL pointer", what);
  int rc = check_device(nullptr);
  if (rc != VFB_OK) return rc;
  const bool vec = (K % 8 == 0) && (ldx % 8 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(codes) % 8 == 0);
  if (vec) {
    const int64_t nvec = K / 8;
    int tpr = static_cast<int>((nvec + kVecPerThread - 1) / kVecPerThread);
    tpr = (tpr + 31) / 32 * 32;
    const int rows_per_block = tpr >= kBlockThreads ? 1 : kBlockThreads / tpr;
    const int threads = tpr * rows_per_block;
    const int64_t blocks = (M_pad + rows_per_block - 1) / rows_per_block;
    const size_t smem = static_cast<size_t>(rows_per_block) * (tpr / 32) * sizeof(uint32_t);
    fp8_quant_rows_vec<<<static_cast<unsigned>(blocks), threads, smem, s>>>(
        static_cast<const __nv_bfloat16 *>(x), M, K, ldx, static_cast<uint8_t *>(codes), scales,
        M_pad, tpr, amax_in, amax_out);
  } else {
    fp8_quant_rows_scalar<<<static_cast<unsigned>(M_pad), kScalarThreads, 0, s>>>(
        static_cast<const __nv_bfloat16 *>(x), M, K, ldx, static_cast<uint8_t *>(codes), scales,
        M_pad, amax_in, amax_out);
  }
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_error(VFB_ECUDA, "%s launch: %s", what, cudaGetErrorString(err));
  return VFB_OK;
}

}  // namespace
}  // namespace vfb

extern "C" int vfb_fp8_quant_rows(const void *x, int64_t M, int64_t K, int64_t ldx, void *codes,
                                  float *scales, int64_t M_pad, void *stream) {
  if (M_pad > 0 && (codes == nullptr || scales == nullptr))
    return vfb::set_error(VFB_EINVAL, "vfb_fp8_quant_rows: NULL pointer");
  return vfb::launch_quant("vfb_fp8_quant_rows", x, M, K, ldx, codes, scales, M_pad, nullptr,
                           nullptr, static_cast<cudaStream_t>(stream));
}

extern "C" int vfb_fp8_row_absmax(const void *x, int64_t M, int64_t K, int64_t ldx, float *amax,
                                  void *stream) {
  if (M > 0 && amax == nullptr) return vfb::set_error(VFB_EINVAL, "vfb_fp8_row_absmax: NULL pointer");
  return vfb::launch_quant("vfb_fp8_row_absmax", x, M, K, ldx, nullptr, nullptr, M, nullptr, amax,
                           static_cast<cudaStream_t>(stream));
}

extern "C" int vfb_fp8_quant_rows_amax(const void *x, int64_t M, int64_t K, int64_t ldx,
                                       const float *amax, void *codes, float *scales, int64_t M_pad,
                                       void *stream) {
  if (M_pad > 0 && (codes == nullptr || scales == nullptr || (M > 0 && amax == nullptr)))
    return vfb::set_error(VFB_EINVAL, "vfb_fp8_quant_rows_amax: NULL pointer");
  return vfb::launch_quant("vfb_fp8_quant_rows_amax", x, M, K, ldx, codes, scales, M_pad, amax,
                           nullptr, static_cast<cudaStream_t>(stream));
}

extern "C" int vfb_fp8_norm_modulate_quant(const void *x, int64_t M, int64_t K, int64_t ldx,
                                           const void *norm_weight, float eps, const void *scale,
                                           int64_t scale_token_stride, const void *shift,
                                           int64_t shift_token_stride, int64_t tokens, void *codes,
                                           float *scales, int64_t M_pad, void *stream) {
  using namespace vfb;
  if (M < 0 || K < 8 || K > 32768 || K % 8 || ldx < K || M_pad < M || tokens <= 0 ||
      scale_token_stride < 0 || shift_token_stride < 0 || !(eps >= 0.0f))
    return set_error(VFB_EINVAL,
                     "vfb_fp8_norm_modulate_quant: need 8 <= K <= 32768, K %% 8 == 0, ldx >= K, "
                     "M_pad >= M, tokens > 0, strides >= 0, eps >= 0");
  if (M_pad == 0) return VFB_OK;
  if ((M > 0 && (!x || !scale || !shift)) || !codes || !scales)
    return set_error(VFB_EINVAL, "vfb_fp8_norm_modulate_quant: NULL pointer");
  const auto al16 = [](const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (!al16(x) || ldx % 8 || (norm_weight && !al16(norm_weight)) || !al16(scale) || !al16(shift) ||
      scale_token_stride % 8 || shift_token_stride % 8 || reinterpret_cast<uintptr_t>(codes) % 8)
    return set_error(VFB_EINVAL,
                     "vfb_fp8_norm_modulate_quant: rows of x, weight, scale and shift must be "
                     "16-byte aligned (strides %% 8 == 0) and codes 8-byte aligned");
  int rc = check_device(nullptr);
  if (rc != VFB_OK) return rc;
  const int64_t nvec = K / 8;
  int tpr = static_cast<int>((nvec + kNormVecPerThread - 1) / kNormVecPerThread);
  tpr = (tpr + 31) / 32 * 32;
  const int rows_per_block = tpr >= kBlockThreads ? 1 : kBlockThreads / tpr;
  const int threads = tpr * rows_per_block;
  const int64_t blocks = (M_pad + rows_per_block - 1) / rows_per_block;
  const size_t smem = static_cast<size_t>(rows_per_block) * (tpr / 32) * sizeof(uint32_t);
  fp8_norm_modulate_quant_vec<<<static_cast<unsigned>(blocks), threads, smem,
                                static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16 *>(x), M, K, ldx, static_cast<const __nv_bfloat16 *>(norm_weight),
      eps, static_cast<const __nv_bfloat16 *>(scale), scale_token_stride,
      static_cast<const __nv_bfloat16 *>(shift), shift_token_stride, tokens, static_cast<uint8_t *>(codes),
      scales, M_pad, tpr);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return set_error(VFB_ECUDA, "vfb_fp8_norm_modulate_quant launch: %s", cudaGetErrorString(err));
  return VFB_OK;
}
