// The fused FP8 FFN as C entry points: per-token quantiser (except
// vfb_fp8_ffn_quantized), then up GEMM + activation, per-token requantisation
// of the bf16 intermediate and down GEMM + bias / gated residual.
//
// vfb_fp8_ffn runs those three steps as three launches (up GEMM with the
// activation epilogue, vfb_fp8_quant_rows, down GEMM with the residual
// epilogue), the fastest order measured on the B200 at the benchmark's size.
// vfb_fp8_ffn_one_kernel runs them as ONE persistent launch (ffn_fused.cu)
// that requantises the intermediate in place, when the width tiles it (GELU:
// F % 256 == 0, SwiGLU: F % 128 == 0).  Both give the same bits.
// Intermediates live in a caller-owned workspace (vfb_fp8_ffn_workspace_bytes):
// nothing is allocated.
#include <cstdint>

#include "common.cuh"
#include "ffn_fused.h"

namespace vfb {
namespace {

constexpr int64_t kAlign = 256;

int64_t align_up(int64_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

int64_t pad16(int64_t m) { return (m + 15) / 16 * 16; }

// Workspace layout (each region 256-byte aligned):
//   x codes   e4m3 [pad16(M), H]     x scales   fp32 [pad16(M)]
//   mid       bf16 [M, F]
//   mid codes e4m3 [pad16(M), F]     mid scales fp32 [pad16(M)]
//   row maxima u32 [M], then the fused kernel's counters int [1 + 2 ceil(M/256)]
//   (one zeroed region)
struct FfnWorkspace {
  int64_t x_codes, x_scales, mid, mid_codes, mid_scales, amax, counters, zero_bytes, total;
};

FfnWorkspace ffn_layout(int64_t M, int64_t H, int64_t F) {
  FfnWorkspace w{};
  const int64_t mp = pad16(M);
  int64_t at = 0;
  w.x_codes = at;
  at = align_up(at + mp * H);
  w.x_scales = at;
  at = align_up(at + mp * 4);
  w.mid = at;
  at = align_up(at + M * F * 2);
  w.mid_codes = at;
  at = align_up(at + mp * F);
  w.mid_scales = at;
  at = align_up(at + mp * 4);
  w.amax = at;
  w.counters = at + M * 4;
  at = align_up(w.counters + (1 + 2 * ((M + 255) / 256)) * 4);
  w.zero_bytes = at - w.amax;
  w.total = at;
  return w;
}

bool ffn_shape_ok(int64_t M, int64_t H, int64_t F) {
  return M >= 0 && M <= ((int64_t)1 << 31) && H >= 16 && H <= 32768 && H % 32 == 0 && F >= 32 &&
         F <= 32768 && F % 32 == 0;
}

// Shared body of vfb_fp8_ffn and vfb_fp8_ffn_quantized; xc / xs are the
// quantised input (in the workspace for vfb_fp8_ffn).
int ffn_body(const char *fn, const void *xc, const float *xs, int64_t M, int64_t H, const void *w_up,
             const float *s_up, int64_t n_up, const void *w_down, const float *s_down, int32_t activation,
             const void *bias_up, const void *bias_down, const void *residual, int64_t ldr, const void *gate,
             int64_t gate_token_stride, int64_t tokens, void *out, int64_t ldo, uint8_t *ws,
             const FfnWorkspace &lay, int64_t F, bool one_kernel, void *stream) {
  if (one_kernel && ffn_fused_supported(activation, H, F)) {
    FfnFusedArgs a{};
    a.M = M;
    a.H = H;
    a.F = F;
    a.activation = activation;
    a.x_codes = xc;
    a.x_scales = xs;
    a.w_up = w_up;
    a.s_up = s_up;
    a.w_down = w_down;
    a.s_down = s_down;
    a.bias_up = bias_up;
    a.bias_down = bias_down;
    a.residual = residual;
    a.ldr = ldr;
    a.gate = gate;
    a.gate_token_stride = gate_token_stride;
    a.tokens = tokens;
    a.out = out;
    a.ldo = ldo;
    a.mid = ws + lay.mid;
    a.mid_codes = ws + lay.mid_codes;
    a.amax_bits = reinterpret_cast<uint32_t *>(ws + lay.amax);
    a.counters = reinterpret_cast<int *>(ws + lay.counters);
    a.zero_bytes = lay.zero_bytes;
    a.lead = -1;
    return launch_ffn_fused(a, stream);
  }
  (void)fn;
  const int64_t mp = pad16(M);
  void *mid = ws + lay.mid;
  void *mc = ws + lay.mid_codes;
  float *ms = reinterpret_cast<float *>(ws + lay.mid_scales);
  vfb_epilogue up{};
  up.kind = activation;
  up.out = mid;
  up.ldo = F;
  up.bias = bias_up;
  int rc = vfb_fp8_gemm(xc, H, xs, w_up, H, s_up, M, n_up, H, &up, stream);
  if (rc != VFB_OK) return rc;
  rc = vfb_fp8_quant_rows(mid, M, F, F, mc, ms, mp, stream);
  if (rc != VFB_OK) return rc;
  vfb_epilogue down{};
  down.kind = residual != nullptr ? VFB_EPI_RESIDUAL : VFB_EPI_STORE;
  down.out = out;
  down.ldo = ldo;
  down.bias = bias_down;
  if (residual != nullptr) {
    down.residual = residual;
    down.ldr = ldr;
    down.gate = gate;
    down.gate_token_stride = gate_token_stride;
    down.gate_hidden_stride = 1;
    down.tokens = gate != nullptr ? tokens : 0;
  }
  return vfb_fp8_gemm(mc, F, ms, w_down, F, s_down, M, H, F, &down, stream);
}

// Argument checks shared by both entry points; sets F.
int ffn_check(const char *fn, int64_t M, int64_t H, int64_t n_up, int32_t activation, const void *w_up,
              const float *s_up, const void *w_down, const float *s_down, const void *bias_up,
              const void *bias_down, const void *residual, int64_t ldr, const void *gate,
              int64_t gate_token_stride, int64_t tokens, const void *out, int64_t ldo, int64_t *F) {
  if (activation != VFB_EPI_GELU_TANH && activation != VFB_EPI_SWIGLU)
    return set_error(VFB_EINVAL, "%s: activation must be VFB_EPI_GELU_TANH or VFB_EPI_SWIGLU", fn);
  *F = activation == VFB_EPI_SWIGLU ? n_up / 2 : n_up;
  if (n_up <= 0 || (activation == VFB_EPI_SWIGLU && n_up % 2) || !ffn_shape_ok(M, H, *F))
    return set_error(VFB_EINVAL, "%s: need 16 <= H <= 32768 and 32 <= F <= 32768, both multiples of "
                                 "32 (F = n_up, or n_up / 2 for SWIGLU), M >= 0 (M=%lld H=%lld n_up=%lld)",
                     fn, (long long)M, (long long)H, (long long)n_up);
  if (gate != nullptr && (residual == nullptr || tokens <= 0 || gate_token_stride < H))
    return set_error(VFB_EINVAL, "%s: a gate needs a residual, tokens > 0 and a token stride >= H", fn);
  if (M == 0) return VFB_OK;
  if (w_up == nullptr || s_up == nullptr || w_down == nullptr || s_down == nullptr || out == nullptr)
    return set_error(VFB_EINVAL, "%s: NULL operand", fn);
  if (!aligned16(w_up) || !aligned16(w_down) || !aligned16(s_up) || !aligned16(s_down) || !aligned16(out) ||
      ldo < H || ldo % 8 || (bias_up && !aligned16(bias_up)) || (bias_down && !aligned16(bias_down)))
    return set_error(VFB_EINVAL, "%s: weights, scales, biases and out need 16-byte alignment, ldo >= H, "
                                 "ldo %% 8 == 0", fn);
  if (residual != nullptr && (!aligned16(residual) || ldr < H || ldr % 8))
    return set_error(VFB_EINVAL, "%s: residual needs a 16-byte aligned [M, H] view", fn);
  if (gate != nullptr && (!aligned16(gate) || gate_token_stride % 8))
    return set_error(VFB_EINVAL, "%s: gate rows need 16-byte alignment", fn);
  return VFB_OK;
}

}  // namespace
}  // namespace vfb

extern "C" int64_t vfb_fp8_ffn_workspace_bytes(int64_t M, int64_t H, int64_t F) {
  using namespace vfb;
  if (!ffn_shape_ok(M, H, F)) return -1;
  return ffn_layout(M, H, F).total;
}

namespace vfb {
namespace {

int ffn_entry(const char *fn, bool one_kernel, const void *x, int64_t M, int64_t H, int64_t ldx,
              const void *w_up, const float *s_up, int64_t n_up, const void *w_down, const float *s_down,
              int32_t activation, const void *bias_up, const void *bias_down, const void *residual, int64_t ldr,
              const void *gate, int64_t gate_token_stride, int64_t tokens, void *out, int64_t ldo,
              void *workspace, int64_t workspace_bytes, void *stream) {
  int64_t F = 0;
  int rc = ffn_check(fn, M, H, n_up, activation, w_up, s_up, w_down, s_down, bias_up, bias_down, residual, ldr,
                     gate, gate_token_stride, tokens, out, ldo, &F);
  if (rc != VFB_OK) return rc;
  const FfnWorkspace lay = ffn_layout(M, H, F);
  if (workspace == nullptr || workspace_bytes < lay.total || reinterpret_cast<uintptr_t>(workspace) % kAlign)
    return set_error(VFB_EINVAL, "%s: workspace must be 256-byte aligned and hold %lld bytes", fn,
                     (long long)lay.total);
  if (M == 0) return VFB_OK;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  void *xc = ws + lay.x_codes;
  float *xs = reinterpret_cast<float *>(ws + lay.x_scales);
  rc = vfb_fp8_quant_rows(x, M, H, ldx, xc, xs, pad16(M), stream);
  if (rc != VFB_OK) return rc;
  return ffn_body(fn, xc, xs, M, H, w_up, s_up, n_up, w_down, s_down, activation, bias_up, bias_down, residual,
                  ldr, gate, gate_token_stride, tokens, out, ldo, ws, lay, F, one_kernel, stream);
}

}  // namespace
}  // namespace vfb

extern "C" int vfb_fp8_ffn(const void *x, int64_t M, int64_t H, int64_t ldx, const void *w_up, const float *s_up,
                           int64_t n_up, const void *w_down, const float *s_down, int32_t activation,
                           const void *bias_up, const void *bias_down, const void *residual, int64_t ldr,
                           const void *gate, int64_t gate_token_stride, int64_t tokens, void *out, int64_t ldo,
                           void *workspace, int64_t workspace_bytes, void *stream) {
  return vfb::ffn_entry("vfb_fp8_ffn", false, x, M, H, ldx, w_up, s_up, n_up, w_down, s_down, activation, bias_up,
                        bias_down, residual, ldr, gate, gate_token_stride, tokens, out, ldo, workspace,
                        workspace_bytes, stream);
}

extern "C" int vfb_fp8_ffn_one_kernel(const void *x, int64_t M, int64_t H, int64_t ldx, const void *w_up,
                                      const float *s_up, int64_t n_up, const void *w_down, const float *s_down,
                                      int32_t activation, const void *bias_up, const void *bias_down,
                                      const void *residual, int64_t ldr, const void *gate,
                                      int64_t gate_token_stride, int64_t tokens, void *out, int64_t ldo,
                                      void *workspace, int64_t workspace_bytes, void *stream) {
  return vfb::ffn_entry("vfb_fp8_ffn_one_kernel", true, x, M, H, ldx, w_up, s_up, n_up, w_down, s_down,
                        activation, bias_up, bias_down, residual, ldr, gate, gate_token_stride, tokens, out, ldo,
                        workspace, workspace_bytes, stream);
}

extern "C" int vfb_fp8_ffn_quantized(const void *x_codes, const float *x_scales, int64_t M, int64_t H,
                                     const void *w_up, const float *s_up, int64_t n_up, const void *w_down,
                                     const float *s_down, int32_t activation, const void *bias_up,
                                     const void *bias_down, const void *residual, int64_t ldr, const void *gate,
                                     int64_t gate_token_stride, int64_t tokens, void *out, int64_t ldo,
                                     void *workspace, int64_t workspace_bytes, void *stream) {
  using namespace vfb;
  int64_t F = 0;
  int rc = ffn_check("vfb_fp8_ffn_quantized", M, H, n_up, activation, w_up, s_up, w_down, s_down, bias_up,
                     bias_down, residual, ldr, gate, gate_token_stride, tokens, out, ldo, &F);
  if (rc != VFB_OK) return rc;
  const FfnWorkspace lay = ffn_layout(M, H, F);
  if (workspace == nullptr || workspace_bytes < lay.total || reinterpret_cast<uintptr_t>(workspace) % kAlign)
    return set_error(VFB_EINVAL, "vfb_fp8_ffn_quantized: workspace must be 256-byte aligned and hold %lld bytes",
                     (long long)lay.total);
  if (M == 0) return VFB_OK;
  if (x_codes == nullptr || x_scales == nullptr || !aligned16(x_codes))
    return set_error(VFB_EINVAL, "vfb_fp8_ffn_quantized: x codes need a 16-byte aligned [M, H] matrix");
  return ffn_body("vfb_fp8_ffn_quantized", x_codes, x_scales, M, H, w_up, s_up, n_up, w_down, s_down, activation,
                  bias_up, bias_down, residual, ldr, gate, gate_token_stride, tokens, out, ldo,
                  static_cast<uint8_t *>(workspace), lay, F, false, stream);
}
