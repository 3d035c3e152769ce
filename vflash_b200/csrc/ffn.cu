// The fused FP8 FFN as one C entry point: per-token quantiser, up GEMM with
// the activation in its epilogue, per-token requantisation of the bf16
// intermediate, down GEMM with bias / gated residual in its epilogue.
//
// The same four launches RowFP8Execution.ffn issues, sequenced here on the
// caller's stream, so a host without Python gets the whole FFN in one call
// and the results are the same bits.  Intermediates live in a caller-owned
// workspace (vfb_fp8_ffn_workspace_bytes): nothing is allocated.
#include <cstdint>

#include "common.cuh"

namespace vfb {
namespace {

constexpr int64_t kAlign = 256;

int64_t align_up(int64_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

int64_t pad16(int64_t m) { return (m + 15) / 16 * 16; }

// Workspace layout (each region 256-byte aligned):
//   x codes  e4m3 [pad16(M), H]   x scales  fp32 [pad16(M)]
//   mid      bf16 [M, F]
//   mid codes e4m3 [pad16(M), F]  mid scales fp32 [pad16(M)]
struct FfnWorkspace {
  int64_t x_codes, x_scales, mid, mid_codes, mid_scales, total;
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
  w.total = at;
  return w;
}

bool ffn_shape_ok(int64_t M, int64_t H, int64_t F) {
  return M >= 0 && M <= ((int64_t)1 << 31) && H >= 16 && H <= 32768 && H % 32 == 0 && F >= 32 &&
         F <= 32768 && F % 32 == 0;
}

}  // namespace
}  // namespace vfb

extern "C" int64_t vfb_fp8_ffn_workspace_bytes(int64_t M, int64_t H, int64_t F) {
  using namespace vfb;
  if (!ffn_shape_ok(M, H, F)) return -1;
  return ffn_layout(M, H, F).total;
}

extern "C" int vfb_fp8_ffn(const void *x, int64_t M, int64_t H, int64_t ldx, const void *w_up, const float *s_up,
                           int64_t n_up, const void *w_down, const float *s_down, int32_t activation,
                           const void *bias_up, const void *bias_down, const void *residual, int64_t ldr,
                           const void *gate, int64_t gate_token_stride, int64_t tokens, void *out, int64_t ldo,
                           void *workspace, int64_t workspace_bytes, void *stream) {
  using namespace vfb;
  if (activation != VFB_EPI_GELU_TANH && activation != VFB_EPI_SWIGLU)
    return set_error(VFB_EINVAL, "vfb_fp8_ffn: activation must be VFB_EPI_GELU_TANH or VFB_EPI_SWIGLU");
  const int64_t F = activation == VFB_EPI_SWIGLU ? n_up / 2 : n_up;
  if (n_up <= 0 || (activation == VFB_EPI_SWIGLU && n_up % 2) || !ffn_shape_ok(M, H, F))
    return set_error(VFB_EINVAL, "vfb_fp8_ffn: need 16 <= H <= 32768 and 32 <= F <= 32768, both multiples of "
                                 "32 (F = n_up, or n_up / 2 for SWIGLU), M >= 0 (M=%lld H=%lld n_up=%lld)",
                     (long long)M, (long long)H, (long long)n_up);
  if (gate != nullptr && (residual == nullptr || tokens <= 0 || gate_token_stride < H))
    return set_error(VFB_EINVAL, "vfb_fp8_ffn: a gate needs a residual, tokens > 0 and a token stride >= H");
  const FfnWorkspace lay = ffn_layout(M, H, F);
  if (workspace == nullptr || workspace_bytes < lay.total || reinterpret_cast<uintptr_t>(workspace) % kAlign)
    return set_error(VFB_EINVAL, "vfb_fp8_ffn: workspace must be 256-byte aligned and hold %lld bytes",
                     (long long)lay.total);
  if (M == 0) return VFB_OK;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  const int64_t mp = pad16(M);
  void *xc = ws + lay.x_codes;
  float *xs = reinterpret_cast<float *>(ws + lay.x_scales);
  void *mid = ws + lay.mid;
  void *mc = ws + lay.mid_codes;
  float *ms = reinterpret_cast<float *>(ws + lay.mid_scales);

  int rc = vfb_fp8_quant_rows(x, M, H, ldx, xc, xs, mp, stream);
  if (rc != VFB_OK) return rc;

  vfb_epilogue up{};
  up.kind = activation;
  up.out = mid;
  up.ldo = F;
  up.bias = bias_up;
  rc = vfb_fp8_gemm(xc, H, xs, w_up, H, s_up, M, n_up, H, &up, stream);
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
