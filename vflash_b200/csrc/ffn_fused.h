// Host interface of the fused FFN kernel (ffn_fused.cu), used by the C entry
// points in ffn.cu.
#pragma once

#include <stdint.h>

namespace vfb {

struct FfnFusedArgs {
  int64_t M, H, F;          // rows, hidden, intermediate width
  int32_t activation;       // VFB_EPI_GELU_TANH or VFB_EPI_SWIGLU
  const void *x_codes;      // e4m3 [M, H], row stride H
  const float *x_scales;    // [M]
  const void *w_up;         // e4m3 [F or 2F, H]
  const float *s_up;
  const void *w_down;       // e4m3 [H, F]
  const float *s_down;
  const void *bias_up;      // bf16 or NULL
  const void *bias_down;
  const void *residual;     // bf16 [M, H] (row stride ldr) or NULL
  int64_t ldr;
  const void *gate;         // bf16 [tokens, H] or NULL
  int64_t gate_token_stride;
  int64_t tokens;
  void *out;                // bf16 [M, H], row stride ldo
  int64_t ldo;
  const void *mid;          // workspace: bf16 [M, F]
  void *mid_codes;          // workspace: e4m3 [M, F]
  uint32_t *amax_bits;      // workspace: [M], followed by the counters; zeroed by the launch
  int *counters;            // workspace: 1 + 2 * ceil(M / 256)
  int64_t zero_bytes;       // bytes from amax_bits to the end of the counters
  // schedule overrides (<= 0 / < 0: defaults)
  int group;
  int band_up;
  int band_down;
  int lead;
  int lag;
};

// Whether the fused kernel handles these widths (GELU: F % 256 == 0; SwiGLU: F % 128 == 0; H % 32 == 0).
int ffn_fused_supported(int32_t activation, int64_t H, int64_t F);

// Zeroes the row maxima and counters, then launches the fused kernel on `stream`.
int launch_ffn_fused(const FfnFusedArgs &args, void *stream);

}  // namespace vfb
