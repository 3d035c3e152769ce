// Epilogue building blocks shared by the tcgen05 GEMM kernels (fp8_gemm.cu,
// ffn_fused.cu): the activations written from their definitions, vector loads
// of the per-column operands, the row x column scale + bias step with the
// reference's two bf16 roundings, and the 32 x 32 output box written through
// 64-byte-swizzled shared memory and a TMA store.
#pragma once

#include "common.cuh"

namespace vfb {

constexpr int EPI_BOX_BYTES = 32 * 32 * 2;  // one 32 x 32 bf16 output box

// Weight slab kept in L2 per band of the tile order: 24 MiB.  Measured on the
// config 1 GEMM (K = 4096, 1 MiB of weight per 256-row tile): bands of 24
// tiles ran 5 % faster than the N-fastest order over all 48 tiles and 2 %
// faster than bands of 12.
constexpr int64_t kBandBytes = 24ll << 20;

// Weight tiles (256 rows of K bytes each) per band: as many as fit kBandBytes.
inline int band_width(int num_n_tiles, int64_t k_bytes) {
  int64_t band = kBandBytes / (256 * k_bytes);
  if (band < 1) band = 1;
  return band < num_n_tiles ? static_cast<int>(band) : num_n_tiles;
}

// Coordinates of the tile-th output tile in the banded order: bands of `band`
// weight tiles, row-block by row-block inside a band, weight tile fastest.
// The last band may be narrower.
__device__ __forceinline__ void band_coords(int tile, int num_m_tiles, int num_n_tiles, int band, int &m,
                                            int &n) {
  const int b = tile / (num_m_tiles * band);
  const int r = tile - b * num_m_tiles * band;
  const int w = min(band, num_n_tiles - b * band);
  m = r / w;
  n = b * band + r % w;
}

__device__ __forceinline__ float gelu_tanh(float y) {
  // 0.5 y (1 + tanh(sqrt(2/pi) (y + 0.044715 y^3)))
  const float k_beta = 0.7978845608028654f;
  const float k_kappa = 0.044715f;
  const float cube = y * y * y;
  const float inner = k_beta * (y + k_kappa * cube);
  return 0.5f * y * (1.0f + tanhf(inner));
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

__device__ __forceinline__ void load_f32x32(const float *__restrict__ p, float (&r)[32]) {
  const float4 *q = reinterpret_cast<const float4 *>(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 t = __ldg(q + i);
    r[4 * i] = t.x;
    r[4 * i + 1] = t.y;
    r[4 * i + 2] = t.z;
    r[4 * i + 3] = t.w;
  }
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16 *p, float (&r)[32]) {
  const uint4 *q = reinterpret_cast<const uint4 *>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 t = __ldg(q + i);
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&t);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      r[8 * i + 2 * j] = f.x;
      r[8 * i + 2 * j + 1] = f.y;
    }
  }
}

// Writes one 32 x 32 output box: lane i holds row i of the warp's 32 rows.
// The rows go to shared memory in the 64-byte swizzle the output tensor map
// uses (conflict-free 16-byte stores), then lane 0 issues one TMA store.
// Each warp cycles through EPI_BOXES staging boxes; a box is rewritten only
// after the store issued from it EPI_BOXES chunks earlier has read it.
// Exact packing of two bf16-representable floats (their low 16 bits are zero).
__device__ __forceinline__ uint32_t pack_exact_bf16x2(float lo, float hi) {
  return __byte_perm(__float_as_uint(lo), __float_as_uint(hi), 0x7632);
}


// KEEP = true stores with an evict_last L2 policy (data this kernel reads back
// soon, e.g. the FFN intermediate); otherwise evict_first (final outputs).
// ROUNDED = true: every y is already a bf16 value, so the halves are packed by
// a byte permute instead of a conversion (the conversion pipe is the busiest
// unit of the activation epilogues).
template <int BOXES, bool KEEP = false, bool ROUNDED = false>
__device__ __forceinline__ void store_box(uint8_t *warp_smem, int &box, const CUtensorMap *map,
                                          const float (&y)[32], int lane, int32_t col, int32_t row0,
                                          int32_t plane, bool any_row) {
  uint8_t *buf = warp_smem + box * EPI_BOX_BYTES;
  if (lane == 0) bulk_wait_group_read<BOXES - 1>();
  __syncwarp();
  uint4 *row = reinterpret_cast<uint4 *>(buf + lane * 64);
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 t;
    if constexpr (ROUNDED) {
      t.x = pack_exact_bf16x2(y[8 * j + 0], y[8 * j + 1]);
      t.y = pack_exact_bf16x2(y[8 * j + 2], y[8 * j + 3]);
      t.z = pack_exact_bf16x2(y[8 * j + 4], y[8 * j + 5]);
      t.w = pack_exact_bf16x2(y[8 * j + 6], y[8 * j + 7]);
    } else {
      t.x = pack_bf16x2(y[8 * j + 0], y[8 * j + 1]);
      t.y = pack_bf16x2(y[8 * j + 2], y[8 * j + 3]);
      t.z = pack_bf16x2(y[8 * j + 4], y[8 * j + 5]);
      t.w = pack_bf16x2(y[8 * j + 6], y[8 * j + 7]);
    }
    row[j ^ sw] = t;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0 && any_row) {
    tma_store_3d_hint(map, buf, col, row0, plane, KEEP ? l2_policy_evict_last() : l2_policy_evict_first());
    bulk_commit_group();
  }
  box = box + 1 == BOXES ? 0 : box + 1;
}

// y = bf16(acc * sa * sw) then bf16(y + bias): the _scaled_mm output followed
// by the separate bias add of the reference.  Unscaled (bf16 operands):
// y = bf16(acc), the F.linear output, then the bias the same way.
template <bool SCALED = true>
__device__ __forceinline__ void scale_bias(float (&v)[32], float sa, const float *sw,
                                           const __nv_bfloat16 *bias) {
  if constexpr (SCALED) {
    float w[32];
    load_f32x32(sw, w);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = v[j] * sa * w[j];
  }
  bf16r_x32(v);
  if (bias != nullptr) {
    float b[32];
    load_bf16x32(bias, b);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = v[j] + b[j];
    bf16r_x32(v);
  }
}

}  // namespace vfb
