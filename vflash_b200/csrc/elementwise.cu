// Strict-BF16 elementwise steps of the H3 block (HBM-bound).
//
// Each kernel keeps the BF16 rounding boundaries of the reference's Triton
// kernel it replaces (src/vflash/native/h3_fused_ops.py):
//   silu_mul              out = bf16(v * bf16(silu(g)))                  (185-224)
//   gate_residual         out = bf16(r + bf16(gate * p))                 (125-170)
//   qkv_direct_merge      base_b = bf16(base_b + bf16(a_b * s_b)), in place (901-949)
//   ffn_adapter_silu      v = bf16(bv + bf16(av * s)), g = bf16(bg + bf16(ag * s)),
//                         out = bf16(v * bf16(silu(g)))                  (254-284)
//   adapter_merge         out = bf16(base + bf16(a * s_branch))          (298-339)
//   adapter_gate_residual out = bf16(r + bf16(gate * bf16(base + bf16(a * s)))) (342-415)
//   modulate              out = bf16(bf16(x * bf16(1 + scale)) + shift)  (52-122, 575-611)
//   rotary                out = bf16(bf16(x * cos) + bf16(partner * sin)) on the first
//                         rotary_dim values of each head (split-half)   (421-510, 1031-1085)
// Work is split into 8-element groups along the contiguous last dimension;
// when every pointer and row stride allows, a group is one 16-byte load or
// store, otherwise the same kernel runs with scalar accesses.  Offsets are
// 64-bit.  A grid-stride loop sized to the SM count covers any length.
#include "common.cuh"

namespace vfb {
namespace {

constexpr int kThreads = 256;

template <bool VEC>
struct Group {
  float v[8];
  __device__ __forceinline__ void load(const __nv_bfloat16 *p) {
    if (VEC) {
      uint4 t = __ldg(reinterpret_cast<const uint4 *>(p));
      const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&t);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __bfloat162float(p[j]);
    }
  }
  __device__ __forceinline__ void store(__nv_bfloat16 *p) const {
    if (VEC) {
      uint4 t;
      t.x = pack_bf16x2(v[0], v[1]);
      t.y = pack_bf16x2(v[2], v[3]);
      t.z = pack_bf16x2(v[4], v[5]);
      t.w = pack_bf16x2(v[6], v[7]);
      *reinterpret_cast<uint4 *>(p) = t;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) p[j] = __float2bfloat16_rn(v[j]);
    }
  }
};

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// Row-structured index: group i of a [rows, width] matrix with width % 8 == 0.
struct RowIndex {
  int64_t row;
  int64_t col;
};

__device__ __forceinline__ RowIndex split(int64_t group, int64_t groups_per_row) {
  RowIndex r;
  r.row = group / groups_per_row;
  r.col = (group - r.row * groups_per_row) * 8;
  return r;
}

template <bool VEC>
__global__ void __launch_bounds__(kThreads) silu_mul_kernel(const __nv_bfloat16 *packed, int64_t rows,
                                                            int64_t width, __nv_bfloat16 *out,
                                                            int64_t out_ld) {
  const int64_t gpr = width / 8;
  const int64_t total = rows * gpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const RowIndex ix = split(i, gpr);
    const __nv_bfloat16 *base = packed + ix.row * 2 * width + ix.col;
    Group<VEC> v, g;
    v.load(base);
    g.load(base + width);
#pragma unroll
    for (int j = 0; j < 8; ++j) v.v[j] = v.v[j] * bf16r(silu(g.v[j]));
    v.store(out + ix.row * out_ld + ix.col);
  }
}

template <bool VEC>
__global__ void __launch_bounds__(kThreads) ffn_adapter_silu_kernel(
    const __nv_bfloat16 *base, const __nv_bfloat16 *adapter, int64_t rows, int64_t width,
    float scaling, __nv_bfloat16 *out, int64_t out_ld) {
  const int64_t gpr = width / 8;
  const int64_t total = rows * gpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const RowIndex ix = split(i, gpr);
    const int64_t off = ix.row * 2 * width + ix.col;
    Group<VEC> bv, bg, av, ag;
    bv.load(base + off);
    bg.load(base + off + width);
    av.load(adapter + off);
    ag.load(adapter + off + width);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float value = bf16r(bv.v[j] + bf16r(av.v[j] * scaling));
      const float gate = bf16r(bg.v[j] + bf16r(ag.v[j] * scaling));
      bv.v[j] = value * bf16r(silu(gate));
    }
    bv.store(out + ix.row * out_ld + ix.col);
  }
}

// residual/projected [batch*tokens, hidden] contiguous; gate [tokens, hidden]
// with row stride gate_ts and unit column stride.
template <bool VEC>
__global__ void __launch_bounds__(kThreads) gate_residual_kernel(
    const __nv_bfloat16 *residual, const __nv_bfloat16 *gate, int64_t gate_ts,
    const __nv_bfloat16 *projected, int64_t rows, int64_t tokens, int64_t hidden,
    __nv_bfloat16 *out) {
  const int64_t gpr = hidden / 8;
  const int64_t total = rows * gpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const RowIndex ix = split(i, gpr);
    const int64_t off = ix.row * hidden + ix.col;
    Group<VEC> r, g, p;
    r.load(residual + off);
    g.load(gate + (ix.row % tokens) * gate_ts + ix.col);
    p.load(projected + off);
#pragma unroll
    for (int j = 0; j < 8; ++j) r.v[j] = r.v[j] + bf16r(g.v[j] * p.v[j]);
    r.store(out + off);
  }
}

// value [rows, hidden] contiguous; scale / shift [tokens, hidden] with row
// strides scale_ts / shift_ts (0 broadcasts one row) and unit column stride.
template <bool VEC>
__global__ void __launch_bounds__(kThreads) modulate_kernel(
    const __nv_bfloat16 *value, const __nv_bfloat16 *scale, int64_t scale_ts,
    const __nv_bfloat16 *shift, int64_t shift_ts, int64_t rows, int64_t tokens, int64_t hidden,
    __nv_bfloat16 *out) {
  const int64_t gpr = hidden / 8;
  const int64_t total = rows * gpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const RowIndex ix = split(i, gpr);
    const int64_t off = ix.row * hidden + ix.col;
    const int64_t token = ix.row % tokens;
    Group<VEC> x, sc, sh;
    x.load(value + off);
    sc.load(scale + token * scale_ts + ix.col);
    sh.load(shift + token * shift_ts + ix.col);
#pragma unroll
    for (int j = 0; j < 8; ++j) x.v[j] = bf16r(x.v[j] * bf16r(1.0f + sc.v[j])) + sh.v[j];
    x.store(out + off);
  }
}

// value [rows, heads, head_dim] contiguous; cos / sin [tokens, rotary_dim]
// with row strides cos_ts / sin_ts and unit column stride.  For d < half the
// partner is -x[d + half], otherwise x[d - half]; d >= rotary_dim is copied.
__global__ void __launch_bounds__(kThreads) rotary_kernel(
    const __nv_bfloat16 *value, const __nv_bfloat16 *cos, int64_t cos_ts, const __nv_bfloat16 *sin,
    int64_t sin_ts, int64_t rows, int64_t tokens, int64_t heads, int64_t head_dim, int64_t rotary_dim,
    __nv_bfloat16 *out) {
  const int64_t total = rows * heads * head_dim;
  const int64_t half = rotary_dim / 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t d = i % head_dim;
    const float x = __bfloat162float(value[i]);
    if (d >= rotary_dim) {
      out[i] = value[i];
      continue;
    }
    const int64_t token = (i / (heads * head_dim)) % tokens;
    const float partner = d < half ? -__bfloat162float(value[i + half]) : __bfloat162float(value[i - half]);
    const float c = __bfloat162float(cos[token * cos_ts + d]);
    const float s = __bfloat162float(sin[token * sin_ts + d]);
    out[i] = __float2bfloat16_rn(bf16r(x * c) + bf16r(partner * s));
  }
}

template <bool VEC>
__global__ void __launch_bounds__(kThreads) adapter_gate_residual_kernel(
    const __nv_bfloat16 *base, const __nv_bfloat16 *adapter, const __nv_bfloat16 *residual,
    const __nv_bfloat16 *gate, int64_t gate_ts, int64_t rows, int64_t tokens, int64_t hidden,
    float scaling, __nv_bfloat16 *out) {
  const int64_t gpr = hidden / 8;
  const int64_t total = rows * gpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const RowIndex ix = split(i, gpr);
    const int64_t off = ix.row * hidden + ix.col;
    Group<VEC> b, a, r, g;
    b.load(base + off);
    a.load(adapter + off);
    r.load(residual + off);
    g.load(gate + (ix.row % tokens) * gate_ts + ix.col);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float adapted = bf16r(b.v[j] + bf16r(a.v[j] * scaling));
      r.v[j] = r.v[j] + bf16r(g.v[j] * adapted);
    }
    r.store(out + off);
  }
}

// base/adapter [rows, width]; `branches` equal-width column branches with
// their own scaling.  out may alias base (in-place merge).
template <bool VEC>
__global__ void __launch_bounds__(kThreads) adapter_merge_kernel(
    const __nv_bfloat16 *base, const __nv_bfloat16 *adapter, int64_t rows, int64_t width,
    int64_t branch_width, float s0, float s1, float s2, __nv_bfloat16 *out) {
  const int64_t gpr = width / 8;
  const int64_t total = rows * gpr;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const RowIndex ix = split(i, gpr);
    const int64_t off = ix.row * width + ix.col;
    Group<VEC> b, a;
    b.load(base + off);
    a.load(adapter + off);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t branch = (ix.col + j) / branch_width;
      const float s = branch == 0 ? s0 : (branch == 1 ? s1 : s2);
      b.v[j] = b.v[j] + bf16r(a.v[j] * s);
    }
    b.store(out + off);
  }
}

// In-place merge of three separate branch adapters [rows, width] into the
// packed base [rows, 3*width].
template <bool VEC>
__global__ void __launch_bounds__(kThreads) qkv_direct_merge_kernel(
    __nv_bfloat16 *base, const __nv_bfloat16 *a0, const __nv_bfloat16 *a1,
    const __nv_bfloat16 *a2, int64_t rows, int64_t width, float s0, float s1, float s2) {
  const int64_t gpr = width / 8;
  const int64_t per_branch = rows * gpr;
  const int64_t total = 3 * per_branch;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int branch = static_cast<int>(i / per_branch);
    const RowIndex ix = split(i - branch * per_branch, gpr);
    const __nv_bfloat16 *ad = branch == 0 ? a0 : (branch == 1 ? a1 : a2);
    const float s = branch == 0 ? s0 : (branch == 1 ? s1 : s2);
    __nv_bfloat16 *dst = base + ix.row * 3 * width + branch * width + ix.col;
    Group<VEC> b, a;
    b.load(dst);
    a.load(ad + ix.row * width + ix.col);
#pragma unroll
    for (int j = 0; j < 8; ++j) b.v[j] = b.v[j] + bf16r(a.v[j] * s);
    b.store(dst);
  }
}

bool a16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

int grid_for(int64_t groups) {
  int sms = 0;
  if (check_device(&sms) != VFB_OK) return -1;
  int64_t blocks = (groups + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sms) * 16;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : static_cast<int>(blocks);
}

int finish(const char *what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_error(VFB_ECUDA, "%s launch: %s", what, cudaGetErrorString(err));
  return VFB_OK;
}

}  // namespace
}  // namespace vfb

using vfb::a16;

extern "C" int vfb_silu_mul(const void *packed, int64_t rows, int64_t width, void *out,
                            int64_t out_ld, void *stream) {
  using namespace vfb;
  if (rows < 0 || width <= 0 || width % 8 || out_ld < width || packed == nullptr || out == nullptr)
    return set_error(VFB_EINVAL, "vfb_silu_mul: need rows >= 0, width %% 8 == 0, out_ld >= width");
  if (rows == 0) return VFB_OK;
  const int grid = grid_for(rows * (width / 8));
  if (grid < 0) return VFB_EDEVICE;
  const auto *p = static_cast<const __nv_bfloat16 *>(packed);
  auto *o = static_cast<__nv_bfloat16 *>(out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a16(p) && a16(o) && out_ld % 8 == 0)
    silu_mul_kernel<true><<<grid, kThreads, 0, s>>>(p, rows, width, o, out_ld);
  else
    silu_mul_kernel<false><<<grid, kThreads, 0, s>>>(p, rows, width, o, out_ld);
  return finish("vfb_silu_mul");
}

extern "C" int vfb_ffn_adapter_silu(const void *base, const void *adapter, int64_t rows,
                                    int64_t width, float scaling, void *out, int64_t out_ld,
                                    void *stream) {
  using namespace vfb;
  if (rows < 0 || width <= 0 || width % 8 || out_ld < width || !base || !adapter || !out)
    return set_error(VFB_EINVAL, "vfb_ffn_adapter_silu: need width %% 8 == 0, out_ld >= width");
  if (rows == 0) return VFB_OK;
  const int grid = grid_for(rows * (width / 8));
  if (grid < 0) return VFB_EDEVICE;
  const auto *b = static_cast<const __nv_bfloat16 *>(base);
  const auto *a = static_cast<const __nv_bfloat16 *>(adapter);
  auto *o = static_cast<__nv_bfloat16 *>(out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a16(b) && a16(a) && a16(o) && out_ld % 8 == 0)
    ffn_adapter_silu_kernel<true><<<grid, kThreads, 0, s>>>(b, a, rows, width, scaling, o, out_ld);
  else
    ffn_adapter_silu_kernel<false><<<grid, kThreads, 0, s>>>(b, a, rows, width, scaling, o, out_ld);
  return finish("vfb_ffn_adapter_silu");
}

extern "C" int vfb_gate_residual(const void *residual, const void *gate, int64_t gate_token_stride,
                                 const void *projected, int64_t rows, int64_t tokens,
                                 int64_t hidden, void *out, void *stream) {
  using namespace vfb;
  if (rows < 0 || tokens <= 0 || hidden <= 0 || hidden % 8 || gate_token_stride < 0 ||
      !residual || !gate || !projected || !out)
    return set_error(VFB_EINVAL, "vfb_gate_residual: need hidden %% 8 == 0, tokens > 0");
  if (rows == 0) return VFB_OK;
  const int grid = grid_for(rows * (hidden / 8));
  if (grid < 0) return VFB_EDEVICE;
  const auto *r = static_cast<const __nv_bfloat16 *>(residual);
  const auto *g = static_cast<const __nv_bfloat16 *>(gate);
  const auto *p = static_cast<const __nv_bfloat16 *>(projected);
  auto *o = static_cast<__nv_bfloat16 *>(out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a16(r) && a16(g) && a16(p) && a16(o) && gate_token_stride % 8 == 0)
    gate_residual_kernel<true><<<grid, kThreads, 0, s>>>(r, g, gate_token_stride, p, rows, tokens, hidden, o);
  else
    gate_residual_kernel<false><<<grid, kThreads, 0, s>>>(r, g, gate_token_stride, p, rows, tokens, hidden, o);
  return finish("vfb_gate_residual");
}

extern "C" int vfb_adapter_gate_residual(const void *base, const void *adapter, const void *residual,
                                         const void *gate, int64_t gate_token_stride, int64_t rows,
                                         int64_t tokens, int64_t hidden, float scaling, void *out,
                                         void *stream) {
  using namespace vfb;
  if (rows < 0 || tokens <= 0 || hidden <= 0 || hidden % 8 || gate_token_stride < 0 ||
      !base || !adapter || !residual || !gate || !out)
    return set_error(VFB_EINVAL, "vfb_adapter_gate_residual: need hidden %% 8 == 0, tokens > 0");
  if (rows == 0) return VFB_OK;
  const int grid = grid_for(rows * (hidden / 8));
  if (grid < 0) return VFB_EDEVICE;
  const auto *b = static_cast<const __nv_bfloat16 *>(base);
  const auto *a = static_cast<const __nv_bfloat16 *>(adapter);
  const auto *r = static_cast<const __nv_bfloat16 *>(residual);
  const auto *g = static_cast<const __nv_bfloat16 *>(gate);
  auto *o = static_cast<__nv_bfloat16 *>(out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a16(b) && a16(a) && a16(r) && a16(g) && a16(o) && gate_token_stride % 8 == 0)
    adapter_gate_residual_kernel<true><<<grid, kThreads, 0, s>>>(b, a, r, g, gate_token_stride, rows,
                                                                 tokens, hidden, scaling, o);
  else
    adapter_gate_residual_kernel<false><<<grid, kThreads, 0, s>>>(b, a, r, g, gate_token_stride, rows,
                                                                  tokens, hidden, scaling, o);
  return finish("vfb_adapter_gate_residual");
}

extern "C" int vfb_adapter_merge(const void *base, const void *adapter, int64_t rows, int64_t width,
                                 int32_t branches, const float *scalings, void *out, void *stream) {
  using namespace vfb;
  if (rows < 0 || width <= 0 || width % 8 || branches < 1 || branches > 3 || width % branches ||
      (width / branches) % 8 || !base || !adapter || !out || !scalings)
    return set_error(VFB_EINVAL,
                     "vfb_adapter_merge: need 1..3 branches of equal width, multiples of 8");
  if (rows == 0) return VFB_OK;
  const int grid = grid_for(rows * (width / 8));
  if (grid < 0) return VFB_EDEVICE;
  const auto *b = static_cast<const __nv_bfloat16 *>(base);
  const auto *a = static_cast<const __nv_bfloat16 *>(adapter);
  auto *o = static_cast<__nv_bfloat16 *>(out);
  const float s0 = scalings[0], s1 = branches > 1 ? scalings[1] : s0, s2 = branches > 2 ? scalings[2] : s0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a16(b) && a16(a) && a16(o))
    adapter_merge_kernel<true><<<grid, kThreads, 0, s>>>(b, a, rows, width, width / branches, s0, s1, s2, o);
  else
    adapter_merge_kernel<false><<<grid, kThreads, 0, s>>>(b, a, rows, width, width / branches, s0, s1, s2, o);
  return finish("vfb_adapter_merge");
}

extern "C" int vfb_qkv_direct_merge(void *base, const void *adapter_q, const void *adapter_k,
                                    const void *adapter_v, int64_t rows, int64_t width,
                                    const float *scalings, void *stream) {
  using namespace vfb;
  if (rows < 0 || width <= 0 || width % 8 || !base || !adapter_q || !adapter_k || !adapter_v ||
      !scalings)
    return set_error(VFB_EINVAL, "vfb_qkv_direct_merge: need width %% 8 == 0 and three adapters");
  if (rows == 0) return VFB_OK;
  const int grid = grid_for(3 * rows * (width / 8));
  if (grid < 0) return VFB_EDEVICE;
  auto *b = static_cast<__nv_bfloat16 *>(base);
  const auto *q = static_cast<const __nv_bfloat16 *>(adapter_q);
  const auto *k = static_cast<const __nv_bfloat16 *>(adapter_k);
  const auto *v = static_cast<const __nv_bfloat16 *>(adapter_v);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a16(b) && a16(q) && a16(k) && a16(v))
    qkv_direct_merge_kernel<true><<<grid, kThreads, 0, s>>>(b, q, k, v, rows, width, scalings[0],
                                                            scalings[1], scalings[2]);
  else
    qkv_direct_merge_kernel<false><<<grid, kThreads, 0, s>>>(b, q, k, v, rows, width, scalings[0],
                                                             scalings[1], scalings[2]);
  return finish("vfb_qkv_direct_merge");
}

extern "C" int vfb_modulate(const void *value, const void *scale, int64_t scale_token_stride,
                            const void *shift, int64_t shift_token_stride, int64_t rows, int64_t tokens,
                            int64_t hidden, void *out, void *stream) {
  using namespace vfb;
  if (rows < 0 || tokens <= 0 || hidden <= 0 || hidden % 8 || scale_token_stride < 0 ||
      shift_token_stride < 0 || !value || !scale || !shift || !out)
    return set_error(VFB_EINVAL, "vfb_modulate: need hidden %% 8 == 0, tokens > 0, strides >= 0");
  if (rows == 0) return VFB_OK;
  const int grid = grid_for(rows * (hidden / 8));
  if (grid < 0) return VFB_EDEVICE;
  const auto *x = static_cast<const __nv_bfloat16 *>(value);
  const auto *sc = static_cast<const __nv_bfloat16 *>(scale);
  const auto *sh = static_cast<const __nv_bfloat16 *>(shift);
  auto *o = static_cast<__nv_bfloat16 *>(out);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a16(x) && a16(sc) && a16(sh) && a16(o) && scale_token_stride % 8 == 0 && shift_token_stride % 8 == 0)
    modulate_kernel<true><<<grid, kThreads, 0, s>>>(x, sc, scale_token_stride, sh, shift_token_stride, rows,
                                                    tokens, hidden, o);
  else
    modulate_kernel<false><<<grid, kThreads, 0, s>>>(x, sc, scale_token_stride, sh, shift_token_stride, rows,
                                                     tokens, hidden, o);
  return finish("vfb_modulate");
}

extern "C" int vfb_rotary(const void *value, const void *cos, int64_t cos_token_stride, const void *sin,
                          int64_t sin_token_stride, int64_t rows, int64_t tokens, int64_t heads,
                          int64_t head_dim, int64_t rotary_dim, void *out, void *stream) {
  using namespace vfb;
  if (rows < 0 || tokens <= 0 || heads <= 0 || head_dim <= 0 || rotary_dim <= 0 ||
      rotary_dim > head_dim || rotary_dim % 2 || cos_token_stride < 0 || sin_token_stride < 0 ||
      !value || !cos || !sin || !out)
    return set_error(VFB_EINVAL, "vfb_rotary: need 0 < rotary_dim <= head_dim, rotary_dim even, tokens > 0");
  if (rows == 0) return VFB_OK;
  const int grid = grid_for(rows * heads * head_dim);
  if (grid < 0) return VFB_EDEVICE;
  rotary_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16 *>(value), static_cast<const __nv_bfloat16 *>(cos), cos_token_stride,
      static_cast<const __nv_bfloat16 *>(sin), sin_token_stride, rows, tokens, heads, head_dim, rotary_dim,
      static_cast<__nv_bfloat16 *>(out));
  return finish("vfb_rotary");
}
