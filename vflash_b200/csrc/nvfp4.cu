// NVFP4 (e2m1 with one ue4m3 scale per 16 elements) activation quantiser and
// block-scaled GEMM for sm_100a.
//
// Quantiser — replaces FlashInfer nvfp4_quantize(x, global_scale,
// sfLayout=128x4, do_shuffle=False) as called by NVFP4Execution.linear
// (src/vflash/native/h3_nvfp4_linear.py:102).  Per group of 16 elements
// (FlashInfer 0.6.18's default, non-TE-exact recipe, restated from its
// published source quantization_utils.cuh:294-380):
//   amax   = max |x|
//   sf     = e4m3_rn_satfinite(gsf * (amax * rcp(6)))
//   scale  = amax != 0 ? rcp(float(sf) * rcp(gsf)) : 0
//   code_i = e2m1_rn_satfinite(x_i * scale)        (element 2i in the low nibble)
// with rcp = rcp.approx.ftz.f32, so the codes and scales match that kernel bit
// for bit.  Scales are written in the 128x4 layout: for row m and 16-element
// group k, byte offset
//   (m/128)*(kt*512) + (k/4)*512 + (m%32)*16 + ((m%128)/32)*4 + k%4,
// kt = ceil(K/64); rows up to ceil128(M) and groups up to 4*kt exist, and the
// padding entries are written as 0.  One thread handles one 16-element group
// (two 16-byte loads, one 8-byte store of codes, one scale byte).  The
// multiplies flush subnormals (mul.ftz), as the reference's fast-math build
// does.
//
// GEMM — replaces FlashInfer mm_fp4(codes, packed.T, scales, scales_w.T,
// alpha, bf16, backend="cutlass") plus the bias add
// (h3_nvfp4_linear.py:118-139):
//   out[m,n] = bf16(alpha * sum_k e2m1(A[m,k]) sfA[m,k/16] e2m1(W[n,k]) sfW[n,k/16])
//   out      = bf16(out + bias[n])                       if bias != NULL
// One persistent CTA per SM, 128 x 256 tiles, K staged 256 elements (128
// bytes) at a time: TMA loads the packed codes (128-byte swizzle) and bulk
// copies load the matching 512-byte scale blocks, which the MMA thread moves
// into TMEM with tcgen05.cp before issuing four tcgen05.mma kind::mxf4nvf4
// (K = 64 each).  The two 256-column accumulators overlap by 64 TMEM columns
// ([0,256) and [192,448)) so that 64 columns remain for the scale factors; the
// epilogue drains the shared 64 columns of a tile first (reverse column
// order for even tiles, forward for odd tiles) and then releases the next
// tile's MMAs while it finishes the rest.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

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

// Multiplication with subnormal inputs and results flushed to zero, as the
// reference quantiser's fast-math build performs it.
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

__device__ __forceinline__ float e4m3_value(uint32_t byte) {
  // exact decode of a non-negative finite e4m3 byte
  const uint32_t e = (byte >> 3) & 0xF, m = byte & 0x7;
  if (e == 0) return static_cast<float>(m) * 0.001953125f;  // m * 2^-9
  return __uint_as_float(((e + 120u) << 23) | (m << 20));
}

__device__ __forceinline__ int64_t sf_offset(int64_t m, int64_t k, int64_t ktiles) {
  return (m >> 7) * (ktiles * 512) + (k >> 2) * 512 + (m & 31) * 16 + ((m & 127) >> 5) * 4 + (k & 3);
}

template <bool FP16, bool VEC>
__global__ void __launch_bounds__(256) nvfp4_quant_kernel(const uint16_t *__restrict__ x, int64_t M,
                                                          int64_t K, int64_t ldx,
                                                          const float *__restrict__ gsf_ptr,
                                                          uint8_t *__restrict__ codes,
                                                          uint8_t *__restrict__ sf, int64_t rows_pad,
                                                          int64_t groups_pad) {
  const float gsf = __ldg(gsf_ptr);
  const float rcp6 = rcp_approx_ftz(6.0f);
  const float rcp_gsf = rcp_approx_ftz(gsf);
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
      float amax = 0.0f;
#pragma unroll
      for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
      const float sf_value = mul_ftz(gsf, mul_ftz(amax, rcp6));
      sf_byte = e4m3_byte(sf_value);
      // amax != 0 compared after flushing a subnormal amax to zero
      const float scale =
          mul_ftz(amax, 1.0f) != 0.0f ? rcp_approx_ftz(mul_ftz(e4m3_value(sf_byte), rcp_gsf)) : 0.0f;
      float lo[8], hi[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        lo[j] = mul_ftz(v[j], scale);
        hi[j] = mul_ftz(v[8 + j], scale);
      }
      uint2 packed = make_uint2(pack_e2m1x8(lo), pack_e2m1x8(hi));
      *reinterpret_cast<uint2 *>(codes + m * (K / 2) + k * 8) = packed;
    }
    sf[sf_offset(m, k, ktiles)] = static_cast<uint8_t>(sf_byte);
  }
}

// ---------------------------------------------------------------------------
// GEMM
// ---------------------------------------------------------------------------
constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK_BYTES = 128;              // 256 e2m1 elements per stage
constexpr int KB_PER_STAGE = 4;            // MMAs (K = 64) per stage
constexpr int STAGES = 3;
constexpr int A_STAGE = BM * BK_BYTES;     // 16 KB
constexpr int B_STAGE = BN * BK_BYTES;     // 32 KB
constexpr int SFA_STAGE = KB_PER_STAGE * 512;      // 2 KB
constexpr int SFB_STAGE = 2 * KB_PER_STAGE * 512;  // 4 KB (two 128-row blocks)
constexpr int STAGE_BYTES = A_STAGE + B_STAGE + SFA_STAGE + SFB_STAGE;
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 512;
constexpr uint32_t ACC1_COL = 192;         // second accumulator overlaps the first by 64
constexpr uint32_t SFA_COL = 448;          // 4 columns per K = 64 block
constexpr uint32_t SFB_COL = 464;          // 8 columns per K = 64 block
constexpr int EPI_BOXES = 4;
constexpr int EPI_BOX_BYTES = 32 * 32 * 2;
constexpr int EPI_SMEM = 4 * EPI_BOXES * EPI_BOX_BYTES;
constexpr size_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_SMEM + 256;

struct Params {
  int64_t M, N, K;
  const uint8_t *sfa;     // activation scales, 128x4 layout
  const uint8_t *sfw;     // weight scales, 128x4 layout
  const float *alpha;     // device scalar
  const __nv_bfloat16 *bias;
  int32_t plane_width;
  int num_m_tiles, num_n_tiles, ktiles;  // ktiles = K / 64
  int *status;
};

__device__ __forceinline__ void store_box(uint8_t *warp_smem, int &box, const CUtensorMap *map,
                                          const float (&y)[32], int lane, int32_t col, int32_t row0,
                                          int32_t plane, bool any_row) {
  uint8_t *buf = warp_smem + box * EPI_BOX_BYTES;
  if (lane == 0) bulk_wait_group_read<EPI_BOXES - 1>();
  __syncwarp();
  uint4 *row = reinterpret_cast<uint4 *>(buf + lane * 64);
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 t;
    t.x = pack_bf16x2(y[8 * j + 0], y[8 * j + 1]);
    t.y = pack_bf16x2(y[8 * j + 2], y[8 * j + 3]);
    t.z = pack_bf16x2(y[8 * j + 4], y[8 * j + 5]);
    t.w = pack_bf16x2(y[8 * j + 6], y[8 * j + 7]);
    row[j ^ sw] = t;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0 && any_row) {
    tma_store_3d_hint(map, buf, col, row0, plane, l2_policy_evict_first());
    bulk_commit_group();
  }
  box = box + 1 == EPI_BOXES ? 0 : box + 1;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmOut, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  // per stage: A | B | SFA | SFB (all offsets multiples of 1024)
  uint8_t *sEpi = smem + STAGES * STAGE_BYTES;
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(sEpi + EPI_SMEM);
  uint64_t *empty_bar = full_bar + STAGES;
  uint64_t *tfull_bar = empty_bar + STAGES;  // one phase per tile
  uint64_t *tfree_bar = tfull_bar + 1;       // one phase per tile: shared columns drained
  uint64_t *drain_bar = tfree_bar + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain_bar + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tfree_bar, 128);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmOut);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = p.num_m_tiles * p.num_n_tiles;
  const int kstages = (p.ktiles + KB_PER_STAGE - 1) / KB_PER_STAGE;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer ----------------
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_phase[STAGES];
      bool issued[STAGES];
      for (int i = 0; i < STAGES; ++i) issued[i] = false;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m_tile = tile / p.num_n_tiles;
        const int n_tile = tile % p.num_n_tiles;
        for (int ks = 0; ks < kstages; ++ks) {
          if (!mbar_wait(&empty_bar[s], ph ^ 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          const int kb_here = min(KB_PER_STAGE, p.ktiles - ks * KB_PER_STAGE);
          // the tile's second 128-row weight block exists only when N reaches it
          const int w_blocks = (2 * n_tile + 1) * 128 < p.N ? 2 : 1;
          uint8_t *st = smem + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&full_bar[s], A_STAGE + B_STAGE + (1 + w_blocks) * kb_here * 512);
          tma_load_2d(st, &tmA, &full_bar[s], ks * BK_BYTES, m_tile * BM);
          // every tile row re-reads the whole weight: keep it resident in L2
          tma_load_2d_hint(st + A_STAGE, &tmB, &full_bar[s], ks * BK_BYTES, n_tile * BN,
                           l2_policy_evict_last());
          const int64_t kt0 = static_cast<int64_t>(ks) * KB_PER_STAGE;
          bulk_load(st + A_STAGE + B_STAGE, p.sfa + (m_tile * (int64_t)p.ktiles + kt0) * 512,
                    kb_here * 512, &full_bar[s]);
          for (int h = 0; h < w_blocks; ++h)
            bulk_load(st + A_STAGE + B_STAGE + SFA_STAGE + h * (KB_PER_STAGE * 512),
                      p.sfw + ((2 * n_tile + h) * (int64_t)p.ktiles + kt0) * 512, kb_here * 512,
                      &full_bar[s]);
          issued[s] = true;
          issued_phase[s] = ph;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      for (int i = 0; i < STAGES; ++i)
        if (issued[i]) mbar_wait(&full_bar[i], issued_phase[i], abort_flag, p.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = idesc_nvf4_f32(BM, BN);
      int s = 0;
      uint32_t ph = 0;
      int t = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++t) {
        // the previous tile's epilogue must have drained the shared columns
        // (and, by program order, everything of the tile before it)
        if (t > 0 && !mbar_wait(tfree_bar, (t - 1) & 1, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ((t & 1) ? ACC1_COL : 0u);
        for (int ks = 0; ks < kstages; ++ks) {
          if (!mbar_wait(&full_bar[s], ph, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int kb_here = min(KB_PER_STAGE, p.ktiles - ks * KB_PER_STAGE);
          uint8_t *st = smem + s * STAGE_BYTES;
          const uint32_t sfa_smem = smem_u32(st + A_STAGE + B_STAGE);
          const uint32_t sfb_smem = sfa_smem + SFA_STAGE;
          for (int kb = 0; kb < kb_here; ++kb) {
            tmem_cp_32x128b_warpx4(tmem_base + SFA_COL + 4 * kb, sf_block_desc(sfa_smem + kb * 512));
            tmem_cp_32x128b_warpx4(tmem_base + SFB_COL + 8 * kb, sf_block_desc(sfb_smem + kb * 512));
            tmem_cp_32x128b_warpx4(tmem_base + SFB_COL + 8 * kb + 4,
                                   sf_block_desc(sfb_smem + KB_PER_STAGE * 512 + kb * 512));
          }
          const uint64_t a_desc = sw128_kmajor_desc(smem_u32(st));
          const uint64_t b_desc = sw128_kmajor_desc(smem_u32(st + A_STAGE));
          for (int kb = 0; kb < kb_here; ++kb) {
            mma_mxf4nvf4(d_tmem, a_desc + 2 * kb, b_desc + 2 * kb, idesc,
                         tmem_base + SFA_COL + 4 * kb, tmem_base + SFB_COL + 8 * kb,
                         (ks | kb) != 0);
          }
          tc_commit(&empty_bar[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(tfull_bar);
      }
      tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, abort_flag, p.status);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    uint8_t *warp_smem = sEpi + q * EPI_BOXES * EPI_BOX_BYTES;
    int box = 0;
    const float alpha = __ldg(p.alpha);
    int t = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++t) {
      if (!mbar_wait(tfull_bar, t & 1, abort_flag, p.status)) break;
      tc_fence_after();
      const int m_tile = tile / p.num_n_tiles;
      const int n_tile = tile % p.num_n_tiles;
      const int64_t row0 = static_cast<int64_t>(m_tile) * BM + q * 32;
      const bool live = row0 + lane < p.M;
      const bool any_row = row0 < p.M;
      const bool odd = t & 1;
      const uint32_t t_row = tmem_base + (odd ? ACC1_COL : 0u) + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
      for (int i = 0; i < BN / 32; ++i) {
        // even tiles: columns 224..0 (shared 192..255 first); odd: 0..224
        const int c = odd ? i : (BN / 32 - 1 - i);
        const int32_t n = n_tile * BN + c * 32;
        float v[32];
        tmem_ld_32x32b_x32(t_row + c * 32, v);
        if (i == 1) {
          // the 64 shared columns are in registers or stored: release them
          tc_fence_before();
          mbar_arrive(tfree_bar);
        }
        if (n >= p.N) continue;  // warp-uniform
        const int32_t plane = n / p.plane_width;
        const int32_t col = n - plane * p.plane_width;
        if (live) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = bf16r(alpha * v[j]);
          if (p.bias != nullptr) {
            const uint4 *bq = reinterpret_cast<const uint4 *>(p.bias + n);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint4 bt = __ldg(bq + g);
              const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&bt);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float2 f = __bfloat1622float2(h[e]);
                v[8 * g + 2 * e] = bf16r(v[8 * g + 2 * e] + f.x);
                v[8 * g + 2 * e + 1] = bf16r(v[8 * g + 2 * e + 1] + f.y);
              }
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.0f;
        }
        store_box(warp_smem, box, &tmOut, v, lane, col, static_cast<int32_t>(row0), plane, any_row);
      }
    }
    if (lane == 0) bulk_wait_group_all();
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

int map_codes(CUtensorMap *map, const void *base, int64_t rows, int64_t row_bytes, int box_rows) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return set_error(VFB_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK_BYTES), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides,
                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VFB_ECUDA, "cuTensorMapEncodeTiled (nvfp4) failed (%d)", (int)r);
  return VFB_OK;
}

int map_out(CUtensorMap *map, void *base, int64_t width, int64_t rows, int64_t planes,
            int64_t plane_stride) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return set_error(VFB_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(planes)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(width) * 2, static_cast<cuuint64_t>(plane_stride) * 2};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                      CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VFB_ECUDA, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
  return VFB_OK;
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

extern "C" int vfb_nvfp4_gemm(const void *A, const void *sfa, const void *W, const void *sfw,
                              const float *alpha, int64_t M, int64_t N, int64_t K, const void *bias,
                              void *out, int64_t planes, void *stream) {
  using namespace vfb;
  if (M < 0 || N <= 0 || K <= 0 || K % 64 || N % 128 || planes < 1 || planes > 3 || N % planes ||
      (N / planes) % 32)
    return set_error(VFB_EINVAL,
                     "vfb_nvfp4_gemm: need K %% 64 == 0, N %% 128 == 0, 1..3 planes of width %% 32");
  if (M == 0) return VFB_OK;
  if (!A || !sfa || !W || !sfw || !alpha || !out)
    return set_error(VFB_EINVAL, "vfb_nvfp4_gemm: NULL operand");
  if (!a16(A) || !a16(W) || !a16(sfa) || !a16(sfw) || !a16(out) || (bias && !a16(bias)))
    return set_error(VFB_EINVAL, "vfb_nvfp4_gemm: operands must be 16-byte aligned");
  if ((K / 2) % 16) return set_error(VFB_EINVAL, "vfb_nvfp4_gemm: K/2 must be a multiple of 16 bytes");
  int sms = 0;
  int rc = check_device(&sms);
  if (rc != VFB_OK) return rc;
  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.sfa = static_cast<const uint8_t *>(sfa);
  p.sfw = static_cast<const uint8_t *>(sfw);
  p.alpha = alpha;
  p.bias = static_cast<const __nv_bfloat16 *>(bias);
  p.plane_width = static_cast<int32_t>(N / planes);
  p.num_m_tiles = static_cast<int>((M + BM - 1) / BM);
  p.num_n_tiles = static_cast<int>((N + BN - 1) / BN);
  p.ktiles = static_cast<int>(K / 64);
  p.status = device_status_ptr();
  CUtensorMap ta, tb, to;
  if ((rc = map_codes(&ta, A, M, K / 2, BM)) != VFB_OK) return rc;
  if ((rc = map_codes(&tb, W, N, K / 2, BN)) != VFB_OK) return rc;
  if ((rc = map_out(&to, out, N / planes, M, planes, M * (N / planes))) != VFB_OK) return rc;
  cudaError_t err =
      cudaFuncSetAttribute(nvfp4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (err != cudaSuccess) return set_error(VFB_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(err));
  const int tiles = p.num_m_tiles * p.num_n_tiles;
  const int grid = tiles < sms ? tiles : sms;
  nvfp4_gemm_kernel<<<grid, NUM_THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(ta, tb, to, p);
  err = cudaGetLastError();
  if (err != cudaSuccess) return set_error(VFB_ECUDA, "vfb_nvfp4_gemm launch: %s", cudaGetErrorString(err));
  return VFB_OK;
}
