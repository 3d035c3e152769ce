// NVFP4 block-scaled GEMM for sm_100a (e2m1 x e2m1 with one ue4m3 scale per
// 16 K-elements, fp32 accumulate, bf16 out).
//
// Replaces FlashInfer mm_fp4(codes, packed.T, scales, weight_scales.T, alpha,
// bf16, backend="cutlass") plus the bias add of NVFP4Execution.linear
// (src/vflash/native/h3_nvfp4_linear.py:118-139):
//   out[m,n] = bf16(alpha * sum_k e2m1(A[m,k]) sfA[m,k/16] e2m1(W[n,k]) sfW[n,k/16])
//   out      = bf16(out + bias[n])                       if bias != NULL
//
// Structure: persistent CTA pairs (cta_group::2), 256 x 256 output tile per
// pair in the banded order of the FP8 GEMM (epilogue.cuh: band_coords), K
// staged 256 elements (128 bytes of codes) at a time.  Each CTA TMA-
// loads its own 128 A rows and 128 of the tile's 256 weight rows (128-byte
// swizzle, no multicast), its A rows' scale blocks and the scale blocks of all
// 256 weight rows (512-byte blocks in the 128x4 layout, loaded through 2-D
// tensor maps over those blocks so that rows past the end read as zero).  One
// elected lane of the leader's converged MMA warp moves each K = 64 block's
// scales into both CTAs' TMEM
// with tcgen05.cp.cta_group::2.32x128b.warpx4 and issues
// tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 (M = 256,
// N = 256, K = 64).  TMEM per CTA: two 256-column accumulators overlapping by
// 64 columns ([0,256) and [192,448)) and 48 columns of scales at [448,496).
// Eight epilogue warps (two groups of four, each half of a tile's columns):
// the group holding a tile's 64 shared columns reads them first (reverse
// column order for even tiles, forward for odd) and then lets the next tile's
// MMAs start.
// Launched as a programmatic dependent of the previous kernel (the quantiser):
// setup overlaps its last wave; grid_dependency_wait() precedes every global access.
#include <cudaTypedefs.h>

#include <atomic>

#include "common.cuh"
#include "epilogue.cuh"
#include "nvfp4_quant.cuh"

namespace vfb {
namespace {

constexpr int BM = 128;                    // A rows per CTA (pair: 256)
constexpr int BN = 256;                    // output columns per pair tile
constexpr int BN_HALF = BN / 2;            // weight rows per CTA
constexpr int BK_BYTES = 128;              // 256 e2m1 elements per stage
constexpr int KB_PER_STAGE = 4;            // MMAs (K = 64) per stage
constexpr int STAGES = 5;
constexpr int A_STAGE = BM * BK_BYTES;                 // 16 KB
constexpr int B_STAGE = BN_HALF * BK_BYTES;            // 16 KB
constexpr int SFA_STAGE = KB_PER_STAGE * 512;          // 2 KB: own 128 rows
constexpr int SFB_STAGE = 2 * KB_PER_STAGE * 512;      // 4 KB: all 256 weight rows
constexpr int STAGE_BYTES = A_STAGE + B_STAGE + SFA_STAGE + SFB_STAGE;
// Warps 0 (TMA) and 1 (MMA) plus the epilogue warps: one group of four (one
// per TMEM lane quarter) per EPI_GROUPS, each group taking an equal share of
// the tile's 32-column chunks.
constexpr int EPI_GROUPS = 2;
constexpr int EPI_WARPS = 4 * EPI_GROUPS;
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
constexpr int TMEM_COLS = 512;
constexpr uint32_t ACC1_COL = 192;
constexpr uint32_t SFA_COL = 448;          // 4 columns per K = 64 block
constexpr uint32_t SFB_COL = 464;          // 8 columns per K = 64 block
constexpr int EPI_BOXES = 2;
constexpr int EPI_SMEM = EPI_WARPS * EPI_BOXES * EPI_BOX_BYTES;
constexpr size_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_SMEM + 256;

struct Params {
  int64_t M, N, K;  // N: GEMM output columns (the packed 2F for SWIGLU)
  const float *alpha;
  const float *alpha_div;  // NULL, or alpha is divided by it (IEEE division, once per thread)
  const __nv_bfloat16 *bias;
  int32_t plane_width;
  int32_t F;               // SWIGLU: output width
  const __nv_bfloat16 *adapter[3];  // STORE: LoRA branch per plane (NULL = none)
  int64_t adapter_ld;
  float scaling[3];
  const __nv_bfloat16 *residual;    // RESIDUAL
  int64_t ldr;
  const __nv_bfloat16 *gate;
  int64_t gate_ts;
  int64_t gate_hs;
  int64_t tokens;
  int num_m_tiles, num_n_tiles, ktiles;  // ktiles = K / 64
  int band_n;                            // weight tiles per band of the tile order
  int *status;
  // quantised output (vfb_nvfp4_gemm_quant): e2m1 codes [M, q_ld] and 128x4
  // scales of the bf16 result, for the next NVFP4 linear
  uint8_t *q_codes;
  uint8_t *q_sf;
  const float *q_gsf;
  int64_t q_ld;        // code bytes per row (output width / 2)
  int64_t q_rows_pad;  // ceil128(M): scale rows that exist
  int64_t q_ktiles;    // output width / 64
};

// The bf16 values of 32 output columns of row m, quantised as the next
// NVFP4 linear's quantiser would (nvfp4_group, the same arithmetic as
// vfb_nvfp4_quant_rows): 16 code bytes and two scale bytes.  Rows past M
// inside the padded scale rows get zero scales, as the quantiser writes them.
__device__ __forceinline__ void store_nvfp4(const Params &p, float (&v)[32], int64_t m, bool live, int32_t col,
                                            const Nvfp4Consts &c) {
  if (m >= p.q_rows_pad) return;
  uint32_t s0 = 0, s1 = 0;
  if (live) {
    bf16r_x32(v);  // the value a bf16 output would hold
    uint2 c0, c1;
    s0 = nvfp4_group(v, c, c0);
    s1 = nvfp4_group(v + 16, c, c1);
    *reinterpret_cast<uint4 *>(p.q_codes + m * p.q_ld + col / 2) = make_uint4(c0.x, c0.y, c1.x, c1.y);
  }
  // col % 32 == 0: groups k0 and k0 + 1 are adjacent bytes of the 128x4 layout
  *reinterpret_cast<uint16_t *>(p.q_sf + sf_offset(m, col / 16, p.q_ktiles)) = static_cast<uint16_t>(s0 | (s1 << 8));
}

// y = bf16(alpha * acc) then bf16(y + bias): mm_fp4's output, then the
// separate bias add of NVFP4Execution.linear (h3_nvfp4_linear.py:139).
__device__ __forceinline__ void alpha_bias(float (&v)[32], float alpha, const __nv_bfloat16 *bias) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = alpha * v[j];
  bf16r_x32(v);
  if (bias != nullptr) {
    float b[32];
    load_bf16x32(bias, b);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = v[j] + b[j];
    bf16r_x32(v);
  }
}

template <int EPI, bool QUANT = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ CUtensorMap tmSFA,
                      const __grid_constant__ CUtensorMap tmSFB, const __grid_constant__ CUtensorMap tmOut,
                      const Params p) {
  constexpr bool kSwiglu = EPI == VFB_EPI_SWIGLU;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  // per stage: A | B | SFA | SFB (every offset a multiple of 1024)
  uint8_t *sEpi = smem + STAGES * STAGE_BYTES;
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(sEpi + EPI_SMEM);
  uint64_t *empty_bar = full_bar + STAGES;
  uint64_t *tfull_bar = empty_bar + STAGES;  // per CTA, one phase per tile
  uint64_t *tfree_bar = tfull_bar + 1;       // leader: both epilogues drained the shared columns
  uint64_t *drain_bar = tfree_bar + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain_bar + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x / 2;
  const int num_pairs = gridDim.x / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, 1);
    // every epilogue thread of both CTAs arrives once per tile: the group that
    // holds the shared columns after reading them, the others at the tile's
    // start (they are done with the previous tile by then)
    mbar_init(tfree_bar, 2 * 32 * EPI_WARPS);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (kSwiglu) tma_prefetch_desc(&tmB2);
    tma_prefetch_desc(&tmSFA);
    tma_prefetch_desc(&tmSFB);
    tma_prefetch_desc(&tmOut);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dependency_wait();  // the previous kernel's outputs (A, its scales) are complete
  const int num_tiles = p.num_m_tiles * p.num_n_tiles;
  const int kstages = (p.ktiles + KB_PER_STAGE - 1) / KB_PER_STAGE;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer (both CTAs) ----------------
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_phase[STAGES];
      bool issued[STAGES];
      for (int i = 0; i < STAGES; ++i) issued[i] = false;
      bool ok = true;
      const uint64_t keep = l2_policy_evict_last();
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
        int m_tile, n_tile;
        band_coords(tile, p.num_m_tiles, p.num_n_tiles, p.band_n, m_tile, n_tile);
        const int m_block = 2 * m_tile + static_cast<int>(rank);  // this CTA's 128-row block
        for (int ks = 0; ks < kstages; ++ks) {
          if (!mbar_wait(&empty_bar[s], ph ^ 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = map_to_rank(smem_u32(&full_bar[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[s], 2 * STAGE_BYTES);
          uint8_t *st = smem + s * STAGE_BYTES;
          const int32_t kt0 = ks * KB_PER_STAGE;
          tma_load_2d_pair(st, &tmA, full_leader, ks * BK_BYTES, m_block * BM);
          if (kSwiglu) {
            // leader: value rows [n*128, +128); peer: the matching gate rows (second half of W)
            tma_load_2d_pair_hint(st + A_STAGE, rank == 0 ? &tmB : &tmB2, full_leader, ks * BK_BYTES,
                                  n_tile * BN_HALF, keep);
          } else {
            tma_load_2d_pair_hint(st + A_STAGE, &tmB, full_leader, ks * BK_BYTES,
                                  n_tile * BN + static_cast<int32_t>(rank) * BN_HALF, keep);
          }
          // scale blocks: rows of 256 bytes, two per 512-byte block
          tma_load_2d_pair(st + A_STAGE + B_STAGE, &tmSFA, full_leader, 0,
                           (m_block * p.ktiles + kt0) * 2);
          for (int h = 0; h < 2; ++h) {
            // the 128-row weight block of each half of the tile's 256 B rows
            const int w_block = kSwiglu ? (h == 0 ? n_tile : p.F / BN_HALF + n_tile) : 2 * n_tile + h;
            tma_load_2d_pair_hint(st + A_STAGE + B_STAGE + SFA_STAGE + h * (KB_PER_STAGE * 512), &tmSFB,
                                  full_leader, 0, (w_block * p.ktiles + kt0) * 2, keep);
          }
          issued[s] = true;
          issued_phase[s] = ph;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (rank == 0)
        for (int i = 0; i < STAGES; ++i)
          if (issued[i]) mbar_wait(&full_bar[i], issued_phase[i], abort_flag, p.status);
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // ---------------- MMA issuer (leader CTA only): whole warp, one elected lane ----------------
      constexpr uint32_t idesc = idesc_nvf4_f32(2 * BM, BN);
      const bool leader = elect_one();  // the same lane issues and commits every tcgen05 op
      int s = 0;
      uint32_t ph = 0;
      int t = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs, ++t) {
        if (t > 0 && !warp_wait(tfree_bar, (t - 1) & 1, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ((t & 1) ? ACC1_COL : 0u);
        for (int ks = 0; ks < kstages; ++ks) {
          if (!warp_wait(&full_bar[s], ph, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int kb_here = min(KB_PER_STAGE, p.ktiles - ks * KB_PER_STAGE);
          uint8_t *st = smem + s * STAGE_BYTES;
          const uint32_t sfa_smem = smem_u32(st + A_STAGE + B_STAGE);
          const uint32_t sfb_smem = sfa_smem + SFA_STAGE;
          const uint64_t a_desc = sw128_kmajor_desc(smem_u32(st));
          const uint64_t b_desc = sw128_kmajor_desc(smem_u32(st + A_STAGE));
          const uint64_t sfa_d = sf_block_desc(sfa_smem);
          const uint64_t sfb_d = sf_block_desc(sfb_smem);
          if (leader) {
            if (kb_here == KB_PER_STAGE) {
#pragma unroll
              for (int kb = 0; kb < KB_PER_STAGE; ++kb) {
                tmem_cp_32x128b_warpx4_pair(tmem_base + SFA_COL + 4 * kb, sfa_d + (kb * 512 >> 4));
                tmem_cp_32x128b_warpx4_pair(tmem_base + SFB_COL + 8 * kb, sfb_d + (kb * 512 >> 4));
                tmem_cp_32x128b_warpx4_pair(tmem_base + SFB_COL + 8 * kb + 4, sfb_d + ((KB_PER_STAGE * 512 + kb * 512) >> 4));
              }
#pragma unroll
              for (int kb = 0; kb < KB_PER_STAGE; ++kb)
                mma_mxf4nvf4_pair(d_tmem, a_desc + 2 * kb, b_desc + 2 * kb, idesc,
                                  tmem_base + SFA_COL + 4 * kb, tmem_base + SFB_COL + 8 * kb, (ks | kb) != 0);
            } else {
              for (int kb = 0; kb < kb_here; ++kb) {
                tmem_cp_32x128b_warpx4_pair(tmem_base + SFA_COL + 4 * kb, sfa_d + (kb * 512 >> 4));
                tmem_cp_32x128b_warpx4_pair(tmem_base + SFB_COL + 8 * kb, sfb_d + (kb * 512 >> 4));
                tmem_cp_32x128b_warpx4_pair(tmem_base + SFB_COL + 8 * kb + 4, sfb_d + ((KB_PER_STAGE * 512 + kb * 512) >> 4));
              }
              for (int kb = 0; kb < kb_here; ++kb)
                mma_mxf4nvf4_pair(d_tmem, a_desc + 2 * kb, b_desc + 2 * kb, idesc,
                                  tmem_base + SFA_COL + 4 * kb, tmem_base + SFB_COL + 8 * kb, (ks | kb) != 0);
            }
            tc_commit_pair(smem_u32(&empty_bar[s]));
            tc_commit_pair(map_to_rank(smem_u32(&empty_bar[s]), 1));
          }
          __syncwarp();
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        if (leader) {
          tc_commit_pair(smem_u32(tfull_bar));
          tc_commit_pair(map_to_rank(smem_u32(tfull_bar), 1));
        }
        __syncwarp();
      }
      if (leader) {
        tc_commit_pair(smem_u32(drain_bar));
        mbar_wait(drain_bar, 0, abort_flag, p.status);
      }
      __syncwarp();
    }
  } else {
    // ---------------- epilogue (warps 2.. of both CTAs) ----------------
    const int q = warp & 3;              // TMEM lane quarter: this warp's 32 rows
    const int group = (warp - 2) >> 2;   // which share of the tile's chunks
    uint8_t *warp_smem = sEpi + (warp - 2) * EPI_BOXES * EPI_BOX_BYTES;
    int box = 0;
    float alpha = __ldg(p.alpha);
    if (p.alpha_div != nullptr) alpha = __fdiv_rn(alpha, __ldg(p.alpha_div));
    const Nvfp4Consts qc = nvfp4_consts(QUANT ? __ldg(p.q_gsf) : 1.0f);
    const uint32_t tfree_leader = map_to_rank(smem_u32(tfree_bar), 0);
    // chunks of 32 columns per tile; SWIGLU pairs value chunk c with gate chunk c + 4
    constexpr int kChunks = kSwiglu ? BN_HALF / 32 : BN / 32;
    constexpr int kGroupChunks = kChunks / EPI_GROUPS;
    static_assert(kGroupChunks >= 2, "the group holding the shared columns reads two chunks first");
    int t = 0;
    for (int tile = pair; tile < num_tiles; tile += num_pairs, ++t) {
      if (!mbar_wait(tfull_bar, t & 1, abort_flag, p.status)) break;
      tc_fence_after();
      int m_tile, n_tile;
      band_coords(tile, p.num_m_tiles, p.num_n_tiles, p.band_n, m_tile, n_tile);
      const int64_t row0 = static_cast<int64_t>(m_tile) * (2 * BM) + rank * BM + q * 32;
      const int64_t m = row0 + lane;
      const bool live = m < p.M;
      const bool any_row = row0 < p.M;
      const bool odd = t & 1;
      const uint32_t t_row = tmem_base + (odd ? ACC1_COL : 0u) + (static_cast<uint32_t>(q * 32) << 16);
      // The 64 columns the two accumulators share are the last of an even
      // tile and the first of an odd one (for SWIGLU: gate chunks 2-3 or
      // value chunks 0-1), in the last group's share or the first's.  That
      // group reads both shared chunks first, with one wait (even tiles go in
      // reverse chunk order), and then releases them to the next tile's MMAs;
      // the other groups release at the tile's start.
      const bool holder = group == (odd ? 0 : EPI_GROUPS - 1);
      if (!holder) {
        tc_fence_before();
        mbar_arrive_cluster(tfree_leader);
      }
      uint32_t held[32];  // the second shared chunk, loaded together with the first
#pragma unroll 1
      for (int i = 0; i < kGroupChunks; ++i) {
        const int c = group * kGroupChunks + (odd ? i : (kGroupChunks - 1 - i));
        const bool first_shared = holder && i == 0, second_shared = holder && i == 1;
        float v[32];
        if constexpr (kSwiglu) {
          float g[32];
          uint32_t rv[32], rg[32];
          if (first_shared) {
            // this chunk's value and gate columns and the second shared chunk
            // (gate c - 1 of an even tile, value 1 of an odd one), one wait
            tmem_ld_32x32b_x32_issue(t_row + c * 32, rv);
            tmem_ld_32x32b_x32_issue(t_row + BN_HALF + c * 32, rg);
            tmem_ld_32x32b_x32_issue(odd ? t_row + 32 : t_row + BN_HALF + (c - 1) * 32, held);
            tmem_ld_wait();
            tmem_ld_fence(rv);
            tmem_ld_fence(rg);
            tmem_ld_fence(held);
            tc_fence_before();
            mbar_arrive_cluster(tfree_leader);
          } else if (second_shared) {
            // the shared half was loaded with chunk 0; load the other one
            if (odd) {
              tmem_ld_32x32b_x32_issue(t_row + BN_HALF + c * 32, rg);
              tmem_ld_wait();
              tmem_ld_fence(rg);
#pragma unroll
              for (int j = 0; j < 32; ++j) rv[j] = held[j];
            } else {
              tmem_ld_32x32b_x32_issue(t_row + c * 32, rv);
              tmem_ld_wait();
              tmem_ld_fence(rv);
#pragma unroll
              for (int j = 0; j < 32; ++j) rg[j] = held[j];
            }
          } else {
            tmem_ld_32x32b_x32_issue(t_row + c * 32, rv);
            tmem_ld_32x32b_x32_issue(t_row + BN_HALF + c * 32, rg);
            tmem_ld_wait();
            tmem_ld_fence(rv);
            tmem_ld_fence(rg);
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            v[j] = __uint_as_float(rv[j]);
            g[j] = __uint_as_float(rg[j]);
          }
          const int32_t f = n_tile * BN_HALF + c * 32;
          if (f >= p.F) continue;  // warp-uniform
          if (live) {
            alpha_bias(v, alpha, p.bias ? p.bias + f : nullptr);
            alpha_bias(g, alpha, p.bias ? p.bias + p.F + f : nullptr);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = v[j] * bf16r(silu(g[j]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.0f;
          }
          if constexpr (QUANT)
            store_nvfp4(p, v, m, live, f, qc);
          else
            store_box<EPI_BOXES>(warp_smem, box, &tmOut, v, lane, f, static_cast<int32_t>(row0), 0, any_row);
        } else {
          uint32_t r[32];
          if (first_shared) {
            // both shared chunks with one wait, then release them
            tmem_ld_32x32b_x32_issue(t_row + c * 32, r);
            tmem_ld_32x32b_x32_issue(t_row + (odd ? 1 : kChunks - 2) * 32, held);
            tmem_ld_wait();
            tmem_ld_fence(r);
            tmem_ld_fence(held);
            tc_fence_before();
            mbar_arrive_cluster(tfree_leader);
          } else if (second_shared) {
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = held[j];
          } else {
            tmem_ld_32x32b_x32_issue(t_row + c * 32, r);
            tmem_ld_wait();
            tmem_ld_fence(r);
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          const int32_t n = n_tile * BN + c * 32;
          if (n >= p.N) continue;  // warp-uniform
          const int32_t plane = n / p.plane_width;
          const int32_t col = n - plane * p.plane_width;
          if (live) {
            alpha_bias(v, alpha, p.bias ? p.bias + n : nullptr);
            if constexpr (EPI == VFB_EPI_STORE) {
              // triton_strict_bf16_qkv_direct_merge (h3_fused_ops.py:901-949)
              const __nv_bfloat16 *ad = plane < 3 ? p.adapter[plane] : nullptr;
              if (ad != nullptr) {
                float av[32];
                load_bf16x32(ad + m * p.adapter_ld + col, av);
                const float sc = p.scaling[plane];
#pragma unroll
                for (int j = 0; j < 32; ++j) av[j] = av[j] * sc;
                bf16r_x32(av);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = v[j] + av[j];
                bf16r_x32(v);  // the merge's own rounding (the store packs exact bf16 values)
              }
            } else if constexpr (EPI == VFB_EPI_GELU_TANH) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
            } else if constexpr (EPI == VFB_EPI_RESIDUAL) {
              // triton_strict_bf16_gate_residual (h3_fused_ops.py:125-170)
              if (p.gate != nullptr) {
                const __nv_bfloat16 *gp = p.gate + (m % p.tokens) * p.gate_ts + n * p.gate_hs;
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __bfloat162float(gp[j * p.gate_hs]) * v[j];
                bf16r_x32(v);
              }
              float r[32];
              load_bf16x32(p.residual + m * p.ldr + n, r);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = r[j] + v[j];
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.0f;
          }
          // STORE values are bf16 already (alpha_bias / the merge rounded them)
          if constexpr (QUANT)
            store_nvfp4(p, v, m, live, col, qc);
          else
            store_box<EPI_BOXES, false, EPI == VFB_EPI_STORE>(warp_smem, box, &tmOut, v, lane, col,
                                                              static_cast<int32_t>(row0), plane, any_row);
        }
      }
    }
    if (lane == 0) bulk_wait_group_all();
  }

  __syncthreads();
  __syncwarp();
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

int map_u8(CUtensorMap *map, const void *base, int64_t rows, int64_t row_bytes, int box_x, int box_rows,
           CUtensorMapSwizzle swizzle) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return set_error(VFB_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_x), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides,
                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(VFB_ECUDA, "cuTensorMapEncodeTiled (nvfp4) failed (%d)", (int)r);
  return VFB_OK;
}

bool a16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

template <int EPI, bool QUANT = false>
int launch(const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &tb2, const CUtensorMap &tsa,
           const CUtensorMap &tsb, const CUtensorMap &to, const Params &p, int sms, cudaStream_t stream) {
  auto kernel = nvfp4_gemm_kernel<EPI, QUANT>;
  // the shared-memory opt-in is a function attribute of the device's context: set it once per context
  static std::atomic<uint64_t> smem_set[kMaxAttrDevices];
  int rc = ensure_smem_optin(reinterpret_cast<const void *>(kernel), static_cast<int>(SMEM_BYTES), smem_set);
  if (rc != VFB_OK) return rc;
  const int tiles = p.num_m_tiles * p.num_n_tiles;
  const int max_pairs = sms / 2;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // scheduled while the previous kernel (the quantiser) finishes; waits in the kernel for its results
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, ta, tb, tb2, tsa, tsb, to, p);
  if (err != cudaSuccess) return set_error(VFB_ECUDA, "vfb_nvfp4_gemm launch: %s", cudaGetErrorString(err));
  return VFB_OK;
}

// quant: the result goes out as NVFP4 codes and scales (q_gsf its global
// scale) instead of bf16 (ep->out, ldo and planes are not used).
int nvfp4_impl(const char *fn, const void *A, const void *sfa, const void *W, const void *sfw, const float *alpha,
               const float *alpha_div, int64_t M, int64_t N, int64_t K, const vfb_epilogue *ep, void *stream,
               bool quant = false, const float *q_gsf = nullptr, void *q_codes = nullptr, void *q_sf = nullptr) {
  if (ep == nullptr) return set_error(VFB_EINVAL, "%s: epilogue is NULL", fn);
  const int kind = ep->kind;
  if (kind != VFB_EPI_STORE && kind != VFB_EPI_GELU_TANH && kind != VFB_EPI_SWIGLU && kind != VFB_EPI_RESIDUAL)
    return set_error(VFB_EINVAL, "%s: epilogue kind %d is not STORE, GELU_TANH, SWIGLU or RESIDUAL", fn, kind);
  if (ep->wire_chunks != 0) return set_error(VFB_EINVAL, "%s: no wire layout for NVFP4 outputs", fn);
  if (M < 0 || N <= 0 || K <= 0 || K % 64 || N % 128 || K > (int64_t)1 << 20 || N > (int64_t)1 << 24)
    return set_error(VFB_EINVAL, "%s: need K %% 64 == 0 and N %% 128 == 0 (M=%lld N=%lld K=%lld)", fn,
                     (long long)M, (long long)N, (long long)K);
  if (kind == VFB_EPI_SWIGLU && ((N / 2) % 128 || (!quant && ep->ldo < N / 2)))
    return set_error(VFB_EINVAL, "%s: SWIGLU needs the packed N = 2F with F %% 128 == 0 and ldo >= F", fn);
  if (quant) {
    const int64_t width = kind == VFB_EPI_SWIGLU ? N / 2 : N;
    if (kind == VFB_EPI_RESIDUAL || width % 64 || (kind != VFB_EPI_SWIGLU && ep->plane_width != 0 &&
                                                   ep->plane_width != N))
      return set_error(VFB_EINVAL, "%s: the NVFP4 output needs a STORE, GELU_TANH or SWIGLU epilogue with one "
                                   "plane whose width is a multiple of 64", fn);
    for (int i = 0; i < 3; ++i)
      if (ep->adapter[i] != nullptr) return set_error(VFB_EINVAL, "%s: no adapter merge for the NVFP4 output", fn);
  }
  if (M == 0) return VFB_OK;
  if (!A || !sfa || !W || !sfw || !alpha || (!quant && !ep->out))
    return set_error(VFB_EINVAL, "%s: NULL operand", fn);
  if (quant && (q_gsf == nullptr || q_codes == nullptr || q_sf == nullptr || !a16(q_codes) || !a16(q_sf)))
    return set_error(VFB_EINVAL, "%s: the NVFP4 output needs its global scale and 16-byte aligned codes and "
                                 "scales", fn);
  if (!a16(A) || !a16(W) || !a16(sfa) || !a16(sfw) || (!quant && !a16(ep->out)) || (ep->bias && !a16(ep->bias)) ||
      (!quant && ep->ldo % 8))
    return set_error(VFB_EINVAL, "%s: operands must be 16-byte aligned, ldo %% 8 == 0", fn);
  int sms = 0;
  int rc = check_device(&sms);
  if (rc != VFB_OK) return rc;
  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.alpha = alpha;
  p.alpha_div = alpha_div;
  p.bias = static_cast<const __nv_bfloat16 *>(ep->bias);
  p.num_m_tiles = static_cast<int>((M + 2 * BM - 1) / (2 * BM));
  p.ktiles = static_cast<int>(K / 64);
  p.status = device_status_ptr();
  const int64_t a_blocks = (M + 127) / 128;  // 128-row scale blocks of the activation
  const int64_t w_blocks = N / 128;
  CUtensorMap ta, tb, tb2, tsa, tsb, to{};  // `to` stays unused for the NVFP4 output
  if ((rc = map_u8(&ta, A, M, K / 2, BK_BYTES, BM, CU_TENSOR_MAP_SWIZZLE_128B)) != VFB_OK) return rc;
  if (kind == VFB_EPI_SWIGLU) {
    const int64_t F = N / 2;
    p.F = static_cast<int32_t>(F);
    p.plane_width = static_cast<int32_t>(F);
    p.num_n_tiles = static_cast<int>(F / BN_HALF);
    if ((rc = map_u8(&tb, W, F, K / 2, BK_BYTES, BN_HALF, CU_TENSOR_MAP_SWIZZLE_128B)) != VFB_OK) return rc;
    if ((rc = map_u8(&tb2, static_cast<const uint8_t *>(W) + F * (K / 2), F, K / 2, BK_BYTES, BN_HALF,
                     CU_TENSOR_MAP_SWIZZLE_128B)) != VFB_OK)
      return rc;
    if (!quant && (rc = make_map_out(&to, ep->out, F, M, 1, ep->ldo, M * ep->ldo)) != VFB_OK) return rc;
  } else if (quant) {
    p.plane_width = static_cast<int32_t>(N);
    p.num_n_tiles = static_cast<int>((N + BN - 1) / BN);
    if ((rc = map_u8(&tb, W, N, K / 2, BK_BYTES, BN_HALF, CU_TENSOR_MAP_SWIZZLE_128B)) != VFB_OK) return rc;
    tb2 = tb;
  } else {
    if (ep->plane_width < 0 || (ep->plane_width > 0 && (ep->plane_width % 32 || N % ep->plane_width)))
      return set_error(VFB_EINVAL, "%s: plane_width must be 0 or a multiple of 32 dividing N", fn);
    const int64_t width = ep->plane_width > 0 ? ep->plane_width : N;
    const int64_t planes = N / width;
    if (ep->ldo < width) return set_error(VFB_EINVAL, "%s: ldo smaller than the plane width", fn);
    const int64_t plane_stride = planes > 1 ? ep->plane_stride : M * ep->ldo;
    if (plane_stride % 8 || (planes > 1 && plane_stride < M * ep->ldo))
      return set_error(VFB_EINVAL, "%s: plane_stride must be a multiple of 8 and >= M*ldo", fn);
    p.plane_width = static_cast<int32_t>(width);
    p.num_n_tiles = static_cast<int>((N + BN - 1) / BN);
    if ((rc = map_u8(&tb, W, N, K / 2, BK_BYTES, BN_HALF, CU_TENSOR_MAP_SWIZZLE_128B)) != VFB_OK) return rc;
    tb2 = tb;
    if ((rc = make_map_out(&to, ep->out, width, M, planes, ep->ldo, plane_stride)) != VFB_OK) return rc;
    if (kind == VFB_EPI_STORE) {
      for (int i = 0; i < 3; ++i) {
        p.adapter[i] = static_cast<const __nv_bfloat16 *>(ep->adapter[i]);
        p.scaling[i] = ep->scaling[i];
        if (p.adapter[i] != nullptr &&
            (i >= planes || !a16(p.adapter[i]) || ep->adapter_ld % 8 || ep->adapter_ld < width))
          return set_error(VFB_EINVAL, "%s: adapter %d misaligned or beyond the planes", fn, i);
      }
      p.adapter_ld = ep->adapter_ld;
    }
    if (kind == VFB_EPI_RESIDUAL) {
      if (ep->residual == nullptr || !a16(ep->residual) || ep->ldr % 8 || ep->ldr < N || planes != 1)
        return set_error(VFB_EINVAL, "%s: RESIDUAL needs a 16-byte aligned [M,N] residual and one plane", fn);
      p.residual = static_cast<const __nv_bfloat16 *>(ep->residual);
      p.ldr = ep->ldr;
      p.gate = static_cast<const __nv_bfloat16 *>(ep->gate);
      if (p.gate != nullptr) {
        if (ep->tokens <= 0) return set_error(VFB_EINVAL, "%s: gate needs tokens > 0", fn);
        p.gate_ts = ep->gate_token_stride;
        p.gate_hs = ep->gate_hidden_stride;
        p.tokens = ep->tokens;
      }
    }
  }
  p.band_n = band_width(p.num_n_tiles, K / 2);
  // scale buffers viewed as rows of 256 bytes (two rows per 512-byte block)
  if ((rc = map_u8(&tsa, sfa, a_blocks * p.ktiles * 2, 256, 256, 2 * KB_PER_STAGE,
                   CU_TENSOR_MAP_SWIZZLE_NONE)) != VFB_OK)
    return rc;
  if ((rc = map_u8(&tsb, sfw, w_blocks * p.ktiles * 2, 256, 256, 2 * KB_PER_STAGE,
                   CU_TENSOR_MAP_SWIZZLE_NONE)) != VFB_OK)
    return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (quant) {
    const int64_t width = kind == VFB_EPI_SWIGLU ? N / 2 : N;
    p.q_codes = static_cast<uint8_t *>(q_codes);
    p.q_sf = static_cast<uint8_t *>(q_sf);
    p.q_gsf = q_gsf;
    p.q_ld = width / 2;
    p.q_rows_pad = (M + 127) / 128 * 128;
    p.q_ktiles = width / 64;
    switch (kind) {
      case VFB_EPI_GELU_TANH:
        return launch<VFB_EPI_GELU_TANH, true>(ta, tb, tb2, tsa, tsb, to, p, sms, s);
      case VFB_EPI_SWIGLU:
        return launch<VFB_EPI_SWIGLU, true>(ta, tb, tb2, tsa, tsb, to, p, sms, s);
      default:
        return launch<VFB_EPI_STORE, true>(ta, tb, tb2, tsa, tsb, to, p, sms, s);
    }
  }
  switch (kind) {
    case VFB_EPI_GELU_TANH:
      return launch<VFB_EPI_GELU_TANH>(ta, tb, tb2, tsa, tsb, to, p, sms, s);
    case VFB_EPI_SWIGLU:
      return launch<VFB_EPI_SWIGLU>(ta, tb, tb2, tsa, tsb, to, p, sms, s);
    case VFB_EPI_RESIDUAL:
      return launch<VFB_EPI_RESIDUAL>(ta, tb, tb2, tsa, tsb, to, p, sms, s);
    default:
      return launch<VFB_EPI_STORE>(ta, tb, tb2, tsa, tsb, to, p, sms, s);
  }
}

}  // namespace
}  // namespace vfb

extern "C" int vfb_nvfp4_gemm(const void *A, const void *sfa, const void *W, const void *sfw,
                              const float *alpha, int64_t M, int64_t N, int64_t K, const void *bias,
                              void *out, int64_t planes, void *stream) {
  using namespace vfb;
  if (planes < 1 || planes > 3 || N <= 0 || N % planes || (N / planes) % 32)
    return set_error(VFB_EINVAL, "vfb_nvfp4_gemm: need K %% 64 == 0, N %% 128 == 0, 1..3 planes of width %% 32");
  vfb_epilogue ep{};
  ep.kind = VFB_EPI_STORE;
  ep.out = out;
  ep.ldo = N / planes;
  ep.plane_width = planes > 1 ? N / planes : 0;
  ep.plane_stride = M * (N / planes);
  ep.bias = bias;
  return nvfp4_impl("vfb_nvfp4_gemm", A, sfa, W, sfw, alpha, nullptr, M, N, K, &ep, stream);
}

extern "C" int vfb_nvfp4_gemm_ex(const void *A, const void *sfa, const void *W, const void *sfw,
                                 const float *alpha, const float *alpha_div, int64_t M, int64_t N, int64_t K,
                                 const vfb_epilogue *ep, void *stream) {
  return vfb::nvfp4_impl("vfb_nvfp4_gemm_ex", A, sfa, W, sfw, alpha, alpha_div, M, N, K, ep, stream);
}

extern "C" int vfb_nvfp4_gemm_quant(const void *A, const void *sfa, const void *W, const void *sfw,
                                    const float *alpha, const float *alpha_div, int64_t M, int64_t N, int64_t K,
                                    const vfb_epilogue *ep, const float *out_global_scale, void *out_codes,
                                    void *out_sf, void *stream) {
  return vfb::nvfp4_impl("vfb_nvfp4_gemm_quant", A, sfa, W, sfw, alpha, alpha_div, M, N, K, ep, stream, true,
                         out_global_scale, out_codes, out_sf);
}
