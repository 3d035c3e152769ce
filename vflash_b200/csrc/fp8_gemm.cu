// Row-scaled FP8 (e4m3 x e4m3 -> fp32) GEMM for sm_100a with fused epilogues.
//
// Replaces torch._scaled_mm(codes, weight.t(), scale_a, scale_b.t(), bf16)
// and the bias add that follows it (src/vflash/native/h3_fp8_linear.py:109-121),
// plus the strict-BF16 elementwise launch that the H3 block runs next
// (src/vflash/native/h3_fused_ops.py: silu_mul 185-224, gate_residual
// 125-170, qkv_direct_merge 901-949).  Every BF16 rounding boundary of those
// eager/Triton sequences is kept: the GEMM result is rounded to BF16 first,
// then each elementwise step rounds where the reference rounds.
//
// Structure: persistent CTA pairs (2-CTA clusters, one CTA per SM), one
// 256 x 256 output tile per pair at a time, K staged 128 bytes per stage.
//   warp 0      TMA producer in both CTAs: its own 128 A rows and 128 of the
//               tile's 256 weight rows per stage (128-byte swizzle, weights with
//               an evict_last L2 policy) into a 5-deep shared-memory ring; the
//               bytes of both CTAs complete on the leader's full barrier.
//   warp 1      allocates 512 TMEM columns per CTA (two 256-column fp32
//               accumulators); in the leader CTA the whole warp runs the issue
//               loop and one elected lane issues tcgen05.mma.cta_group::2
//               kind::f8f6f4 (M=256, N=256, K=32; four per stage), committing
//               each stage to both CTAs' empty barriers and each finished tile to
//               both CTAs' epilogues.
//   warps 2-5   epilogue (2-9 for QKV_NORM_ROPE, one group of four per head, and
//               for SWIGLU, one group per half of the tile; 2-17 for bf16
//               operands, one group per quarter):
//               tcgen05.ld 32 columns at a time (warp w reads TMEM lanes
//               32*(w%4)..+31 = tile rows), scales / bias / activation /
//               residual / QK-norm + rotary in registers, 32 x 32 bf16 boxes
//               staged in 64-byte-swizzled shared memory and written by TMA
//               stores (evict_first).  The second accumulator lets the epilogue
//               of tile i overlap the main loop of tile i+1.
// Tiles are visited in bands of band_n weight tiles (the weight slab of a band,
// band_n x 256 rows x K bytes, is sized on the host to stay in L2), M-block by
// M-block inside a band with the N index fastest: the pairs running at the
// same time share one A row-block, and each band's weights are fetched from
// DRAM once instead of once per row-block.
// No TMA multicast is used: every CTA loads its own operands.
// Launched with programmatic stream serialisation: setup (barriers, TMEM,
// descriptor prefetch) may overlap the previous kernel (the quantiser), and
// every thread waits in grid_dependency_wait() before touching global memory.
#include <cudaTypedefs.h>

#include <atomic>

#include <mutex>

#include "common.cuh"
#include "epilogue.cuh"

namespace vfb {
namespace {

constexpr int BM = 128;       // A rows per CTA (a CTA pair covers 256 rows)
constexpr int BN = 256;       // output columns per pair tile
constexpr int BN_HALF = BN / 2;  // weight rows each CTA of the pair loads
constexpr int BK = 128;       // bytes per stage: 128 e4m3 or 64 bf16 elements of K
constexpr int UMMA_K = 32;    // bytes of K per MMA: 32 e4m3 (kind::f8f6f4) or 16 bf16 (kind::f16)
// operand types of the kernel: row-scaled e4m3 (the FP8 linear) or plain bf16
// (the low-rank adapter products, F.linear in bf16)
constexpr int OPS_E4M3 = 0;
constexpr int OPS_BF16 = 1;
constexpr int STAGES = 5;
constexpr int A_STAGE_BYTES = BM * BK;       // 16 KB
constexpr int B_STAGE_BYTES = BN_HALF * BK;  // 16 KB
// Warps 0 (TMA) and 1 (MMA) plus the epilogue warps: four (one per TMEM lane
// quarter) for the light epilogues, eight for QK-norm + rotary, where each
// 256-column tile is two 128-column heads and each head gets its own four
// warps, sixteen for bf16 operands, whose products are mostly output writes
// (each group of four stores one 64-column quarter of the tile, so four warps
// per lane quarter hide each other's TMEM-load and store latency; eight gave
// 0.292 ms and sixteen 0.261 ms -- 0.222 ms with one proxy fence per two boxes -- for three rank-32 up products at config 1's
// shape), and eight for
// SwiGLU, whose precise silu (expf and an IEEE divide per element) made the
// four-warp epilogue the longer side of each tile (measured at the packed
// FFN shape: 3.78 -> 3.28-3.33 ms for the up projection).
template <int EPI, int OPS = OPS_E4M3>
__host__ __device__ constexpr int epi_warps() {
  return OPS == OPS_BF16 ? 16 : EPI == VFB_EPI_QKV_NORM_ROPE || EPI == VFB_EPI_SWIGLU ? 8 : 4;
}
template <int EPI, int OPS = OPS_E4M3>
__host__ __device__ constexpr int num_threads() { return 64 + 32 * epi_warps<EPI, OPS>(); }
constexpr int TMEM_COLS = 512;
// Epilogue staging: per epilogue warp a ring of EPI_BOXES 32 x 32 bf16 boxes
// (2 KB each), so TMA stores drain while the warp fills the next boxes.
constexpr int EPI_BOXES = 4;  // with four epilogue warps; two with eight or sixteen
template <int EPI, int OPS = OPS_E4M3>
__host__ __device__ constexpr int epi_boxes() { return epi_warps<EPI, OPS>() > 8 ? 2 : 16 / epi_warps<EPI, OPS>(); }
template <int EPI, int OPS = OPS_E4M3>
__host__ __device__ constexpr int epi_smem_bytes() { return epi_warps<EPI, OPS>() * epi_boxes<EPI, OPS>() * EPI_BOX_BYTES; }
template <int EPI, int OPS = OPS_E4M3>
__host__ __device__ constexpr size_t smem_bytes() {
  return 1024 + STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + epi_smem_bytes<EPI, OPS>() + 256;
}
static_assert(smem_bytes<VFB_EPI_STORE, OPS_BF16>() <= 227 * 1024, "the widest epilogue staging must fit");

struct EpiParams {
  int32_t plane_width;  // columns per output plane (N when there is one plane)
  int32_t wire_chunks;  // > 0: planes stored in the (chunk, destination, qkv) slabs of pack_qkv
  int32_t wire_width;   // columns per slab (plane_width / (2 * wire_chunks))
  const __nv_bfloat16 *bias;
  const __nv_bfloat16 *adapter[3];
  int64_t adapter_ld;
  float scaling[3];
  const __nv_bfloat16 *residual;
  int64_t ldr;
  const __nv_bfloat16 *gate;
  int64_t gate_ts;
  int64_t gate_hs;
  int64_t tokens;
  // QKV_NORM_ROPE
  const __nv_bfloat16 *q_norm;
  const __nv_bfloat16 *k_norm;
  const __nv_bfloat16 *rope_cos;
  const __nv_bfloat16 *rope_sin;
  int64_t rope_ts;
  float qk_eps;
};

struct GemmParams {
  int64_t M;
  int64_t N;  // output columns of the GEMM (packed 2F for SWIGLU)
  int64_t K;
  const float *sa;
  const float *sw;
  int num_m_tiles;
  int num_n_tiles;
  int band_n;  // weight tiles per band of the tile order
  int num_kb;
  int *status;
  EpiParams ep;
};

// Output coordinate (column, plane index of the tensor map) of a 32-column
// box that starts at column col of plane `plane`.  Without the wire layout the
// planes are the tensor map's planes.  With it, plane p's columns are split
// into 2 * wire_chunks groups of wire_width (group g = destination *
// wire_chunks + chunk, i.e. heads in destination-major, chunk-minor order)
// and group g goes to slab (chunk * 2 + destination) * 3 + p: the
// (chunk, destination, qkv, rows, heads, dim) layout of pack_qkv
// (src/vflash/native/h3_parallel_relayout.py:214-256).  A box never
// straddles two groups (wire_width % 32 == 0).
__device__ __forceinline__ void out_coord(const EpiParams &ep, int32_t plane, int32_t col, int32_t &ocol,
                                          int32_t &oplane) {
  if (ep.wire_chunks == 0) {
    ocol = col;
    oplane = plane;
    return;
  }
  const int32_t g = col / ep.wire_width;
  const int32_t chunk = g % ep.wire_chunks;
  const int32_t dest = g / ep.wire_chunks;
  ocol = col - g * ep.wire_width;
  oplane = (chunk * 2 + dest) * 3 + plane;
}

// STORE value of 32 columns: scale_bias, then the plane's LoRA branch if any.
template <bool SCALED = true>
__device__ __forceinline__ void store_value(float (&v)[32], float sa, const float *sw, const EpiParams &ep,
                                            int32_t n, int32_t plane, int32_t col, int64_t m) {
  scale_bias<SCALED>(v, sa, SCALED ? sw + n : nullptr, ep.bias ? ep.bias + n : nullptr);
  const __nv_bfloat16 *ad = plane < 3 ? ep.adapter[plane] : nullptr;
  if (ad != nullptr) {
    float a[32];
    load_bf16x32(ad + m * ep.adapter_ld + col, a);
    const float sc = ep.scaling[plane];
#pragma unroll
    for (int j = 0; j < 32; ++j) a[j] = a[j] * sc;
    bf16r_x32(a);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = v[j] + a[j];
    bf16r_x32(v);  // the merge's own rounding (the store then packs exact bf16 values)
  }
}


__device__ __forceinline__ uint4 ld8(const __nv_bfloat16 *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }

__device__ __forceinline__ __nv_bfloat162 as_bf162(uint32_t u) { return *reinterpret_cast<__nv_bfloat162 *>(&u); }


// QK-norm + rotary output of one 32-column chunk of a head (k in 0..3) from
// the head's 128 bf16 values packed in hp[64] (hp[i] = columns 2i, 2i+1):
//   n = bf16((x * rstd) * w)                      fp32 products, one rounding
//   out[d] = bf16(bf16(n[d] * cos[d]) + bf16(partner[d] * sin[d]))
//   partner[d] = -n[d + 64] for d < 64, n[d - 64] otherwise.
// The rotary products are bf16 x bf16, exact in fp32, so rounding the fp32
// product equals one mul.rn.bf16x2 of the packed operands; the sum stays fp32
// and is rounded at the store, as in the reference.
__device__ __forceinline__ void qk_norm_rope_chunk(const uint32_t (&hp)[64], float rstd, int k,
                                                   const __nv_bfloat16 *w, const __nv_bfloat16 *cs,
                                                   const __nv_bfloat16 *sn, float (&out)[32]) {
  const uint4 one = make_uint4(0x3f803f80u, 0x3f803f80u, 0x3f803f80u, 0x3f803f80u);
  const int kp = k ^ 2;  // the partner chunk (64 columns away)
  const bool first = k < 2;
  // eight columns per step: 16-byte loads of the norm weights and of this
  // row's cos / sin (each lane reads its own token's row)
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int d = 32 * k + 8 * g;   // this chunk's columns d .. d+7
    const int dp = 32 * kp + 8 * g;  // partner columns
    const uint4 wv = w ? ld8(w + d) : one, wp = w ? ld8(w + dp) : one;
    const uint4 cv = ld8(cs + d), sv = ld8(sn + d);
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w}, wpw[4] = {wp.x, wp.y, wp.z, wp.w};
    const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w}, sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 x = __bfloat1622float2(as_bf162(hp[16 * k + 4 * g + h]));
      const float2 xp = __bfloat1622float2(as_bf162(hp[16 * kp + 4 * g + h]));
      const float2 fw = __bfloat1622float2(as_bf162(ww[h]));
      const float2 fwp = __bfloat1622float2(as_bf162(wpw[h]));
      const __nv_bfloat162 n = __floats2bfloat162_rn((x.x * rstd) * fw.x, (x.y * rstd) * fw.y);
      __nv_bfloat162 np = __floats2bfloat162_rn((xp.x * rstd) * fwp.x, (xp.y * rstd) * fwp.y);
      if (first) np = __hneg2(np);
      const float2 c = __bfloat1622float2(__hmul2(n, as_bf162(cw[h])));
      const float2 sp = __bfloat1622float2(__hmul2(np, as_bf162(sw[h])));
      out[8 * g + 2 * h] = c.x + sp.x;
      out[8 * g + 2 * h + 1] = c.y + sp.y;
    }
  }
}

template <int EPI, int OPS>
__global__ void __launch_bounds__(num_threads<EPI, OPS>(), 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ CUtensorMap tmOut,
                    const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  uint8_t *sA = smem;
  uint8_t *sB = smem + STAGES * A_STAGE_BYTES;
  uint8_t *sEpi = sB + STAGES * B_STAGE_BYTES;
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(sEpi + epi_smem_bytes<EPI, OPS>());
  uint64_t *empty_bar = full_bar + STAGES;
  uint64_t *tfull_bar = empty_bar + STAGES;
  uint64_t *tempty_bar = tfull_bar + 2;
  uint64_t *drain_bar = tempty_bar + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain_bar + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();  // 0 = leader of the CTA pair
  const int pair = blockIdx.x / 2;
  const int num_pairs = gridDim.x / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);   // leader: one expect_tx arrival + both CTAs' bytes
      mbar_init(&empty_bar[s], 1);  // one commit from the leader's MMA thread
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * 32 * epi_warps<EPI, OPS>());  // leader: every epilogue thread of both CTAs
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (EPI == VFB_EPI_SWIGLU) tma_prefetch_desc(&tmB2);
  }
  if (warp == 2 && lane == 0) tma_prefetch_desc(&tmOut);
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dependency_wait();  // the previous kernel's outputs (A, its scales) are complete

  const int num_tiles = p.num_m_tiles * p.num_n_tiles;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_phase[STAGES];
      bool issued[STAGES];
      for (int i = 0; i < STAGES; ++i) issued[i] = false;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
        int m_tile, n_tile;
        band_coords(tile, p.num_m_tiles, p.num_n_tiles, p.band_n, m_tile, n_tile);
        const int32_t a_row = m_tile * (2 * BM) + static_cast<int32_t>(rank) * BM;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[s], ph ^ 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = map_to_rank(smem_u32(&full_bar[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[s], 2 * (A_STAGE_BYTES + B_STAGE_BYTES));
          tma_load_2d_pair(sA + s * A_STAGE_BYTES, &tmA, full_leader, kb * BK, a_row);
          // every tile row re-reads the whole weight: keep it resident in L2
          const uint64_t keep = l2_policy_evict_last();
          if (EPI == VFB_EPI_SWIGLU) {
            // leader: value rows [n*128, +128); peer: the matching gate rows
            tma_load_2d_pair_hint(sB + s * B_STAGE_BYTES, rank == 0 ? &tmB : &tmB2, full_leader,
                                  kb * BK, n_tile * BN_HALF, keep);
          } else {
            tma_load_2d_pair_hint(sB + s * B_STAGE_BYTES, &tmB, full_leader, kb * BK,
                                  n_tile * BN + static_cast<int32_t>(rank) * BN_HALF, keep);
          }
          issued[s] = true;
          issued_phase[s] = ph;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      // Drain: the leader waits until every load it accounted has landed.
      if (rank == 0)
        for (int i = 0; i < STAGES; ++i)
          if (issued[i]) mbar_wait(&full_bar[i], issued_phase[i], abort_flag, p.status);
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // ---------------- MMA issuer (leader CTA only): whole warp, one elected lane ----------------
      constexpr uint32_t idesc = OPS == OPS_BF16 ? idesc_bf16_f32(2 * BM, BN) : idesc_e4m3_f32(2 * BM, BN);
      const bool leader = elect_one();  // the same lane issues and commits every tcgen05 op
      int s = 0;
      uint32_t ph = 0;
      int t = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs, ++t) {
        const int acc = t & 1;
        const uint32_t acc_ph = (t >> 1) & 1;
        if (!warp_wait(&tempty_bar[acc], acc_ph ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!warp_wait(&full_bar[s], ph, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a_desc = sw128_kmajor_desc(smem_u32(sA + s * A_STAGE_BYTES));
          const uint64_t b_desc = sw128_kmajor_desc(smem_u32(sB + s * B_STAGE_BYTES));
          if (leader) {
#pragma unroll
            for (int k = 0; k < BK / UMMA_K; ++k) {
              // +32 bytes along K inside the swizzled 128-byte row = +2 in 16-byte units.
              if constexpr (OPS == OPS_BF16)
                mma_f16_pair(d_tmem, a_desc + 2 * k, b_desc + 2 * k, idesc, (kb | k) != 0);
              else
                mma_f8f6f4_pair(d_tmem, a_desc + 2 * k, b_desc + 2 * k, idesc, (kb | k) != 0);
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
          tc_commit_pair(smem_u32(&tfull_bar[acc]));
          tc_commit_pair(map_to_rank(smem_u32(&tfull_bar[acc]), 1));
        }
        __syncwarp();
      }
      // Drain: all MMAs issued by the leader lane are complete before TMEM is freed.
      if (leader) {
        tc_commit_pair(smem_u32(drain_bar));
        mbar_wait(drain_bar, 0, abort_flag, p.status);
      }
      __syncwarp();
    }
  } else {
    // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const EpiParams &ep = p.ep;
    constexpr int kBoxes = epi_boxes<EPI, OPS>();
    // which group of four warps: its share of the tile's chunks (QKV_NORM_ROPE: its head)
    const int group = (warp - 2) >> 2;
    // groups of four warps that split the tile's chunks (QK-norm + rotary splits by head instead)
    constexpr int kGroups = EPI == VFB_EPI_QKV_NORM_ROPE ? 1 : epi_warps<EPI, OPS>() / 4;
    constexpr int kChunks = BN / 32 / kGroups;  // 32-column chunks per warp and tile
    uint8_t *warp_smem = sEpi + (q + 4 * group) * kBoxes * EPI_BOX_BYTES;
    int box = 0;
    int t = 0;
    for (int tile = pair; tile < num_tiles; tile += num_pairs, ++t) {
      const int acc = t & 1;
      const uint32_t acc_ph = (t >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_ph, abort_flag, p.status)) break;
      tc_fence_after();
      int m_tile, n_tile;
      band_coords(tile, p.num_m_tiles, p.num_n_tiles, p.band_n, m_tile, n_tile);
      const int64_t row0 = static_cast<int64_t>(m_tile) * (2 * BM) + rank * BM + q * 32;
      const int64_t m = row0 + lane;
      const bool live = m < p.M;
      const bool any_row = row0 < p.M;  // warp-uniform
      constexpr bool kScaled = OPS == OPS_E4M3;
      const float sa = kScaled && live ? __ldg(p.sa + m) : 1.0f;
      const uint32_t t_row = tmem_base + acc * BN + (static_cast<uint32_t>(q * 32) << 16);

      if (EPI == VFB_EPI_QKV_NORM_ROPE) {
        const int hh = group;
        const int32_t n0 = n_tile * BN + hh * 128;
        const int32_t plane = n0 / ep.plane_width;
        const int32_t col0 = n0 - plane * ep.plane_width;
        const uint32_t t_head = t_row + hh * 128;
        if (n0 >= p.N) {
          // past the last head (warp-uniform): nothing to store
        } else if (plane == 2) {  // V: plain store
#pragma unroll 1
            for (int k = 0; k < 4; ++k) {
              float v[32];
              tmem_ld_32x32b_x32(t_head + k * 32, v);
              if (live) {
                store_value(v, sa, p.sw, ep, n0 + 32 * k, plane, col0 + 32 * k, m);
              } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = 0.0f;
              }
              int32_t oc, op;
              out_coord(ep, plane, col0 + 32 * k, oc, op);
              store_box<kBoxes, false, true>(warp_smem, box, &tmOut, v, lane, oc, static_cast<int32_t>(row0), op,
                                             any_row);
            }
        } else {
          // pass 1: this thread's row of the head (bf16 values, packed), sum of squares in fp32
          uint32_t hp[64];
          float ss = 0.0f;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float v[32];
            tmem_ld_32x32b_x32(t_head + k * 32, v);
            if (live) {
              store_value(v, sa, p.sw, ep, n0 + 32 * k, plane, col0 + 32 * k, m);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              ss = fmaf(v[j], v[j], ss);
              ss = fmaf(v[j + 1], v[j + 1], ss);
              hp[16 * k + j / 2] = pack_exact_bf16x2(v[j], v[j + 1]);
            }
          }
          const float mean_eps = __fadd_rn(__fdiv_rn(ss, 128.0f), ep.qk_eps);
          const float rstd = static_cast<float>(1.0 / sqrt(static_cast<double>(mean_eps)));
          const __nv_bfloat16 *w = plane == 0 ? ep.q_norm : ep.k_norm;
          const int64_t token = live ? m % ep.tokens : 0;
          const __nv_bfloat16 *cs = ep.rope_cos + token * ep.rope_ts;
          const __nv_bfloat16 *sn = ep.rope_sin + token * ep.rope_ts;
          // pass 2: norm + rotary from registers, one 32-column chunk at a time
          // (unrolled: hp is indexed with compile-time positions only)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float o[32];
            if (live) {
              qk_norm_rope_chunk(hp, rstd, k, w, cs, sn, o);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) o[j] = 0.0f;
            }
            int32_t oc, op;
            out_coord(ep, plane, col0 + 32 * k, oc, op);
            store_box<kBoxes>(warp_smem, box, &tmOut, o, lane, oc, static_cast<int32_t>(row0), op, any_row);
          }
        }
      } else if (EPI == VFB_EPI_SWIGLU) {
        const int32_t F = ep.plane_width;
#pragma unroll 1
        for (int cc = 0; cc < BN_HALF / 64; ++cc) {
          const int c = group * (BN_HALF / 64) + cc;  // each group of four: half of the value/gate chunk pairs
          const int32_t f = n_tile * BN_HALF + c * 32;
          if (f >= F) break;  // warp-uniform
          float v[32], g[32];
          tmem_ld_32x32b_x32(t_row + c * 32, v);
          tmem_ld_32x32b_x32(t_row + BN_HALF + c * 32, g);
          if (live) {
            scale_bias(v, sa, p.sw + f, ep.bias ? ep.bias + f : nullptr);
            scale_bias(g, sa, p.sw + F + f, ep.bias ? ep.bias + F + f : nullptr);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = v[j] * bf16r(silu(g[j]));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.0f;
          }
          store_box<kBoxes>(warp_smem, box, &tmOut, v, lane, f, static_cast<int32_t>(row0), 0, any_row);
        }
      } else if constexpr (OPS == OPS_BF16) {
        // Plain bf16 store (the low-rank products, bound by their output writes):
        // this warp's two adjacent chunks are staged one after the other in its
        // two boxes, then ONE proxy fence covers both box stores (a fence per
        // box made the fence the kernel's main stall).
        static_assert(kChunks == 2 && kBoxes == 2, "two chunks per warp, one box each");
        const int c0 = group * kChunks;
        const int32_t n = n_tile * BN + c0 * 32;
        if (n < p.N) {  // warp-uniform
          if (lane == 0) bulk_wait_group_read<0>();  // both boxes read by the previous tile's stores
          __syncwarp();
          const int sw = (lane >> 1) & 3;  // 64-byte swizzle of the 64-byte box rows
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            float v[32];
            tmem_ld_32x32b_x32(t_row + (c0 + cc) * 32, v);
            if (live) {
              bf16r_x32(v);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = 0.0f;
            }
            uint4 *r = reinterpret_cast<uint4 *>(warp_smem + cc * EPI_BOX_BYTES + lane * 64);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint4 w;
              w.x = pack_exact_bf16x2(v[8 * j + 0], v[8 * j + 1]);
              w.y = pack_exact_bf16x2(v[8 * j + 2], v[8 * j + 3]);
              w.z = pack_exact_bf16x2(v[8 * j + 4], v[8 * j + 5]);
              w.w = pack_exact_bf16x2(v[8 * j + 6], v[8 * j + 7]);
              r[j ^ sw] = w;
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && any_row) {
            const uint64_t policy = l2_policy_evict_first();  // final outputs, as store_box
            tma_store_3d_hint(&tmOut, warp_smem, n, static_cast<int32_t>(row0), 0, policy);
            if (n + 32 < p.N)
              tma_store_3d_hint(&tmOut, warp_smem + EPI_BOX_BYTES, n + 32, static_cast<int32_t>(row0), 0, policy);
            bulk_commit_group();
          }
        }
      } else {
#pragma unroll 1
        for (int cc = 0; cc < kChunks; ++cc) {
          const int c = group * kChunks + cc;
          const int32_t n = n_tile * BN + c * 32;
          if (n >= p.N) break;  // warp-uniform
          float v[32];
          tmem_ld_32x32b_x32(t_row + c * 32, v);
          const int32_t plane = n / ep.plane_width;
          const int32_t col = n - plane * ep.plane_width;
          if (live) {
            if (EPI == VFB_EPI_STORE) {
              store_value<kScaled>(v, sa, p.sw, ep, n, plane, col, m);
            } else if (EPI == VFB_EPI_GELU_TANH) {
              scale_bias(v, sa, p.sw + n, ep.bias ? ep.bias + n : nullptr);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
            } else if (EPI == VFB_EPI_RESIDUAL) {
              scale_bias(v, sa, p.sw + n, ep.bias ? ep.bias + n : nullptr);
              if (ep.gate != nullptr) {
                const __nv_bfloat16 *gp = ep.gate + (m % ep.tokens) * ep.gate_ts + n * ep.gate_hs;
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __bfloat162float(gp[j * ep.gate_hs]) * v[j];
                bf16r_x32(v);
              }
              float r[32];
              load_bf16x32(ep.residual + m * ep.ldr + n, r);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = r[j] + v[j];
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.0f;
          }
          int32_t oc, op;
          out_coord(ep, plane, col, oc, op);
          // STORE values are bf16 already (scale_bias / the merge rounded them)
          store_box<kBoxes, false, EPI == VFB_EPI_STORE>(warp_smem, box, &tmOut, v, lane, oc,
                                                         static_cast<int32_t>(row0), op, any_row);
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(map_to_rank(smem_u32(&tempty_bar[acc]), 0));
    }
    if (lane == 0) bulk_wait_group_all();  // output stores complete before the CTA exits
  }

  __syncthreads();
  __syncwarp();
  cluster_sync();  // both CTAs are done with TMEM before the pair frees it
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ---- host side ---------------------------------------------------------------



template <int EPI, int OPS = OPS_E4M3>
int launch(const CUtensorMap &a, const CUtensorMap &b, const CUtensorMap &b2, const CUtensorMap &o,
           const GemmParams &p, int sm_count, cudaStream_t stream) {
  auto kernel = fp8_gemm_kernel<EPI, OPS>;
  // the shared-memory opt-in is a function attribute of the device's context: set it once per context
  static std::atomic<uint64_t> smem_set[kMaxAttrDevices];
  int rc = ensure_smem_optin(reinterpret_cast<const void *>(kernel), static_cast<int>(smem_bytes<EPI, OPS>()),
                             smem_set);
  if (rc != VFB_OK) return rc;
  // Persistent grid of CTA pairs, one CTA per SM.
  const int tiles = p.num_m_tiles * p.num_n_tiles;
  const int max_pairs = sm_count / 2;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(num_threads<EPI, OPS>(), 1, 1);
  cfg.dynamicSmemBytes = smem_bytes<EPI, OPS>();
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
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, a, b, b2, o, p);
  if (err != cudaSuccess)
    return set_error(VFB_ECUDA, "vfb_fp8_gemm launch: %s", cudaGetErrorString(err));
  return VFB_OK;
}

// Shared body of vfb_fp8_gemm and vfb_bf16_gemm.  K, lda and ldw are in BYTES
// of the operand rows (= elements for e4m3); fn names the entry point in errors.
int gemm_impl(const char *fn, int ops, const void *A, int64_t lda, const float *sa, const void *W,
              int64_t ldw, const float *sw, int64_t M, int64_t N, int64_t K, const vfb_epilogue *ep,
              void *stream) {
  if (ep == nullptr) return set_error(VFB_EINVAL, "%s: epilogue is NULL", fn);
  const int kind = ep->kind;
  if (kind < VFB_EPI_STORE || kind > VFB_EPI_QKV_NORM_ROPE)
    return set_error(VFB_EINVAL, "%s: unknown epilogue kind %d", fn, kind);
  // bf16 operands: N % 8 (the output boxes clip at N), plain STORE, no scales
  const bool bf16 = ops == OPS_BF16;
  if (M < 0 || N <= 0 || K <= 0 || K % 16 || N % (bf16 ? 8 : 32))
    return set_error(VFB_EINVAL, "%s: need M >= 0, N > 0 with N %% %d == 0, K > 0 with "
                                 "%d-byte rows (M=%lld N=%lld K=%lld)", fn, bf16 ? 8 : 32, 16,
                     (long long)M, (long long)N, (long long)(bf16 ? K / 2 : K));
  if (bf16 && (kind != VFB_EPI_STORE || ep->wire_chunks != 0 || ep->plane_width != 0 ||
               ep->adapter[0] != nullptr || ep->adapter[1] != nullptr || ep->adapter[2] != nullptr ||
               ep->bias != nullptr))
    return set_error(VFB_EINVAL, "%s: bf16 operands take a plain STORE epilogue (one plane, no bias, "
                                 "no adapters)", fn);
  if (M == 0) return VFB_OK;
  if (M > (int64_t)2 * BM * 0x3FFFFF || N > (int64_t)1 << 24 || K > (int64_t)1 << 20)
    return set_error(VFB_EINVAL, "%s: problem too large", fn);
  if (A == nullptr || W == nullptr || (!bf16 && (sa == nullptr || sw == nullptr)) || ep->out == nullptr)
    return set_error(VFB_EINVAL, "%s: NULL operand", fn);
  if (lda < K || ldw < K || lda % 16 || ldw % 16 || !aligned16(A) || !aligned16(W))
    return set_error(VFB_EINVAL, "%s: A/W need 16-byte aligned bases and row strides", fn);
  if ((!bf16 && !aligned16(sw)) || !aligned16(ep->out) || ep->ldo % 8)
    return set_error(VFB_EINVAL, "%s: sw/out need 16-byte alignment, ldo %% 8 == 0", fn);
  if (ep->bias != nullptr && !aligned16(ep->bias))
    return set_error(VFB_EINVAL, "%s: bias needs 16-byte alignment", fn);
  if (ep->wire_chunks < 0 || ep->wire_chunks > 1024 ||
      (ep->wire_chunks > 0 && kind != VFB_EPI_STORE && kind != VFB_EPI_QKV_NORM_ROPE))
    return set_error(VFB_EINVAL, "%s: wire_chunks must be 0..1024, and 0 unless the epilogue is "
                                 "STORE or QKV_NORM_ROPE", fn);
  if (kind == VFB_EPI_SWIGLU && N % 64)
    return set_error(VFB_EINVAL, "%s: SWIGLU needs the packed width N = 2F, F %% 32 == 0", fn);
  if (kind == VFB_EPI_SWIGLU && ep->ldo < N / 2) return set_error(VFB_EINVAL, "%s: SWIGLU output ldo < F", fn);

  int sm_count = 0;
  int rc = check_device(&sm_count);
  if (rc != VFB_OK) return rc;

  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.sa = sa;
  p.sw = sw;
  p.num_m_tiles = static_cast<int>((M + 2 * BM - 1) / (2 * BM));
  p.num_kb = static_cast<int>((K + BK - 1) / BK);
  p.status = device_status_ptr();
  EpiParams &e = p.ep;
  e.bias = static_cast<const __nv_bfloat16 *>(ep->bias);

  CUtensorMap ta, tb, tb2, to;
  rc = make_map_u8(&ta, A, M, K, lda, BM);
  if (rc != VFB_OK) return rc;

  if (kind == VFB_EPI_SWIGLU) {
    const int64_t F = N / 2;
    e.plane_width = static_cast<int32_t>(F);
    p.num_n_tiles = static_cast<int>((F + BN_HALF - 1) / BN_HALF);
    if ((rc = make_map_out(&to, ep->out, F, M, 1, ep->ldo, M * ep->ldo)) != VFB_OK) return rc;
    const uint8_t *gate_rows = static_cast<const uint8_t *>(W) + F * ldw;
    if ((rc = make_map_u8(&tb, W, F, K, ldw, BN_HALF)) != VFB_OK) return rc;
    if ((rc = make_map_u8(&tb2, gate_rows, F, K, ldw, BN_HALF)) != VFB_OK) return rc;
  } else {
    if (ep->plane_width < 0 || (ep->plane_width > 0 && (ep->plane_width % 32 || N % ep->plane_width)))
      return set_error(VFB_EINVAL, "%s: plane_width must be 0 or a multiple of 32 dividing N", fn);
    const int64_t width = ep->plane_width > 0 ? ep->plane_width : N;
    const int64_t planes = N / width;
    const int64_t chunks = ep->wire_chunks;
    if (chunks > 0 && (planes != 3 || width % (2 * chunks) || (width / (2 * chunks)) % 32))
      return set_error(VFB_EINVAL, "%s: the wire layout needs three planes whose width splits into "
                                   "2 * wire_chunks groups of a multiple of 32 columns", fn);
    // the tensor map's planes: the output planes, or the 6 * wire_chunks slabs of the wire layout
    const int64_t out_width = chunks > 0 ? width / (2 * chunks) : width;
    const int64_t slabs = chunks > 0 ? 6 * chunks : planes;
    if (ep->ldo < out_width) return set_error(VFB_EINVAL, "%s: ldo smaller than the plane width", fn);
    const int64_t plane_stride = slabs > 1 ? ep->plane_stride : M * ep->ldo;
    if (plane_stride % 8 || (slabs > 1 && plane_stride < M * ep->ldo))
      return set_error(VFB_EINVAL, "%s: plane_stride must be a multiple of 8 and >= M*ldo", fn);
    e.plane_width = static_cast<int32_t>(width);
    e.wire_chunks = static_cast<int32_t>(chunks);
    e.wire_width = static_cast<int32_t>(out_width);
    if ((rc = make_map_out(&to, ep->out, out_width, M, slabs, ep->ldo, plane_stride)) != VFB_OK) return rc;
    p.num_n_tiles = static_cast<int>((N + BN - 1) / BN);
    if ((rc = make_map_u8(&tb, W, N, K, ldw, BN_HALF)) != VFB_OK) return rc;
    tb2 = tb;
    if (kind == VFB_EPI_QKV_NORM_ROPE) {
      const auto a16p = [](const void *q) { return q == nullptr || aligned16(q); };
      if (planes != 3 || width % 128)
        return set_error(VFB_EINVAL, "%s: QKV_NORM_ROPE needs three planes of 128-column heads", fn);
      if (ep->rope_cos == nullptr || ep->rope_sin == nullptr || !aligned16(ep->rope_cos) ||
          !aligned16(ep->rope_sin) || ep->rope_token_stride < 0 || ep->rope_token_stride % 8 ||
          (ep->tokens > 1 && ep->rope_token_stride < 128) || ep->tokens <= 0)
        return set_error(VFB_EINVAL, "%s: rotary cos/sin need 16-byte aligned [tokens, 128] rows, tokens > 0", fn);
      if (!a16p(ep->q_norm) || !a16p(ep->k_norm) || !(ep->qk_eps > 0.0f))
        return set_error(VFB_EINVAL, "%s: QK-norm weights need 16-byte alignment, qk_eps > 0", fn);
      e.q_norm = static_cast<const __nv_bfloat16 *>(ep->q_norm);
      e.k_norm = static_cast<const __nv_bfloat16 *>(ep->k_norm);
      e.rope_cos = static_cast<const __nv_bfloat16 *>(ep->rope_cos);
      e.rope_sin = static_cast<const __nv_bfloat16 *>(ep->rope_sin);
      e.rope_ts = ep->rope_token_stride;
      e.qk_eps = ep->qk_eps;
      e.tokens = ep->tokens;
    }
    if (kind == VFB_EPI_STORE || kind == VFB_EPI_QKV_NORM_ROPE) {
      for (int i = 0; i < 3; ++i) {
        e.adapter[i] = static_cast<const __nv_bfloat16 *>(ep->adapter[i]);
        e.scaling[i] = ep->scaling[i];
        if (e.adapter[i] != nullptr) {
          if (i >= planes || !aligned16(e.adapter[i]) || ep->adapter_ld % 8 || ep->adapter_ld < width)
            return set_error(VFB_EINVAL, "%s: adapter %d misaligned or beyond the planes", fn, i);
        }
      }
      e.adapter_ld = ep->adapter_ld;
    }
    if (kind == VFB_EPI_RESIDUAL) {
      if (ep->residual == nullptr || !aligned16(ep->residual) || ep->ldr % 8 || ep->ldr < N)
        return set_error(VFB_EINVAL, "%s: residual needs a 16-byte aligned [M,N] view", fn);
      if (planes != 1)
        return set_error(VFB_EINVAL, "%s: RESIDUAL writes one plane", fn);
      e.residual = static_cast<const __nv_bfloat16 *>(ep->residual);
      e.ldr = ep->ldr;
      e.gate = static_cast<const __nv_bfloat16 *>(ep->gate);
      if (e.gate != nullptr) {
        if (ep->tokens <= 0)
          return set_error(VFB_EINVAL, "%s: gate needs tokens > 0", fn);
        e.gate_ts = ep->gate_token_stride;
        e.gate_hs = ep->gate_hidden_stride;
        e.tokens = ep->tokens;
      }
    }
  }

  p.band_n = band_width(p.num_n_tiles, K);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bf16) return launch<VFB_EPI_STORE, OPS_BF16>(ta, tb, tb2, to, p, sm_count, s);
  switch (kind) {
    case VFB_EPI_STORE:
      return launch<VFB_EPI_STORE>(ta, tb, tb2, to, p, sm_count, s);
    case VFB_EPI_GELU_TANH:
      return launch<VFB_EPI_GELU_TANH>(ta, tb, tb2, to, p, sm_count, s);
    case VFB_EPI_SWIGLU:
      return launch<VFB_EPI_SWIGLU>(ta, tb, tb2, to, p, sm_count, s);
    case VFB_EPI_QKV_NORM_ROPE:
      return launch<VFB_EPI_QKV_NORM_ROPE>(ta, tb, tb2, to, p, sm_count, s);
    default:
      return launch<VFB_EPI_RESIDUAL>(ta, tb, tb2, to, p, sm_count, s);
  }
}

}  // namespace
}  // namespace vfb

extern "C" int vfb_fp8_gemm(const void *A, int64_t lda, const float *sa, const void *W, int64_t ldw,
                            const float *sw, int64_t M, int64_t N, int64_t K,
                            const vfb_epilogue *ep, void *stream) {
  return vfb::gemm_impl("vfb_fp8_gemm", vfb::OPS_E4M3, A, lda, sa, W, ldw, sw, M, N, K, ep, stream);
}

extern "C" int vfb_bf16_gemm(const void *A, int64_t lda, const void *W, int64_t ldw, int64_t M, int64_t N,
                             int64_t K, const vfb_epilogue *ep, void *stream) {
  using namespace vfb;
  if (K <= 0 || K % 8 || lda < K || ldw < K || lda % 8 || ldw % 8 || K > (int64_t)1 << 19)
    return set_error(VFB_EINVAL, "vfb_bf16_gemm: need 0 < K <= 2^19 with K %% 8 == 0 and row strides "
                                 ">= K, multiples of 8 (K=%lld lda=%lld ldw=%lld)",
                     (long long)K, (long long)lda, (long long)ldw);
  // the operands travel as bytes: 2 per element
  return gemm_impl("vfb_bf16_gemm", OPS_BF16, A, 2 * lda, nullptr, W, 2 * ldw, nullptr, M, N, 2 * K, ep,
                   stream);
}
