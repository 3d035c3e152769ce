// Fused FP8 FFN for sm_100a: up GEMM + activation, per-token requantisation of
// the bf16 intermediate, down GEMM + bias / gated residual, in one persistent
// launch whose intermediate stays in L2.
//
// Arithmetic (the same bits as the separate steps, and as the reference's
// chain: src/vflash/native/h3_fp8_linear.py:92-121 per linear,
// h3_fused_ops.py:185-224 for SwiGLU, h3_fp8_activation.py:16-19 for the
// requantisation of the intermediate over its full row):
//   mid[m,f]  = act(bf16(bf16(sx[m] * s_up[f] * sum_h X[m,h] W_up[f,h]) + bias_up[f]))   rounded to bf16
//   codes     = e4m3(mid / scale[m]), scale[m] = max(max_f |mid[m,f]| / 448, FLT_MIN) (1 for 0 or NaN)
//   out[m,n]  = epilogue(bf16(bf16(scale[m] * s_down[n] * sum_f codes[m,f] W_down[n,f]) + bias_down[n]))
// with act = GELU-tanh, or value * bf16(silu(gate)) over the packed [2F, H]
// up weight, and the down epilogue a plain store or bf16(residual + bf16(gate * y)).
//
// Structure: persistent CTA pairs (cta_group::2, 256 x 256 tiles, the FP8
// GEMM's TMA ring, MMA issue and TMEM double buffer; fp8_gemm.cu).  The pairs
// take work items from one global counter in the order of ffn_plan.h: up
// tiles of a group of row blocks in weight bands, then down tiles of that
// group interleaved with up tiles of the next.  The leader CTA's producer
// thread takes the item and publishes it to both CTAs' item rings.
//   up tile:   the epilogue stores the bf16 intermediate (evict_last: it is
//              read back within a few tiles), takes each row's maximum of
//              |mid| on the bf16 bit patterns and merges it into the row's
//              global maximum with atomicMax, then counts the tile done for
//              its row block.  Once every up tile of the row block is done
//              (all row maxima final), the warp that stored a region converts
//              that same region to e4m3 codes, drops the bf16 lines from L2
//              without write-back, and counts the conversion done.
//   down tile: the producer waits until its row block is converted, then
//              TMA-loads the codes like any GEMM operand; the epilogue takes
//              the row scale from the row maximum.
// Waits on flags in global memory are bounded (4 s, then VFB_ETIMEOUT) like
// every mbarrier wait; an item only waits on items that running pairs took
// earlier from the counter, so the order cannot deadlock whether or not
// every pair of the grid is resident.  No TMA multicast is used.
#include <cudaTypedefs.h>

#include <atomic>

#include "common.cuh"
#include "epilogue.cuh"
#include "ffn_fused.h"
#include "ffn_plan.h"
#include "quant.cuh"

namespace vfb {
namespace {

constexpr int BM = 128;          // A rows per CTA (pair: 256)
constexpr int BN = 256;          // output columns per pair tile (SwiGLU: 128 value + 128 gate)
constexpr int BN_HALF = BN / 2;  // weight rows per CTA
constexpr int BK = 128;          // bytes of K per stage
constexpr int UMMA_K = 32;
constexpr int STAGES = 5;
constexpr int A_STAGE = BM * BK;
constexpr int B_STAGE = BN_HALF * BK;
constexpr int EPI_WARPS = 8;     // two per TMEM lane quarter: group 0 and 1 take one half of the tile's columns
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
constexpr int TMEM_COLS = 512;
constexpr int BOXES = 2;         // staging boxes per epilogue warp
constexpr int EPI_SMEM = EPI_WARPS * BOXES * EPI_BOX_BYTES;
constexpr int RING = 8;          // published work items in flight
// Stored regions awaiting conversion, per epilogue warp, kept in shared memory.
// A warp holds one entry per up tile from the first tile of a row block until
// that row block is complete; the FIFO must never fill in practice, because a
// full FIFO makes the warp wait for its oldest row block, whose last up tile
// may be queued behind this very warp (the wait is bounded, not a hang, but
// it costs the time limit).  64 entries cover many groups of row blocks.
constexpr int PENDING = 64;
constexpr int PENDING_SMEM = EPI_WARPS * PENDING * 4;
constexpr size_t SMEM_BYTES = 1024 + STAGES * (A_STAGE + B_STAGE) + EPI_SMEM + PENDING_SMEM + 512;

struct FfnParams {
  int64_t M, H, F;
  FfnPlan plan;
  int done_target;  // per row block: up tiles x 2 CTAs x EPI_WARPS signals (stored, converted)
  const float *x_scales;
  const float *s_up;
  const float *s_down;
  const __nv_bfloat16 *bias_up;
  const __nv_bfloat16 *bias_down;
  const __nv_bfloat16 *residual;
  int64_t ldr;
  const __nv_bfloat16 *gate;
  int64_t gate_ts;
  int64_t tokens;
  const __nv_bfloat16 *mid;  // [M, F]
  uint8_t *mid_codes;        // [M, F]
  uint32_t *amax_bits;       // [M]: max |mid| per row as bf16 bits (zeroed before the launch)
  int *queue;                // work-item counter (zeroed)
  int *up_done;              // [R] (zeroed)
  int *conv_done;            // [R] (zeroed)
  int *status;
};

// Bounded wait until *flag >= target (acquire).  Returns false on abort or timeout.
__device__ __forceinline__ bool wait_flag(const int *flag, int target, volatile int *abort_flag, int *status) {
  if (ld_acquire_gpu(flag) >= target) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t spin = 1;; ++spin) {
    __nanosleep(128);
    if (ld_acquire_gpu(flag) >= target) return true;
    if ((spin & 63u) == 0) {
      if (*abort_flag) return false;
      if (global_timer_ns() - start > VFB_WAIT_TIMEOUT_NS) {
        *abort_flag = 1;
        record_status(status, VFB_ETIMEOUT);
        return false;
      }
    }
  }
}

// Maximum of |v| over 32 bf16-representable floats, as bf16 bit patterns
// (sign cleared; NaN patterns order above +inf, as in the quantiser).
__device__ __forceinline__ uint32_t abs_bits_max32(const float (&v)[32], uint32_t acc) {
#pragma unroll
  for (int j = 0; j < 32; ++j) acc = max(acc, (__float_as_uint(v[j]) >> 16) & 0x7fffu);
  return acc;
}

// Per epilogue warp: the regions it stored whose row blocks were not complete
// yet, in the order stored (row blocks complete in about that order).  The
// entries (row block << 9 | tile; a row block has at most 256 up tiles) live
// in shared memory; head and count are warp-uniform registers, and lane 0
// writes the entries.
struct Pending {
  uint32_t *entry;  // PENDING entries of this warp
  int head = 0;
  int count = 0;
  __device__ __forceinline__ int r() const { return static_cast<int>(entry[head] >> 9); }
  __device__ __forceinline__ int t() const { return static_cast<int>(entry[head] & 0x1ffu); }
};

template <int ACT>
struct Ffn {
  static constexpr bool kSwiglu = ACT == VFB_EPI_SWIGLU;
  // columns of the intermediate one epilogue warp stores (and converts) per up tile
  static constexpr int kWarpCols = kSwiglu ? 64 : 128;

  // Converts this warp's region of up tile (r, t) to e4m3 codes.  The row
  // maxima are final (every up tile of row block r is done).
  static __device__ void convert(const FfnParams &p, int r, int t, int rank, int quarter, int group,
                                 int lane) {
    constexpr int LPR = kWarpCols / 8;  // lanes per row (one 16-byte vector of 8 bf16 each)
    constexpr int RPI = 32 / LPR;       // rows per pass
    constexpr int PASSES = 32 / RPI;
    const int64_t col0 = kSwiglu ? static_cast<int64_t>(t) * 128 + group * 64
                                 : static_cast<int64_t>(t) * 256 + group * 128;
    // this warp's TMA stores of the region have landed and are visible to plain loads
    if (lane == 0) {
      bulk_wait_group_all();
      fence_proxy_async_global();
    }
    __syncwarp();
    const int64_t base = static_cast<int64_t>(r) * 256 + rank * BM + quarter * 32 + lane / LPR;
    const int part = lane % LPR;
    constexpr int BATCH = 4;  // loads in flight per lane
#pragma unroll 1
    for (int i0 = 0; i0 < PASSES; i0 += BATCH) {
      uint4 v[BATCH];
      uint32_t bits[BATCH];
#pragma unroll
      for (int i = 0; i < BATCH; ++i) {
        const int64_t m = base + (i0 + i) * RPI;
        if (m < p.M) {
          bits[i] = __ldcg(p.amax_bits + m);
          v[i] = __ldcg(reinterpret_cast<const uint4 *>(p.mid + m * p.F + col0) + part);
        }
      }
#pragma unroll
      for (int i = 0; i < BATCH; ++i) {
        const int64_t m = base + (i0 + i) * RPI;
        if (m < p.M) {
          const float scale = row_scale_from_bits(bits[i]);
          const bool fast = markstein_ok(scale);
          const uint2 out = fast ? quantize8(v[i], scale, __frcp_rn(scale)) : quantize8_ieee(v[i], scale);
          *reinterpret_cast<uint2 *>(p.mid_codes + m * p.F + col0 + part * 8) = out;
        }
      }
    }
    __syncwarp();
    // the bf16 intermediate of this region is dead: drop its L2 lines unwritten
    if ((part * 16) % 128 == 0) {
#pragma unroll
      for (int i = 0; i < PASSES; ++i) {
        const int64_t m = base + i * RPI;
        if (m < p.M) discard_l2_line(p.mid + m * p.F + col0 + part * 8);
      }
    }
    // the codes are read by other CTAs' TMA loads (async proxy)
    __threadfence();
    fence_proxy_async_global();
    __syncwarp();
    if (lane == 0) red_release_gpu_add(p.conv_done + r, 1);
  }

  static __device__ __forceinline__ bool front_ready(const FfnParams &p, const Pending &pend, int lane) {
    int ready = 0;
    if (lane == 0) ready = ld_acquire_gpu(p.up_done + pend.r()) >= p.done_target;
    ready = __shfl_sync(0xffffffffu, ready, 0);
    __syncwarp();
    return ready != 0;
  }

  static __device__ __forceinline__ void pop_convert(const FfnParams &p, Pending &pend, int rank, int quarter,
                                                     int group, int lane) {
    convert(p, pend.r(), pend.t(), rank, quarter, group, lane);
    pend.head = (pend.head + 1) % PENDING;
    --pend.count;
  }

  // Converts every pending region whose row block is complete.
  static __device__ void convert_ready(const FfnParams &p, Pending &pend, int rank, int quarter, int group,
                                       int lane) {
    while (pend.count > 0 && front_ready(p, pend, lane)) pop_convert(p, pend, rank, quarter, group, lane);
  }

  // Converts the oldest pending region, waiting (bounded) for its row block.
  static __device__ bool convert_oldest(const FfnParams &p, Pending &pend, int rank, int quarter, int group,
                                        int lane, volatile int *abort_flag) {
    bool ok = true;
    if (lane == 0) ok = wait_flag(p.up_done + pend.r(), p.done_target, abort_flag, p.status);
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    __syncwarp();
    if (!ok) return false;
    pop_convert(p, pend, rank, quarter, group, lane);
    return true;
  }

  // Waits (bounded) for an mbarrier phase; while it is not complete, converts
  // pending regions whose row blocks are done (the row-block counter is
  // polled every 4th spin).
  static __device__ bool wait_converting(uint64_t *bar, uint32_t parity, bool cluster_acquire,
                                         const FfnParams &p, Pending &pend, int rank, int quarter, int group,
                                         int lane, volatile int *abort_flag) {
    const uint64_t start = global_timer_ns();
    for (uint32_t spin = 1;; ++spin) {
      const bool done = cluster_acquire ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
      if (__any_sync(0xffffffffu, done)) {
        // complete for every lane now; each lane acquires it itself
        const bool ok = cluster_acquire ? mbar_wait_cluster(bar, parity, abort_flag, p.status)
                                        : mbar_wait(bar, parity, abort_flag, p.status);
        return __all_sync(0xffffffffu, ok);
      }
      if ((spin & 3u) == 0 && pend.count > 0 && front_ready(p, pend, lane)) {
        pop_convert(p, pend, rank, quarter, group, lane);
        continue;
      }
      if ((spin & 255u) == 0) {
        int stop = 0;
        if (lane == 0) {
          if (*abort_flag) {
            stop = 1;
          } else if (global_timer_ns() - start > VFB_WAIT_TIMEOUT_NS) {
            *abort_flag = 1;
            record_status(p.status, VFB_ETIMEOUT);
            stop = 1;
          }
        }
        if (__shfl_sync(0xffffffffu, stop, 0)) return false;
      }
    }
  }
};

template <int ACT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    ffn_kernel(const __grid_constant__ CUtensorMap tmAx, const __grid_constant__ CUtensorMap tmAm,
               const __grid_constant__ CUtensorMap tmBu, const __grid_constant__ CUtensorMap tmBu2,
               const __grid_constant__ CUtensorMap tmBd, const __grid_constant__ CUtensorMap tmMid,
               const __grid_constant__ CUtensorMap tmOut, const FfnParams p) {
  using F = Ffn<ACT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  uint8_t *sA = smem;
  uint8_t *sB = smem + STAGES * A_STAGE;
  uint8_t *sEpi = sB + STAGES * B_STAGE;
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(sEpi + EPI_SMEM + PENDING_SMEM);
  uint64_t *empty_bar = full_bar + STAGES;
  uint64_t *tfull_bar = empty_bar + STAGES;
  uint64_t *tempty_bar = tfull_bar + 2;
  uint64_t *item_full = tempty_bar + 2;   // per CTA: the leader's producer published an item
  uint64_t *item_empty = item_full + RING;  // leader: every consumer of both CTAs read it
  uint64_t *drain_bar = item_empty + RING;
  volatile int *items = reinterpret_cast<volatile int *>(drain_bar + 1);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(const_cast<int *>(items) + RING);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * 32 * EPI_WARPS);
    }
    for (int i = 0; i < RING; ++i) {
      mbar_init(&item_full[i], 1);
      // the peer's producer, the MMA warp, and one lane of every epilogue warp of both CTAs
      mbar_init(&item_empty[i], 2 + 2 * EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmAx);
    tma_prefetch_desc(&tmAm);
    tma_prefetch_desc(&tmBu);
    if (F::kSwiglu) tma_prefetch_desc(&tmBu2);
    tma_prefetch_desc(&tmBd);
  }
  if (warp == 2 && lane == 0) {
    tma_prefetch_desc(&tmMid);
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
  const int kb_up = static_cast<int>((p.H + BK - 1) / BK);
  const int kb_down = static_cast<int>((p.F + BK - 1) / BK);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- work items and TMA producer (both CTAs) ----------------
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_phase[STAGES];
      bool issued[STAGES];
      for (int i = 0; i < STAGES; ++i) issued[i] = false;
      const uint64_t keep = l2_policy_evict_last();
      bool ok = true;
      for (int i = 0; ok; ++i) {
        const int slot = i % RING;
        const uint32_t iph = (i / RING) & 1;
        int q;
        if (rank == 0) {
          // every consumer of both CTAs has read the item this slot held
          if (!mbar_wait_cluster(&item_empty[slot], iph ^ 1, abort_flag, p.status)) break;
          // an item is taken only when this pair can start it: an item taken
          // ahead would hold up the row blocks whose conversions others wait for
          q = atomicAdd(p.queue, 1);
          if (q >= p.plan.total) q = -1;
          items[slot] = q;
          st_shared_cluster_u32(map_to_rank(smem_u32(const_cast<int *>(&items[slot])), 1), static_cast<uint32_t>(q));
          mbar_arrive(&item_full[slot]);
          mbar_arrive_cluster(map_to_rank(smem_u32(&item_full[slot]), 1));
        } else {
          if (!mbar_wait_cluster(&item_full[slot], iph, abort_flag, p.status)) break;
          q = items[slot];
          mbar_arrive_cluster(map_to_rank(smem_u32(&item_empty[slot]), 0));
        }
        if (q < 0) break;
        int kind, r, t;
        ffn_item(p.plan, q, kind, r, t);
        const int32_t a_row = r * (2 * BM) + static_cast<int32_t>(rank) * BM;
        const CUtensorMap *ma, *mb;
        int32_t b_row;
        int nkb;
        if (kind == kFfnUp) {
          ma = &tmAx;
          nkb = kb_up;
          if (F::kSwiglu) {
            mb = rank == 0 ? &tmBu : &tmBu2;  // leader: value rows, peer: the matching gate rows
            b_row = t * BN_HALF;
          } else {
            mb = &tmBu;
            b_row = t * BN + static_cast<int32_t>(rank) * BN_HALF;
          }
        } else {
          ma = &tmAm;
          mb = &tmBd;
          nkb = kb_down;
          b_row = t * BN + static_cast<int32_t>(rank) * BN_HALF;
          // the row block's codes are written (plain stores) and published
          if (!wait_flag(p.conv_done + r, p.done_target, abort_flag, p.status)) break;
          fence_proxy_async_global();
        }
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty_bar[s], ph ^ 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = map_to_rank(smem_u32(&full_bar[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[s], 2 * (A_STAGE + B_STAGE));
          tma_load_2d_pair(sA + s * A_STAGE, ma, full_leader, kb * BK, a_row);
          tma_load_2d_pair_hint(sB + s * B_STAGE, mb, full_leader, kb * BK, b_row, keep);
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
      // ---------------- MMA issuer (leader CTA): whole warp, one elected lane ----------------
      constexpr uint32_t idesc = idesc_e4m3_f32(2 * BM, BN);
      const bool leader = elect_one();
      int s = 0;
      uint32_t ph = 0;
      int t = 0;
      bool ok = true;
      for (int i = 0; ok; ++i) {
        const int slot = i % RING;
        const uint32_t iph = (i / RING) & 1;
        if (!warp_wait(&item_full[slot], iph, abort_flag, p.status)) break;
        const int q = items[slot];
        __syncwarp();
        if (leader) mbar_arrive(&item_empty[slot]);
        if (q < 0) break;
        int kind, r, tt;
        ffn_item(p.plan, q, kind, r, tt);
        const int nkb = kind == kFfnUp ? kb_up : kb_down;
        const int acc = t & 1;
        const uint32_t acc_ph = (t >> 1) & 1;
        if (!warp_wait(&tempty_bar[acc], acc_ph ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!warp_wait(&full_bar[s], ph, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a_desc = sw128_kmajor_desc(smem_u32(sA + s * A_STAGE));
          const uint64_t b_desc = sw128_kmajor_desc(smem_u32(sB + s * B_STAGE));
          if (leader) {
#pragma unroll
            for (int k = 0; k < BK / UMMA_K; ++k)
              mma_f8f6f4_pair(d_tmem, a_desc + 2 * k, b_desc + 2 * k, idesc, (kb | k) != 0);
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
        ++t;
      }
      if (leader) {
        tc_commit_pair(smem_u32(drain_bar));
        mbar_wait(drain_bar, 0, abort_flag, p.status);
      }
      __syncwarp();
    }
  } else {
    // ---------------- epilogue (warps 2..9 of both CTAs) ----------------
    const int ew = warp - 2;
    const int quarter = warp & 3;  // TMEM lane quarter: this warp's 32 rows of the tile
    const int group = ew >> 2;     // which half of the tile's columns
    uint8_t *warp_smem = sEpi + ew * BOXES * EPI_BOX_BYTES;
    const uint32_t tempty_leader = map_to_rank(smem_u32(&tempty_bar[0]), 0);
    Pending pend;
    pend.entry = reinterpret_cast<uint32_t *>(sEpi + EPI_SMEM) + ew * PENDING;
    int box = 0;
    int t = 0;
    for (int i = 0;; ++i) {
      const int slot = i % RING;
      const uint32_t iph = (i / RING) & 1;
      if (!F::wait_converting(&item_full[slot], iph, rank != 0, p, pend, rank, quarter, group, lane, abort_flag))
        break;
      const int q = items[slot];
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(&item_empty[slot]);
        else
          mbar_arrive_cluster(map_to_rank(smem_u32(&item_empty[slot]), 0));
      }
      if (q < 0) break;
      int kind, r, tt;
      ffn_item(p.plan, q, kind, r, tt);
      const int acc = t & 1;
      const uint32_t acc_ph = (t >> 1) & 1;
      if (!F::wait_converting(&tfull_bar[acc], acc_ph, false, p, pend, rank, quarter, group, lane, abort_flag))
        break;
      tc_fence_after();
      const int64_t row0 = static_cast<int64_t>(r) * (2 * BM) + rank * BM + quarter * 32;
      const int64_t m = row0 + lane;
      const bool live = m < p.M;
      const bool any_row = row0 < p.M;
      const uint32_t t_row = tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      if (kind == kFfnUp) {
        const float sa = live ? __ldg(p.x_scales + m) : 1.0f;
        uint32_t rmax = 0;
        if (F::kSwiglu) {
#pragma unroll 1
          for (int cc = 0; cc < 2; ++cc) {
            const int c = group * 2 + cc;
            const int64_t f = static_cast<int64_t>(tt) * BN_HALF + c * 32;
            float v[32], g[32];
            tmem_ld_32x32b_x32(t_row + c * 32, v);
            tmem_ld_32x32b_x32(t_row + BN_HALF + c * 32, g);
            if (live) {
              scale_bias(v, sa, p.s_up + f, p.bias_up ? p.bias_up + f : nullptr);
              scale_bias(g, sa, p.s_up + p.F + f, p.bias_up ? p.bias_up + p.F + f : nullptr);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = v[j] * bf16r(silu(g[j]));
              bf16r_x32(v);
              rmax = abs_bits_max32(v, rmax);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = 0.0f;
            }
            store_box<BOXES, true, true>(warp_smem, box, &tmMid, v, lane, static_cast<int32_t>(f),
                                   static_cast<int32_t>(row0), 0, any_row);
          }
        } else {
#pragma unroll 1
          for (int cc = 0; cc < 4; ++cc) {
            const int c = group * 4 + cc;
            const int64_t n = static_cast<int64_t>(tt) * BN + c * 32;
            float v[32];
            tmem_ld_32x32b_x32(t_row + c * 32, v);
            if (live) {
              scale_bias(v, sa, p.s_up + n, p.bias_up ? p.bias_up + n : nullptr);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
              bf16r_x32(v);
              rmax = abs_bits_max32(v, rmax);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = 0.0f;
            }
            store_box<BOXES, true, true>(warp_smem, box, &tmMid, v, lane, static_cast<int32_t>(n),
                                   static_cast<int32_t>(row0), 0, any_row);
          }
        }
        tc_fence_before();
        mbar_arrive_cluster(tempty_leader + acc * sizeof(uint64_t));
        // this tile's row maxima, then the tile counts as stored for its row block
        if (live && rmax != 0) atomicMax(p.amax_bits + m, rmax);
        __threadfence();
        __syncwarp();
        if (lane == 0) red_release_gpu_add(p.up_done + r, 1);
        if (pend.count == PENDING && !F::convert_oldest(p, pend, rank, quarter, group, lane, abort_flag)) break;
        if (lane == 0) pend.entry[(pend.head + pend.count) % PENDING] = (static_cast<uint32_t>(r) << 9) | tt;
        __syncwarp();
        ++pend.count;
      } else {
        // the row block's maxima are final (its conversions are published)
        bool ready = true;
        if (lane == 0) ready = ld_acquire_gpu(p.conv_done + r) >= p.done_target;
        __syncwarp();
        if (!__shfl_sync(0xffffffffu, ready ? 1 : 0, 0)) {
          record_status(p.status, VFB_ETIMEOUT);  // cannot happen: the producer waited for it
          *abort_flag = 1;
          break;
        }
        const float sa = live ? row_scale_from_bits(__ldcg(p.amax_bits + m)) : 1.0f;
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          const int c = group * 4 + cc;
          const int64_t n = static_cast<int64_t>(tt) * BN + c * 32;
          if (n >= p.H) break;  // warp-uniform
          float v[32];
          tmem_ld_32x32b_x32(t_row + c * 32, v);
          if (live) {
            scale_bias(v, sa, p.s_down + n, p.bias_down ? p.bias_down + n : nullptr);
            if (p.residual != nullptr) {
              if (p.gate != nullptr) {
                const __nv_bfloat16 *gp = p.gate + (m % p.tokens) * p.gate_ts + n;
                float gv[32];
                load_bf16x32(gp, gv);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = gv[j] * v[j];
                bf16r_x32(v);
              }
              float res[32];
              load_bf16x32(p.residual + m * p.ldr + n, res);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = res[j] + v[j];
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.0f;
          }
          store_box<BOXES, false>(warp_smem, box, &tmOut, v, lane, static_cast<int32_t>(n),
                                  static_cast<int32_t>(row0), 0, any_row);
        }
        tc_fence_before();
        mbar_arrive_cluster(tempty_leader + acc * sizeof(uint64_t));
      }
      ++t;
      F::convert_ready(p, pend, rank, quarter, group, lane);
    }
    // every up tile has been handed out: finish this warp's conversions
    while (pend.count > 0 && !*abort_flag)
      if (!F::convert_oldest(p, pend, rank, quarter, group, lane, abort_flag)) break;
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

}  // namespace

int ffn_fused_supported(int32_t activation, int64_t H, int64_t F) {
  return H % 32 == 0 && (activation == VFB_EPI_SWIGLU ? F % BN_HALF == 0 : F % BN == 0);
}

int launch_ffn_fused(const FfnFusedArgs &a, void *stream) {
  int sm_count = 0;
  int rc = check_device(&sm_count);
  if (rc != VFB_OK) return rc;
  const bool swiglu = a.activation == VFB_EPI_SWIGLU;
  FfnParams p{};
  p.M = a.M;
  p.H = a.H;
  p.F = a.F;
  FfnPlan &pl = p.plan;
  pl.rows_blocks = static_cast<int>((a.M + 2 * BM - 1) / (2 * BM));
  pl.ju = static_cast<int>(swiglu ? a.F / BN_HALF : a.F / BN);
  pl.jd = static_cast<int>((a.H + BN - 1) / BN);
  pl.group = a.group > 0 ? a.group : 8;
  pl.groups = (pl.rows_blocks + pl.group - 1) / pl.group;
  // half the GEMM's band budget for each weight: both bands, a group's
  // intermediate and its codes share L2
  pl.band_up = a.band_up > 0 ? a.band_up : band_width(pl.ju, 2 * a.H);
  pl.band_down = a.band_down > 0 ? a.band_down : band_width(pl.jd, 2 * a.F);
  const int pairs_max = sm_count / 2;
  // measured at config 2: interleaving down tiles with the next group's up
  // tiles made them wait for conversions (lead 0: 7.1 ms, 148: 5.5 ms, a
  // whole group: 4.3-4.5 ms), so by default a group's down tiles follow the
  // next group's up tiles
  pl.lead = a.lead >= 0 ? a.lead : 1 << 30;
  pl.lag = a.lag > 0 ? a.lag : 1;
  pl.total = pl.rows_blocks * (pl.ju + pl.jd);
  p.done_target = pl.ju * 2 * EPI_WARPS;
  p.x_scales = a.x_scales;
  p.s_up = a.s_up;
  p.s_down = a.s_down;
  p.bias_up = static_cast<const __nv_bfloat16 *>(a.bias_up);
  p.bias_down = static_cast<const __nv_bfloat16 *>(a.bias_down);
  p.residual = static_cast<const __nv_bfloat16 *>(a.residual);
  p.ldr = a.ldr;
  p.gate = static_cast<const __nv_bfloat16 *>(a.gate);
  p.gate_ts = a.gate_token_stride;
  p.tokens = a.tokens > 0 ? a.tokens : 1;
  p.mid = static_cast<const __nv_bfloat16 *>(a.mid);
  p.mid_codes = static_cast<uint8_t *>(a.mid_codes);
  p.amax_bits = a.amax_bits;
  p.queue = a.counters;
  p.up_done = a.counters + 1;
  p.conv_done = a.counters + 1 + pl.rows_blocks;
  p.status = device_status_ptr();

  CUtensorMap tax, tam, tbu, tbu2, tbd, tmid, tout;
  if ((rc = make_map_u8(&tax, a.x_codes, a.M, a.H, a.H, BM)) != VFB_OK) return rc;
  if ((rc = make_map_u8(&tam, a.mid_codes, a.M, a.F, a.F, BM)) != VFB_OK) return rc;
  if (swiglu) {
    if ((rc = make_map_u8(&tbu, a.w_up, a.F, a.H, a.H, BN_HALF)) != VFB_OK) return rc;
    if ((rc = make_map_u8(&tbu2, static_cast<const uint8_t *>(a.w_up) + a.F * a.H, a.F, a.H, a.H, BN_HALF)) !=
        VFB_OK)
      return rc;
  } else {
    if ((rc = make_map_u8(&tbu, a.w_up, a.F, a.H, a.H, BN_HALF)) != VFB_OK) return rc;
    tbu2 = tbu;
  }
  if ((rc = make_map_u8(&tbd, a.w_down, a.H, a.F, a.F, BN_HALF)) != VFB_OK) return rc;
  if ((rc = make_map_out(&tmid, const_cast<void *>(a.mid), a.F, a.M, 1, a.F, a.M * a.F)) != VFB_OK) return rc;
  if ((rc = make_map_out(&tout, a.out, a.H, a.M, 1, a.ldo, a.M * a.ldo)) != VFB_OK) return rc;

  // the row maxima and the counters start at zero
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err = cudaMemsetAsync(a.amax_bits, 0, a.zero_bytes, s);
  if (err != cudaSuccess) return set_error(VFB_ECUDA, "vfb_fp8_ffn: zeroing: %s", cudaGetErrorString(err));

  auto kernel = swiglu ? ffn_kernel<VFB_EPI_SWIGLU> : ffn_kernel<VFB_EPI_GELU_TANH>;
  static std::atomic<uint64_t> smem_set[2][kMaxAttrDevices];
  if ((rc = ensure_smem_optin(reinterpret_cast<const void *>(kernel), static_cast<int>(SMEM_BYTES),
                              smem_set[swiglu ? 1 : 0])) != VFB_OK)
    return rc;
  const int items = pl.total;
  const int pairs = items < pairs_max ? items : pairs_max;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, kernel, tax, tam, tbu, tbu2, tbd, tmid, tout, p);
  if (err != cudaSuccess) return set_error(VFB_ECUDA, "vfb_fp8_ffn launch: %s", cudaGetErrorString(err));
  return VFB_OK;
}

}  // namespace vfb
