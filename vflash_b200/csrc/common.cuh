// Device-side building blocks shared by the sm_100a kernels: mbarriers with
// bounded waits, TMA tile loads, tcgen05 (TMEM allocation, MMA issue, commit,
// TMEM loads) and strict BF16 rounding helpers.  Every wait in this file gives
// up after VFB_WAIT_TIMEOUT_NS of wall time, records VFB_ETIMEOUT in the
// device status word and returns false, so a broken pipeline ends the kernel
// instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "vflash_b200.h"

#define VFB_WAIT_TIMEOUT_NS (4000000000ull)  // 4 s: far above any legitimate wait

namespace vfb {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier -------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// try_wait with acquire semantics at cluster scope: for a barrier whose
// arrivals come from the peer CTA of the pair along with data it wrote into
// this CTA's shared memory.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Record the first error code of this device (kept until the host clears it).
__device__ __forceinline__ void record_status(int *status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

// Wait until the phase with the given parity has completed.  Returns false if
// the wait expired or another role of this CTA already gave up (`abort_flag`).
__device__ __forceinline__ bool mbar_wait_for(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                              int *status, uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 255u) == 0) {
      if (*abort_flag) return false;
      if (global_timer_ns() - start > timeout_ns) {
        *abort_flag = 1;
        record_status(status, VFB_ETIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                          int *status) {
  return mbar_wait_for(bar, parity, abort_flag, status, VFB_WAIT_TIMEOUT_NS);
}

// mbar_wait with cluster-scope acquire (see mbar_try_wait_cluster).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                                  int *status) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((spin & 255u) == 0) {
      if (*abort_flag) return false;
      if (global_timer_ns() - start > VFB_WAIT_TIMEOUT_NS) {
        *abort_flag = 1;
        record_status(status, VFB_ETIMEOUT);
        return false;
      }
    }
  }
}

// ---- global-memory flags between CTAs ----------------------------------------
__device__ __forceinline__ int ld_acquire_gpu(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(int *p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Orders this thread's generic-proxy accesses of global memory with async-proxy
// (TMA) accesses: data written by plain stores and then read by a TMA load
// elsewhere, or written by a TMA store and then read by plain loads.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Drops one 128-byte L2 line without writing it back (its contents become
// undefined): for scratch data that is dead once read.
__device__ __forceinline__ void discard_l2_line(const void *p) {
  asm volatile("discard.global.L2 [%0], 128;" ::"l"(p) : "memory");
}

// 32-bit store into the shared memory of a CTA of this cluster (shared::cluster address).
__device__ __forceinline__ void st_shared_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

// ---- programmatic dependent launch ----------------------------------------
// The GEMMs are launched with programmatic stream serialisation: one may be
// scheduled while the kernel before it in the stream (the quantiser that wrote
// its A operand and row scales) is still running, set up its barriers and
// TMEM, and then wait here.  The wait returns once every prerequisite grid has
// completed and its memory operations are visible to this grid; for a kernel
// launched without the attribute it returns at once.  Every thread waits
// before it touches global memory that an earlier kernel may write or read.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Lets the next kernel in the stream be scheduled once every block of this
// grid has issued it (or exited).  Only a kernel launched with programmatic
// serialisation is affected, and it still waits in grid_dependency_wait() for
// this grid to complete, so a block may issue it before writing anything.
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- TMA ------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of one box into shared memory; completion is signalled on
// `bar` as transaction bytes.  x is the innermost (contiguous) coordinate.
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// L2 eviction policies for TMA traffic: weights are re-read by every tile row
// of a GEMM and should outlive the streamed activations and outputs.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// tma_load_2d with an L2 cache policy.
__device__ __forceinline__ void tma_load_2d_hint(void *smem_dst, const CUtensorMap *map, uint64_t *bar,
                                                 int32_t x, int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// 3-D tiled store with an L2 cache policy (see tma_store_3d).
__device__ __forceinline__ void tma_store_3d_hint(const CUtensorMap *map, const void *smem_src,
                                                  int32_t x, int32_t y, int32_t z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3, %4}], [%1], %5;" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}

// 3-D tiled store of one shared-memory box to global memory (bulk-group
// completion).  Coordinates outside the tensor are not written.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *smem_src, int32_t x,
                                             int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N bulk groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until every bulk group of this thread has completed.
__device__ __forceinline__ void bulk_wait_group_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Make this thread's shared-memory writes visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05 ----------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T for 8-bit float operands (kind::f8f6f4).
__device__ __forceinline__ void mma_f8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle (rows of 128 bytes, 8-row groups 1024 bytes apart), as TMA
// writes it with CU_TENSOR_MAP_SWIZZLE_128B.  The tile base must be 1024-byte
// aligned; advancing along K inside the 128-byte row adds bytes/16 to the
// start-address field.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t desc = 0;
  desc |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);  // start address  [0,14)
  desc |= static_cast<uint64_t>(1) << 16;                       // leading offset [16,30) (unused)
  desc |= static_cast<uint64_t>(1024 >> 4) << 32;               // stride offset  [32,46)
  desc |= static_cast<uint64_t>(1) << 46;                       // descriptor version (sm_100)
  desc |= static_cast<uint64_t>(2) << 61;                       // layout: 128-byte swizzle
  return desc;
}

// Instruction descriptor: e4m3 x e4m3 -> f32, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int m, int n) {
  return (1u << 4)                                  // D format f32
         | (0u << 7) | (0u << 10)                   // A, B format e4m3
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// Instruction descriptor (kind::f16): bf16 x bf16 -> f32, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
  return (1u << 4)                                  // D format f32
         | (1u << 7) | (1u << 10)                   // A, B format bf16
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// 32 lanes x 32 consecutive 32-bit TMEM columns; thread i gets lane base+i.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  __syncwarp();  // .sync.aligned: the whole warp must issue it together
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Split-phase TMEM loads: issue several loads, wait once (tmem_ld_wait), then
// pass each destination through tmem_ld_fence so that no use of its registers
// is scheduled before the wait (the empty asm statements "rewrite" them and
// stay ordered after the wait like every volatile asm).
__device__ __forceinline__ void tmem_ld_32x32b_x32_issue(uint32_t taddr, uint32_t (&r)[32]) {
  __syncwarp();
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld_fence(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

// ---- block-scaled (NVFP4) helpers --------------------------------------------
// Contiguous global -> shared copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned) counted as transaction bytes on `bar`.
__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gmem_src, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gmem_src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory descriptor of a 512-byte scale-factor block: 32 rows of 16
// bytes, no swizzle (8-row core matrices 128 bytes apart).
__device__ __forceinline__ uint64_t sf_block_desc(uint32_t smem_addr) {
  uint64_t desc = 0;
  desc |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  desc |= static_cast<uint64_t>(1) << 16;          // leading offset (one 16-byte column)
  desc |= static_cast<uint64_t>(128 >> 4) << 32;   // stride offset between 8-row groups
  desc |= static_cast<uint64_t>(1) << 46;          // descriptor version (sm_100)
  return desc;                                     // layout 0: no swizzle
}

// Copy one 32 x 128-bit shared block into TMEM lanes 0-31 and replicate it to
// the other three 32-lane sub-partitions (4 columns of 32 bits).
__device__ __forceinline__ void tmem_cp_32x128b_warpx4(uint32_t taddr, uint64_t src_desc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src_desc)
               : "memory");
}

// D[tmem] (+)= (A * SFA) (B * SFB)^T for e2m1 operands with one ue4m3 scale
// per 16 K-elements (kind::mxf4nvf4, block16), scales read from TMEM.
__device__ __forceinline__ void mma_mxf4nvf4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::
          "r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Instruction descriptor: e2m1 x e2m1 with ue4m3 block scales, f32 accumulate,
// both operands K-major, K = 64 per instruction.
__host__ __device__ constexpr uint32_t idesc_nvf4_f32(int m, int n) {
  return (1u << 7) | (1u << 10)                     // A, B format e2m1
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (0u << 23)                               // scale format ue4m3
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// Approximate reciprocal with denormals flushed (PTX rcp.approx.ftz.f32).
__device__ __forceinline__ float rcp_approx_ftz(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Eight floats -> eight e2m1 codes (round to nearest even, saturating to
// +-6), element 2i in the low nibble of byte i.
__device__ __forceinline__ uint32_t pack_e2m1x8(const float (&v)[8]) {
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(r)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return r;
}

// ---- warp-wide issue ----------------------------------------------------------
// The tcgen05 issuer runs as a whole converged warp and one elected lane
// issues: the operands (descriptors, TMEM addresses, loop state) are then
// warp-uniform, which a single-lane branch (`if (lane == 0)`) hides from the
// compiler.  Measured on the block-scaled GEMM: 2.7 -> 4.7 PFLOP/s.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// Every lane waits (bounded); the warp proceeds only if all lanes saw the phase.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                          int *status) {
  const bool ok = mbar_wait(bar, parity, abort_flag, status);
  return __all_sync(0xffffffffu, ok);
}

// ---- CTA pairs (2-CTA clusters) ---------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

// Arrive on an mbarrier given by its shared::cluster address (own or peer CTA).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// 2-D tiled load into this CTA's shared memory whose completion is counted on
// an mbarrier of the pair's leader CTA (`bar_cluster_addr`, a shared::cluster
// address).  No multicast: each CTA loads its own tile.
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const CUtensorMap *map,
                                                 uint32_t bar_cluster_addr, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}

// tma_load_2d_pair with an L2 cache policy.
__device__ __forceinline__ void tma_load_2d_pair_hint(void *smem_dst, const CUtensorMap *map,
                                                      uint32_t bar_cluster_addr, int32_t x, int32_t y,
                                                      uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Arrive once on the mbarrier at `bar_cluster_addr` (this CTA's or the peer's)
// when every pair-wide tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cluster_addr)
               : "memory");
}

// Pair-wide D (+)= A * B^T, 8-bit float operands: A rows split across the two
// CTAs (M/2 each), B rows (the N dimension) split likewise; each CTA's TMEM
// receives its M/2 rows of D.
__device__ __forceinline__ void mma_f8f6f4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Pair-wide D (+)= A * B^T with 16-bit operands (kind::f16; both operands
// bf16, as the instruction descriptor says): K = 16 elements = 32 bytes per
// instruction, the same byte step as the 8-bit form.
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Pair version of tmem_cp_32x128b_warpx4: issued by the leader, each CTA of
// the pair copies the block at this shared offset into its own TMEM.
__device__ __forceinline__ void tmem_cp_32x128b_warpx4_pair(uint32_t taddr, uint64_t src_desc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src_desc)
               : "memory");
}

// Pair-wide block-scaled e2m1 MMA (M = 256 over the two CTAs).
__device__ __forceinline__ void mma_mxf4nvf4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                  uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::
          "r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// ---- numerics -------------------------------------------------------------
// Round to BF16 (nearest-even) and widen back: one eager BF16 rounding boundary.
__device__ __forceinline__ float bf16r(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Rounds 32 floats to bf16 values in place, two per cvt.rn.bf16x2.f32: the same
// per-element rounding as bf16r with half the conversion instructions (the
// conversions share the XU pipe, which the GEMM epilogues otherwise saturate).
__device__ __forceinline__ void bf16r_x32(float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float2 f = __bfloat1622float2(__floats2bfloat162_rn(v[j], v[j + 1]));
    v[j] = f.x;
    v[j + 1] = f.y;
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

// Two floats -> two e4m3 bytes (round to nearest even, saturating to +-448);
// `lo` lands in the low byte (lower address).
__device__ __forceinline__ uint16_t pack_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

}  // namespace vfb

// Devices whose per-device kernel attributes are cached (others set them per launch).
constexpr int kMaxAttrDevices = 64;

// Host-side helpers implemented in capi.cu.
#include <cudaTypedefs.h>

#include <atomic>
namespace vfb {
int set_error(int code, const char *fmt, ...);
int check_device(int *sm_count);
uint64_t current_context_id();
int *device_status_ptr();
int ensure_smem_optin(const void *kernel, int bytes, std::atomic<uint64_t> *done);
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();
// Tensor map over an 8-bit [rows, cols] matrix (row stride ld bytes), boxes of
// box_rows x 128 bytes with the 128-byte swizzle.
int make_map_u8(CUtensorMap *map, const void *base, int64_t rows, int64_t cols, int64_t ld, int box_rows);
// Tensor map over a bf16 output [planes][rows][width] (strides in elements),
// 32 x 32 boxes with the 64-byte swizzle of the epilogue's staging boxes.
int make_map_out(CUtensorMap *map, void *base, int64_t width, int64_t rows, int64_t planes, int64_t ld,
                 int64_t plane_stride);
bool aligned16(const void *ptr);
}  // namespace vfb
