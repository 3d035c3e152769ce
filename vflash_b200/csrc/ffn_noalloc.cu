// vfb_fp8_ffn_noalloc: the fused FP8 FFN for callers that cannot allocate.
//
// vfb_fp8_ffn needs a workspace for its intermediates (the quantised input,
// the bf16 intermediate and its quantised copy), which the caller allocates.
// Some callers cannot: a host that embeds this library inside a runtime
// which has already reserved the device memory for its own pool, or code
// that runs where cudaMalloc's implicit device synchronisation is not
// allowed (a latency-critical loop, a host callback).  This entry point
// takes the same inputs and outputs and keeps the intermediates in one
// fixed array of device memory that belongs to the library.
//
// The array is a file-scope __device__ variable of kScratchBytes: every GPU
// that loads this library holds it until the process exits, and calls whose
// intermediates need more are rejected.  Host code reaches it only through
// cudaGetSymbolAddress (the host-side name is a stand-in, not a device
// address), looked up once per device, with that device current, on the
// first call made on that device -- and again on the first call after a
// cudaDeviceReset, whose new context places the array at a new address (the
// cached address is kept with the id of the context it belongs to).
//
// All calls on a device share the array.  Two calls whose kernels overlap on
// the GPU (different streams, or different host threads without ordering)
// overwrite each other's intermediates: callers order them, e.g. on one
// stream.  Nothing in the array needs to start at zero: every byte a call
// reads was written earlier in the same call (the quantiser also writes the
// padding rows), so the contents left by the previous call do no harm.
#include <cstdint>
#include <mutex>

#include "common.cuh"

namespace vfb {
namespace {

constexpr int64_t kScratchBytes = 64ll << 20;  // 64 MiB per device

static __device__ __align__(256) uint8_t g_ffn_scratch[kScratchBytes];

std::mutex g_scratch_mutex;
void *g_scratch_ptr[kMaxAttrDevices] = {};
uint64_t g_scratch_ctx[kMaxAttrDevices] = {};  // id of the context g_scratch_ptr[dev] belongs to

// Device address of the array on the current device, looked up once per
// device and context.
int scratch_address(void **out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return set_error(VFB_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxAttrDevices)
    return set_error(VFB_EINVAL, "vfb_fp8_ffn_noalloc: device %d is beyond the supported %d", dev,
                     kMaxAttrDevices);
  const uint64_t ctx = current_context_id();
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr || ctx == 0 || g_scratch_ctx[dev] != ctx) {
    void *ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_ffn_scratch);
    if (err != cudaSuccess || ptr == nullptr)
      return set_error(VFB_ECUDA, "vfb_fp8_ffn_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(err));
    g_scratch_ptr[dev] = ptr;
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_ptr[dev];
  return VFB_OK;
}

}  // namespace
}  // namespace vfb

extern "C" int vfb_fp8_ffn_noalloc(const void *x, int64_t M, int64_t H, int64_t ldx, const void *w_up,
                                   const float *s_up, int64_t n_up, const void *w_down, const float *s_down,
                                   int32_t activation, const void *bias_up, const void *bias_down,
                                   const void *residual, int64_t ldr, const void *gate, int64_t gate_token_stride,
                                   int64_t tokens, void *out, int64_t ldo, void *stream) {
  using namespace vfb;
  if (activation != VFB_EPI_GELU_TANH && activation != VFB_EPI_SWIGLU)
    return set_error(VFB_EINVAL, "vfb_fp8_ffn_noalloc: activation must be VFB_EPI_GELU_TANH or VFB_EPI_SWIGLU");
  const int64_t width = activation == VFB_EPI_SWIGLU ? n_up / 2 : n_up;
  const int64_t need = vfb_fp8_ffn_workspace_bytes(M, H, width);
  if (need < 0 || (activation == VFB_EPI_SWIGLU && n_up % 2))
    return set_error(VFB_EINVAL, "vfb_fp8_ffn_noalloc: need 16 <= H <= 32768 and 32 <= F <= 32768, both "
                                 "multiples of 32 (F = n_up, or n_up / 2 for SWIGLU), M >= 0 (M=%lld H=%lld "
                                 "n_up=%lld)", (long long)M, (long long)H, (long long)n_up);
  if (need > kScratchBytes)
    return set_error(VFB_EINVAL,
                     "vfb_fp8_ffn_noalloc: these shapes need %lld bytes of intermediates, more than the "
                     "library's fixed %lld-byte scratch; use vfb_fp8_ffn with a workspace, or fewer rows",
                     (long long)need, (long long)kScratchBytes);
  void *scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != VFB_OK) return rc;
  // shape and argument checks are vfb_fp8_ffn's own
  return vfb_fp8_ffn(x, M, H, ldx, w_up, s_up, n_up, w_down, s_down, activation, bias_up, bias_down, residual, ldr,
                     gate, gate_token_stride, tokens, out, ldo, scratch, kScratchBytes, stream);
}
