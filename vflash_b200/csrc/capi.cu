// Error reporting, device checks and the device status word of the C ABI.
#include <cstdarg>
#include <cstdio>
#include <atomic>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "common.cuh"

namespace {

thread_local char g_last_error[512] = "";

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
int g_sm_count[kMaxDevices];          // 0 = not queried yet
int *g_status_ptr[kMaxDevices];       // device address of g_device_status ...
uint64_t g_status_ctx[kMaxDevices];   // ... in the context with this id

}  // namespace

// One status word per device; kernels receive its address as an argument.
static __device__ int g_device_status = 0;

namespace vfb {

int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

// Checks that the current device is a compute capability 10.0 part (B200)
// and returns its SM count.
int check_device(int *sm_count) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return set_error(VFB_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices) return set_error(VFB_EDEVICE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_sm_count[dev] == 0) {
    int major = 0, minor = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return set_error(VFB_ECUDA, "cudaDeviceGetAttribute failed on device %d", dev);
    if (major != 10 || minor != 0)
      return set_error(VFB_EDEVICE,
                       "vflash_b200 kernels are built for sm_100a only; device %d is sm_%d%d", dev,
                       major, minor);
    g_sm_count[dev] = sms;
  }
  if (sm_count) *sm_count = g_sm_count[dev];
  return VFB_OK;
}

// Unique id (never 0) of the calling thread's current CUDA context, or 0 if
// it cannot be read.  Device addresses of the library's __device__ variables
// and the kernels' shared-memory opt-ins belong to one context: a
// cudaDeviceReset ends it and the next runtime call creates a new primary
// context with a new id, so every per-device cache below is keyed by this id.
uint64_t current_context_id() {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &qres) == cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(ptr);
    ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &ptr, cudaEnableDefault, &qres) == cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(ptr);
  });
  if (get_current == nullptr || get_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
    // no context is current yet: make the current device's primary context
    // current (cudaSetDevice initialises it) and read it again
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess) return 0;
    if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  }
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return static_cast<uint64_t>(id) + 1;
}

// Device address of this device's status word, looked up once per device and
// context (again after a device reset).
int *device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  const uint64_t ctx = current_context_id();
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_status_ptr[dev] == nullptr || ctx == 0 || g_status_ctx[dev] != ctx) {
    void *ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_device_status) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<int *>(ptr);
    g_status_ctx[dev] = ctx;
  }
  return g_status_ptr[dev];
}

// Sets the dynamic shared-memory opt-in of `kernel` once per device and
// context; `done` holds, per device, the context id it was last set in.
int ensure_smem_optin(const void *kernel, int bytes, std::atomic<uint64_t> *done) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return set_error(VFB_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(err));
  const uint64_t ctx = current_context_id();
  const bool cached = dev >= 0 && dev < kMaxAttrDevices && ctx != 0;
  if (cached && done[dev].load(std::memory_order_acquire) == ctx) return VFB_OK;
  err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err != cudaSuccess) return set_error(VFB_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(err));
  if (cached) done[dev].store(ctx, std::memory_order_release);
  return VFB_OK;
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime
// (no link-time dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) ==
            cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Tensor map over an 8-bit [rows, cols] matrix (row stride ld bytes) with a
// 128-byte-swizzled box of box_rows x 128 bytes (one K stage of the GEMMs).
int make_map_u8(CUtensorMap *map, const void *base, int64_t rows, int64_t cols, int64_t ld,
                int box_rows) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return set_error(VFB_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {128, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims,
                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(VFB_ECUDA, "cuTensorMapEncodeTiled failed (%d) rows=%lld cols=%lld ld=%lld",
                     static_cast<int>(r), (long long)rows, (long long)cols, (long long)ld);
  return VFB_OK;
}

// Tensor map over the bf16 output viewed as [planes][rows][width] (row stride
// ld elements, plane stride plane_stride elements), 32 x 32 boxes with the
// 64-byte swizzle the epilogue writes its staging boxes in.
int make_map_out(CUtensorMap *map, void *base, int64_t width, int64_t rows, int64_t planes,
                 int64_t ld, int64_t plane_stride) {
  auto encode = tensor_map_encoder();
  if (encode == nullptr) return set_error(VFB_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(planes)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 2, static_cast<cuuint64_t>(plane_stride) * 2};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                      CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(VFB_ECUDA, "cuTensorMapEncodeTiled (output) failed (%d)", static_cast<int>(r));
  return VFB_OK;
}

bool aligned16(const void *ptr) { return reinterpret_cast<uintptr_t>(ptr) % 16 == 0; }

}  // namespace vfb

extern "C" const char *vfb_last_error(void) { return g_last_error; }

extern "C" const char *vfb_version(void) { return "vflash_b200 0.1.0 sm_100a"; }

extern "C" int vfb_device_status(int *status, int clear) {
  if (status == nullptr) return vfb::set_error(VFB_EINVAL, "vfb_device_status: status is NULL");
  int rc = vfb::check_device(nullptr);
  if (rc != VFB_OK) return rc;
  int *ptr = vfb::device_status_ptr();
  if (ptr == nullptr) return vfb::set_error(VFB_ECUDA, "cannot resolve the device status word");
  cudaError_t err = cudaDeviceSynchronize();
  if (err != cudaSuccess)
    return vfb::set_error(VFB_ECUDA, "cudaDeviceSynchronize: %s", cudaGetErrorString(err));
  err = cudaMemcpy(status, ptr, sizeof(int), cudaMemcpyDeviceToHost);
  if (err != cudaSuccess) return vfb::set_error(VFB_ECUDA, "status read: %s", cudaGetErrorString(err));
  if (clear) {
    err = cudaMemset(ptr, 0, sizeof(int));
    if (err != cudaSuccess) return vfb::set_error(VFB_ECUDA, "status clear: %s", cudaGetErrorString(err));
    err = cudaDeviceSynchronize();
    if (err != cudaSuccess) return vfb::set_error(VFB_ECUDA, "status clear sync: %s", cudaGetErrorString(err));
  }
  return VFB_OK;
}

// ---------------------------------------------------------------------------
// Bounded-wait self-test: one thread waits on an mbarrier that nothing ever
// arrives at.  The wait gives up after timeout_ns, records VFB_ETIMEOUT in the
// device status word and the kernel returns normally (no trap, no fault), so
// the context stays usable; this is the path every pipeline wait in the GEMMs
// takes when a peer role stops making progress.
// ---------------------------------------------------------------------------
namespace vfb {
namespace {
__global__ void wait_selftest_kernel(uint64_t timeout_ns, int *status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_for(&bar, 0, &abort_flag, status, timeout_ns);
}
}  // namespace
}  // namespace vfb

extern "C" int vfb_wait_selftest(int64_t timeout_ns, void *stream) {
  using namespace vfb;
  if (timeout_ns < 1000000 || timeout_ns > 10000000000ll)
    return set_error(VFB_EINVAL, "vfb_wait_selftest: timeout must be 1 ms .. 10 s");
  int rc = check_device(nullptr);
  if (rc != VFB_OK) return rc;
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint64_t>(timeout_ns),
                                                                       device_status_ptr());
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_error(VFB_ECUDA, "vfb_wait_selftest launch: %s", cudaGetErrorString(err));
  return VFB_OK;
}
