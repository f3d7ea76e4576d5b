// Status/error plumbing, device checks and the device-side error word.
#include "common.cuh"

#include <mutex>
#include <string>
#include <vector>

// Written by kernels whose bounded waits expired; read by the host.
__device__ int musc_device_error = 0;

namespace musc {

static thread_local std::string g_last_error;

int fail(int status, const std::string& message) {
  g_last_error = message;
  return status;
}

int cuda_fail(cudaError_t err, const char* what) {
  std::string msg = std::string(what) + ": " + cudaGetErrorName(err) + " (" +
                    cudaGetErrorString(err) + ")";
  return fail(MUSC_B200_ERR_CUDA, msg);
}

namespace {
struct DeviceInfo {
  int major = -1, minor = -1, sms = 0, smem_optin = 0;
};
std::mutex g_info_mutex;
std::vector<DeviceInfo> g_info;

int device_info(DeviceInfo* out) {
  int dev = 0;
  MUSC_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_info_mutex);
  if ((int)g_info.size() <= dev) g_info.resize(dev + 1);
  DeviceInfo& d = g_info[dev];
  if (d.major < 0) {
    MUSC_CUDA(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev));
    MUSC_CUDA(cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev));
    MUSC_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
    MUSC_CUDA(cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  }
  *out = d;
  return MUSC_B200_OK;
}
}  // namespace

int require_sm100(void) {
  DeviceInfo d;
  MUSC_TRY(device_info(&d));
  if (d.major != 10 || d.minor != 0)
    return fail(MUSC_B200_ERR_DEVICE, "musc_b200 kernels are built for sm_100a; current device is sm_" +
                                          std::to_string(d.major) + std::to_string(d.minor));
  return MUSC_B200_OK;
}

int sm_count(void) {
  DeviceInfo d;
  if (device_info(&d) != MUSC_B200_OK) return 0;
  return d.sms;
}

int smem_optin(void) {
  DeviceInfo d;
  if (device_info(&d) != MUSC_B200_OK) return 0;
  return d.smem_optin;
}

// Looked up on every call (a host-side query) instead of cached, so a context
// that was torn down and recreated never leaves a stale address behind.
int* device_error_ptr(void) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, musc_device_error) != cudaSuccess) return nullptr;
  return static_cast<int*>(p);
}

}  // namespace musc

extern "C" int musc_b200_abi_version(void) { return 3; }

extern "C" const char* musc_b200_last_error(void) { return musc::g_last_error.c_str(); }

extern "C" int musc_b200_take_device_error(int* code) {
  if (!code) return musc::fail(MUSC_B200_ERR_INVALID, "take_device_error: null output pointer");
  MUSC_CUDA(cudaDeviceSynchronize());
  int value = 0, zero = 0;
  MUSC_CUDA(cudaMemcpyFromSymbol(&value, musc_device_error, sizeof(int)));
  MUSC_CUDA(cudaMemcpyToSymbol(musc_device_error, &zero, sizeof(int)));
  *code = value;
  return MUSC_B200_OK;
}

// ---------------------------------------------------------------------------
// Self-test of the bounded-wait path every pipelined kernel uses: one thread
// initialises an mbarrier and waits on it with a time limit.  With `arrive`
// == 0 nothing ever arrives, the wait expires after limit_ns, the kernel
// records MUSC_B200_ERR_TIMEOUT in the device error word and returns -- the
// context stays usable.  With `arrive` != 0 the thread arrives first and the
// wait completes at once.
// ---------------------------------------------------------------------------
namespace musc {
__global__ void selftest_wait_kernel(long long limit_ns, int arrive, int* err) {
  __shared__ uint64_t bar;
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(&bar));
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(a) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  if (arrive) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
  const uint64_t start = global_ns();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a)
        : "memory");
    if (done) return;
    if ((long long)(global_ns() - start) > limit_ns) {
      atomicExch(err, MUSC_B200_ERR_TIMEOUT);
      return;
    }
  }
}
}  // namespace musc

extern "C" int musc_b200_selftest_wait(long long limit_ns, int arrive, musc_b200_stream stream) {
  if (limit_ns <= 0 || limit_ns > 10000000000LL)
    return musc::fail(MUSC_B200_ERR_INVALID, "selftest_wait: limit_ns must be in (0, 1e10]");
  MUSC_TRY(musc::require_sm100());
  int* err = musc::device_error_ptr();
  if (!err) return musc::fail(MUSC_B200_ERR_CUDA, "selftest_wait: device error word unavailable");
  musc::selftest_wait_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(limit_ns, arrive, err);
  return musc::check_launch("selftest_wait_kernel");
}
