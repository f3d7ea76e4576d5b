// Copy-engine exchange between the GPUs of one node: the multi-GPU pool
// scoring moves each bank's planes and each bank's screen tables between ranks
// with peer copies (copy engines, no SMs) ordered by flags in device memory,
// instead of NCCL collectives that must wait for the persistent GEMM to free
// SMs.  The reference is single-device; this is the transport of this
// library's query-image sharding.
//
//   musc_b200_ipc_get / _open / _close: CUDA IPC of a device buffer, by its
//       allocation's handle plus the offset of the buffer inside it (buffers from
//       a caching allocator are sub-allocations).
//   musc_b200_stream_signal / _wait: stream-ordered write / wait of a 32-bit
//       counter in device memory (the writer's prior work made visible first; the
//       wait returns once the counter is >= the value, cyclically).  A rank
//       signals into a peer's flag array through the IPC mapping and waits on its
//       own flags.
//   musc_b200_copy_async: one cudaMemcpyAsync between any two device pointers of
//       the unified address space (a peer's mapped buffer included).
#include "common.cuh"

#include <cuda.h>

#include <mutex>

namespace musc {
namespace {

using WaitFn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
using WriteFn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
using RangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

template <typename Fn>
int driver_fn(const char* name, Fn* out) {
  void* ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint(name, &ptr, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !ptr)
    return fail(MUSC_B200_ERR_CUDA, std::string(name) + " is unavailable from the driver");
  *out = reinterpret_cast<Fn>(ptr);
  return MUSC_B200_OK;
}

struct DriverFns {
  WaitFn wait = nullptr;
  WriteFn write = nullptr;
  RangeFn range = nullptr;
};

int driver_fns(DriverFns* out) {
  static std::mutex m;
  static DriverFns fns;
  static bool ok = false;
  std::lock_guard<std::mutex> lock(m);
  if (!ok) {
    MUSC_TRY(driver_fn("cuStreamWaitValue32", &fns.wait));
    MUSC_TRY(driver_fn("cuStreamWriteValue32", &fns.write));
    MUSC_TRY(driver_fn("cuMemGetAddressRange", &fns.range));
    ok = true;
  }
  *out = fns;
  return MUSC_B200_OK;
}

int driver_status(CUresult r, const char* what) {
  if (r == CUDA_SUCCESS) return MUSC_B200_OK;
  return fail(MUSC_B200_ERR_CUDA, std::string(what) + " failed: CUresult " + std::to_string((int)r));
}

}  // namespace
}  // namespace musc

using namespace musc;

extern "C" int musc_b200_ipc_get(const void* ptr, void* handle, size_t* offset) {
  if (!ptr || !handle || !offset) return fail(MUSC_B200_ERR_INVALID, "ipc_get: null pointer");
  DriverFns fns;
  MUSC_TRY(driver_fns(&fns));
  CUdeviceptr base = 0;
  size_t size = 0;
  MUSC_TRY(driver_status(fns.range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)), "cuMemGetAddressRange"));
  cudaIpcMemHandle_t h;
  MUSC_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = (size_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return MUSC_B200_OK;
}

extern "C" int musc_b200_ipc_open(const void* handle, size_t offset, void** base, void** ptr) {
  if (!handle || !base || !ptr) return fail(MUSC_B200_ERR_INVALID, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  MUSC_CUDA(cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess));
  *base = b;
  *ptr = static_cast<uint8_t*>(b) + offset;
  return MUSC_B200_OK;
}

extern "C" int musc_b200_ipc_close(void* base) {
  if (!base) return fail(MUSC_B200_ERR_INVALID, "ipc_close: null pointer");
  MUSC_CUDA(cudaIpcCloseMemHandle(base));
  return MUSC_B200_OK;
}

extern "C" int musc_b200_stream_signal(unsigned int* flag, unsigned int value, musc_b200_stream stream) {
  if (!flag) return fail(MUSC_B200_ERR_INVALID, "stream_signal: null flag");
  if (reinterpret_cast<uintptr_t>(flag) % 4 != 0) return fail(MUSC_B200_ERR_INVALID, "stream_signal: misaligned flag");
  DriverFns fns;
  MUSC_TRY(driver_fns(&fns));
  return driver_status(fns.write(reinterpret_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(flag), value,
                                 CU_STREAM_WRITE_VALUE_DEFAULT),
                       "cuStreamWriteValue32");
}

extern "C" int musc_b200_stream_wait(const unsigned int* flag, unsigned int value, musc_b200_stream stream) {
  if (!flag) return fail(MUSC_B200_ERR_INVALID, "stream_wait: null flag");
  if (reinterpret_cast<uintptr_t>(flag) % 4 != 0) return fail(MUSC_B200_ERR_INVALID, "stream_wait: misaligned flag");
  DriverFns fns;
  MUSC_TRY(driver_fns(&fns));
  return driver_status(fns.wait(reinterpret_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(flag), value,
                                CU_STREAM_WAIT_VALUE_GEQ),
                       "cuStreamWaitValue32");
}

extern "C" int musc_b200_copy_async(void* dst, const void* src, size_t bytes, musc_b200_stream stream) {
  if (bytes == 0) return MUSC_B200_OK;
  if (!dst || !src) return fail(MUSC_B200_ERR_INVALID, "copy_async: null pointer");
  MUSC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, reinterpret_cast<cudaStream_t>(stream)));
  return MUSC_B200_OK;
}
