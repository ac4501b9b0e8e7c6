// Host-side plumbing of the C ABI: error messages, launch status, SM count and
// the device status word.
#include <cuda.h>
#include <string.h>

#include "lr_host.h"

namespace lr {

namespace {
thread_local char g_message[512] = "";
}

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_message, sizeof(g_message), fmt, ap);
  va_end(ap);
  return status;
}

int launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return LR_OK;
  return set_error(LR_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int sm_count() {
  static int counts[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

int read_status_elementwise(unsigned int* bits, int clear);
int read_status_gemm(unsigned int* bits, int clear);
int read_status_flash(unsigned int* bits, int clear);
int read_status_attention(unsigned int* bits, int clear);

}  // namespace lr

extern "C" int lr_version(void) { return 100; }

extern "C" const char* lr_last_error(void) { return lr::g_message; }

extern "C" int lr_device_status(unsigned int* bits, int clear) {
  LR_REQUIRE(bits != nullptr, "device_status: null output");
  *bits = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return lr::launch_status("device_status: synchronize");
  int st = lr::read_status_elementwise(bits, clear);
  if (st) return st;
  st = lr::read_status_gemm(bits, clear);
  if (st) return st;
  st = lr::read_status_flash(bits, clear);
  if (st) return st;
  return lr::read_status_attention(bits, clear);
}

// ------------------------------------------------------------- CUDA IPC
// Peer mapping of device buffers between the processes of one node (one
// process per GPU): a buffer is exported as the IPC handle of the allocation
// that holds it plus its offset in that allocation, and imported by mapping
// the allocation (peer access over NVLink enabled lazily).
namespace {
typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(p);
  }
  return fn;
}
}  // namespace

static_assert(sizeof(cudaIpcMemHandle_t) == LR_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int lr_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  LR_REQUIRE(ptr != nullptr && handle != nullptr && offset != nullptr, "ipc_export: null argument");
  auto range = address_range_fn();
  if (range == nullptr) return lr::set_error(LR_ERR_CUDA, "ipc_export: cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return lr::set_error(LR_ERR_INVALID_ARGUMENT, "ipc_export: %p is not device memory of this context", ptr);
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess)
    return lr::launch_status("ipc_export: cudaIpcGetMemHandle (the allocation must come from cudaMalloc)");
  memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return LR_OK;
}

extern "C" int lr_ipc_import(const void* handle, int64_t offset, void** ptr) {
  LR_REQUIRE(handle != nullptr && ptr != nullptr && offset >= 0, "ipc_import: invalid argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return lr::launch_status("ipc_import: cudaIpcOpenMemHandle");
  *ptr = static_cast<char*>(base) + offset;
  return LR_OK;
}

extern "C" int lr_ipc_release(void* ptr, int64_t offset) {
  LR_REQUIRE(ptr != nullptr && offset >= 0, "ipc_release: invalid argument");
  if (cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset) != cudaSuccess)
    return lr::launch_status("ipc_release: cudaIpcCloseMemHandle");
  return LR_OK;
}
