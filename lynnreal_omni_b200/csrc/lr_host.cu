// Host-side plumbing of the C ABI: error messages, launch status, SM count and
// the device status word.
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
