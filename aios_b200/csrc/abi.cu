// C-ABI infrastructure: version, per-thread error message, launch checking.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "abi_util.h"

namespace {
thread_local char g_msg[512] = {0};
thread_local int g_code = 0;
}  // namespace

namespace aiosb {
int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  g_code = code;
  return code;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(AIOSB_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return AIOSB_OK;
}
}  // namespace aiosb

extern "C" int aiosb_version(void) { return 100; }

extern "C" int aiosb_host_device_pointer(void* host, void** device) {
  AIOSB_REQUIRE(host != nullptr && device != nullptr, AIOSB_ERR_INVALID_ARG, "host_device_pointer: null pointer");
  cudaError_t e = cudaHostGetDevicePointer(device, host, 0);
  if (e != cudaSuccess)
    return aiosb::set_error(AIOSB_ERR_INVALID_ARG, "host_device_pointer: %s (is the buffer page-locked?)",
                     cudaGetErrorString(e));
  return AIOSB_OK;
}

extern "C" int aiosb_last_error(char* buf, size_t len) {
  if (buf != nullptr && len > 0) {
    strncpy(buf, g_msg, len - 1);
    buf[len - 1] = 0;
  }
  return g_code;
}
