// Library-wide C-ABI plumbing: error messages, version, device properties.
#include <stdarg.h>
#include <stdio.h>

#include "mi_common.cuh"

namespace mi {

static thread_local char g_err[512] = "";

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MI_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return MI_OK;
}

int num_sms() {
  // Per-device cache; the SM count of the current device.
  static thread_local int cached_dev = -1, cached_sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev != cached_dev) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached_dev = dev;
    cached_sms = n;
  }
  return cached_sms;
}

}  // namespace mi

extern "C" const char *mi_last_error(void) { return mi::g_err; }

extern "C" int mi_version(void) { return 100; }
