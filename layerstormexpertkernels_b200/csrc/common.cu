// Status plumbing shared by every entry point of liblsek.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "common.cuh"

namespace lsek {

namespace {
thread_local char t_last_error[512] = "no error";
}

lsek_status fail(lsek_status st, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return st;
}

lsek_status check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(LSEK_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return LSEK_OK;
}

int num_sms() {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace lsek

extern "C" const char* lsek_last_error(void) { return lsek::t_last_error; }

extern "C" const char* lsek_version(void) { return "lsek 0.1.0 sm_100a"; }
