// Host-side error state and version of the kdn_b200 C ABI.
#include <stdarg.h>
#include <stdio.h>

#include "kdn_common.cuh"

namespace {
thread_local char g_last_error[512] = "";
}

namespace kdn {

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    return set_error(KDN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
  }
  return KDN_OK;
}

}  // namespace kdn

extern "C" {

int kdn_version(void) { return 101; }

const char* kdn_last_error(void) { return g_last_error; }

}  // extern "C"
