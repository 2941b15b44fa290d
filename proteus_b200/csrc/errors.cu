// Host-side error state of the C ABI (one message per host thread).
#include <stdarg.h>

#include "common.cuh"

namespace atlas {

static thread_local char g_err[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(ATLAS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return ATLAS_OK;
}

}  // namespace atlas

extern "C" const char* atlas_last_error(void) { return atlas::g_err; }
extern "C" int atlas_abi_version(void) { return 2; }
