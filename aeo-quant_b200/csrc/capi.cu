// Error plumbing and version for the C ABI.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace aeoq {

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(AEOQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return AEOQ_OK;
}

}  // namespace aeoq

extern "C" int aeoq_version(void) { return 100; }

extern "C" const char* aeoq_last_error(void) { return aeoq::g_err; }
