// Error plumbing and version for the C ABI.
#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <utility>

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

static std::mutex g_setup_mu;

int func_smem_attr(const void* func, size_t bytes, int carveout, const char* what) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return set_error(AEOQ_ERR_CUDA, "%s: no current CUDA device", what);
  }
  static std::map<std::pair<int, const void*>, size_t> done;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  size_t& have = done[{dev, func}];
  if (have >= bytes && have != 0) return AEOQ_OK;
  cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess && carveout >= 0)
    e = cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout, carveout);
  if (e != cudaSuccess) {
    cudaGetLastError();   // do not leave the error for the next launch check
    return set_error(AEOQ_ERR_CUDA, "%s: shared memory attribute (%zu B): %s", what, bytes, cudaGetErrorString(e));
  }
  have = bytes > 0 ? bytes : 1;
  return AEOQ_OK;
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 148;
  }
  static std::map<int, int> sms;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  auto it = sms.find(dev);
  if (it != sms.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = 148;
  }
  sms[dev] = n;
  return n;
}

}  // namespace aeoq

extern "C" int aeoq_version(void) { return 100; }

extern "C" const char* aeoq_last_error(void) { return aeoq::g_err; }
