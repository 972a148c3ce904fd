// Error convention, version string and device queries of libmxq_b200.so.
#include "common.cuh"

#include <mutex>
#include <string>

namespace mxq {

static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MXQ_OK;
  return set_error(MXQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int sm_count() {
  static std::mutex mu;
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace mxq

extern "C" const char* mxq_version(void) { return "mxq_b200 0.1.0 (sm_100a)"; }

extern "C" const char* mxq_last_error(void) { return mxq::g_last_error.c_str(); }
