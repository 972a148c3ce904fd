// Plumbing shared by every translation unit of libmxq_b200.so: the C-ABI error convention (status code plus a
// thread-local message), argument checks, and launch helpers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/mxq_b200.h"

namespace mxq {

// Records `fmt` as this thread's last error message and returns `code`.
int set_error(int code, const char* fmt, ...);
// Turns a CUDA status into an mxq status (MXQ_ERR_CUDA with the runtime's message) or MXQ_OK.
int check_cuda(cudaError_t e, const char* what);
// Number of SMs of the current device (cached per device).
int sm_count();
// A number naming the calling thread's current CUDA context, unique for the life of the process (a context made
// after cudaDeviceReset gets a new one), so per-device state uploaded once can tell that it must be uploaded again;
// 0 when the driver cannot say.
unsigned long long context_id();

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Grid size for a grid-stride loop over n items: enough CTAs to fill every SM `per_sm` times, never more than the
// work needs.
inline unsigned grid_for(int64_t n, int threads, int per_sm = 8) {
  int64_t want = (n + threads - 1) / threads;
  int64_t cap = (int64_t)sm_count() * per_sm;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  return (unsigned)want;
}

}  // namespace mxq

#define MXQ_REQUIRE(cond, code, ...)                                   \
  do {                                                                 \
    if (!(cond)) return ::mxq::set_error((code), __VA_ARGS__);         \
  } while (0)

#define MXQ_LAUNCH_CHECK(what) ::mxq::check_cuda(cudaGetLastError(), (what))
