// Error convention, version string and device queries of libmxq_b200.so.
#include "common.cuh"
#include "tma.cuh"

#include <cudaTypedefs.h>

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

unsigned long long context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static std::once_flag once;
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode_tmap_f32(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                    const uint32_t* box) {
  auto fn = encode_fn();
  if (!fn) return set_error(MXQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; i++) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i > 0) s[i - 1] = strides[i - 1];
  }
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(MXQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MXQ_OK;
}

unsigned* wait_status_word() {
  static std::mutex mu;
  static unsigned* word = nullptr;
  static int alloc_dev = -1;
  static unsigned long long alloc_ctx = 0;
  std::lock_guard<std::mutex> lock(mu);
  if (word != nullptr && alloc_ctx != 0) {
    // a cudaDeviceReset of the device whose context allocated the word freed it with that context: make a new one
    int dev = -1;
    if (cudaGetDevice(&dev) == cudaSuccess && dev == alloc_dev && context_id() != alloc_ctx) word = nullptr;
  }
  if (word == nullptr) {
    void* p = nullptr;
    if (check_cuda(cudaHostAlloc(&p, 64, cudaHostAllocMapped | cudaHostAllocPortable), "wait-status word"))
      return nullptr;
    void* d = nullptr;
    if (check_cuda(cudaHostGetDevicePointer(&d, p, 0), "wait-status word: device address") || d != p) {
      // unified addressing gives mapped host memory one address on the host and every device; the kernels are
      // handed the host address, so anything else is refused
      if (d != p) set_error(MXQ_ERR_CUDA, "wait-status word: mapped host memory has a different device address");
      cudaFreeHost(p);
      return nullptr;
    }
    *static_cast<volatile unsigned*>(p) = 0u;
    word = static_cast<unsigned*>(p);
    if (cudaGetDevice(&alloc_dev) != cudaSuccess) alloc_dev = -1;
    alloc_ctx = context_id();
  }
  return word;
}

}  // namespace mxq

extern "C" int mxq_wait_status_word(uint32_t** out) {
  if (!out) return mxq::set_error(MXQ_ERR_VALUE, "wait_status_word: null output");
  unsigned* w = mxq::wait_status_word();
  if (!w) return MXQ_ERR_CUDA;
  *out = reinterpret_cast<uint32_t*>(w);
  return MXQ_OK;
}

extern "C" const char* mxq_version(void) { return "mxq_b200 0.1.0 (sm_100a)"; }

extern "C" const char* mxq_last_error(void) { return mxq::g_last_error.c_str(); }
