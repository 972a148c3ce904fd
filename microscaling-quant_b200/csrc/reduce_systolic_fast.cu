// Specialised systolic kernels (filled in below as they are added). Until then every configuration takes the
// generic kernel.
#include "common.cuh"
#include "reduce_common.cuh"

namespace mxq {
int systolic_fast(const float*, const float*, const float*, const float*, float*, int64_t, int64_t, int64_t, int64_t,
                  int, const ArithP&, const LaneTable&, cudaStream_t) {
  return MXQ_ERR_UNSUPPORTED;
}
}  // namespace mxq
