// C-ABI entry points of the reducers: the reference's argument checks (mxq/matmul/_common.py, _systolic.py:33-36,
// _adder.py:114-120, _anchor.py:234-254), then the specialised kernel where one exists, else the generic one.
#include "common.cuh"
#include "numerics.cuh"
#include "reduce_common.cuh"

using namespace mxq;

namespace {

ArithP to_arith(const mxq_arith* a) {
  ArithP p;
  p.kind = a->kind;
  p.prod_e = a->prod_e;
  p.prod_m = a->prod_m;
  p.has_floor = a->has_floor;
  p.floor_thr = a->floor_thr;
  p.sat_limit = a->sat_limit;
  p.sat_value = a->sat_value;
  return p;
}

int check_dims(int64_t K, int64_t M, int64_t N, int64_t block, int64_t size, const char* what) {
  MXQ_REQUIRE(K >= 0 && M >= 0 && N >= 0, MXQ_ERR_VALUE, "%s: negative extent", what);
  MXQ_REQUIRE(block >= 1 && size >= 1, MXQ_ERR_VALUE, "%s: size and block size must be positive", what);
  MXQ_REQUIRE(block % size == 0, MXQ_ERR_VALUE, "size %lld must divide block size %lld", (long long)size,
              (long long)block);
  return MXQ_OK;
}

int fill_lanes(LaneTable& t, const int32_t* e, const int32_t* m, int64_t n, const char* what) {
  MXQ_REQUIRE(n <= kMaxLanes, MXQ_ERR_UNSUPPORTED, "%s: at most %d accumulator positions, got %lld", what,
              kMaxLanes, (long long)n);
  for (int64_t i = 0; i < n; i++) {
    bool ok = (e[i] == 8 && m[i] == 23) || (e[i] >= 1 && e[i] <= 8 && m[i] >= 1 && m[i] <= 22);
    MXQ_REQUIRE(ok, MXQ_ERR_VALUE, "unsupported widths e=%d, m=%d", e[i], m[i]);
    t.e[i] = (int8_t)e[i];
    t.m[i] = (int8_t)m[i];
  }
  return MXQ_OK;
}

}  // namespace

extern "C" {

int mxq_systolic(const float* PA, const float* XA, const float* PB, const float* XB, float* Y, int64_t K, int64_t M,
                 int64_t N, int64_t block, int64_t size, const mxq_arith* arith, const int32_t* sched_e,
                 const int32_t* sched_m, void* stream) {
  if (int r = check_dims(K, M, N, block, size, "systolic")) return r;
  if (int r = check_arith(arith, "systolic")) return r;
  LaneTable lanes;
  if (int r = fill_lanes(lanes, sched_e, sched_m, size, "systolic")) return r;
  if (M == 0 || N == 0) return MXQ_OK;
  ArithP A = to_arith(arith);
  cudaStream_t st = as_stream(stream);
  int r = systolic_fast(PA, XA, PB, XB, Y, K, M, N, block, (int)size, A, lanes, st);
  if (r != MXQ_ERR_UNSUPPORTED) return r;
  return systolic_generic(PA, XA, PB, XB, Y, K, M, N, block, (int)size, A, lanes, st);
}

int mxq_systolic_batched(const float* PA, const float* XA, const float* PB, const float* XB, float* Y,
                         int64_t batch, int64_t K, int64_t M, int64_t N, int64_t block, int64_t size,
                         const mxq_arith* arith, const int32_t* sched_e, const int32_t* sched_m, void* stream) {
  MXQ_REQUIRE(batch >= 0, MXQ_ERR_VALUE, "systolic: negative batch");
  if (int r = check_dims(K, M, N, block, size, "systolic")) return r;
  if (int r = check_arith(arith, "systolic")) return r;
  LaneTable lanes;
  if (int r = fill_lanes(lanes, sched_e, sched_m, size, "systolic")) return r;
  if (M == 0 || N == 0 || batch == 0) return MXQ_OK;
  ArithP A = to_arith(arith);
  cudaStream_t st = as_stream(stream);
  const int64_t nb = (K + block - 1) / block;
  const Batch bt{K * M, nb * M, K * N, nb * N, M * N};
  for (int64_t z0 = 0; z0 < batch; z0 += 65535) {           // gridDim.z holds at most 65535 problems
    const int zb = (int)(batch - z0 < 65535 ? batch - z0 : 65535);
    int r = systolic_fast(PA + z0 * bt.pa, XA + z0 * bt.xa, PB + z0 * bt.pb, XB + z0 * bt.xb, Y + z0 * bt.y, K, M, N,
                          block, (int)size, A, lanes, st, zb, bt);
    if (r == MXQ_ERR_UNSUPPORTED) {                           // no specialised kernel: one generic launch each
      for (int64_t z = z0; z < z0 + zb; z++) {
        r = systolic_generic(PA + z * bt.pa, XA + z * bt.xa, PB + z * bt.pb, XB + z * bt.xb, Y + z * bt.y, K, M, N,
                             block, (int)size, A, lanes, st);
        if (r) return r;
      }
    } else if (r) {
      return r;
    }
  }
  return MXQ_OK;
}

int mxq_adder_tree(const float* PA, const float* XA, const float* PB, const float* XB, float* Y, int64_t K, int64_t M,
                   int64_t N, int64_t block, int64_t size, const mxq_arith* arith, const int32_t* level_e,
                   const int32_t* level_m, void* stream) {
  int levels = 0;
  while (levels < 62 && ((int64_t)1 << levels) < size) levels++;
  MXQ_REQUIRE(size >= 2 && ((int64_t)1 << levels) == size, MXQ_ERR_VALUE, "size %lld must be a power of two >= 2",
              (long long)size);
  if (int r = check_dims(K, M, N, block, size, "adder_tree")) return r;
  MXQ_REQUIRE(levels <= kMaxLevels, MXQ_ERR_UNSUPPORTED, "adder_tree: at most %d levels", kMaxLevels);
  if (int r = check_arith(arith, "adder_tree")) return r;
  LaneTable lv;
  if (int r = fill_lanes(lv, level_e, level_m, levels, "adder_tree")) return r;
  if (M == 0 || N == 0) return MXQ_OK;
  ArithP A = to_arith(arith);
  cudaStream_t st = as_stream(stream);
  int r = adder_fast(PA, XA, PB, XB, Y, K, M, N, block, (int)size, levels, A, lv, st);
  if (r != MXQ_ERR_UNSUPPORTED) return r;
  return adder_generic(PA, XA, PB, XB, Y, K, M, N, block, (int)size, levels, A, lv, st);
}

int mxq_anchor_tree(const float* PA, const float* XA, const float* PB, const float* XB, float* Y, int64_t K,
                    int64_t M, int64_t N, int64_t block, int64_t size, const mxq_arith* arith, const int32_t* tree_e,
                    const int32_t* tree_m, const mxq_anchor_spec* anchor, const int32_t* tree_bits, void* stream) {
  MXQ_REQUIRE(anchor != nullptr, MXQ_ERR_VALUE, "anchor_tree: no anchor spec");
  const mxq_anchor_spec& a = *anchor;
  MXQ_REQUIRE(a.width >= 1 && size % a.width == 0 && block % size == 0, MXQ_ERR_VALUE,
              "width %d must divide size %lld, and size must divide block size %lld", a.width, (long long)size,
              (long long)block);
  if (int r = check_dims(K, M, N, block, size, "anchor_tree")) return r;
  int64_t trees = size / a.width;
  MXQ_REQUIRE(a.width <= kMaxWidth && trees <= kMaxTrees && a.nbits >= 1 && a.nbits <= kMaxBits,
              MXQ_ERR_UNSUPPORTED, "anchor_tree: width <= %d, trees <= %d and <= %d levels supported", kMaxWidth,
              kMaxTrees, kMaxBits);
  if (int r = check_arith(arith, "anchor_tree")) return r;
  AnchorTable at;
  at.width = a.width;
  at.nbits = a.nbits;
  at.drop_rne = a.drop_rne;
  at.headroom = a.headroom;
  at.has_emin = a.has_emin;
  at.emin = a.emin;
  LaneTable lanes;
  if (int r = fill_lanes(lanes, tree_e, tree_m, trees, "anchor_tree")) return r;
  for (int64_t t = 0; t < trees; t++) {
    at.tree_e[t] = lanes.e[t];
    at.tree_m[t] = lanes.m[t];
    for (int l = 0; l < a.nbits; l++) {
      int32_t b = tree_bits[t * a.nbits + l];
      MXQ_REQUIRE(b >= 1 && b <= 24 && (l == 0 || b <= tree_bits[t * a.nbits + l - 1]), MXQ_ERR_VALUE,
                  "bits needs %d non-increasing entries, each <= 24", a.nbits);
      at.bits[t * a.nbits + l] = (int8_t)b;
    }
  }
  if (M == 0 || N == 0) return MXQ_OK;
  ArithP A = to_arith(arith);
  cudaStream_t st = as_stream(stream);
  int r = anchor_fast(PA, XA, PB, XB, Y, K, M, N, block, (int)size, A, at, st);
  if (r != MXQ_ERR_UNSUPPORTED) return r;
  return anchor_generic(PA, XA, PB, XB, Y, K, M, N, block, (int)size, A, at, st);
}

int mxq_fp64_accum(const float* PA, const float* XA, const float* PB, const float* XB, float* Y, int64_t K, int64_t M,
                   int64_t N, int64_t block, void* stream) {
  if (int r = check_dims(K, M, N, block, 1, "fp64_accum")) return r;
  if (M == 0 || N == 0) return MXQ_OK;
  return fp64_accum(PA, XA, PB, XB, Y, K, M, N, block, as_stream(stream));
}

}  // extern "C"
