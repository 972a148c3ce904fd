// Elementwise entry points: the public per-element functions of the reference (rounding, float_em, the
// microxcaling element step, scale rules, arith, the Arithmetic stages), one fused kernel each. Each kernel is a
// grid-stride loop over n values; every value is one call of the numerics.cuh function that restates the
// reference function named in include/mxq_b200.h.
#include "common.cuh"
#include "numerics.cuh"

using namespace mxq;

namespace {

constexpr int kThreads = 256;

template <typename F>
__global__ void __launch_bounds__(kThreads) k_map(int64_t n, F f) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) f(i);
}

template <typename F>
int launch_map(int64_t n, void* stream, const char* what, F f) {
  MXQ_REQUIRE(n >= 0, MXQ_ERR_VALUE, "%s: negative size", what);
  if (n == 0) return MXQ_OK;
  k_map<<<grid_for(n, kThreads), kThreads, 0, as_stream(stream)>>>(n, f);
  return MXQ_LAUNCH_CHECK(what);
}

int check_mode(int mode, const char* what) {
  MXQ_REQUIRE(mode >= 0 && mode <= 2, MXQ_ERR_VALUE, "%s: unknown rounding mode %d", what, mode);
  return MXQ_OK;
}

int check_em(int e, int m, int grid, const char* what) {
  MXQ_REQUIRE(grid >= 0 && grid <= 2, MXQ_ERR_VALUE, "%s: unknown grid %d", what, grid);
  if (e == 8 && m == 23) return MXQ_OK;
  MXQ_REQUIRE(e >= 1 && e <= 8 && m >= 1 && m <= 22, MXQ_ERR_VALUE, "unsupported widths e=%d, m=%d", e, m);
  MXQ_REQUIRE(grid != GRID_OCP || ocp_max_norm(e, m) > 0.0f, MXQ_ERR_VALUE,
              "grid='ocp' is defined only for the OCP element formats, not (e=%d, m=%d)", e, m);
  return MXQ_OK;
}

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

}  // namespace

namespace mxq {
int check_arith(const mxq_arith* a, const char* what) {
  MXQ_REQUIRE(a != nullptr, MXQ_ERR_VALUE, "%s: no Arithmetic", what);
  MXQ_REQUIRE(a->kind == MXQ_ARITH_MXQUANT || a->kind == MXQ_ARITH_MXGEMMINI, MXQ_ERR_VALUE,
              "%s: unknown Arithmetic kind %d", what, a->kind);
  if (a->kind == MXQ_ARITH_MXQUANT) {
    MXQ_REQUIRE((a->prod_e == 8 && a->prod_m == 23) || (a->prod_e >= 1 && a->prod_e <= 8 && a->prod_m >= 1 &&
                                                         a->prod_m <= 22),
                MXQ_ERR_VALUE, "unsupported widths e=%d, m=%d", a->prod_e, a->prod_m);
  } else {
    MXQ_REQUIRE(a->prod_m >= 0, MXQ_ERR_VALUE, "%s: negative product mantissa width", what);
  }
  return MXQ_OK;
}
}  // namespace mxq

extern "C" {

int mxq_round_pattern(const int64_t* bits, const int64_t* drop, int64_t drop_s, const int64_t* mask, int64_t mask_s,
                      const int64_t* half, int64_t half_s, int64_t* out, int64_t n, int32_t mode, void* stream) {
  if (int r = check_mode(mode, "rounding bits")) return r;
  return launch_map(n, stream, "rounding bits", [=] __device__(int64_t i) {
    out[i] = round_pattern_i64(bits[i], drop ? drop[i] : drop_s, mask ? mask[i] : mask_s, half ? half[i] : half_s,
                               mode);
  });
}

int mxq_round_bits(const int64_t* bits, const int64_t* keep, int32_t keep_scalar, int64_t* out, int64_t n,
                   int32_t mode, void* stream) {
  if (int r = check_mode(mode, "round_bits")) return r;
  MXQ_REQUIRE(keep != nullptr || (keep_scalar >= 0 && keep_scalar <= 22), MXQ_ERR_VALUE,
              "keep must be in [0, 22] (23 = identity is not a rounding)");
  return launch_map(n, stream, "round_bits", [=] __device__(int64_t i) {
    out[i] = round_bits_i64(bits[i], keep ? (int)keep[i] : keep_scalar, mode);
  });
}

int mxq_round_int_f32(const float* k, float* out, int64_t n, int32_t mode, void* stream) {
  if (int r = check_mode(mode, "round_int")) return r;
  return launch_map(n, stream, "round_int", [=] __device__(int64_t i) { out[i] = round_int_f(k[i], mode); });
}

int mxq_round_int_f64(const double* k, double* out, int64_t n, int32_t mode, void* stream) {
  if (int r = check_mode(mode, "round_int")) return r;
  return launch_map(n, stream, "round_int", [=] __device__(int64_t i) { out[i] = round_int_d(k[i], mode); });
}

int mxq_bf16(const float* x, float* out, int64_t n, void* stream) {
  return launch_map(n, stream, "bf16", [=] __device__(int64_t i) { out[i] = bf16_rne(x[i]); });
}

int mxq_float_em_f32(const float* z, float* out, int64_t n, int32_t e, int32_t m, int32_t mode, int32_t grid,
                     void* stream) {
  if (int r = check_mode(mode, "float_em")) return r;
  if (int r = check_em(e, m, grid, "float_em")) return r;
  return launch_map(n, stream, "float_em", [=] __device__(int64_t i) { out[i] = q_float_em(z[i], e, m, mode, grid); });
}

int mxq_float_em_f64(const double* z, float* out, int64_t n, int32_t e, int32_t m, int32_t mode, int32_t grid,
                     void* stream) {
  if (int r = check_mode(mode, "float_em")) return r;
  if (int r = check_em(e, m, grid, "float_em")) return r;
  return launch_map(n, stream, "float_em",
                    [=] __device__(int64_t i) { out[i] = q_float_em_d(z[i], e, m, mode, grid); });
}

int mxq_microsoft(const float* A, float* out, int64_t n, int32_t bits, int32_t exp_bits, float max_norm,
                  int32_t round, int32_t saturate_normals, void* stream) {
  MXQ_REQUIRE(round >= 0 && round <= 2, MXQ_ERR_VALUE, "Unrecognized round method %d", round);
  MXQ_REQUIRE(bits >= 2 && bits <= 24 && exp_bits >= 0 && exp_bits <= 8, MXQ_ERR_VALUE,
              "microsoft: unsupported format bits=%d exp_bits=%d", bits, exp_bits);
  bool sat = saturate_normals != 0;
  return launch_map(n, stream, "microsoft", [=] __device__(int64_t i) {
    out[i] = q_microsoft(A[i], bits, exp_bits, max_norm, round, sat);
  });
}

int mxq_scale_mxquant(const float* amax, float* X, int64_t n, float floor, void* stream) {
  return launch_map(n, stream, "scale_mxquant", [=] __device__(int64_t i) { X[i] = scale_mxquant(amax[i], floor); });
}

int mxq_scale_ocp(const float* amax, float* X, int64_t n, int32_t emax, float scale_emax, void* stream) {
  return launch_map(n, stream, "scale_ocp",
                    [=] __device__(int64_t i) { X[i] = scale_ocp(amax[i], emax, scale_emax); });
}

int mxq_scale_ocp_no_clip(const float* amax, float* X, int64_t n, int32_t e, int32_t m, int32_t round,
                          float scale_emax, void* stream) {
  MXQ_REQUIRE(ocp_max_norm(e, m) > 0.0f, MXQ_ERR_VALUE, "ocp_no_clip: (e=%d, m=%d) is not an OCP format", e, m);
  MXQ_REQUIRE(round >= 0 && round <= 2, MXQ_ERR_VALUE, "Unrecognized round method %d", round);
  return launch_map(n, stream, "scale_ocp_no_clip",
                    [=] __device__(int64_t i) { X[i] = scale_ocp_no_clip(amax[i], e, m, round, scale_emax); });
}

int mxq_exact_add(const float* a, const float* b, float* out, int64_t n, int32_t e, int32_t m, int32_t mode,
                  int32_t grid, void* stream) {
  if (int r = check_mode(mode, "exact_add")) return r;
  if (int r = check_em(e, m, grid, "exact_add")) return r;
  return launch_map(n, stream, "exact_add",
                    [=] __device__(int64_t i) { out[i] = exact_add_any(a[i], b[i], e, m, mode, grid); });
}

int mxq_truncate_significand(const float* x, float* out, int64_t n, int32_t m, void* stream) {
  MXQ_REQUIRE(m >= 0, MXQ_ERR_VALUE, "truncate_significand: negative width %d", m);
  return launch_map(n, stream, "truncate_significand",
                    [=] __device__(int64_t i) { out[i] = truncate_significand(x[i], m); });
}

int mxq_flush_product(const float* x, float* out, int64_t n, float thr, void* stream) {
  return launch_map(n, stream, "flush_product", [=] __device__(int64_t i) { out[i] = flush_below(x[i], thr); });
}

int mxq_saturate(const float* x, float* out, int64_t n, float limit, float value, void* stream) {
  return launch_map(n, stream, "saturate", [=] __device__(int64_t i) { out[i] = saturate(x[i], limit, value); });
}

int mxq_arith_product(const float* a, const float* b, float* out, int64_t n, const mxq_arith* arith, void* stream) {
  if (int r = check_arith(arith, "product")) return r;
  ArithP A = to_arith(arith);
  return launch_map(n, stream, "product", [=] __device__(int64_t i) { out[i] = ar_product(A, a[i], b[i]); });
}

int mxq_arith_acc_add(const float* S, const float* p, float* out, int64_t n, const mxq_arith* arith, int32_t e,
                      int32_t m, void* stream) {
  if (int r = check_arith(arith, "acc_add")) return r;
  if (int r = check_em(e, m, GRID_IEEE, "acc_add")) return r;
  ArithP A = to_arith(arith);
  return launch_map(n, stream, "acc_add", [=] __device__(int64_t i) { out[i] = ar_acc_add(A, S[i], p[i], e, m); });
}

int mxq_arith_tile_add(const float* C, const float* t, float* out, int64_t n, const mxq_arith* arith, void* stream) {
  if (int r = check_arith(arith, "tile_add")) return r;
  ArithP A = to_arith(arith);
  return launch_map(n, stream, "tile_add", [=] __device__(int64_t i) { out[i] = ar_tile_add(A, C[i], t[i]); });
}

}  // extern "C"
