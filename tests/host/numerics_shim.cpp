// Test shim: the CUDA kernels' element math (microscaling-quant_b200/csrc/numerics.cuh) compiled for the host,
// exported under the oracle's signatures (h_* for o_*) so tests/test_numerics_host.py can run it through the
// same golden checks and compare it with the oracle on large corpora without a GPU.
#include <math.h>
#include "../../microscaling-quant_b200/csrc/numerics.cuh"

using namespace mxq;
#define X extern "C" __attribute__((visibility("default")))

X void h_round_bits(const int64_t* bits, const int64_t* keep, int64_t n, int mode, int64_t* out) {
  for (int64_t i = 0; i < n; i++) out[i] = round_bits_i64(bits[i], (int)keep[i], mode);
}
X void h_round_int_f32(const float* k, int64_t n, int mode, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = round_int_f(k[i], mode);
}
X void h_round_int_f64(const double* k, int64_t n, int mode, double* out) {
  for (int64_t i = 0; i < n; i++) out[i] = round_int_d(k[i], mode);
}
X void h_bf16(const float* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = bf16_rne(x[i]);
}
X void h_float_em_f32(const float* z, int64_t n, int e, int m, int mode, int grid, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = q_float_em(z[i], e, m, mode, grid);
}
X void h_float_em_f64(const double* z, int64_t n, int e, int m, int mode, int grid, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = q_float_em_d(z[i], e, m, mode, grid);
}
X void h_microsoft(const float* A, int64_t n, int bits, int exp_bits, float max_norm, int round, int sat, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = q_microsoft(A[i], bits, exp_bits, max_norm, round, sat != 0);
}
X void h_scale_mxquant(const float* amax, int64_t n, float fl, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = scale_mxquant(amax[i], fl);
}
X void h_scale_ocp(const float* amax, int64_t n, int emax, float scale_emax, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = scale_ocp(amax[i], emax, scale_emax);
}
X void h_scale_ocp_no_clip(const float* amax, int64_t n, int e, int m, int round, float scale_emax, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = scale_ocp_no_clip(amax[i], e, m, round, scale_emax);
}
X void h_exact_add(const float* a, const float* b, int64_t n, int e, int m, int mode, int grid, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = exact_add_any(a[i], b[i], e, m, mode, grid);
}
X void h_truncate_significand(const float* x, int64_t n, int m, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = truncate_significand(x[i], m);
}
X void h_flush_product(const float* x, int64_t n, float thr, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = flush_below(x[i], thr);
}
X void h_saturate(const float* x, int64_t n, float limit, float value, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = saturate(x[i], limit, value);
}
// floor_log2_rn against floor(RN32(log2 x)) computed through libm's double log2, over bit patterns [lo, hi)
X int64_t h_log2_mismatches(uint32_t lo, uint32_t hi) {
  int64_t bad = 0;
  for (uint32_t u = lo; u < hi; u++) {
    float x = u2f(u);
    float ref = floorf((float)log2((double)x));
    if ((float)floor_log2_rn(x) != ref) bad++;
  }
  return bad;
}
// the thresholds floor_log2_rn implies: smallest bit pattern reading k, for k in [-149, 128]
X void h_log2_thresholds(uint32_t* out) {
  for (int k = -149; k <= 128; k++) {
    uint32_t lo = 1, hi = 0x7f800000u;                     // first u with floor_log2_rn(u2f(u)) >= k
    while (lo < hi) {
      uint32_t mid = lo + (hi - lo) / 2;
      if (floor_log2_rn(u2f(mid)) >= k) hi = mid; else lo = mid + 1;
    }
    out[k + 149] = lo;
  }
}
// the block quantizer's fast element forms against the general ones, over bit patterns lo, lo+stride, ... < hi
X int64_t h_fast_forms_mismatches(uint64_t lo, uint64_t hi, uint64_t stride, int which, int e, int m, int mode) {
  int64_t bad = 0;
  float mn = ocp_max_norm(e, m);
  for (uint64_t v = lo; v < hi; v += stride) {
    float x = u2f((uint32_t)v);
    float a, b;
    if (which == 0) { a = q_ocp_bits(x, e, m, mode, mn); b = q_ocp_f(x, e, m, mode, mn); }
    else { a = q_microsoft_sat(x, m + 2, e, mn, mode); b = q_microsoft(x, m + 2, e, mn, mode, true); }
    bool an = (f2u(a) & 0x7fffffffu) > 0x7f800000u, bn = (f2u(b) & 0x7fffffffu) > 0x7f800000u;
    if (an != bn || (!an && f2u(a) != f2u(b))) bad++;
  }
  return bad;
}
// the one-add forms of clean tiles (|x| < 2^17) against the general ones, over bit patterns lo, lo+stride, ... < hi
// (patterns with |x| >= 2^17 skipped): which 0 q_ocp_small / q_ocp_bits, 1 q_microsoft_ocp_small / _core
X int64_t h_small_forms_mismatches(uint64_t lo, uint64_t hi, uint64_t stride, int which, int e, int m, int mode) {
  int64_t bad = 0;
  float mn = ocp_max_norm(e, m);
  for (uint64_t v = lo; v < hi; v += stride) {
    if (((uint32_t)v & 0x7fffffffu) >= 0x48000000u) continue;
    float x = u2f((uint32_t)v);
    float a, b;
    if (which == 0) { a = q_ocp_small(x, e, m, mode, mn); b = q_ocp_bits(x, e, m, mode, mn); }
    else { a = q_microsoft_ocp_small(x, m + 2, e, mn, mode); b = q_microsoft_ocp_core(x, m + 2, e, mn, mode); }
    if (f2u(a) != f2u(b)) bad++;
  }
  return bad;
}
// q_ieee_small against q_ieee_f on patterns with |x| < 2^17, over bit patterns lo, lo+stride, ... < hi
X int64_t h_ieee_small_mismatches(uint64_t lo, uint64_t hi, uint64_t stride, int e, int m, int mode) {
  int64_t bad = 0;
  for (uint64_t v = lo; v < hi; v += stride) {
    if (((uint32_t)v & 0x7fffffffu) >= 0x48000000u) continue;
    float x = u2f((uint32_t)v);
    if (f2u(q_ieee_small(x, e, m, mode)) != f2u(q_ieee_f(x, e, m, mode))) bad++;
  }
  return bad;
}
// q_microsoft_ocp against q_microsoft (saturating) over bit patterns lo, lo+stride, ... < hi
X int64_t h_ms_ocp_mismatches(uint64_t lo, uint64_t hi, uint64_t stride, int e, int m, int mode) {
  int64_t bad = 0;
  float mn = ocp_max_norm(e, m);
  for (uint64_t v = lo; v < hi; v += stride) {
    float x = u2f((uint32_t)v);
    float a = q_microsoft_ocp(x, m + 2, e, mn, mode), b = q_microsoft(x, m + 2, e, mn, mode, true);
    bool an = (f2u(a) & 0x7fffffffu) > 0x7f800000u, bn = (f2u(b) & 0x7fffffffu) > 0x7f800000u;
    if (an != bn || (!an && f2u(a) != f2u(b))) bad++;
  }
  return bad;
}
