// Element arithmetic of the block quantizers shared by the TMA quantizer (quantize_tma.cu) and block.lut's fused
// kernel (lut.cu): the OCP grid rounding of block.mxgemmini and block.ocp (float_em._ocp), the reciprocal that makes a
// power-of-two scale's division a multiply, and an element's OCP code byte.
#pragma once
#include "common.cuh"
#include "numerics.cuh"

using namespace mxq;

namespace {

template <int E, int M>
struct Fmt {
  static constexpr int BIAS = (1 << (E - 1)) - 1;
  static constexpr float MAX_NORM = (E == 4 && M == 3) ? 448.0f
                                    : (E == 5 && M == 2) ? 57344.0f
                                    : (E == 3 && M == 2) ? 28.0f
                                    : (E == 2 && M == 3) ? 7.5f
                                                         : 6.0f;
  static constexpr int EMAX = (E == 5) ? 15 : (E == 4) ? 8 : (E == 3) ? 4 : 2;   // microxcaling emax
};

// float_em._ocp (float_em.py:113-134): q_ocp_bits with the format's constants folded; the core for finite x
template <int E, int M>
__device__ __forceinline__ float ocp_grid_core(float x, int mode) {
  constexpr uint32_t LO = (uint32_t)(128 - Fmt<E, M>::BIAS) << 23;     // biased emin in place
  const uint32_t u = f2u(x), a = u & 0x7fffffffu;
  const uint32_t e23 = (a & 0x7f800000u) > LO ? (a & 0x7f800000u) : LO;
  const float k = round_nonneg(__fmul_rn(u2f(a), u2f(((uint32_t)(254 + M) << 23) - e23)), mode);
  const float val = fminf(__fmul_rn(k, u2f(e23 - ((uint32_t)M << 23))), Fmt<E, M>::MAX_NORM);
  const float r = u2f(f2u(val) | (u & 0x80000000u));
  return a == 0u ? 0.0f : r;
}
template <int E, int M>
__device__ __forceinline__ float ocp_grid(float x, int mode) {
  return (f2u(x) & 0x7fffffffu) >= 0x7f800000u ? x : ocp_grid_core<E, M>(x, mode);
}

// the reciprocal that turns v / X into an exact multiply, or 0 when the division must be a division (X not a
// normal power of two, or -- for the qtorch family, whose codes see NaN sign bits -- a block holding a NaN)
template <int FAM>
__device__ __forceinline__ float reciprocal_of(float x, bool nan_block) {
  const uint32_t u = f2u(x);
  const bool pow2 = ((u & 0x807fffffu) == 0u && u >= 0x00800000u && u < 0x7f800000u) || u == 0x00400000u;
  if (!pow2 || (FAM == MXQ_FAMILY_MXQUANT && nan_block)) return 0.0f;
  return pow2f(-ilogb_f(x));
}

// an OCP element code's bit pattern (sign at bit E + M); `bad` set for what the format lacks (Inf, and NaN in FP6 /
// FP4; E4M3 keeps NaN as S.1111.111, E5M2 Inf as S.11111.00 and NaN as S.11111.11)
template <int E, int M>
__device__ __forceinline__ uint32_t ocp_code(float v, bool& bad) {
  constexpr int BIAS = (1 << (E - 1)) - 1;
  const uint32_t u = f2u(v), a = u & 0x7fffffffu, s = (u >> 31) << (E + M);
  if (a >= 0x7f800000u) {
    if (E == 5 && M == 2) return s | (a == 0x7f800000u ? 0x7cu : 0x7fu);
    if (E == 4 && M == 3 && a > 0x7f800000u) return s | 0x7fu;
    bad = true;
    return s;
  }
  const int ev = (int)(a >> 23) - 127;
  uint32_t c;
  if (ev >= 1 - BIAS) {
    c = ((uint32_t)(ev + BIAS) << M) | ((a >> (23 - M)) & ((1u << M) - 1u));
  } else {                                     // below the format's normal range: a multiple of its subnormal step
    const int sh = 24 - BIAS - M - ev;
    c = a == 0u ? 0u : (((a & 0x007fffffu) | 0x00800000u) >> (sh < 31 ? sh : 31));
  }
  return s | c;
}

// the same for a finite code on the format's grid (a clean tile's), branch-free: a normal code's bits are the
// float's exponent and top mantissa bits re-biased; a code below the normal range is the integer |v| / 2^(1-BIAS-M),
// read from a float add at 2^23
template <int E, int M>
__device__ __forceinline__ uint32_t ocp_code_finite(float v) {
  constexpr int BIAS = (1 << (E - 1)) - 1;
  constexpr uint32_t MIN_NORMAL = (uint32_t)(128 - BIAS) << 23;
  const uint32_t u = f2u(v), a = u & 0x7fffffffu;
  const uint32_t normal = (a >> (23 - M)) - ((uint32_t)(127 - BIAS) << M);
  const float scaled = __fmul_rn(u2f(a), u2f((uint32_t)(126 + BIAS + M) << 23));      // |v| * 2^(BIAS - 1 + M)
  const uint32_t sub = f2u(__fadd_rn(scaled, 8388608.0f)) - 0x4b000000u;
  return ((u >> 31) << (E + M)) | (a >= MIN_NORMAL ? normal : sub);
}

// ocp_code_finite(q_ocp_small(z, E, M, MODE, MAX_NORM)) for a finite |z| < 2^17, without the value: the rounding
// add of step_round leaves C + k q (C its magic constant, q the step), so k = bits(a + C) - bits(C) is the rounded
// magnitude in steps (Sterbenz: the subtraction step_round does is exact), and a code of a format's binade is k plus
// the binade's first code (k runs over [2^M, 2^(M+1)] in a normal binade, [0, 2^(M+1)] in the lowest, and reaching
// 2^(M+1) carries into the next binade's exponent as the code of the value would); saturation at MAX_NORM is the
// minimum with its code (codes grow with the value), and a zero input is +0 (q_ocp_small drops its sign)
// ZERO_SIGN: a zero keeps its sign (the negative-zero code for -0), one select fewer -- for block.lut's internal
// codes, where both zeros count into the same grid rank and look up the same table entry
template <int E, int M, int MODE, bool ZERO_SIGN = false>
__device__ __forceinline__ uint32_t code_clean(float z) {
  constexpr int BIAS = (1 << (E - 1)) - 1;
  constexpr uint32_t LO = (uint32_t)(128 - BIAS) << 23;               // the lowest binade's exponent field in place
  constexpr uint32_t MAXC = (E == 4 && M == 3) ? 0x7eu : (1u << (E + M)) - 1u - ((E == 5 && M == 2) ? 4u : 0u);
  const uint32_t u = f2u(z), a = u & 0x7fffffffu;
  const uint32_t e23 = (a & 0x7f800000u) > LO ? (a & 0x7f800000u) : LO;
  const uint32_t cb = e23 + (((uint32_t)(23 - M) << 23) | 0x400000u);
  const float c = u2f(cb);
  float s;
  if (MODE == RM_RNE) s = __fadd_rn(u2f(a), c);
  else if (MODE == RM_TRUNCATE) s = __fadd_rz(u2f(a), c);
  else s = __fadd_rz(__fadd_rn(u2f(a), u2f(e23 - ((uint32_t)(M + 1) << 23))), c);
  const uint32_t k = f2u(s) - cb;
  const uint32_t mag = min(k + ((e23 - LO) >> (23 - M)), MAXC);
  if (ZERO_SIGN) return ((u >> 31) << (E + M)) | mag;
  return a == 0u ? 0u : (((u >> 31) << (E + M)) | mag);
}

// A code for block.lut's table fit: the OCP bit pattern, read back in the LUT code space, where every E4M3 byte is a
// finite value (0x7F / 0xFF are +-480, formats.py:91-96) so E4M3's NaN has no code there: it counts as one the format
// cannot hold, as a NaN code does in the fit of float codes
template <int E, int M>
__device__ __forceinline__ uint32_t lut_code(float v, bool& bad) {
  if (E == 4 && M == 3 && (f2u(v) & 0x7fffffffu) > 0x7f800000u) bad = true;
  return ocp_code<E, M>(v, bad);
}

}  // namespace
