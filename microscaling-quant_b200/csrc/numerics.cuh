// Element arithmetic of the mxq hot path, written once for the CUDA kernels (nvcc) and for host-side
// exhaustive tests (g++, built with -ffp-contract=off). Every function here is a bit-exact restatement of
// one reference function; the citations name the file:line in chloe-wong/microscaling-quant (mxq/...).
//
// Rules every function follows:
//   * IEEE single/double operations only through add_rn/mul_rn/div_rn (never contracted into an FMA);
//   * no flush-to-zero: subnormals are data (the default scale floor 1e-38 is itself a float32 subnormal);
//   * NaN is data. Where the reference's x86 NaN bits leak into a non-NaN result (qtorch's bit rounding maps a
//     NaN to +-max by its sign bit) the x86_* operations reproduce the host's NaN propagation: the first NaN
//     operand (quieted) wins, an invalid operation yields the default NaN 0xFFC00000.
#pragma once
#include <stdint.h>
#include <string.h>
#include <math.h>

#if defined(__CUDACC__)
#define MXQ_HD __host__ __device__ __forceinline__
#else
#define MXQ_HD static inline
#endif

namespace mxq {

// ------------------------------------------------------------------------------------------------ enums
// rounding modes (mxq/rounding/__init__.py:25 MODES = ties_away, rne, truncate)
enum RoundMode : int { RM_TIES_AWAY = 0, RM_RNE = 1, RM_TRUNCATE = 2 };
// microxcaling's names (mxq/microxcaling/elemwise.py:29-60): nearest (ties away), floor (toward zero), even
enum MsRound : int { MS_NEAREST = 0, MS_FLOOR = 1, MS_EVEN = 2 };

// ------------------------------------------------------------------------------------------------ bits
MXQ_HD uint32_t f2u(float x) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(x);
#else
  uint32_t u; memcpy(&u, &x, 4); return u;
#endif
}
MXQ_HD float u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float x; memcpy(&x, &u, 4); return x;
#endif
}
MXQ_HD uint64_t d2u(double x) {
#if defined(__CUDA_ARCH__)
  return (uint64_t)__double_as_longlong(x);
#else
  uint64_t u; memcpy(&u, &x, 8); return u;
#endif
}
MXQ_HD double u2d(uint64_t u) {
#if defined(__CUDA_ARCH__)
  return __longlong_as_double((long long)u);
#else
  double x; memcpy(&x, &u, 8); return x;
#endif
}
MXQ_HD int clz32(uint32_t u) {   // u != 0
#if defined(__CUDA_ARCH__)
  return __clz(u);
#else
  return __builtin_clz(u);
#endif
}
MXQ_HD int clz64(uint64_t u) {   // u != 0
#if defined(__CUDA_ARCH__)
  return __clzll((long long)u);
#else
  return __builtin_clzll(u);
#endif
}

MXQ_HD bool isnan_f(float x) { return (f2u(x) & 0x7fffffffu) > 0x7f800000u; }
MXQ_HD bool isinf_f(float x) { return (f2u(x) & 0x7fffffffu) == 0x7f800000u; }
MXQ_HD bool finite_f(float x) { return (f2u(x) & 0x7fffffffu) < 0x7f800000u; }
MXQ_HD bool isnan_d(double x) { return (d2u(x) & 0x7fffffffffffffffull) > 0x7ff0000000000000ull; }
MXQ_HD bool finite_d(double x) { return (d2u(x) & 0x7fffffffffffffffull) < 0x7ff0000000000000ull; }
MXQ_HD float abs_f(float x) { return u2f(f2u(x) & 0x7fffffffu); }                 // torch.abs clears the sign
MXQ_HD double abs_d(double x) { return u2d(d2u(x) & 0x7fffffffffffffffull); }
MXQ_HD float copysign_f(float v, float s) { return u2f((f2u(v) & 0x7fffffffu) | (f2u(s) & 0x80000000u)); }
MXQ_HD double copysign_d(double v, double s) {
  return u2d((d2u(v) & 0x7fffffffffffffffull) | (d2u(s) & 0x8000000000000000ull));
}
MXQ_HD float inf_f() { return u2f(0x7f800000u); }
MXQ_HD double inf_d() { return u2d(0x7ff0000000000000ull); }
MXQ_HD float qnan_f() { return u2f(0x7fc00000u); }
// torch.sign: (0 < x) - (x < 0); sign(+-0) = +0, sign(NaN) = 0 (probed: both vector and scalar paths)
MXQ_HD float sign_f(float x) { return (x > 0.0f) ? 1.0f : ((x < 0.0f) ? -1.0f : 0.0f); }

// ------------------------------------------------------------------------------- uncontracted IEEE ops
MXQ_HD float add_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fadd_rn(a, b);
#else
  return a + b;
#endif
}
MXQ_HD float sub_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fsub_rn(a, b);
#else
  return a - b;
#endif
}
MXQ_HD float mul_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}
MXQ_HD float div_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fdiv_rn(a, b);
#else
  return a / b;
#endif
}
MXQ_HD double dadd_rn(double a, double b) {
#if defined(__CUDA_ARCH__)
  return __dadd_rn(a, b);
#else
  return a + b;
#endif
}
MXQ_HD double dsub_rn(double a, double b) {
#if defined(__CUDA_ARCH__)
  return __dsub_rn(a, b);
#else
  return a - b;
#endif
}
MXQ_HD double dmul_rn(double a, double b) {
#if defined(__CUDA_ARCH__)
  return __dmul_rn(a, b);
#else
  return a * b;
#endif
}
MXQ_HD double ddiv_rn(double a, double b) {
#if defined(__CUDA_ARCH__)
  return __ddiv_rn(a, b);
#else
  return a / b;
#endif
}
MXQ_HD float floor_f(float x) { return floorf(x); }    // exact operations (no rounding involved)
MXQ_HD float trunc_f(float x) { return truncf(x); }
MXQ_HD float rint_f(float x) { return rintf(x); }      // round half to even = torch.round
// floor / rint of a float32 0 <= s < 2^23 with adds at a fixed exponent, which the device runs on the full-rate
// FP32 pipe rather than the conversion pipe: s + 2^23 lies in [2^23, 2^24), where float32 values are the integers,
// so the add's own rounding (toward zero, or to nearest even) is the rounding of s and subtracting 2^23 is exact.
// Infinities and NaN pass through unchanged, as with floorf / rintf. (Negative s: a defined value that callers
// discard.)
MXQ_HD float floor_small(float s) {
#if defined(__CUDA_ARCH__)
  return __fsub_rn(__fadd_rz(s, 8388608.0f), 8388608.0f);
#else
  return floorf(s);
#endif
}
MXQ_HD float rint_small(float s) { return sub_rn(add_rn(s, 8388608.0f), 8388608.0f); }
// a + b rounded toward zero (the host form: the TwoSum error of the nearest sum says whether it overshot)
MXQ_HD float add_rz(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fadd_rz(a, b);
#else
  const float r = a + b, bb = r - a, err = (a - (r - bb)) + (b - bb);     // a + b = r + err exactly
  return (err != 0.0f && ((err < 0.0f) != (r < 0.0f))) ? nextafterf(r, 0.0f) : r;
#endif
}
MXQ_HD double floor_d(double x) { return floor(x); }
MXQ_HD double trunc_d(double x) { return trunc(x); }
MXQ_HD double rint_d(double x) { return rint(x); }

// ------------------------------------------------------------------------------ x86 NaN propagation
constexpr uint32_t X86_DEFAULT_NAN = 0xffc00000u;
MXQ_HD float x86_fix(float a, float b, float r) {
  uint32_t ua = f2u(a), ub = f2u(b);
  if ((ua & 0x7fffffffu) > 0x7f800000u) return u2f(ua | 0x00400000u);
  if ((ub & 0x7fffffffu) > 0x7f800000u) return u2f(ub | 0x00400000u);
  if ((f2u(r) & 0x7fffffffu) > 0x7f800000u) return u2f(X86_DEFAULT_NAN);
  return r;
}
MXQ_HD float x86_mul(float a, float b) { return x86_fix(a, b, mul_rn(a, b)); }
MXQ_HD float x86_add(float a, float b) { return x86_fix(a, b, add_rn(a, b)); }
MXQ_HD float x86_div(float a, float b) { return x86_fix(a, b, div_rn(a, b)); }
// float64 -> float32 as the host converts (cvtsd2ss): RN; a NaN keeps its sign and the top 22 payload bits, quieted
MXQ_HD float x86_d2f(double x) {
  uint64_t u = d2u(x);
  if ((u & 0x7fffffffffffffffull) > 0x7ff0000000000000ull)
    return u2f((uint32_t)(u >> 32 & 0x80000000u) | 0x7fc00000u | (uint32_t)((u >> 29) & 0x003fffffu));
#if defined(__CUDA_ARCH__)
  return __double2float_rn(x);
#else
  return (float)x;
#endif
}

// ----------------------------------------------------------------------------------- powers of two
MXQ_HD float pow2f(int t) {            // 2^t in float32, saturating to 0 / inf like torch.exp2 and torch.pow
  if (t > 127) return inf_f();
  if (t >= -126) return u2f((uint32_t)(t + 127) << 23);
  if (t >= -149) return u2f(1u << (t + 149));
  return 0.0f;
}
MXQ_HD double pow2d(int t) {
  if (t > 1023) return inf_d();
  if (t >= -1022) return u2d((uint64_t)(t + 1023) << 52);
  if (t >= -1074) return u2d(1ull << (t + 1074));
  return 0.0;
}
// exact floor(log2 |x|) of a finite nonzero value, from the bits (torch.frexp's exponent minus one)
MXQ_HD int ilogb_f(float x) {
  uint32_t a = f2u(x) & 0x7fffffffu;
  if (a >= 0x00800000u) return (int)(a >> 23) - 127;
  return (31 - clz32(a)) - 149;
}
MXQ_HD int ilogb_d(double x) {
  uint64_t a = d2u(x) & 0x7fffffffffffffffull;
  if (a >= 0x0010000000000000ull) return (int)(a >> 52) - 1023;
  return (63 - clz64(a)) - 1074;
}

// ------------------------------------------------------------------------------ floor(log2 x) as torch
// torch.floor(torch.log2(x)) on float32 is floor(RN32(log2 x)): a correctly rounded float32 log2, so a value
// within d ulps below 2^k already reads k (log2 x = k - eps rounds to k). d depends on the float32 spacing at k
// only: by the bit length of |k| (k - 1 for k > 0) it is 0,0,1,2,5,11,22,44 for lengths 0..7; the binades
// reaching into the subnormal range have fewer ulps below 2^k. Verified exhaustively against torch 2.11 on all
// positive float32 (tests/test_numerics_host.py). Used by scale_factor.mxquant/ocp (mxq/scale_factor.py:43, :54)
// and the microxcaling element step (mxq/microxcaling/elemwise.py:116-117).
MXQ_HD int floor_log2_rn(float x) {     // x finite, > 0
  uint32_t u = f2u(x);
  int e = (u >= 0x00800000u) ? (int)(u >> 23) - 127 : (31 - clz32(u)) - 149;
  int k = e + 1;
  uint32_t start = (k >= -126) ? ((uint32_t)(k + 127) << 23) : (1u << (k + 149));
  uint32_t d;
  if (k >= -125) {
    uint32_t a = (k > 0) ? (uint32_t)(k - 1) : (uint32_t)(-k);
    int bl = a ? 32 - clz32(a) : 0;
    d = (uint32_t)((0x2C160B0502010000ull >> (8 * bl)) & 0xffu);
  } else {
    d = (k == -126) ? 22u : (k == -127 || k == -128) ? 11u : (k == -129) ? 5u : (k == -130) ? 2u : (k == -131) ? 1u : 0u;
  }
  return (u >= start - d) ? k : e;
}
// the same as a float, with torch's special values: log2(+inf) = inf, log2(NaN) = NaN, log2(0) = -inf,
// log2(x < 0) = NaN (SLEEF returns the positive quiet NaN there).
MXQ_HD float floor_log2_torch(float x) {
  if (isnan_f(x)) return u2f(f2u(x) | 0x00400000u);
  if (x == 0.0f) return u2f(0xff800000u);
  if (x < 0.0f) return qnan_f();
  if (isinf_f(x)) return inf_f();
  return (float)floor_log2_rn(x);
}
// torch.pow(2, t) / 2 ** t for an integer-valued (or infinite / NaN) float32 t: exact (probed)
MXQ_HD float exp2_torch(float t) {
  if (isnan_f(t)) return u2f(f2u(t) | 0x00400000u);
  if (t >= 128.0f) return inf_f();
  if (t <= -150.0f) return 0.0f;
  return pow2f((int)t);
}

// ------------------------------------------------------------------------------ rounding primitives
// mxq/rounding/__init__.py:51-55 round_bits on an int64 holding any integer; keep in [0, 22]
// the three modules' bits(bits, drop, mask, half) on int64 (no reduction to 32 bits); a shift outside [0, 63] fills
// with the sign, as torch's >> does
MXQ_HD int64_t round_pattern_i64(int64_t bits, int64_t drop, int64_t mask, int64_t half, int mode) {
  if (mode == RM_TIES_AWAY) return (bits + half) & ~mask;                                   // ties_away.py:5-6
  if (mode == RM_RNE) {                                                                     // rne.py:6-8
    const int sh = (drop < 0 || drop > 63) ? 63 : (int)drop;
    return (bits + half - 1 + ((bits >> sh) & 1)) & ~mask;
  }
  return bits & ~mask;                                                                      // truncate.py:5-6
}
MXQ_HD int64_t round_bits_i64(int64_t bits, int keep, int mode) {
  int drop = 23 - keep;
  int64_t mask = ((int64_t)1 << drop) - 1, half = (int64_t)1 << (drop - 1);
  return round_pattern_i64(bits, drop, mask, half, mode) & 0xffffffffll;
}
// mxq/rounding/__init__.py:58-61 round_int on an integer-valued quantity
MXQ_HD float round_int_f(float k, int mode) {
  if (mode == RM_RNE) return rint_f(k);                                          // rne.py:11-12 torch.round
  if (mode == RM_TRUNCATE) return trunc_f(k);                                    // truncate.py:9-10
  float s = sign_f(k);                                                           // ties_away.py:9-10
  return x86_mul(s, floor_f(add_rn(abs_f(k), 0.5f)));
}
MXQ_HD double round_int_d(double k, int mode) {
  if (mode == RM_RNE) return rint_d(k);
  if (mode == RM_TRUNCATE) return trunc_d(k);
  double s = (k > 0.0) ? 1.0 : ((k < 0.0) ? -1.0 : 0.0);
  if (isnan_d(k)) return k;
  return dmul_rn(s, floor_d(dadd_rn(abs_d(k), 0.5)));
}
// mxq/rounding/__init__.py:64-85 bf16: RNE to 7 fraction bits on the bit pattern; NaN passes through
MXQ_HD float bf16_rne(float x) {
  uint32_t u = f2u(x);
  if ((u & 0x7fffffffu) > 0x7f800000u) return x;
  return u2f((u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u);
}

// ------------------------------------------------------------------------------ float_em grids
MXQ_HD int bias_of(int e) { return (1 << (e - 1)) - 1; }                         // float_em.py:45-47

// float_em._qtorch (mxq/element_quant/float_em.py:64-84): round the float32 pattern at m fraction bits,
// then clip the exponent to [127-L, 127+L] with one fake-subnormal binade.
MXQ_HD float q_qtorch(float z, int e, int m, int mode) {
  uint32_t bits = f2u(z);
  uint32_t drop = 23u - (uint32_t)m, mask = (1u << drop) - 1u, half = 1u << (drop - 1u);
  uint32_t q;
  if (mode == RM_TIES_AWAY) q = (bits + half) & ~mask;
  else if (mode == RM_RNE) q = (bits + half - 1u + ((bits >> drop) & 1u)) & ~mask;
  else q = bits & ~mask;
  uint32_t L = (1u << (e - 1)) - 1u;
  uint32_t min_store = 127u - L, max_store = 127u + L;
  uint32_t exp_store = (q >> 23) & 0xffu;
  uint32_t sign = bits & 0x80000000u;
  uint32_t max_num = sign | (max_store << 23) | (0x007fffffu & ~((1u << (23 - m)) - 1u));
  uint32_t min_num = sign | (min_store << 23);
  uint32_t middle = (min_store - 1u) << 23;
  uint32_t q_mag = q & 0x7fffffffu;
  uint32_t r = q;
  if (exp_store > max_store) r = max_num;
  if (exp_store < min_store) r = (q_mag > middle) ? min_num : 0u;
  return u2f(r);
}

// float_em._ieee (float_em.py:87-110), float32 arithmetic (e < 8): scaled integer on step 2^(max(E,emin)-m),
// true subnormals, overflow -> inf, underflow -> +0, +-0 / inf / NaN pass through.
MXQ_HD float q_ieee_f(float x, int e, int m, int mode) {
  uint32_t a = f2u(x) & 0x7fffffffu;
  if (a == 0u || a >= 0x7f800000u) return x;
  int b = bias_of(e), emin = 1 - b, emax = b;
  int E = ilogb_f(x);
  int s = (E > emin ? E : emin) - m;
  float k = mul_rn(u2f(a), pow2f(-s));                        // exact: division by a power of two
  k = round_int_f(k, mode);
  float val = mul_rn(k, pow2f(s));
  if (val >= pow2f(emax + 1)) val = inf_f();
  if (val == 0.0f) return 0.0f;
  return copysign_f(val, x);
}
// the same in float64 (e = 8, or a float64 input: float_em.py:94); keep_signed_zero is the e = 8 rule
MXQ_HD double q_ieee_d(double x, int e, int m, int mode) {
  uint64_t a = d2u(x) & 0x7fffffffffffffffull;
  if (a == 0ull || a >= 0x7ff0000000000000ull) return x;
  int b = bias_of(e), emin = 1 - b, emax = b;
  int E = ilogb_d(x);
  int s = (E > emin ? E : emin) - m;
  double k = dmul_rn(u2d(a), pow2d(-s));
  k = round_int_d(k, mode);
  double val = dmul_rn(k, pow2d(s));
  if (val >= pow2d(emax + 1)) val = inf_d();
  if (val == 0.0 && e < 8) return 0.0;
  return copysign_d(val, x);
}
// float_em.quantize(z, e, m, mode, "ieee") for a float32 input, float32 out (float_em.py:50-61)
MXQ_HD float q_ieee(float x, int e, int m, int mode) {
  if (e == 8 && m == 23) return x;
  if (e < 8) return q_ieee_f(x, e, m, mode);
  return x86_d2f(q_ieee_d((double)x, e, m, mode));
}
// float64 input (float_em.py:56-57, :94): computed in float64, then float32
MXQ_HD float q_ieee_from_d(double x, int e, int m, int mode) { return x86_d2f(q_ieee_d(x, e, m, mode)); }

// float_em._ocp (float_em.py:113-134): the OCP element grid (ieee's emin/step), saturate at max_norm,
// exact +-0 -> +0, a negative value that rounds to zero stays -0, inf / NaN pass through.
MXQ_HD float q_ocp_f(float x, int e, int m, int mode, float max_norm) {
  uint32_t a = f2u(x) & 0x7fffffffu;
  if (a == 0u) return 0.0f;
  if (a >= 0x7f800000u) return x;
  int emin = 1 - bias_of(e);
  int E = ilogb_f(x);
  int s = (E > emin ? E : emin) - m;
  float k = round_int_f(mul_rn(u2f(a), pow2f(-s)), mode);
  float val = mul_rn(k, pow2f(s));
  if (val > max_norm) val = max_norm;
  return copysign_f(val, x);
}
MXQ_HD float q_ocp_from_d(double x, int e, int m, int mode, double max_norm) {
  uint64_t a = d2u(x) & 0x7fffffffffffffffull;
  if (a == 0ull) return 0.0f;
  if (a >= 0x7ff0000000000000ull) return x86_d2f(x);
  int emin = 1 - bias_of(e);
  int E = ilogb_d(x);
  int s = (E > emin ? E : emin) - m;
  double k = round_int_d(dmul_rn(u2d(a), pow2d(-s)), mode);
  double val = dmul_rn(k, pow2d(s));
  if (val > max_norm) val = max_norm;
  return x86_d2f(copysign_d(val, x));
}

// ------------------------------------------------------------------------ microxcaling element step
// _quantize_elemwise_core (mxq/microxcaling/elemwise.py:63-151) with allow_denorm=True, as block.ocp and
// scale_factor.ocp_no_clip call it: private exponent floor(log2|A|) clipped at min_exp, scale so bits-2 fraction
// bits are integral, round (_round_mantissa :29-60), unscale, clamp (saturate) or overflow to +-inf.
// exp_bits = 0 is the integer formats (no private exponent, always clamped).
MXQ_HD float q_microsoft(float A, int bits, int exp_bits, float max_norm, int round, bool saturate) {
  float out;
  float pe = 0.0f, p = 1.0f;
  if (exp_bits != 0) {
    float t = (A == 0.0f) ? 1.0f : abs_f(A);                  // |A| + (A == 0)
    pe = floor_log2_torch(t);
    float min_exp = (float)(2 - (1 << (exp_bits - 1)));
    if (pe < min_exp) pe = min_exp;                            // clip(min=): NaN stays NaN
    p = exp2_torch(pe);
    // A / 2^pe * 2^(bits-2); for pe in [min_exp, 127] the reciprocal is exact, so multiplying is the division
    if (finite_f(pe) && pe <= 127.0f) out = mul_rn(A, pow2f(-(int)pe));
    else out = div_rn(A, p);
  } else {
    out = A;
  }
  out = mul_rn(out, pow2f(bits - 2));
  float absA = abs_f(out), sgn = sign_f(out), r;
  if (round == MS_FLOOR) {
    r = mul_rn(sgn, floor_f(absA));
  } else if (round == MS_NEAREST) {
    r = mul_rn(sgn, floor_f(add_rn(absA, 0.5f)));
  } else {
    float y = sub_rn(absA, 0.5f);                              // (|A| - 0.5) % 2 == 0: y an even integer >= 0
    float h = mul_rn(y, 0.5f);
    float mask = (y >= 0.0f && finite_f(y) && floor_f(h) == h) ? 1.0f : 0.0f;
    r = mul_rn(sgn, sub_rn(floor_f(add_rn(absA, 0.5f)), mask));
  }
  out = mul_rn(r, pow2f(-(bits - 2)));                         // / 2^(bits-2), exact
  if (exp_bits != 0) out = mul_rn(out, p);
  if (saturate || exp_bits == 0) {
    if (out < -max_norm) out = -max_norm;
    if (out > max_norm) out = max_norm;
  } else if (abs_f(out) > max_norm) {
    out = copysign_f(inf_f(), out);
  }
  if (isinf_f(A)) out = A;                                     // out[A == +-inf] = +-inf
  return out;
}

// ------------------------------------------------------------------------------ scale rules (step 1)
// scale_factor.mxquant (mxq/scale_factor.py:40-44): 2^floor(log2 max(amax, floor)), then max(., floor);
// `fl` is the floor as float32 (torch casts the Python scalar to the tensor dtype).
MXQ_HD float scale_mxquant(float amax, float fl) {
  float c = (isnan_f(amax) || !(amax < fl)) ? amax : fl;       // clamp(min=fl), NaN propagates
  float sc = exp2_torch(floor_log2_torch(c));
  return (isnan_f(sc) || !(sc < fl)) ? sc : fl;
}
// scale_factor.ocp (scale_factor.py:47-59): 2^(floor(log2(amax + 2^-126 [amax==0])) - emax), NaN above the E8M0
// range, clamped at -scale_emax below it.
// scale_emax = float32(2^(scale_bits-1) - 1), as torch casts the Python integer it is compared with.
MXQ_HD float scale_ocp(float amax, int emax, float scale_emax) {
  float t = (amax == 0.0f) ? u2f(0x00800000u) : amax;
  float se = floor_log2_torch(t);
  se = sub_rn(se, (float)emax);
  if (se > scale_emax) se = qnan_f();
  if (se < -scale_emax) se = -scale_emax;
  return exp2_torch(se);
}

// ------------------------------------------------------------------------------ PE arithmetic (arith.py)
// _fits_float32 (mxq/arith.py:21-30)
MXQ_HD bool fits_float32(int e, int m) { return (1 << e) - 1 + m <= 24; }

// _round_pair (arith.py:41-65): s + t (exact, t the TwoSum residual) rounded RNE to float(e, m), e <= 7
MXQ_HD float round_pair(float s, float t, int e, int m) {
  uint32_t a = f2u(s) & 0x7fffffffu;
  if (a == 0u || a >= 0x7f800000u) return s;
  int b = bias_of(e), emin = 1 - b, emax = b;
  int E = ilogb_f(s);
  int sh = (E > emin ? E : emin) - m;
  float k = mul_rn(u2f(a), pow2f(-sh));
  float kf = floor_f(k);
  bool tie = sub_rn(k, kf) == 0.5f;
  bool up = mul_rn(sign_f(s), t) > 0.0f;
  float ko = (tie && t != 0.0f) ? (up ? add_rn(kf, 1.0f) : kf) : rint_f(k);
  float val = mul_rn(ko, pow2f(sh));
  if (val >= pow2f(emax + 1)) val = inf_f();
  if (val == 0.0f) return 0.0f;
  return copysign_f(val, s);
}

// exact_add (arith.py:68-103) with rounding_mode="rne", grid="ieee": a + b exactly, one RNE rounding to
// float(e, m); a zero addend returns the other operand unchanged.
MXQ_HD float exact_add_rne(float a, float b, int e, int m) {
  if (a == 0.0f) return b;
  if (b == 0.0f) return a;
  if (e == 8 && m == 23) return x86_d2f(dadd_rn((double)a, (double)b));   // float64 path, quantize = cast
  if (fits_float32(e, m)) return q_ieee_f(add_rn(a, b), e, m, RM_RNE);
  if (e <= 7) {
    float s = add_rn(a, b);                                     // _two_sum (arith.py:33-38)
    float bb = sub_rn(s, a);
    float t = add_rn(sub_rn(a, sub_rn(s, bb)), sub_rn(b, bb));
    return round_pair(s, t, e, m);
  }
  return q_ieee_from_d(dadd_rn((double)a, (double)b), e, m, RM_RNE);
}

// truncate_significand (arith.py:106-117): keep m fraction bits of the significand (subnormals normalised
// first), toward zero; +-0, inf, NaN pass through.
MXQ_HD float truncate_significand(float x, int m) {
  uint32_t u = f2u(x), a = u & 0x7fffffffu;
  if (a == 0u || a >= 0x7f800000u) return x;
  if (m >= 23) return x;
  int lead = (a >= 0x00800000u) ? 23 : (31 - clz32(a));        // bit index of the leading one
  int drop = lead - m;
  if (drop <= 0) return x;
  return u2f(u & ~((1u << drop) - 1u));
}
// flush_product (arith.py:120-124): |x| < thr -> +0 (thr = float32(2^floor_exp))
MXQ_HD float flush_below(float x, float thr) { return (abs_f(x) < thr) ? 0.0f : x; }
// saturate (arith.py:127-137): sign(x) * (|x| > limit ? value : |x|); -0 -> +0, NaN stays NaN
MXQ_HD float saturate(float x, float limit, float value) {
  float ax = abs_f(x);
  return x86_mul(sign_f(x), (ax > limit) ? value : ax);
}
// MXGEMMINI's _unsigned_zero (mxq/matmul/_arithmetic.py:105-108)
MXQ_HD float unsigned_zero(float x) { return (x == 0.0f) ? 0.0f : x; }

// ------------------------------------------------------------------------------ dispatchers
enum Grid : int { GRID_QTORCH = 0, GRID_IEEE = 1, GRID_OCP = 2 };
// OCP element formats (mxq/element_quant/formats.py:23-29): max_norm by (e, m); 0 if not an OCP format
MXQ_HD float ocp_max_norm(int e, int m) {
  if (e == 4 && m == 3) return 448.0f;
  if (e == 5 && m == 2) return 57344.0f;
  if (e == 3 && m == 2) return 28.0f;
  if (e == 2 && m == 3) return 7.5f;
  if (e == 2 && m == 1) return 6.0f;
  return 0.0f;
}
MXQ_HD int ocp_emax(int e, int m) {        // microxcaling emax (mxq/microxcaling/formats.py:92-106)
  if (e == 5) return 15;
  if (e == 4) return 8;
  if (e == 3) return 4;
  return 2;
}
// float_em.quantize(z, e, m, mode, grid) for a float32 input (float_em.py:50-61)
MXQ_HD float q_float_em(float z, int e, int m, int mode, int grid) {
  if (e == 8 && m == 23) return z;
  if (grid == GRID_QTORCH) return q_qtorch(z, e, m, mode);
  if (grid == GRID_IEEE) return q_ieee(z, e, m, mode);
  return q_ocp_f(z, e, m, mode, ocp_max_norm(e, m));
}
// ... for a float64 input: the ieee and ocp grids round from float64; qtorch casts to float32 first
MXQ_HD float q_float_em_d(double z, int e, int m, int mode, int grid) {
  if (e == 8 && m == 23) return q_ieee_from_d(z, 8, 23, mode);
  if (grid == GRID_QTORCH) return q_qtorch(x86_d2f(z), e, m, mode);
  if (grid == GRID_IEEE) return q_ieee_from_d(z, e, m, mode);
  return q_ocp_from_d(z, e, m, mode, (double)ocp_max_norm(e, m));
}
// exact_add (arith.py:68-103) for any rounding mode and grid: rne/ieee takes the float32 paths, every other
// combination the float64 one.
MXQ_HD float exact_add_any(float a, float b, int e, int m, int mode, int grid) {
  if (mode == RM_RNE && grid == GRID_IEEE) return exact_add_rne(a, b, e, m);
  if (a == 0.0f) return b;
  if (b == 0.0f) return a;
  return q_float_em_d(dadd_rn((double)a, (double)b), e, m, mode, grid);
}
// scale_factor.ocp_no_clip (mxq/scale_factor.py:68-81): the ocp scale, doubled where amax / X rounded to the
// format without saturation overflows
MXQ_HD float scale_ocp_no_clip(float amax, int e, int m, int round, float scale_emax) {
  float X = scale_ocp(amax, ocp_emax(e, m), scale_emax);
  float r = q_microsoft(x86_div(amax, X), m + 2, e, ocp_max_norm(e, m), round, false);
  return isinf_f(r) ? mul_rn(X, 2.0f) : X;
}

// ------------------------------------------------------------------------ Arithmetic (_arithmetic.py)
// The two datapaths of mxq/matmul/_arithmetic.py as plain parameters (mirrors mxq_arith of include/mxq_b200.h).
struct ArithP {
  int kind;               // 0 MXQUANT, 1 MXGEMMINI
  int prod_e, prod_m;
  int has_floor;
  float floor_thr, sat_limit, sat_value;
};
// product: MXQUANT (:70) qtorch ties-away of the float32 product; MXGEMMINI (:131) truncate, flush, saturate
MXQ_HD float ar_product(const ArithP& A, float a, float b) {
  if (A.kind == 0) return q_qtorch(x86_mul(a, b), A.prod_e, A.prod_m, RM_TIES_AWAY);
  float x = truncate_significand(mul_rn(a, b), A.prod_m);
  if (A.has_floor) x = flush_below(x, A.floor_thr);
  return saturate(x, A.sat_limit, A.sat_value);
}
// MXGEMMINI's lane rounding (:125-127): bf16 on the bits for (8, 7), the ieee grid otherwise; -0 -> +0
MXQ_HD float lane_round(float x, int e, int m) {
  float r = (e == 8 && m == 7) ? bf16_rne(x) : q_ieee(x, e, m, RM_RNE);
  return unsigned_zero(r);
}
// acc_add: MXQUANT (:71) qtorch ties-away of the float32 sum; MXGEMMINI (:132) exact sum of the two lane values
MXQ_HD float ar_acc_add(const ArithP& A, float S, float p, int e, int m) {
  if (A.kind == 0) return q_float_em(x86_add(S, p), e, m, RM_TIES_AWAY, GRID_QTORCH);
  return exact_add_rne(lane_round(S, e, m), lane_round(p, e, m), e, m);
}
// tile_add: MXQUANT (:72) float32 add; MXGEMMINI (:133) exact bf16 add of the two bf16-rounded values
MXQ_HD float ar_tile_add(const ArithP& A, float C, float t) {
  if (A.kind == 0) return add_rn(C, t);
  return exact_add_rne(lane_round(C, 8, 7), lane_round(t, 8, 7), 8, 7);
}

// ------------------------------------------------------------------ fast forms for the block quantizer
// The same results as q_ocp_f / q_microsoft for EVERY float32 input (checked exhaustively on the host against
// them), with the powers of two built from the exponent field: the scale factors of these grids are always normal
// float32 numbers, and the two exact power-of-two multiplications of the microxcaling step fold into one.
MXQ_HD float round_nonneg(float k, int mode) {        // round_int of a value 0 <= k < 2^22
  if (mode == RM_RNE) return rint_small(k);
  if (mode == RM_TRUNCATE) return floor_small(k);
  return floor_small(add_rn(k, 0.5f));
}
MXQ_HD float q_ocp_bits(float x, int e, int m, int mode, float max_norm) {
  uint32_t u = f2u(x), a = u & 0x7fffffffu;
  // the binade's biased exponent field in place, clipped below at emin (float32 subnormals read biased 0); the
  // step is 2^s with biased field sb = eb - m (normal)
  const uint32_t lo = (uint32_t)(128 - bias_of(e)) << 23;
  const uint32_t e23 = (a & 0x7f800000u) > lo ? (a & 0x7f800000u) : lo;
  float k = round_nonneg(mul_rn(u2f(a), u2f(((uint32_t)(254 + m) << 23) - e23)), mode);     // |x| / 2^s
  float val = fminf(mul_rn(k, u2f(e23 - ((uint32_t)m << 23))), max_norm);                   // k * 2^s
  float r = u2f(f2u(val) | (u & 0x80000000u));
  return a == 0u ? 0.0f : (a >= 0x7f800000u ? x : r);
}
// A finite a >= 0 rounded to a multiple of the step q = 2^(E - 127 - m) by one float add, E << 23 = e23 the
// binade's biased exponent field in place (a < 2^(E - 126)): C = 1.5 * 2^23 * q has ulp q and a is far below C's
// binade width, so a + C lands on C + (a rounded to a multiple of q) in the add's own rounding (to nearest even, or
// toward zero = down), and subtracting C is exact (Sterbenz). Ties away (RM_TIES_AWAY) first adds q / 2 rounded to
// nearest, which is the reference's fl(a / q + 0.5) scaled by q, then rounds down. Needs m <= 21 (a + C must stay
// in C's binade, a < C / 3, which a < 2^(E - 126) gives when m <= 21) and C and q / 2 normal (E >= m + 2); callers
// keep a < 2^17.
MXQ_HD float step_round(float a, uint32_t e23, int m, int mode) {
  const float c = u2f(e23 + (((uint32_t)(23 - m) << 23) | 0x400000u));
  if (mode == RM_RNE) return sub_rn(add_rn(a, c), c);
  if (mode == RM_TRUNCATE) return sub_rn(add_rz(a, c), c);
  return sub_rn(add_rz(add_rn(a, u2f(e23 - ((uint32_t)(m + 1) << 23))), c), c);
}
// q_ocp_bits for finite |x| < 2^17 (a block quantizer's scaled value in a tile whose scales are powers of two):
// the same grid, its rounding by step_round
MXQ_HD float q_ocp_small(float x, int e, int m, int mode, float max_norm) {
  const uint32_t u = f2u(x), a = u & 0x7fffffffu;
  const uint32_t lo = (uint32_t)(128 - bias_of(e)) << 23;
  const uint32_t e23 = (a & 0x7f800000u) > lo ? (a & 0x7f800000u) : lo;
  const float val = fminf(step_round(u2f(a), e23, m, mode), max_norm);
  return a == 0u ? 0.0f : u2f(f2u(val) | (u & 0x80000000u));
}

// q_ieee_f for finite |x| < 2^17, m <= 21 and bias(e) + m <= 126 (every such float(e, m) with e <= 7): the same step
// 2^(max(E, emin) - m), its rounding by step_round; overflow past 2^(emax + 1) to Inf, a nonzero value that rounds
// to zero to +0, a zero unchanged
MXQ_HD float q_ieee_small(float x, int e, int m, int mode) {
  const uint32_t u = f2u(x), a = u & 0x7fffffffu;
  if (a == 0u) return x;
  const int b = bias_of(e);
  const uint32_t lo = (uint32_t)(128 - b) << 23;
  const uint32_t e23 = (a & 0x7f800000u) > lo ? (a & 0x7f800000u) : lo;
  float val = step_round(u2f(a), e23, m, mode);
  if (f2u(val) >= (uint32_t)(128 + b) << 23) val = inf_f();                 // >= 2^(emax + 1)
  return val == 0.0f ? 0.0f : u2f(f2u(val) | (u & 0x80000000u));
}

// q_microsoft with saturate_normals=True and exp_bits > 0
MXQ_HD float q_microsoft_sat(float A, int bits, int exp_bits, float max_norm, int round) {
  uint32_t u = f2u(A), a = u & 0x7fffffffu;
  if (a >= 0x7f7fffd4u) return q_microsoft(A, bits, exp_bits, max_norm, round, true);  // inf, NaN, log2 -> 128
  int min_exp = 2 - (1 << (exp_bits - 1));
  int pe = a ? floor_log2_rn(u2f(a)) : 0;              // floor(log2(|A| + (A == 0)))
  pe = pe > min_exp ? pe : min_exp;
  float t = mul_rn(A, u2f((uint32_t)(125 + bits - pe) << 23));          // A / 2^pe * 2^(bits-2)
  float absA = abs_f(t), r;
  if (round == MS_FLOOR) {                             // |t| < 2^(bits-1): the small-value roundings apply
    r = floor_small(absA);
  } else if (round == MS_NEAREST) {
    r = floor_small(add_rn(absA, 0.5f));
  } else {
    float y = sub_rn(absA, 0.5f), h = mul_rn(y, 0.5f);
    r = sub_rn(floor_small(add_rn(absA, 0.5f)), (y >= 0.0f && floor_small(h) == h) ? 1.0f : 0.0f);
  }
  r = u2f(f2u(r) | (u & 0x80000000u));                 // sign(A) * r: -0 for a negative value rounding to zero
  float out = mul_rn(r, u2f((uint32_t)(129 - bits + pe) << 23));        // / 2^(bits-2) * 2^pe
  out = fminf(fmaxf(out, -max_norm), max_norm);
  return a == 0u ? 0.0f : out;
}

// The microxcaling step for an OCP element format (exp_bits 2..5, so min_exp >= -14), saturating: q_microsoft's
// result for every float32 input, cheaper.
//   * nearest / even: the private exponent may be the exact floor(log2|A|) instead of the reference's rounded-up
//     log2 -- they differ only within 44 ulps below a power of two 2^k, where both step sizes round to 2^k;
//     floor mode keeps the reference's rule (there the two steps floor to different values);
//   * float32 subnormals take the clipped exponent min_exp either way.
// The rounding itself stays the reference's float32 formula: |t| + 0.5 is rounded before the floor, which is not
// rint (t = 0.5 - 2^-25 gives 1), so "even" keeps its mask on exact even ties.
// q_microsoft_ocp_core is the part for |A| < 0x7f7fffd4 (finite, log2 below 128); q_microsoft_ocp adds the rest.
MXQ_HD float q_microsoft_ocp_core(float A, int bits, int exp_bits, float max_norm, int round) {
  const uint32_t u = f2u(A), a = u & 0x7fffffffu;
  const int min_exp = 2 - (1 << (exp_bits - 1));
  // e23: the private exponent's biased field in place, E << 23 with E = pe + 127 (pe clipped below at min_exp)
  uint32_t e23;
  if (round == MS_FLOOR) {
    int pe = a ? floor_log2_rn(u2f(a)) : 0;
    e23 = (uint32_t)((pe > min_exp ? pe : min_exp) + 127) << 23;
  } else {
    const uint32_t lo = (uint32_t)(min_exp + 127) << 23;
    e23 = (a & 0x7f800000u) > lo ? (a & 0x7f800000u) : lo;
  }
  const float t = mul_rn(u2f(a), u2f(((uint32_t)(252 + bits) << 23) - e23));  // |A| / 2^pe * 2^(bits-2), < 2^(bits-1)
  float r;
  if (round == MS_FLOOR) {
    r = floor_small(t);
  } else if (round == MS_NEAREST) {
    r = floor_small(add_rn(t, 0.5f));
  } else {
    // floor(fl(t + 0.5)) minus 1 when t - 0.5 is an even integer: for every t >= 0 that is rint(t) (ties to even),
    // except t = 0.5 - 2^-25, the one value whose float32 sum with 0.5 ties up to 1.0
    r = add_rn(rint_small(t), f2u(t) == 0x3effffffu ? 1.0f : 0.0f);
  }
  const float val = fminf(mul_rn(r, u2f(e23 - ((uint32_t)(bits - 2) << 23))), max_norm);   // r * 2^(pe-bits+2)
  return a == 0u ? 0.0f : u2f(f2u(val) | (u & 0x80000000u));
}
// q_microsoft_ocp_core for |A| < 2^17 with the rounding by step_round (step 2^(pe - bits + 2)): nearest is
// floor(fl(t + 0.5)) = ties away, floor rounds down, and even is RNE except at t = 0.5 - 2^-25 (only reached with
// pe clipped at min_exp, i.e. at one value of |A|), which rounds up to one step.
MXQ_HD float q_microsoft_ocp_small(float A, int bits, int exp_bits, float max_norm, int round) {
  const uint32_t u = f2u(A), a = u & 0x7fffffffu;
  const int min_exp = 2 - (1 << (exp_bits - 1)), m = bits - 2;
  const uint32_t lo = (uint32_t)(min_exp + 127) << 23;
  uint32_t e23;
  if (round == MS_FLOOR) {
    int pe = a ? floor_log2_rn(u2f(a)) : 0;
    e23 = (uint32_t)((pe > min_exp ? pe : min_exp) + 127) << 23;
  } else {
    e23 = (a & 0x7f800000u) > lo ? (a & 0x7f800000u) : lo;
  }
  float r;
  if (round == MS_FLOOR) {
    r = step_round(u2f(a), e23, m, RM_TRUNCATE);
  } else if (round == MS_NEAREST) {
    r = step_round(u2f(a), e23, m, RM_TIES_AWAY);
  } else {
    const uint32_t a_star = lo - ((uint32_t)(m + 2) << 23) + 0x7fffffu;     // (0.5 - 2^-25) * 2^(min_exp - m)
    r = step_round(u2f(a), e23, m, RM_RNE);
    if (a == a_star) r = u2f(lo - ((uint32_t)m << 23));
  }
  const float val = fminf(r, max_norm);
  return a == 0u ? 0.0f : u2f(f2u(val) | (u & 0x80000000u));
}
MXQ_HD float q_microsoft_ocp(float A, int bits, int exp_bits, float max_norm, int round) {
  if ((f2u(A) & 0x7fffffffu) >= 0x7f7fffd4u) return q_microsoft(A, bits, exp_bits, max_norm, round, true);
  return q_microsoft_ocp_core(A, bits, exp_bits, max_norm, round);
}

}  // namespace mxq
