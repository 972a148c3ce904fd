/* TEST INFRASTRUCTURE — the CPU oracle for the mxq hot path. Not part of the product: only tests/, the smoke
 * check and bench.py's CPU-baseline leg load it, and only to check or to time against.
 *
 * A literal C restatement of the reference algorithm (chloe-wong/microscaling-quant, paths mxq/...): each
 * function follows the torch operations of the function it cites, in the same order, with float32 or float64
 * arithmetic as the reference has it and libm for frexp/floor/trunc/rint. It deliberately shares no code with
 * the CUDA kernels' numerics header: the two derivations of every rounding check each other, and both are
 * pinned to golden vectors produced by the reference itself (tests/golden/make_golden.py).
 *
 * Two library semantics the reference inherits from torch are restated explicitly:
 *   - floor(torch.log2(x)) on float32 is floor(RN32(log2 x)): computed here as floorf((float)log2((double)x));
 *   - NaN propagation follows the x86 host: first NaN operand, quieted; invalid operation -> 0xFFC00000.
 *     (It matters only where a NaN's sign bit reaches qtorch's bit rounding.)
 * Built with -O2 -ffp-contract=off -fno-fast-math (oracle/Makefile), so every float operation is one IEEE op.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------------------------ helpers */
static inline uint32_t fb(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float bf(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }
static inline uint64_t db(double x) { uint64_t u; memcpy(&u, &x, 8); return u; }
static inline double bd(uint64_t u) { double x; memcpy(&x, &u, 8); return x; }
static inline int is_nan(float x) { return x != x; }
static inline int is_nand(double x) { return x != x; }
static inline float quiet(float x) { return bf(fb(x) | 0x00400000u); }

/* x86 binary operation result for NaN operands */
static inline float nanfix(float a, float b, float r) {
  if (is_nan(a)) return quiet(a);
  if (is_nan(b)) return quiet(b);
  if (is_nan(r)) return bf(0xffc00000u);
  return r;
}
static inline float fmul(float a, float b) { volatile float r = a * b; return nanfix(a, b, r); }
static inline float fadd(float a, float b) { volatile float r = a + b; return nanfix(a, b, r); }
static inline float fsub(float a, float b) { volatile float r = a - b; return nanfix(a, b, r); }
static inline float fdiv(float a, float b) { volatile float r = a / b; return nanfix(a, b, r); }
/* torch.sign */
static inline float tsign(float x) { return (float)((0.0f < x) - (x < 0.0f)); }
static inline double tsignd(double x) { return (double)((0.0 < x) - (x < 0.0)); }
/* torch.log2 on float32: correctly rounded */
static inline float tlog2(float x) {
  if (is_nan(x)) return quiet(x);
  if (x < 0.0f) return bf(0x7fc00000u);
  return (float)log2((double)x);
}
/* torch.pow(2, t) / torch.exp2 of an integer-valued float32: exact power of two */
static inline float texp2f(float t) {
  if (is_nan(t)) return quiet(t);
  return (float)ldexp(1.0, t > 2000.0f ? 2000 : (t < -2000.0f ? -2000 : (int)t));
}
static inline double texp2d(double t) {
  if (is_nand(t)) return t;
  return ldexp(1.0, t > 5000.0 ? 5000 : (t < -5000.0 ? -5000 : (int)t));
}
static inline int bias(int e) { return (1 << (e - 1)) - 1; }                      /* float_em.py:45-47 */

enum { TIES_AWAY = 0, RNE = 1, TRUNCATE = 2 };
enum { GRID_QTORCH = 0, GRID_IEEE = 1, GRID_OCP = 2 };
enum { MS_NEAREST = 0, MS_FLOOR = 1, MS_EVEN = 2 };

/* ------------------------------------------------------------------------------- rounding (mxq/rounding) */
/* round_bits, mxq/rounding/__init__.py:51-55 (+ ties_away.py:5-6, rne.py:6-8, truncate.py:5-6) */
static inline int64_t round_bits1(int64_t bits, int64_t keep, int mode) {
  int64_t drop = 23 - keep, mask = ((int64_t)1 << drop) - 1, half = (int64_t)1 << (drop - 1), r;
  if (mode == TIES_AWAY) r = (bits + half) & ~mask;
  else if (mode == RNE) r = (bits + half - 1 + ((bits >> drop) & 1)) & ~mask;
  else r = bits & ~mask;
  return r & 0xffffffffLL;
}
EXPORT void o_round_bits(const int64_t* bits, const int64_t* keep, int64_t n, int mode, int64_t* out) {
  for (int64_t i = 0; i < n; i++) out[i] = round_bits1(bits[i], keep[i], mode);
}
/* round_int, mxq/rounding/__init__.py:58-61 */
static inline float round_int_f(float k, int mode) {
  if (mode == RNE) return rintf(k);                                  /* torch.round: half to even */
  if (mode == TRUNCATE) return truncf(k);
  return fmul(tsign(k), floorf(fadd(fabsf(k), 0.5f)));               /* ties_away.py:9-10 */
}
static inline double round_int_d(double k, int mode) {
  if (mode == RNE) return rint(k);
  if (mode == TRUNCATE) return trunc(k);
  if (is_nand(k)) return k;
  return tsignd(k) * floor(fabs(k) + 0.5);
}
EXPORT void o_round_int_f32(const float* k, int64_t n, int mode, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = round_int_f(k[i], mode);
}
EXPORT void o_round_int_f64(const double* k, int64_t n, int mode, double* out) {
  for (int64_t i = 0; i < n; i++) out[i] = round_int_d(k[i], mode);
}
/* bf16, mxq/rounding/__init__.py:64-85 */
static inline float bf16_1(float x) {
  if (is_nan(x)) return x;
  int64_t q = round_bits1((int64_t)fb(x), 7, RNE);
  return bf((uint32_t)q);
}
EXPORT void o_bf16(const float* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = bf16_1(x[i]);
}

/* ------------------------------------------------------------------------- float_em (element_quant) */
/* _qtorch, mxq/element_quant/float_em.py:64-84 */
static inline float qtorch1(float z, int e, int m, int mode) {
  int64_t bits = (int64_t)fb(z);
  int64_t q = round_bits1(bits, m, mode);
  int64_t L = bias(e), min_store = 127 - L, max_store = 127 + L;
  int64_t exp_store = (q >> 23) & 0xff, sign = bits & 0x80000000LL;
  int64_t max_num = sign | (max_store << 23) | (0x007fffffLL & ~(((int64_t)1 << (23 - m)) - 1));
  int64_t min_num = sign | (min_store << 23);
  int64_t middle = (min_store - 1) * ((int64_t)1 << 23);
  int64_t q_mag = q & 0x7fffffffLL;
  if (exp_store > max_store) q = max_num;
  int below = exp_store < min_store;
  if (below && q_mag > middle) q = min_num;
  if (below && !(q_mag > middle)) q = 0;
  return bf((uint32_t)(q & 0xffffffffLL));
}
/* _ieee, float_em.py:87-110, in float64 (used for e == 8 and float64 input) */
static double ieee_d(double x, int e, int m, int mode) {
  int b = bias(e), emin = 1 - b, emax = b;
  double ax = fabs(x);
  int finite_nz = isfinite(x) && ax != 0.0;
  int ex;
  frexp(finite_nz ? ax : 1.0, &ex);
  double E = (double)(ex - 1);
  double step = texp2d((E > emin ? E : (double)emin) - m);
  double k = round_int_d(ax / step, mode);
  double val = k * step;
  if (val >= ldexp(1.0, emax + 1)) val = INFINITY;
  double out = finite_nz ? copysign(val, x) : x;
  if (e < 8 && finite_nz && val == 0.0) out = 0.0;
  return out;
}
/* _ieee in float32 (e < 8, float32 input) */
static float ieee_f(float x, int e, int m, int mode) {
  int b = bias(e), emin = 1 - b, emax = b;
  float ax = fabsf(x);
  int finite_nz = isfinite(x) && ax != 0.0f;
  int ex;
  frexpf(finite_nz ? ax : 1.0f, &ex);
  float E = (float)(ex - 1);
  float step = texp2f((E > emin ? E : (float)emin) - m);
  float k = round_int_f(ax / step, mode);
  float val = k * step;
  if (val >= ldexpf(1.0f, emax + 1)) val = INFINITY;
  float out = finite_nz ? copysignf(val, x) : x;
  if (finite_nz && val == 0.0f) out = 0.0f;
  return out;
}
/* the OCP element formats (mxq/element_quant/formats.py:23-29): (e, m) -> max_norm */
static double ocp_max_norm(int e, int m) {
  if (e == 4 && m == 3) return 448.0;
  if (e == 5 && m == 2) return 57344.0;
  if (e == 3 && m == 2) return 28.0;
  if (e == 2 && m == 3) return 7.5;
  if (e == 2 && m == 1) return 6.0;
  return -1.0;
}
/* _ocp, float_em.py:113-134 */
static float ocp_f(float x, int e, int m, int mode) {
  int emin = 1 - bias(e);
  float mn = (float)ocp_max_norm(e, m);
  float ax = fabsf(x);
  int finite_nz = isfinite(x) && ax != 0.0f;
  int ex;
  frexpf(finite_nz ? ax : 1.0f, &ex);
  float E = (float)(ex - 1);
  float step = texp2f((E > emin ? E : (float)emin) - m);
  float val = round_int_f(ax / step, mode) * step;
  if (val > mn) val = mn;                                            /* clamp(max=max_norm) */
  float out = finite_nz ? copysignf(val, x) : x;
  if (x == 0.0f) out = 0.0f;
  return out;
}
static double ocp_d(double x, int e, int m, int mode) {
  int emin = 1 - bias(e);
  double mn = ocp_max_norm(e, m);
  double ax = fabs(x);
  int finite_nz = isfinite(x) && ax != 0.0;
  int ex;
  frexp(finite_nz ? ax : 1.0, &ex);
  double E = (double)(ex - 1);
  double step = texp2d((E > emin ? E : (double)emin) - m);
  double val = round_int_d(ax / step, mode) * step;
  if (val > mn) val = mn;
  double out = finite_nz ? copysign(val, x) : x;
  if (x == 0.0) out = 0.0;
  return out;
}
static inline float d2f(double x) {                                   /* tensor.to(float32) on x86 */
  return (float)x;
}
/* float_em.quantize, float_em.py:50-61, float32 input */
static float float_em1(float z, int e, int m, int mode, int grid) {
  if (e == 8 && m == 23) return z;
  if (grid == GRID_QTORCH) return qtorch1(z, e, m, mode);
  if (grid == GRID_IEEE) return e == 8 ? d2f(ieee_d((double)z, e, m, mode)) : ieee_f(z, e, m, mode);
  return ocp_f(z, e, m, mode);
}
/* float64 input */
static float float_em1_d(double z, int e, int m, int mode, int grid) {
  if (e == 8 && m == 23) return d2f(ieee_d(z, 8, 23, mode));
  if (grid == GRID_QTORCH) return qtorch1(d2f(z), e, m, mode);
  if (grid == GRID_IEEE) return d2f(ieee_d(z, e, m, mode));
  return d2f(ocp_d(z, e, m, mode));
}
EXPORT void o_float_em_f32(const float* z, int64_t n, int e, int m, int mode, int grid, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = float_em1(z[i], e, m, mode, grid);
}
EXPORT void o_float_em_f64(const double* z, int64_t n, int e, int m, int mode, int grid, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = float_em1_d(z[i], e, m, mode, grid);
}

/* --------------------------------------------------------------------------- microxcaling element step */
/* _quantize_elemwise_core, mxq/microxcaling/elemwise.py:63-151 (dense, allow_denorm=True) */
static float microsoft1(float A, int bits, int exp_bits, float max_norm, int round, int saturate) {
  float out = A, pe = 0.0f;
  if (exp_bits != 0) {
    pe = floorf(tlog2(fadd(fabsf(A), A == 0.0f ? 1.0f : 0.0f)));
    float min_exp = (float)(-(1 << (exp_bits - 1)) + 2);
    if (pe < min_exp) pe = min_exp;                                  /* clip(min=): NaN stays */
    out = fmul(fdiv(out, texp2f(pe)), (float)(1 << (bits - 2)));     /* _safe_lshift */
  } else {
    out = fmul(out, (float)(1 << (bits - 2)));
  }
  /* _round_mantissa, elemwise.py:29-60 */
  float absA = fabsf(out);
  if (round == MS_FLOOR) {
    out = fmul(tsign(out), floorf(absA));
  } else if (round == MS_NEAREST) {
    out = fmul(tsign(out), floorf(fadd(absA, 0.5f)));
  } else {
    float y = fsub(absA, 0.5f);
    float md = fmodf(y, 2.0f);                                       /* torch.remainder(y, 2) */
    if (md != 0.0f && md < 0.0f) md = fadd(md, 2.0f);
    float maskA = (md == 0.0f) ? 1.0f : 0.0f;
    out = fmul(tsign(out), fsub(floorf(fadd(absA, 0.5f)), maskA));
  }
  if (exp_bits != 0) out = fmul(fdiv(out, (float)(1 << (bits - 2))), texp2f(pe));   /* _safe_rshift */
  else out = fdiv(out, (float)(1 << (bits - 2)));
  if (saturate || exp_bits == 0) {
    if (!is_nan(out)) out = fminf(fmaxf(out, -max_norm), max_norm);
  } else if (fabsf(out) > max_norm) {
    out = fmul(tsign(out), INFINITY);
  }
  if (A == INFINITY) out = INFINITY;
  if (A == -INFINITY) out = -INFINITY;
  return out;
}
EXPORT void o_microsoft(const float* A, int64_t n, int bits, int exp_bits, float max_norm, int round, int saturate,
                        float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = microsoft1(A[i], bits, exp_bits, max_norm, round, saturate);
}

/* ------------------------------------------------------------------------------ scale rules (step 1) */
/* scale_factor.mxquant, mxq/scale_factor.py:40-44; fl is float32(floor) */
static float scale_mxquant1(float amax, float fl) {
  float c = (is_nan(amax) || !(amax < fl)) ? amax : fl;
  float sc = texp2f(floorf(tlog2(c)));
  return (is_nan(sc) || !(sc < fl)) ? sc : fl;
}
/* scale_factor.ocp, scale_factor.py:47-59 */
static float scale_ocp1(float amax, int emax, float scale_emax) {
  float se = floorf(tlog2(fadd(amax, fmul(0x1p-126f, amax == 0.0f ? 1.0f : 0.0f))));
  se = fsub(se, (float)emax);
  if (se > scale_emax) se = bf(0x7fc00000u);
  if (se < -scale_emax) se = -scale_emax;
  return texp2f(se);
}
EXPORT void o_scale_mxquant(const float* amax, int64_t n, float fl, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = scale_mxquant1(amax[i], fl);
}
EXPORT void o_scale_ocp(const float* amax, int64_t n, int emax, float scale_emax, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = scale_ocp1(amax[i], emax, scale_emax);
}
/* the microxcaling parameters of an OCP format (mxq/microxcaling/formats.py:61-125) */
static void ms_params(int e, int m, int* bits, int* emax, float* max_norm) {
  *bits = m + 2;
  if (e == 4 && m == 3) { *emax = 8; *max_norm = 448.0f; }
  else if (e == 5 && m == 2) { *emax = 15; *max_norm = 57344.0f; }
  else if (e == 3 && m == 2) { *emax = 4; *max_norm = 28.0f; }
  else if (e == 2 && m == 3) { *emax = 2; *max_norm = 7.5f; }
  else { *emax = 2; *max_norm = 6.0f; }
}
/* scale_factor.ocp_no_clip, scale_factor.py:68-81 */
static float scale_ocp_no_clip1(float amax, int e, int m, int round, float scale_emax) {
  int bits, emax; float mn;
  ms_params(e, m, &bits, &emax, &mn);
  float X = scale_ocp1(amax, emax, scale_emax);
  float r = microsoft1(fdiv(amax, X), bits, e, mn, round, 0);
  return isinf(r) ? fmul(X, 2.0f) : X;
}
EXPORT void o_scale_ocp_no_clip(const float* amax, int64_t n, int e, int m, int round, float scale_emax, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = scale_ocp_no_clip1(amax[i], e, m, round, scale_emax);
}

/* ------------------------------------------------------------------------- block quantizers (compose) */
/* One spec for every named quantizer: mxq/block/{mxquant,mxgemmini,ocp}.py on top of _driver.compose. */
typedef struct {
  int32_t family;      /* 0 passthrough (FP32), 1 mxquant, 2 mxgemmini, 3 ocp */
  int32_t e, m;        /* element format */
  int32_t rounding;    /* RoundMode for mxquant/mxgemmini; MsRound for ocp */
  float scale_floor;   /* mxquant / mxgemmini scale floor, as float32 */
  int32_t placement;   /* ocp: 0 top, 1 below_top, 2 no_clip */
  float scale_emax;    /* ocp: float32(2^(scale_bits-1) - 1) */
  int32_t via_e, via_m;/* mxgemmini: pre-round on the ieee grid; via_e = 0 for none */
} OSpec;

static float elem1(const OSpec* s, float z) {
  if (s->family == 1) return float_em1(z, s->e, s->m, TIES_AWAY, GRID_QTORCH);      /* mxquant.py:26-28 */
  if (s->family == 2) {                                                               /* mxgemmini.py:50-59 */
    if (s->via_e) z = float_em1(z, s->via_e, s->via_m, s->rounding, GRID_IEEE);
    return float_em1(z, s->e, s->m, s->rounding, GRID_OCP);
  }
  int bits, emax; float mn;                                                           /* ocp.py:45-46 */
  ms_params(s->e, s->m, &bits, &emax, &mn);
  return microsoft1(z, bits, s->e, mn, s->rounding, 1);
}
static float scale1(const OSpec* s, float amax) {
  if (s->family == 1 || s->family == 2) return scale_mxquant1(amax, s->scale_floor);
  int bits, emax; float mn;
  ms_params(s->e, s->m, &bits, &emax, &mn);
  if (s->placement == 0) return scale_ocp1(amax, emax, s->scale_emax);
  if (s->placement == 1) return scale_ocp1(amax, emax - 1, s->scale_emax);
  return scale_ocp_no_clip1(amax, s->e, s->m, s->rounding, s->scale_emax);
}
/* _driver.compose (mxq/block/_driver.py:45-66) for a tensor viewed as [outer, len, inner] with the blocks along
 * len: amax over each (zero-padded) block, X = scale(amax), P = elem(data / X); X is [outer, nb, inner]. */
EXPORT void o_block_quantize(const float* V, int64_t outer, int64_t len, int64_t inner, int64_t bs, const OSpec* s,
                             float* P, float* X) {
  int64_t nb = (len + bs - 1) / bs;
  for (int64_t o = 0; o < outer; o++)
    for (int64_t b = 0; b < nb; b++)
      for (int64_t j = 0; j < inner; j++) {
        int64_t l0 = b * bs, l1 = l0 + bs < len ? l0 + bs : len;
        float amax = 0.0f;
        int nan = 0;
        for (int64_t l = l0; l < l1; l++) {
          float a = fabsf(V[(o * len + l) * inner + j]);
          if (is_nan(a)) nan = 1;
          else if (a > amax) amax = a;
        }
        if (nan) amax = bf(0x7fc00000u);                   /* amax of a block holding NaN: +NaN (probed) */
        float x = s->family == 0 ? 1.0f : scale1(s, amax);
        X[(o * nb + b) * inner + j] = x;
        for (int64_t l = l0; l < l1; l++) {
          int64_t i = (o * len + l) * inner + j;
          float z = s->family == 0 ? V[i] : fdiv(V[i], x);
          P[i] = s->family == 0 ? z : elem1(s, z);
        }
      }
}

/* ------------------------------------------------------------------------------------ arith (arith.py) */
static inline int fits_float32(int e, int m) { return (1 << e) - 1 + m <= 24; }       /* arith.py:21-30 */
/* _round_pair, arith.py:41-65 */
static float round_pair(float s, float t, int e, int m) {
  int b = bias(e), emin = 1 - b, emax = b;
  float ax = fabsf(s);
  int finite_nz = isfinite(s) && ax != 0.0f;
  int ex;
  frexpf(finite_nz ? ax : 1.0f, &ex);
  float E = (float)(ex - 1);
  float step = texp2f((E > emin ? E : (float)emin) - m);
  float k = ax / step, kf = floorf(k);
  int tie = (k - kf) == 0.5f;
  int up = (tsign(s) * t) > 0.0f;
  float ko = (tie && t != 0.0f) ? (up ? kf + 1.0f : kf) : rintf(k);
  float val = ko * step;
  if (val >= ldexpf(1.0f, emax + 1)) val = INFINITY;
  float out = finite_nz ? copysignf(val, s) : s;
  if (finite_nz && val == 0.0f) out = 0.0f;
  return out;
}
/* exact_add, arith.py:68-103 */
static float exact_add1(float a, float b, int e, int m, int mode, int grid) {
  float q;
  if (mode == RNE && grid == GRID_IEEE && fits_float32(e, m)) {
    q = float_em1(fadd(a, b), e, m, RNE, GRID_IEEE);
  } else if (mode == RNE && grid == GRID_IEEE && e <= 7) {
    volatile float s = a + b;                                         /* _two_sum, arith.py:33-38 */
    volatile float bb = s - a;
    volatile float t1 = s - bb, t2 = a - t1, t3 = b - bb;
    volatile float t = t2 + t3;
    q = round_pair(s, t, e, m);
  } else {
    volatile double s = (double)a + (double)b;
    q = float_em1_d(s, e, m, mode, grid);
  }
  return a == 0.0f ? b : (b == 0.0f ? a : q);
}
EXPORT void o_exact_add(const float* a, const float* b, int64_t n, int e, int m, int mode, int grid, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = exact_add1(a[i], b[i], e, m, mode, grid);
}
/* truncate_significand, arith.py:106-117 */
static float trunc_sig1(float x, int m) {
  float ax = fabsf(x);
  int nz = isfinite(x) && ax != 0.0f;
  int ex;
  float mant = frexpf(nz ? ax : 1.0f, &ex);
  float k = truncf(mant * (float)(1LL << (m + 1)));
  float t = (k / (float)(1LL << m)) * (float)ldexp(1.0, ex - 1);     /* torch.ldexp: x * 2^e */
  return nz ? copysignf(t, x) : x;
}
EXPORT void o_truncate_significand(const float* x, int64_t n, int m, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = trunc_sig1(x[i], m);
}
/* flush_product, arith.py:120-124 */
static inline float flush1(float x, float thr) { return fabsf(x) < thr ? 0.0f : x; }
EXPORT void o_flush_product(const float* x, int64_t n, float thr, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = flush1(x[i], thr);
}
/* saturate, arith.py:127-137 */
static inline float saturate1(float x, float limit, float value) {
  float ax = fabsf(x);
  return fmul(tsign(x), ax > limit ? value : ax);
}
EXPORT void o_saturate(const float* x, int64_t n, float limit, float value, float* out) {
  for (int64_t i = 0; i < n; i++) out[i] = saturate1(x[i], limit, value);
}

/* ------------------------------------------------------------------------ Arithmetic (_arithmetic.py) */
typedef struct {
  int32_t kind;          /* 0 MXQUANT(prod_e, prod_m), 1 MXGEMMINI(prod_e, prod_m, prod_floor) */
  int32_t prod_e, prod_m;
  int32_t has_floor;     /* MXGEMMINI: prod_floor is not None */
  float floor_thr;       /* float32(2^prod_floor) */
  float sat_limit, sat_value;
} OArith;

static inline float product1(const OArith* ar, float a, float b) {
  if (ar->kind == 0)                                                   /* _arithmetic.py:70 */
    return float_em1(fmul(a, b), ar->prod_e, ar->prod_m, TIES_AWAY, GRID_QTORCH);
  float x = trunc_sig1(fmul(a, b), ar->prod_m);                        /* _arithmetic.py:131 */
  if (ar->has_floor) x = flush1(x, ar->floor_thr);
  return saturate1(x, ar->sat_limit, ar->sat_value);
}
static inline float lane1(float x, int e, int m) {                      /* _arithmetic.py:125-127 */
  float r = (e == 8 && m == 7) ? bf16_1(x) : float_em1(x, e, m, RNE, GRID_IEEE);
  return r == 0.0f ? 0.0f : r;
}
static inline float acc_add1(const OArith* ar, float S, float p, int e, int m) {
  if (ar->kind == 0) return float_em1(fadd(S, p), e, m, TIES_AWAY, GRID_QTORCH);   /* :71 */
  return exact_add1(lane1(S, e, m), lane1(p, e, m), e, m, RNE, GRID_IEEE);        /* :132 */
}
static inline float tile_add1(const OArith* ar, float C, float t) {
  if (ar->kind == 0) return fadd(C, t);                                              /* :72 */
  return exact_add1(lane1(C, 8, 7), lane1(t, 8, 7), 8, 7, RNE, GRID_IEEE);          /* :133 */
}

/* ------------------------------------------------------------------------------------------ reducers */
/* systolic, mxq/matmul/_systolic.py:23-62: A K x M, B K x N, X one row per block of K; Y M x N.
 * Every output element is its own K-sum: the loop runs per (i, j) over output rows [m0, m1), so callers can split
 * the rows over threads. */
EXPORT void o_systolic(const float* PA, const float* XA, const float* PB, const float* XB, int64_t K, int64_t M,
                       int64_t N, int64_t bs, int64_t size, const OArith* ar, const int32_t* se, const int32_t* sm,
                       float* Y, int64_t m0, int64_t m1) {
  for (int64_t i = m0; i < m1; i++)
    for (int64_t j = 0; j < N; j++) {
      float C = 0.0f;
      for (int64_t g = 0; g < K; g += bs) {
        int64_t g_end = g + bs < K ? g + bs : K;
        float sc = fmul(XA[(g / bs) * M + i], XB[(g / bs) * N + j]);    /* _common.scale_map */
        for (int64_t kb = g; kb < g_end; kb += size) {
          int64_t ke = kb + size < g_end ? kb + size : g_end;
          float S = 0.0f;
          for (int64_t k = kb; k < ke; k++) {
            float p = product1(ar, PA[k * M + i], PB[k * N + j]);
            S = acc_add1(ar, S, p, se[k % size], sm[k % size]);
          }
          C = tile_add1(ar, C, fmul(S, sc));
        }
      }
      Y[i * N + j] = C;
    }
}

/* adder_tree, mxq/matmul/_adder.py:23-71: `size` products, log2(size) levels of adjacent-pair acc_add */
EXPORT void o_adder_tree(const float* PA, const float* XA, const float* PB, const float* XB, int64_t K, int64_t M,
                         int64_t N, int64_t bs, int64_t size, const OArith* ar, const int32_t* le, const int32_t* lm,
                         float* Y, int64_t m0, int64_t m1) {
  int levels = 0;
  while ((1LL << levels) < size) levels++;
  for (int64_t i = m0; i < m1; i++) {
    float* p = (float*)malloc(sizeof(float) * size);
    for (int64_t j = 0; j < N; j++) {
      float C = 0.0f;
      for (int64_t g = 0; g < K; g += bs) {
        int64_t g_end = g + bs < K ? g + bs : K;
        float sc = fmul(XA[(g / bs) * M + i], XB[(g / bs) * N + j]);
        for (int64_t k0 = g; k0 < g_end; k0 += size) {
          int64_t k1 = k0 + size < g_end ? k0 + size : g_end;
          for (int64_t t = 0; t < size; t++)
            p[t] = (k0 + t < k1) ? product1(ar, PA[(k0 + t) * M + i], PB[(k0 + t) * N + j]) : 0.0f;
          int64_t len = size;
          for (int l = 0; l < levels; l++) {
            for (int64_t t = 0; t < len; t += 2) p[t / 2] = acc_add1(ar, p[t], p[t + 1], le[l], lm[l]);
            len /= 2;
          }
          C = tile_add1(ar, C, fmul(p[0], sc));
        }
      }
      Y[i * N + j] = C;
    }
    free(p);
  }
}

/* anchor_tree, mxq/matmul/_anchor.py:39-138 */
static inline double log2_floor_anchor(float x) {                     /* _anchor.py:39-44 */
  if (!isfinite(x)) x = 0.5f;
  int ex;
  frexpf(fabsf(x), &ex);
  return (double)(ex - 1);
}
static inline double keep1(double x, int drop_rne) { return drop_rne ? rint(x) : trunc(x); }   /* :47-49 */

typedef struct {
  int32_t width, nbits, drop_rne, headroom, has_emin, emin;   /* nbits = levels + 1 entries per tree */
} OAnchor;

/* one tree, _anchor.py:52-67: p/label width products and labels, c the running sum */
static float anchor_tree1(const OArith* ar, const float* p, const double* label, float c, int e, int m,
                          const OAnchor* an, const int32_t* bits) {
  int w = an->width;
  double top = (c != 0.0f) ? log2_floor_anchor(c) - 1.0 : -INFINITY;
  for (int t = 0; t < w; t++) {
    double lk = (p[t] != 0.0f) ? label[t] : -INFINITY;
    top = top > lk ? top : lk;                                          /* torch.maximum */
  }
  double anchor = (isfinite(top) ? top : 0.0) + an->headroom;
  double grid = texp2d(anchor + 2 - bits[0]);
  double x[64];
  int n = w + 1;
  for (int t = 0; t < w; t++) x[t] = keep1((double)p[t] / grid, an->drop_rne);
  x[w] = keep1((double)c / grid, an->drop_rne);
  for (int level = 1; level < an->nbits; level++) {
    int k = 0;
    for (int t = 0; t + 1 < n; t += 2) x[k++] = x[t] + x[t + 1];
    if (n % 2) x[k++] = x[n - 1];
    n = k;
    if (bits[level] != bits[level - 1]) {
      double d = ldexp(1.0, bits[level - 1] - bits[level]);
      for (int t = 0; t < n; t++) x[t] = keep1(x[t] / d, an->drop_rne);
    }
  }
  float s = (float)(x[0] * texp2d(anchor + 2 - bits[an->nbits - 1]));
  return acc_add1(ar, 0.0f, s, e, m);                                  /* S4, _anchor.py:67 */
}

EXPORT void o_anchor_tree(const float* PA, const float* XA, const float* PB, const float* XB, int64_t K, int64_t M,
                          int64_t N, int64_t bs, int64_t size, const OArith* ar, const int32_t* te,
                          const int32_t* tm, const OAnchor* an, const int32_t* tree_bits, float* Y, int64_t m0,
                          int64_t m1) {
  int64_t w = an->width, trees = size / w, nb = an->nbits;
  for (int64_t i = m0; i < m1; i++) {
    float p[64];
    double lab[64];
    for (int64_t j = 0; j < N; j++) {
      float C = 0.0f;
      for (int64_t g = 0; g < K; g += bs) {
        int64_t g_end = g + bs < K ? g + bs : K;
        float sc = fmul(XA[(g / bs) * M + i], XB[(g / bs) * N + j]);
        for (int64_t k0 = g; k0 < g_end; k0 += size) {
          int64_t n = (k0 + size < g_end ? k0 + size : g_end) - k0;
          float c = 0.0f;
          for (int64_t t = 0; t < trees; t++) {
            for (int64_t u = 0; u < w; u++) {
              int64_t k = t * w + u;
              if (k < n) {
                float a = PA[(k0 + k) * M + i], b = PB[(k0 + k) * N + j];
                double la = log2_floor_anchor(a), lb = log2_floor_anchor(b);
                if (an->has_emin) { la = la < an->emin ? an->emin : la; lb = lb < an->emin ? an->emin : lb; }
                p[u] = product1(ar, a, b);
                lab[u] = la + lb;
              } else {
                p[u] = 0.0f;
                lab[u] = 0.0;
              }
            }
            c = anchor_tree1(ar, p, lab, c, te[t], tm[t], an, tree_bits + t * nb);
          }
          C = tile_add1(ar, C, fmul(c, sc));
        }
      }
      Y[i * N + j] = C;
    }
  }
}

/* fp64_accum, mxq/_fp64_accum.py:24-29: dequantize (P * expand(X)) in float32, then a float64 dot product */
EXPORT void o_fp64_accum(const float* PA, const float* XA, const float* PB, const float* XB, int64_t K, int64_t M,
                         int64_t N, int64_t bs, float* Y, int64_t m0, int64_t m1) {
  for (int64_t i = m0; i < m1; i++)
    for (int64_t j = 0; j < N; j++) {
      double acc = 0.0;
      for (int64_t k = 0; k < K; k++) {
        double a = (double)(PA[k * M + i] * XA[(k / bs) * M + i]);
        double b = (double)(PB[k * N + j] * XB[(k / bs) * N + j]);
        acc += a * b;
      }
      Y[i * N + j] = (float)acc;
    }
}
