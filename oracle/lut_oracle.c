/* TEST INFRASTRUCTURE — CPU oracle for MX-Gemmini's look-up tables (mxq/lut/formats.py, mxq/lut/kmeans.py of
 * chloe-wong/microscaling-quant). A literal per-group restatement of the vectorised torch code; only tests/ and
 * bench.py's CPU-baseline leg use it. */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define EXPORT __attribute__((visibility("default")))
#define LUT_SIZE 16                                       /* formats.py:29 SIZE */

static inline uint32_t fbits(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }

/* ---------------------------------------------------------------------------------- formats.py */
/* fixed-point maps of the finder, formats.py:35-68 */
static int64_t fx_e3m2(int v) {
  int sign = (v >> 5) & 1, exp = (v >> 2) & 7, mant = v & 3;
  if (exp == 0 && mant == 0) return 0;
  int s_exp = exp == 0 ? -2 : exp - 3;
  int64_t sig = (exp == 0 ? 0 : 4) | mant;
  int64_t mag = ((sig << ((s_exp + 2) & 7)) & 0x1FF) & 0xFF;
  return sign ? -mag : mag;
}
static int64_t fx_e2m3(int v) {
  int sign = (v >> 5) & 1, exp = (v >> 3) & 3, mant = v & 7;
  int64_t mag = exp == 0 ? mant : ((int64_t)(8 + mant) << (exp - 1));
  return sign ? -mag : mag;
}
static int64_t fx_e5m2(int v) {
  int sign = (v >> 7) & 1, exp = (v >> 2) & 0x1F, mant = v & 3;
  if (exp == 0 && mant == 0) return 0;
  int64_t sig = (exp == 0 ? 0 : 4) | mant;
  int s_exp = exp == 0 ? 1 - 15 : exp - 15;
  int64_t mag = (sig << ((s_exp + 14) & 0x1F)) & 0xFFFFFFFFLL;
  return sign ? -mag : mag;
}
static int64_t fx_e4m3(int v) {
  int sign = (v >> 7) & 1, exp = (v >> 3) & 0xF, mant = v & 7;
  if (exp == 0 && mant == 0) return 0;
  int64_t sig = (exp == 0 ? 0 : 8) | mant;
  int s_exp = exp == 0 ? 1 - 7 : exp - 7;
  int64_t mag = (sig << ((s_exp + 6) & 0xF)) & 0x3FFFF;
  return sign ? -mag : mag;
}
static int64_t fx_of(int e, int m, int c) {
  if (e == 3 && m == 2) return fx_e3m2(c);
  if (e == 2 && m == 3) return fx_e2m3(c);
  if (e == 5 && m == 2) return fx_e5m2(c);
  return fx_e4m3(c);
}
/* the finder's |difference| mask (formats.py:72-73); 0 = none (E2M3) */
static int64_t fx_mask(int e, int m) {
  if (e == 3 && m == 2) return 0x1FF;
  if (e == 2 && m == 3) return 0;
  if (e == 5 && m == 2) return 0x1FFFFFFFFLL;
  return 0x7FFFF;
}
/* _tables (formats.py:83-111): every code's value and fixed point, and the finder-safe values sorted */
EXPORT int o_lut_format_tables(int e, int m, float* vals, int64_t* fx, float* safe) {
  int n = 1 << (1 + e + m), bias = (1 << (e - 1)) - 1, nsafe = 0;
  for (int c = 0; c < n; c++) {
    int s = (c >> (e + m)) & 1, ex = (c >> m) & ((1 << e) - 1), man = c & ((1 << m) - 1);
    double v;
    if (e == 5 && m == 2 && ex == 0x1F) v = man ? NAN : INFINITY;
    else if (ex == 0) v = man * ldexp(1.0, 1 - bias - m);
    else v = (1.0 + (double)man / (1 << m)) * ldexp(1.0, ex - bias);
    vals[c] = (float)(s ? -v : v);
    fx[c] = fx_of(e, m, c);
  }
  /* fixed point -> value, the smaller magnitude wins, in code order */
  int64_t* keys = (int64_t*)malloc(sizeof(int64_t) * n);
  float* kv = (float*)malloc(sizeof(float) * n);
  int nk = 0;
  for (int c = 0; c < n; c++) {
    float v = vals[c];
    if (v != v || isinf(v)) continue;
    int f = -1;
    for (int i = 0; i < nk; i++) if (keys[i] == fx[c]) { f = i; break; }
    if (f < 0) { keys[nk] = fx[c]; kv[nk] = v; nk++; }
    else if (fabsf(v) < fabsf(kv[f])) kv[f] = v;
  }
  /* sorted(set(values)): -0.0 == 0.0 keeps one zero */
  for (int i = 0; i < nk; i++) {
    int dup = 0;
    for (int j = 0; j < nsafe; j++) if (safe[j] == kv[i]) { dup = 1; break; }
    if (!dup) safe[nsafe++] = kv[i];
  }
  for (int i = 1; i < nsafe; i++)
    for (int j = i; j > 0 && safe[j - 1] > safe[j]; j--) { float t = safe[j]; safe[j] = safe[j - 1]; safe[j - 1] = t; }
  for (int i = 0; i < nsafe; i++) if (safe[i] == 0.0f) safe[i] = 0.0f;     /* a Python set keeps the first zero: +0.0 */
  free(keys); free(kv);
  return nsafe;
}

/* encode (formats.py:125-137): exact values -> the lowest code with the same float32 bits; -1 if none */
EXPORT int o_lut_encode(const float* T, int64_t n, int e, int m, int64_t* out) {
  int nc = 1 << (1 + e + m);
  float* vals = (float*)malloc(sizeof(float) * nc);
  int64_t* fx = (int64_t*)malloc(sizeof(int64_t) * nc);
  float safe[512];
  o_lut_format_tables(e, m, vals, fx, safe);
  int bad = 0;
  for (int64_t i = 0; i < n; i++) {
    int64_t code = -1;
    for (int c = 0; c < nc; c++) if (fbits(vals[c]) == fbits(T[i])) { code = c; break; }
    out[i] = code;
    if (code < 0) bad = 1;
  }
  free(vals); free(fx);
  return bad ? -1 : 0;
}

/* decode (formats.py:114-117): table[codes] with torch indexing (negative codes count from the end); -1 when a
   code is outside [-nc, nc) */
EXPORT int o_lut_decode(const int64_t* codes, int64_t n, int e, int m, float* out) {
  int nc = 1 << (1 + e + m);
  float* vals = (float*)malloc(sizeof(float) * nc);
  int64_t* fx = (int64_t*)malloc(sizeof(int64_t) * nc);
  float safe[512];
  o_lut_format_tables(e, m, vals, fx, safe);
  int bad = 0;
  for (int64_t i = 0; i < n; i++) {
    int64_t c = codes[i];
    if (c < -nc || c >= nc) { bad = 1; out[i] = 0.0f; continue; }
    out[i] = vals[c < 0 ? c + nc : c];
  }
  free(vals); free(fx);
  return bad ? -1 : 0;
}

/* finder (formats.py:140-159): nearest in fixed point, |diff| masked, first minimum */
EXPORT int o_lut_finder(const int64_t* codes, const float* T, int64_t K, int64_t n, int group, int e, int m,
                        int64_t* out) {
  int nc = 1 << (1 + e + m);
  int64_t ng = n >> group, mask = fx_mask(e, m);
  float* vals = (float*)malloc(sizeof(float) * nc);
  int64_t* fx = (int64_t*)malloc(sizeof(int64_t) * nc);
  float safe[512];
  o_lut_format_tables(e, m, vals, fx, safe);
  int64_t* tcode = (int64_t*)malloc(sizeof(int64_t) * ng * LUT_SIZE);
  /* fx_all[codes] first (formats.py:152): a code outside [-nc, nc) is an IndexError, a negative one counts from
     the end; then encode(T) (:153) */
  int rc = 0;
  for (int64_t i = 0; i < K * n; i++)
    if (codes[i] < -nc || codes[i] >= nc) rc = -2;
  if (rc == 0) rc = o_lut_encode(T, ng * LUT_SIZE, e, m, tcode);
  if (rc == 0) {
    for (int64_t k = 0; k < K; k++)
      for (int64_t j = 0; j < n; j++) {
        int64_t c = codes[k * n + j];
        int64_t f = fx[c < 0 ? c + nc : c];
        const int64_t* tc = tcode + (j >> group) * LUT_SIZE;
        int64_t best = 0, bd = 0;
        for (int t = 0; t < LUT_SIZE; t++) {
          int64_t d = f - fx[tc[t]];
          d = d < 0 ? -d : d;
          if (mask) d &= mask;
          if (t == 0 || d < bd) { bd = d; best = t; }
        }
        out[k * n + j] = best;
      }
  }
  free(vals); free(fx); free(tcode);
  return rc;
}

/* ---------------------------------------------------------------------------------- kmeans.py */
static int cmp_d(const void* a, const void* b) {
  double x = *(const double*)a, y = *(const double*)b;
  return (x > y) - (x < y);
}
/* _dedupe (kmeans.py:38-43): sorted, equal values merged, +inf after the last centre */
static void dedupe(double* C) {
  qsort(C, LUT_SIZE, sizeof(double), cmp_d);
  int dup[LUT_SIZE] = {0};
  for (int i = 1; i < LUT_SIZE; i++) dup[i] = C[i] == C[i - 1];
  for (int i = 1; i < LUT_SIZE; i++) if (dup[i]) C[i] = INFINITY;
  qsort(C, LUT_SIZE, sizeof(double), cmp_d);
}
/* first index i with a[i] >= v (torch.searchsorted, right=False) */
static int64_t lower_bound_d(const double* a, int64_t n, double v) {
  int64_t lo = 0, hi = n;
  while (lo < hi) { int64_t mid = (lo + hi) / 2; if (a[mid] < v) lo = mid + 1; else hi = mid; }
  return lo;
}
static int64_t lower_bound_f(const float* a, int64_t n, float v) {
  int64_t lo = 0, hi = n;
  while (lo < hi) { int64_t mid = (lo + hi) / 2; if (a[mid] < v) lo = mid + 1; else hi = mid; }
  return lo;
}

/* tables (kmeans.py:46-122): one SIZE-entry table per 2^group columns of P (K x n). Returns 0, or -1 when P holds
 * a value that is not a code of the format. T is ceil(n / 2^group) x SIZE. */
EXPORT int o_lut_tables(const float* P, int64_t K, int64_t n, int group, int max_iters, int e, int m, float* T) {
  int nc = 1 << (1 + e + m);
  float* vals = (float*)malloc(sizeof(float) * nc);
  int64_t* fx = (int64_t*)malloc(sizeof(int64_t) * nc);
  float safe[512];
  int nsafe = o_lut_format_tables(e, m, vals, fx, safe);
  /* grid = torch.unique of the finite code values: sorted, distinct */
  float grid[512];
  int nv = 0;
  for (int c = 0; c < nc; c++) {
    float v = vals[c];
    if (v != v || isinf(v)) continue;
    int dup = 0;
    for (int i = 0; i < nv; i++) if (grid[i] == v) { dup = 1; break; }
    if (!dup) grid[nv++] = v;
  }
  for (int i = 1; i < nv; i++)
    for (int j = i; j > 0 && grid[j - 1] > grid[j]; j--) { float t = grid[j]; grid[j] = grid[j - 1]; grid[j - 1] = t; }
  int64_t ng = (n + (1 << group) - 1) >> group;
  int64_t* counts = (int64_t*)calloc(ng * nv, sizeof(int64_t));
  int bad = 0;
  for (int64_t k = 0; k < K; k++)
    for (int64_t j = 0; j < n; j++) {
      float v = P[k * n + j];
      int64_t b = lower_bound_f(grid, nv, v);
      if (b >= nv || grid[b] != v) { bad = 1; continue; }
      counts[(j >> group) * nv + b]++;
    }
  if (bad) { free(vals); free(fx); free(counts); return -1; }
  double x[512];
  for (int i = 0; i < nv; i++) x[i] = (double)grid[i];
  /* pad order: indices of safe sorted by |value| (stable) */
  int order[512];
  for (int i = 0; i < nsafe; i++) order[i] = i;
  for (int i = 1; i < nsafe; i++)
    for (int j = i; j > 0 && fabsf(safe[order[j - 1]]) > fabsf(safe[order[j]]); j--) {
      int t = order[j]; order[j] = order[j - 1]; order[j - 1] = t;
    }
  for (int64_t g = 0; g < ng; g++) {
    const int64_t* cnt = counts + g * nv;
    double C[LUT_SIZE];
    for (int i = 0; i < LUT_SIZE; i++) C[i] = INFINITY;
    int npres = 0;
    for (int i = 0; i < nv; i++) npres += cnt[i] > 0;
    if (npres <= LUT_SIZE) {                                             /* 2a */
      int r = 0;
      for (int i = 0; i < nv; i++) if (cnt[i] > 0) C[r++] = x[i];
    } else {                                                             /* 2b, 2c */
      double cdf[512], tot = 0.0;
      int64_t cs = 0, sum = 0;
      for (int i = 0; i < nv; i++) sum += cnt[i];
      tot = (double)sum;
      for (int i = 0; i < nv; i++) { cs += cnt[i]; cdf[i] = (double)cs / tot; }
      for (int i = 0; i < LUT_SIZE; i++) {
        double probe = ((double)i + 0.5) / LUT_SIZE;
        int64_t s = lower_bound_d(cdf, nv, probe);
        if (s > nv - 1) s = nv - 1;
        C[i] = x[s];
      }
      dedupe(C);
      for (int it = 0; it < max_iters; it++) {
        double sums[LUT_SIZE] = {0}, wsum[LUT_SIZE] = {0}, nw[LUT_SIZE];
        for (int i = 0; i < nv; i++) {
          int best = 0;
          double bd = fabs(x[i] - C[0]);
          for (int t = 1; t < LUT_SIZE; t++) {
            double d = fabs(x[i] - C[t]);
            if (d < bd) { bd = d; best = t; }
          }
          double w = (double)cnt[i];
          sums[best] += w * x[i];
          wsum[best] += w;
        }
        for (int t = 0; t < LUT_SIZE; t++) nw[t] = wsum[t] > 0 ? sums[t] / wsum[t] : C[t];
        dedupe(nw);
        int same = 1;
        for (int t = 0; t < LUT_SIZE; t++) {
          int valid = isfinite(C[t]);
          if ((isfinite(nw[t]) != 0) != (valid != 0)) same = 0;
          if (valid && !(fabs(nw[t] - C[t]) <= 1e-8 + 1e-5 * fabs(C[t]))) same = 0;
        }
        if (same) break;
        memcpy(C, nw, sizeof(C));
      }
    }
    /* 3: snap each centre to the nearest finder-safe value, ties to the smaller */
    int member[512] = {0}, nmem = 0;
    for (int t = 0; t < LUT_SIZE; t++) {
      if (!isfinite(C[t])) continue;
      int best = 0;
      double bd = fabs(C[t] - (double)safe[0]);
      for (int i = 1; i < nsafe; i++) {
        double d = fabs(C[t] - (double)safe[i]);
        if (d < bd) { bd = d; best = i; }
      }
      member[best] = 1;
    }
    for (int i = 0; i < nsafe; i++) nmem += member[i];
    /* 4: pad with unused values, smallest magnitude first, then sort */
    int need = LUT_SIZE - nmem, taken = 0;
    for (int i = 0; i < nsafe && taken < need; i++)
      if (!member[order[i]]) { member[order[i]] = 1; taken++; }
    int r = 0;
    for (int i = 0; i < nsafe && r < LUT_SIZE; i++) if (member[i]) T[g * LUT_SIZE + r++] = safe[i];
    for (; r < LUT_SIZE; r++) T[g * LUT_SIZE + r] = INFINITY;
  }
  free(vals); free(fx); free(counts);
  return 0;
}

/* pick (kmeans.py:125-138): nearest of the two sorted entries around each code, ties to the lower index */
EXPORT void o_lut_pick(const float* P, const float* T, int64_t K, int64_t n, int group, int64_t width, int64_t* I) {
  for (int64_t k = 0; k < K; k++)
    for (int64_t j = 0; j < n; j++) {
      const float* row = T + (j >> group) * width;
      float v = P[k * n + j];
      int64_t hi = lower_bound_f(row, width, v);
      if (hi < 1) hi = 1;
      if (hi > width - 1) hi = width - 1;
      int64_t lo = hi - 1;
      float dl = fabsf(v - row[lo]), dh = fabsf(row[hi] - v);
      I[k * n + j] = dl <= dh ? lo : hi;
    }
}
/* lookup (kmeans.py:141-146) */
EXPORT void o_lut_lookup(const int64_t* I, const float* T, int64_t K, int64_t n, int group, int64_t width, float* out) {
  for (int64_t k = 0; k < K; k++)
    for (int64_t j = 0; j < n; j++) out[k * n + j] = T[(j >> group) * width + I[k * n + j]];
}
