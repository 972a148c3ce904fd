// MX-Gemmini's look-up tables (mxq/lut/formats.py, mxq/lut/kmeans.py, mxq/block/lut.py): one 16-entry table of
// element values per 2^G columns of a K x n operand, the host's nearest-entry pick, the chip's fixed-point finder,
// and code encode / decode.
//
// Layout: an operand is addressed as element (k, j) = P[k * sk + j * sj], so the row-major K x n operand (sk = n,
// sj = 1) and the transposed one of an axis-1 quantization (sk = 1, sj = K) are read in place.
//
// tables: one CTA per panel of column groups (32 columns, or one whole group when 2^G >= 32). The CTA histograms its
// panel's codes by grid rank in shared memory, then one warp per group fits the table (kmeans.py:46-122): the group's
// distinct codes when there are at most 16; otherwise quantile seeds and weighted Lloyd passes in float64 until two
// passes agree to numpy.allclose or max_iters have run; every centre snapped to the nearest finder-safe value; the
// table padded with unused values of smallest magnitude and sorted. Every sum is exact (codes times counts), so the
// order of the shared-memory atomics does not change a bit.
#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "numerics.cuh"

using namespace mxq;

namespace {

constexpr int LUT = 16;                          // entries per table (formats.py:29 SIZE)
constexpr int MAXV = 256;                        // codes of an 8-bit format
constexpr int NT = 256;

// ---------------------------------------------------------------------------------------- format tables
// The finder's fixed-point view of each code (formats.py:35-68): the chip's shifts and masks, bit for bit.
int64_t fx_code(int e, int m, int v) {
  if (e == 3 && m == 2) {
    int sign = (v >> 5) & 1, ex = (v >> 2) & 7, man = v & 3;
    if (ex == 0 && man == 0) return 0;
    int s_exp = ex == 0 ? -2 : ex - 3;
    int64_t sig = (ex == 0 ? 0 : 4) | man;
    int64_t mag = ((sig << ((s_exp + 2) & 7)) & 0x1FF) & 0xFF;
    return sign ? -mag : mag;
  }
  if (e == 2 && m == 3) {
    int sign = (v >> 5) & 1, ex = (v >> 3) & 3, man = v & 7;
    int64_t mag = ex == 0 ? man : ((int64_t)(8 + man) << (ex - 1));
    return sign ? -mag : mag;
  }
  if (e == 5 && m == 2) {
    int sign = (v >> 7) & 1, ex = (v >> 2) & 0x1F, man = v & 3;
    if (ex == 0 && man == 0) return 0;
    int64_t sig = (ex == 0 ? 0 : 4) | man;
    int s_exp = ex == 0 ? 1 - 15 : ex - 15;
    int64_t mag = (sig << ((s_exp + 14) & 0x1F)) & 0xFFFFFFFFll;
    return sign ? -mag : mag;
  }
  int sign = (v >> 7) & 1, ex = (v >> 3) & 0xF, man = v & 7;   // E4M3
  if (ex == 0 && man == 0) return 0;
  int64_t sig = (ex == 0 ? 0 : 8) | man;
  int s_exp = ex == 0 ? 1 - 7 : ex - 7;
  int64_t mag = (sig << ((s_exp + 6) & 0xF)) & 0x3FFFF;
  return sign ? -mag : mag;
}
int64_t fx_mask(int e, int m) {                 // formats.py:72-73; 0: E2M3's fixed point is exact, no mask
  if (e == 3 && m == 2) return 0x1FF;
  if (e == 2 && m == 3) return 0;
  if (e == 5 && m == 2) return 0x1FFFFFFFFll;
  return 0x7FFFF;
}

struct FormatTables {
  int e = 0, m = 0, ncodes = 0, nv = 0, nsafe = 0;
  float vals[MAXV];            // value of every code (E5M2's top exponent: Inf / NaN)
  int64_t fx[MAXV];            // finder fixed point of every code
  float grid[MAXV];            // sorted distinct finite values
  float safe[MAXV];            // finder-safe values, sorted
  uint8_t order[MAXV];         // safe indices by |value|, stable (negatives first): the padding order
  uint32_t enc_bits[MAXV];     // distinct value bit patterns, sorted ...
  int16_t enc_code[MAXV];      // ... and the lowest code having each
  int nenc = 0;
};

// _tables (formats.py:83-111), built once per format
const FormatTables* format_tables(int e, int m) {
  static std::mutex mu;
  static FormatTables cache[4];
  static bool ready[4] = {false, false, false, false};
  int slot = (e == 3 && m == 2) ? 0 : (e == 2 && m == 3) ? 1 : (e == 5 && m == 2) ? 2 : (e == 4 && m == 3) ? 3 : -1;
  if (slot < 0) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  FormatTables& t = cache[slot];
  if (ready[slot]) return &t;
  t.e = e;
  t.m = m;
  t.ncodes = 1 << (1 + e + m);
  const int bias = (1 << (e - 1)) - 1;
  for (int c = 0; c < t.ncodes; c++) {
    int s = (c >> (e + m)) & 1, ex = (c >> m) & ((1 << e) - 1), man = c & ((1 << m) - 1);
    double v;
    if (e == 5 && m == 2 && ex == 0x1F) v = man ? NAN : INFINITY;
    else if (ex == 0) v = man * ldexp(1.0, 1 - bias - m);
    else v = (1.0 + (double)man / (1 << m)) * ldexp(1.0, ex - bias);
    t.vals[c] = (float)(s ? -v : v);
    t.fx[c] = fx_code(e, m, c);
  }
  // finder-safe values: per fixed point the smallest magnitude (code order breaks no tie: magnitudes differ)
  std::vector<std::pair<int64_t, float>> seen;
  for (int c = 0; c < t.ncodes; c++) {
    float v = t.vals[c];
    if (v != v || std::isinf(v)) continue;
    auto it = std::find_if(seen.begin(), seen.end(), [&](const std::pair<int64_t, float>& p) { return p.first == t.fx[c]; });
    if (it == seen.end()) seen.push_back({t.fx[c], v});
    else if (fabsf(v) < fabsf(it->second)) it->second = v;
  }
  std::vector<float> safe;
  for (auto& p : seen) {
    float v = p.second == 0.0f ? 0.0f : p.second;          // one zero, +0
    if (std::find(safe.begin(), safe.end(), v) == safe.end()) safe.push_back(v);
  }
  std::sort(safe.begin(), safe.end());
  t.nsafe = (int)safe.size();
  for (int i = 0; i < t.nsafe; i++) t.safe[i] = safe[i];
  std::vector<int> order(t.nsafe);
  for (int i = 0; i < t.nsafe; i++) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return fabsf(t.safe[a]) < fabsf(t.safe[b]); });
  for (int i = 0; i < t.nsafe; i++) t.order[i] = (uint8_t)order[i];
  std::vector<float> grid;
  for (int c = 0; c < t.ncodes; c++) {
    float v = t.vals[c];
    if (v != v || std::isinf(v)) continue;
    v = v == 0.0f ? 0.0f : v;
    if (std::find(grid.begin(), grid.end(), v) == grid.end()) grid.push_back(v);
  }
  std::sort(grid.begin(), grid.end());
  t.nv = (int)grid.size();
  for (int i = 0; i < t.nv; i++) t.grid[i] = grid[i];
  // encode: value bits -> lowest code (formats.py:125-137, `lookup.setdefault(bits, c)`)
  std::vector<std::pair<uint32_t, int>> enc;
  for (int c = 0; c < t.ncodes; c++) {
    uint32_t b = f2u(t.vals[c]);
    if (std::find_if(enc.begin(), enc.end(), [&](const std::pair<uint32_t, int>& p) { return p.first == b; }) ==
        enc.end())
      enc.push_back({b, c});
  }
  std::sort(enc.begin(), enc.end());
  t.nenc = (int)enc.size();
  for (int i = 0; i < t.nenc; i++) {
    t.enc_bits[i] = enc[i].first;
    t.enc_code[i] = (int16_t)enc[i].second;
  }
  ready[slot] = true;
  return &t;
}

// ------------------------------------------------------------------------------------------- device side
struct TableParams {                           // by value: what the tables kernel needs of a format
  int nv, nsafe;
  float grid[MAXV];
  float safe[MAXV];
  uint8_t order[MAXV];
};

__device__ __forceinline__ int lower_bound_f(const float* a, int n, float v) {
  int lo = 0, hi = n;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (a[mid] < v) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// sort 16 doubles ascending (inf last), equal values merged into +inf, sorted again (_dedupe, kmeans.py:38-43)
__device__ void dedupe16(double* c) {
  for (int i = 1; i < LUT; i++) {
    double v = c[i];
    int j = i - 1;
    while (j >= 0 && c[j] > v) {
      c[j + 1] = c[j];
      j--;
    }
    c[j + 1] = v;
  }
  bool dup[LUT];
  dup[0] = false;
  for (int i = 1; i < LUT; i++) dup[i] = c[i] == c[i - 1];
  for (int i = 1; i < LUT; i++)
    if (dup[i]) c[i] = INFINITY;
  for (int i = 1; i < LUT; i++) {
    double v = c[i];
    int j = i - 1;
    while (j >= 0 && c[j] > v) {
      c[j + 1] = c[j];
      j--;
    }
    c[j + 1] = v;
  }
}

// groups per CTA for a given G: a 32-column panel, or one group when it is wider
__host__ __device__ __forceinline__ int groups_per_cta(int G) { return G >= 5 ? 1 : (32 >> G); }

__global__ void __launch_bounds__(NT) k_lut_tables(const float* __restrict__ P, int64_t K, int64_t n, int64_t sk,
                                                   int64_t sj, int G, int max_iters, const __grid_constant__ TableParams tp,
                                                   float* __restrict__ T, int* __restrict__ status) {
  extern __shared__ int counts[];                           // [groups_per_cta][nv]
  __shared__ double cent[NT / 32][LUT], sums[NT / 32][LUT], wsum[NT / 32][LUT], cdf[NT / 32][MAXV];
  __shared__ float sgrid[MAXV];
  __shared__ int bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nv = tp.nv;
  const int gpc = groups_per_cta(G);
  const int64_t ng = (n + ((int64_t)1 << G) - 1) >> G;
  const int64_t g0 = (int64_t)blockIdx.x * gpc;
  const int64_t j0 = g0 << G, jend = (g0 + gpc) << G, j1 = jend < n ? jend : n;
  const int64_t W = j1 - j0;
  for (int i = tid; i < gpc * nv; i += NT) counts[i] = 0;
  for (int i = tid; i < nv; i += NT) sgrid[i] = tp.grid[i];
  if (tid == 0) bad = 0;
  __syncthreads();

  // 1. counts of each distinct code per group (kmeans.py:58-64); iterate so consecutive threads read consecutive memory
  const int64_t total = K * W;
  const bool kfast = sk == 1;
  bool mybad = false;
  for (int64_t e = tid; e < total; e += NT) {
    int64_t k = kfast ? e % K : e / W, jj = kfast ? e / K : e % W;
    float v = P[k * sk + (j0 + jj) * sj];
    int b = lower_bound_f(sgrid, nv, v);
    if (b >= nv || sgrid[b] != v) {
      mybad = true;
      continue;
    }
    atomicAdd(&counts[(int)(jj >> G) * nv + b], 1);
  }
  if (mybad) bad = 1;
  __syncthreads();
  if (bad) {
    if (tid == 0) atomicExch(status, 1);
    return;
  }

  // 2-4. one warp per group
  for (int gl = warp; gl < gpc; gl += NT / 32) {
    const int64_t g = g0 + gl;
    if (g >= ng) break;
    const int* cnt = counts + gl * nv;
    double* C = cent[warp];
    // distinct codes present
    int npres = 0;
    for (int b = lane; b < nv; b += 32) npres += cnt[b] > 0;
    for (int s = 16; s > 0; s >>= 1) npres += __shfl_xor_sync(0xffffffffu, npres, s);
    if (lane < LUT) C[lane] = INFINITY;
    __syncwarp();
    if (npres <= LUT) {                                    // 2a: they are the centres, ascending
      int base = 0;
      for (int b0 = 0; b0 < nv; b0 += 32) {
        int b = b0 + lane;
        bool p = b < nv && cnt[b] > 0;
        unsigned mask = __ballot_sync(0xffffffffu, p);
        if (p) C[base + __popc(mask & ((1u << lane) - 1u))] = (double)sgrid[b];
        base += __popc(mask);
      }
      __syncwarp();
    } else {
      // 2b: quantile seeds: the first code whose cumulative weight reaches (i + 0.5) / 16
      long long run = 0;
      long long tot = 0;
      for (int b = lane; b < nv; b += 32) tot += cnt[b];
      for (int s = 16; s > 0; s >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, s);
      for (int b0 = 0; b0 < nv; b0 += 32) {
        int b = b0 + lane;
        long long c = b < nv ? cnt[b] : 0;
        for (int s = 1; s < 32; s <<= 1) {                 // inclusive scan
          long long o = __shfl_up_sync(0xffffffffu, c, s);
          if (lane >= s) c += o;
        }
        if (b < nv) cdf[warp][b] = __ddiv_rn((double)(run + c), (double)tot);
        run += __shfl_sync(0xffffffffu, c, 31);
      }
      __syncwarp();
      if (lane < LUT) {
        double probe = __ddiv_rn((double)lane + 0.5, (double)LUT);
        int lo = 0, hi = nv;
        while (lo < hi) {
          int mid = (lo + hi) >> 1;
          if (cdf[warp][mid] < probe) lo = mid + 1;
          else hi = mid;
        }
        if (lo > nv - 1) lo = nv - 1;
        C[lane] = (double)sgrid[lo];
      }
      __syncwarp();
      if (lane == 0) dedupe16(C);
      __syncwarp();
      // 2c: weighted Lloyd passes over the distinct codes
      for (int it = 0; it < max_iters; it++) {
        if (lane < LUT) {
          sums[warp][lane] = 0.0;
          wsum[warp][lane] = 0.0;
        }
        __syncwarp();
        double c[LUT];
#pragma unroll
        for (int t = 0; t < LUT; t++) c[t] = C[t];
        for (int b = lane; b < nv; b += 32) {
          if (cnt[b] == 0) continue;                       // a zero weight adds nothing to any sum
          double x = (double)sgrid[b];
          int best = 0;
          double bd = fabs(__dsub_rn(x, c[0]));
#pragma unroll
          for (int t = 1; t < LUT; t++) {
            double d = fabs(__dsub_rn(x, c[t]));
            if (d < bd) {
              bd = d;
              best = t;
            }
          }
          double w = (double)cnt[b];
          atomicAdd(&sums[warp][best], __dmul_rn(w, x));
          atomicAdd(&wsum[warp][best], w);
        }
        __syncwarp();
        int same = 1;
        if (lane == 0) {
          double nw[LUT];
          for (int t = 0; t < LUT; t++) nw[t] = wsum[warp][t] > 0.0 ? __ddiv_rn(sums[warp][t], wsum[warp][t]) : c[t];
          dedupe16(nw);
          for (int t = 0; t < LUT; t++) {
            bool valid = finite_d(c[t]);
            if (finite_d(nw[t]) != valid) same = 0;
            if (valid && !(fabs(__dsub_rn(nw[t], c[t])) <= __dadd_rn(1e-8, __dmul_rn(1e-5, fabs(c[t]))))) same = 0;
          }
          if (!same)
            for (int t = 0; t < LUT; t++) C[t] = nw[t];
        }
        same = __shfl_sync(0xffffffffu, same, 0);
        __syncwarp();
        if (same) break;
      }
    }
    // 3. each centre snapped to the nearest finder-safe value, ties to the smaller; 4. pad and sort
    __shared__ unsigned char member[NT / 32][MAXV];
    for (int i = lane; i < tp.nsafe; i += 32) member[warp][i] = 0;
    __syncwarp();
    if (lane < LUT) {
      double cc = C[lane];
      if (finite_d(cc)) {
        int best = 0;
        double bd = fabs(__dsub_rn(cc, (double)tp.safe[0]));
        for (int i = 1; i < tp.nsafe; i++) {
          double d = fabs(__dsub_rn(cc, (double)tp.safe[i]));
          if (d < bd) {
            bd = d;
            best = i;
          }
        }
        member[warp][best] = 1;
      }
    }
    __syncwarp();
    if (lane == 0) {
      int nmem = 0;
      for (int i = 0; i < tp.nsafe; i++) nmem += member[warp][i];
      for (int i = 0; i < tp.nsafe && nmem < LUT; i++) {
        int s = tp.order[i];
        if (!member[warp][s]) {
          member[warp][s] = 1;
          nmem++;
        }
      }
      int r = 0;
      for (int i = 0; i < tp.nsafe && r < LUT; i++)
        if (member[warp][i]) T[g * LUT + r++] = tp.safe[i];
      for (; r < LUT; r++) T[g * LUT + r] = INFINITY;
    }
    __syncwarp();
  }
}

// pick (kmeans.py:125-138): nearest of the two sorted entries around v, ties to the lower index; `out_vals` set:
// write the entry itself (lookup fused, for block.lut), else the index
__global__ void k_lut_pick(const float* __restrict__ P, const float* __restrict__ T, int64_t K, int64_t n, int64_t sk,
                           int64_t sj, int G, int width, int64_t* __restrict__ I, float* __restrict__ out_vals) {
  const int64_t total = K * n;
  const bool kfast = sk == 1;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t k = kfast ? e % K : e / n, j = kfast ? e / K : e % n;
    const int64_t at = k * sk + j * sj;
    const float v = P[at];
    const float* row = T + (j >> G) * width;
    int lo = 0, hi = width;
    while (lo < hi) {
      int mid = (lo + hi) >> 1;
      if (__ldg(row + mid) < v) lo = mid + 1;
      else hi = mid;
    }
    hi = hi < 1 ? 1 : (hi > width - 1 ? width - 1 : hi);
    lo = hi - 1;
    const float rl = __ldg(row + lo), rh = __ldg(row + hi);
    const int idx = abs_f(__fsub_rn(v, rl)) <= abs_f(__fsub_rn(rh, v)) ? lo : hi;
    if (out_vals) out_vals[at] = idx == lo ? rl : rh;
    else I[k * n + j] = idx;
  }
}

// lookup (kmeans.py:141-146)
__global__ void k_lut_lookup(const int64_t* __restrict__ I, const float* __restrict__ T, int64_t K, int64_t n, int G,
                             int width, float* __restrict__ out) {
  const int64_t total = K * n;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    int64_t j = e % n;
    out[e] = __ldg(T + (j >> G) * width + I[e]);
  }
}

struct CodeTables {
  int ncodes, nenc;
  float vals[MAXV];
  long long fx[MAXV];
  uint32_t enc_bits[MAXV];
  int16_t enc_code[MAXV];
};

__device__ __forceinline__ int encode1(const CodeTables& ct, float v) {
  const uint32_t b = f2u(v);
  int lo = 0, hi = ct.nenc;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (ct.enc_bits[mid] < b) lo = mid + 1;
    else hi = mid;
  }
  return (lo < ct.nenc && ct.enc_bits[lo] == b) ? ct.enc_code[lo] : -1;
}

__global__ void k_lut_encode(const float* __restrict__ V, int64_t* __restrict__ out, int64_t n,
                             const __grid_constant__ CodeTables ct, int* __restrict__ status) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int c = encode1(ct, V[i]);
    if (c < 0) atomicExch(status, 1);
    out[i] = c;
  }
}

__global__ void k_lut_decode(const int64_t* __restrict__ codes, float* __restrict__ out, int64_t n,
                             const __grid_constant__ CodeTables ct, int* __restrict__ status) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t c = codes[i];
    if (c < 0 || c >= ct.ncodes) {
      atomicExch(status, 1);
      out[i] = 0.0f;
    } else {
      out[i] = ct.vals[c];
    }
  }
}

// finder (formats.py:140-159): fixed points of the code and of the 16 entries, masked |difference|, first minimum
__global__ void k_lut_finder(const int64_t* __restrict__ codes, const float* __restrict__ T, int64_t K, int64_t n,
                             int G, long long mask, const __grid_constant__ CodeTables ct, int64_t* __restrict__ I,
                             int* __restrict__ status) {
  const int64_t total = K * n;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = e % n, c = codes[e];
    if (c < 0 || c >= ct.ncodes) {
      atomicExch(status, 1);
      I[e] = 0;
      continue;
    }
    const long long f = ct.fx[c];
    const float* row = T + (j >> G) * LUT;
    int best = 0;
    long long bd = 0;
    for (int t = 0; t < LUT; t++) {
      int tc = encode1(ct, __ldg(row + t));
      if (tc < 0) {
        atomicExch(status, 2);
        tc = 0;
      }
      long long d = f - ct.fx[tc];
      d = d < 0 ? -d : d;
      if (mask) d &= mask;
      if (t == 0 || d < bd) {
        bd = d;
        best = t;
      }
    }
    I[e] = best;
  }
}

int fmt_slot_check(int e, int m, const char* what) {
  MXQ_REQUIRE(format_tables(e, m) != nullptr, MXQ_ERR_VALUE,
              "mxq.lut: (e=%d, m=%d) is not a LUT format; MX-Gemmini sends MXFP6_E3M2, MXFP6_E2M3, MXFP8_E5M2, "
              "MXFP8_E4M3 through LUTs (%s)",
              e, m, what);
  return MXQ_OK;
}

CodeTables code_tables(const FormatTables* f) {
  CodeTables ct;
  ct.ncodes = f->ncodes;
  ct.nenc = f->nenc;
  for (int i = 0; i < f->ncodes; i++) {
    ct.vals[i] = f->vals[i];
    ct.fx[i] = f->fx[i];
  }
  for (int i = 0; i < f->nenc; i++) {
    ct.enc_bits[i] = f->enc_bits[i];
    ct.enc_code[i] = f->enc_code[i];
  }
  return ct;
}

}  // namespace

extern "C" {

int mxq_lut_format_tables(int32_t e, int32_t m, float* vals, int64_t* fx, float* safe, int32_t* nsafe) {
  if (int r = fmt_slot_check(e, m, "format_tables")) return r;
  const FormatTables* f = format_tables(e, m);
  if (vals)
    for (int i = 0; i < f->ncodes; i++) vals[i] = f->vals[i];
  if (fx)
    for (int i = 0; i < f->ncodes; i++) fx[i] = f->fx[i];
  if (safe)
    for (int i = 0; i < f->nsafe; i++) safe[i] = f->safe[i];
  if (nsafe) *nsafe = f->nsafe;
  return MXQ_OK;
}

int mxq_lut_tables(const float* P, float* T, int64_t K, int64_t n, int64_t sk, int64_t sj, int32_t group,
                   int32_t max_iters, int32_t e, int32_t m, int32_t* status, void* stream) {
  if (int r = fmt_slot_check(e, m, "tables")) return r;
  MXQ_REQUIRE(group >= 0 && group < 31, MXQ_ERR_VALUE, "mxq.lut: group %d must be a non-negative integer", group);
  MXQ_REQUIRE(max_iters >= 0, MXQ_ERR_VALUE, "mxq.lut: max_iters %d must be a non-negative integer", max_iters);
  MXQ_REQUIRE(status != nullptr, MXQ_ERR_VALUE, "mxq.lut.tables: no status word");
  const FormatTables* f = format_tables(e, m);
  cudaStream_t st = as_stream(stream);
  if (int r = check_cuda(cudaMemsetAsync(status, 0, sizeof(int32_t), st), "lut.tables")) return r;
  const int64_t ng = (n + ((int64_t)1 << group) - 1) >> group;
  if (ng == 0) return MXQ_OK;
  TableParams tp;
  tp.nv = f->nv;
  tp.nsafe = f->nsafe;
  for (int i = 0; i < f->nv; i++) tp.grid[i] = f->grid[i];
  for (int i = 0; i < f->nsafe; i++) {
    tp.safe[i] = f->safe[i];
    tp.order[i] = f->order[i];
  }
  const int gpc = groups_per_cta(group);
  const size_t smem = (size_t)gpc * f->nv * sizeof(int);
  const unsigned grid = (unsigned)((ng + gpc - 1) / gpc);
  // static (~22 KB) plus the histograms can pass the 48 KB default
  if (int r = check_cuda(cudaFuncSetAttribute(k_lut_tables, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                         "lut.tables: shared memory attribute"))
    return r;
  k_lut_tables<<<grid, NT, smem, st>>>(P, K, n, sk, sj, group, max_iters, tp, T, status);
  return MXQ_LAUNCH_CHECK("lut.tables");
}

int mxq_lut_pick(const float* P, const float* T, int64_t* I, int64_t K, int64_t n, int64_t sk, int64_t sj,
                 int32_t group, int32_t width, void* stream) {
  MXQ_REQUIRE(width >= 2, MXQ_ERR_VALUE, "mxq.lut.pick: tables need width >= 2");
  if (K * n == 0) return MXQ_OK;
  k_lut_pick<<<grid_for(K * n, 256), 256, 0, as_stream(stream)>>>(P, T, K, n, sk, sj, group, width, I, nullptr);
  return MXQ_LAUNCH_CHECK("lut.pick");
}

int mxq_lut_pick_lookup(const float* P, const float* T, float* out, int64_t K, int64_t n, int64_t sk, int64_t sj,
                        int32_t group, int32_t width, void* stream) {
  MXQ_REQUIRE(width >= 2, MXQ_ERR_VALUE, "mxq.lut.pick: tables need width >= 2");
  if (K * n == 0) return MXQ_OK;
  k_lut_pick<<<grid_for(K * n, 256), 256, 0, as_stream(stream)>>>(P, T, K, n, sk, sj, group, width, nullptr, out);
  return MXQ_LAUNCH_CHECK("lut.pick_lookup");
}

int mxq_lut_lookup(const int64_t* I, const float* T, float* out, int64_t K, int64_t n, int32_t group, int32_t width,
                   void* stream) {
  if (K * n == 0) return MXQ_OK;
  k_lut_lookup<<<grid_for(K * n, 256), 256, 0, as_stream(stream)>>>(I, T, K, n, group, width, out);
  return MXQ_LAUNCH_CHECK("lut.lookup");
}

int mxq_lut_encode(const float* V, int64_t* codes, int64_t n, int32_t e, int32_t m, int32_t* status, void* stream) {
  if (int r = fmt_slot_check(e, m, "encode")) return r;
  cudaStream_t st = as_stream(stream);
  if (int r = check_cuda(cudaMemsetAsync(status, 0, sizeof(int32_t), st), "lut.encode")) return r;
  if (n == 0) return MXQ_OK;
  k_lut_encode<<<grid_for(n, 256), 256, 0, st>>>(V, codes, n, code_tables(format_tables(e, m)), status);
  return MXQ_LAUNCH_CHECK("lut.encode");
}

int mxq_lut_decode(const int64_t* codes, float* out, int64_t n, int32_t e, int32_t m, int32_t* status, void* stream) {
  if (int r = fmt_slot_check(e, m, "decode")) return r;
  cudaStream_t st = as_stream(stream);
  if (int r = check_cuda(cudaMemsetAsync(status, 0, sizeof(int32_t), st), "lut.decode")) return r;
  if (n == 0) return MXQ_OK;
  k_lut_decode<<<grid_for(n, 256), 256, 0, st>>>(codes, out, n, code_tables(format_tables(e, m)), status);
  return MXQ_LAUNCH_CHECK("lut.decode");
}

int mxq_lut_finder(const int64_t* codes, const float* T, int64_t* I, int64_t K, int64_t n, int32_t group, int32_t e,
                   int32_t m, int32_t* status, void* stream) {
  if (int r = fmt_slot_check(e, m, "finder")) return r;
  cudaStream_t st = as_stream(stream);
  if (int r = check_cuda(cudaMemsetAsync(status, 0, sizeof(int32_t), st), "lut.finder")) return r;
  if (K * n == 0) return MXQ_OK;
  k_lut_finder<<<grid_for(K * n, 256), 256, 0, st>>>(codes, T, K, n, group, (long long)fx_mask(e, m),
                                                     code_tables(format_tables(e, m)), I, status);
  return MXQ_LAUNCH_CHECK("lut.finder");
}

}  // extern "C"
