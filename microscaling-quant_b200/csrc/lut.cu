// MX-Gemmini's look-up tables (mxq/lut/formats.py, mxq/lut/kmeans.py, mxq/block/lut.py): one 16-entry table of
// element values per 2^G columns of a K x n operand, the host's nearest-entry pick, the chip's fixed-point finder,
// and code encode / decode.
//
// Layout: an operand is addressed as element (k, j) = P[k * sk + j * sj], so the row-major K x n operand (sk = n,
// sj = 1) and the transposed one of an axis-1 quantization (sk = 1, sj = K) are read in place.
//
// tables: a thread-block cluster per panel of column groups (32 columns, or one group when a group is wider). The
// cluster's CTAs split the panel's rows and histogram their codes by grid rank in their own shared memory; after a
// cluster barrier each CTA sums its share of the panel's groups over all the cluster's histograms through
// distributed shared memory, and one warp per group fits the table (kmeans.py:46-122) with the work spread over its
// lanes (k_lut_tables). Every sum is exact (integer counts, codes times counts), so no summation order changes a
// bit.
#include <cooperative_groups.h>
#include <type_traits>
#include <cmath>
#include <algorithm>
#include <memory>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "numerics.cuh"
#include "quant_elem.cuh"

using namespace mxq;
namespace cg = cooperative_groups;

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
  int e = 0, m = 0, ncodes = 0, nv = 0, nsafe = 0, nmag = 0;
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
  // the kernel ranks a value by its magnitude code: the grid must be -mag[nmag-1] .. 0 .. mag[nmag-1] with mag[k] the
  // value of code k (true of all four formats; checked here once)
  t.nmag = (t.nv + 1) / 2;
  for (int k = 0; k < t.nmag; k++)
    if (t.grid[t.nmag - 1 + k] != t.vals[k] || t.grid[t.nmag - 1 - k] != -t.vals[k]) t.nmag = -1;
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
constexpr int KEYS = 1 << 12;                  // bit-pattern keys of a code: sign, exponent, top m <= 3 fraction bits
// A format's tables for the tables kernel, in global memory (read with coalesced loads at each CTA's start; kernel
// parameters indexed per lane would be serialised by the constant cache)
struct DevTables {
  float grid[MAXV];                            // sorted distinct finite values
  float safe[MAXV];                            // finder-safe values, sorted
  float vals[MAXV];                            // every code's value (for the code -> entry map of block.lut)
  uint8_t order[MAXV];                         // safe indices by |value|: the padding order
  uint8_t cbin[MAXV];                          // code (its OCP bit pattern) -> grid rank, 0xFF for NaN / Inf
  uint8_t bin[KEYS];                           // key -> grid rank, 0xFF for a pattern that is no code
};
__device__ DevTables g_dev_tables[4];          // one per format slot, per device (module globals are per device)

struct TableParams {                           // by value: what the tables kernel needs of a format
  int nv, nsafe, ncodes;
  int nmag, bias, m;                           // grid = -mag[nmag-1] .. -mag[1], 0, mag[1] .. mag[nmag-1]
  int keyshift;                                // 23 - m: a code's float32 pattern >> keyshift is its key
  uint32_t lowmask;                            // the fraction bits below a code's m: zero in every code
  const DevTables* dt;
};

// block.lut in one launch (the kernel's fused mode): V's block.mxgemmini quantization (blocks of 32 along rows) is
// done in the kernel, its scales written to X and its codes (OCP bytes) to codesT, column-major (byte (k, j) at
// j K + k), for the kernel's own lookup
struct FusedArgs {
  float* X;
  uint8_t* codesT;
  float scale_floor;
  int rounding;
};

// the larger of two floats, NaN when either is (max.NaN: a NaN is never dropped)
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// block.mxgemmini (block.py, mxgemmini.py) of one 32-row block of one column, by one lane: the 32 values col[0],
// col[n], ... (a warp's load is one 128-byte row segment when its lanes take consecutive columns), the block max, the
// scale (to *xout) and its reciprocal, and every code -- the direct code of the short step when the block is finite
// with a power-of-two scale, else the general OCP grid step (the TMA quantizer's two element steps, the same bits)
// -- counted by tally(code) as it is made and stored as 32 bytes (two 16-byte stores) at dst. Returns whether a value
// had no code in the format.
template <int FE, int FM, int QM, class Tally>
__device__ __forceinline__ bool quant_block(const float* col, int64_t n, float* xout, uint8_t* dst, float scale_floor,
                                            int rounding, Tally& tally) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __ldcs(col + i * n);
  // max |v| by a tree of NaN-propagating maxima (a NaN anywhere makes it NaN)
  float t[16];
#pragma unroll
  for (int i = 0; i < 16; i++) t[i] = max_nan(fabsf(v[2 * i]), fabsf(v[2 * i + 1]));
#pragma unroll
  for (int h = 8; h >= 1; h >>= 1)
#pragma unroll
    for (int i = 0; i < h; i++) t[i] = max_nan(t[i], t[i + h]);
  const float mx = t[0];
  const bool nan = mx != mx;
  const float x = scale_mxquant(nan ? qnan_f() : mx, scale_floor);
  const float r = reciprocal_of<MXQ_FAMILY_MXGEMMINI>(x, nan);
  *xout = x;
  uint32_t w[8];
  bool nocode = false;
  if (mx < INFINITY && r != 0.0f) {
#pragma unroll
    for (int i = 0; i < 32; i++) {
      // the sign of a zero kept: both zeros have one grid rank and one table entry
      const uint32_t c = code_clean<FE, FM, QM, true>(__fmul_rn(v[i], r));
      tally(c);
      w[i >> 2] = (i & 3) ? (w[i >> 2] | (c << (8 * (i & 3)))) : c;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; i++) {
      const float z = r != 0.0f ? __fmul_rn(v[i], r) : div_rn(v[i], x);
      const uint32_t c = lut_code<FE, FM>(ocp_grid<FE, FM>(z, rounding), nocode);
      tally(c);
      w[i >> 2] = (i & 3) ? (w[i >> 2] | (c << (8 * (i & 3)))) : c;
    }
  }
  uint4* d = reinterpret_cast<uint4*>(dst);
  d[0] = make_uint4(w[0], w[1], w[2], w[3]);
  d[1] = make_uint4(w[4], w[5], w[6], w[7]);
  return nocode;
}

constexpr int NW = NT / 32;                    // warps per CTA
constexpr double MIN_GAP = 1.16415321826934814453125e-10;   // 2^-33: centres this far apart never tie by rounding

// The grid rank of a value: its magnitude code from the float's bits (sign-magnitude formats whose finite
// magnitudes increase with the code), clamped into [0, nv); the caller checks grid[rank] == v.
__device__ __forceinline__ int grid_rank(float v, const TableParams& tp) {
  const uint32_t u = f2u(v), a = u & 0x7fffffffu;
  const int E = (int)(a >> 23) - 127;
  int k;
  if (E >= 1 - tp.bias) {
    k = ((E + tp.bias) << tp.m) | (int)((a >> (23 - tp.m)) & ((1u << tp.m) - 1u));
  } else {                                     // below the format's normal range: a multiple of its subnormal step
    const int sh = 24 - tp.bias - tp.m - E;
    k = (int)(((a & 0x007fffffu) | 0x00800000u) >> (sh < 31 ? sh : 31));
  }
  int r = (tp.nmag - 1) + ((u >> 31) ? -k : k);
  return r < 0 ? 0 : (r >= tp.nv ? tp.nv - 1 : r);
}

// a count (0 <= c < 2^31) as float64 by its bit pattern: 2^52 + c has c in its low mantissa bits, and subtracting
// 2^52 is exact -- an FP64 add instead of the slower integer conversion
__device__ __forceinline__ double i2d(int c) {
  return __dsub_rn(__hiloint2double(0x43300000, c), 4503599627370496.0);
}

// _dedupe (kmeans.py:38-43) across lanes 0-15 of a warp, lane t holding v_t: sort ascending (by rank, ties in lane
// order), equal neighbours turned into +inf, sort again. `scratch` holds 16 doubles of this warp.
__device__ __forceinline__ double dedupe_lanes(double v, double* scratch) {
  const int lane = threadIdx.x & 31;
  for (int pass = 0; pass < 2; pass++) {
    int rank = 0;
#pragma unroll
    for (int s = 0; s < LUT; s++) {
      const double o = __shfl_sync(0xffffffffu, v, s);
      rank += (o < v) || (o == v && s < lane);
    }
    if (lane < LUT) scratch[rank] = v;
    __syncwarp();
    if (lane < LUT) v = scratch[lane];
    __syncwarp();
    if (pass == 0) {
      const double prev = __shfl_up_sync(0xffffffffu, v, 1);
      if (lane > 0 && lane < LUT && v == prev) v = INFINITY;
    }
  }
  return v;
}

// The warps of a CTA that fit a group: group gl of a cs-CTA cluster's gpc is fitted by CTA gl % cs, warp gl / cs
__host__ __device__ __forceinline__ int fit_warps(int gpc, int cs, int nw) {
  const int w = (gpc + cs - 1) / cs;
  return w < nw ? w : nw;
}

// The tables (kmeans.py:46-122). A cluster of cs CTAs per panel of gpc column groups: (1) the panel's codes
// histogrammed by grid rank, each CTA its rows into its own shared memory, then group gl merged across the cluster by
// CTA gl % cs; then one warp per group: (2) prefix sums of counts and of counts x values over the sorted
// codes (exact in float64: integers times grid values); the centres -- the present codes when there are at most 16,
// else the quantile seeds, deduplicated, and weighted Lloyd passes until two passes agree to numpy.allclose or
// max_iters have run; (3) each centre snapped to the nearest finder-safe value; (4) padded and sorted.
//
// A Lloyd pass in lanes: lane t holds centre t. Codes and centres are sorted and rounding is monotone, so every
// centre takes a run of consecutive codes; lane t finds where its run ends -- the first code closer (rounded
// float64 distance, ties to the lower centre, as argmin) to centre t + 1 -- by binary search, and its sum and weight
// are differences of the prefix sums. That equals the reference's argmin over all 16 centres whenever consecutive
// centres are at least 2^-33 apart (distances below 2^17 then never round to a tie across a centre); a pass that
// finds two closer centres assigns code by code instead.
// TIn: float codes at P[k sk + j sj], or (block.lut) code bytes stored by 32-column panels, byte (k, j) at
// ((j / 32) K + k) 32 + j % 32 (sk, sj unused). QM >= 0: the fused block.lut (FE, FM the element format, QM the
// rounding mode of its clean blocks): P is V (row-major K x n, K a multiple of 32, panels of at most 32 columns), and
// the codes are made here (FusedArgs)
template <typename TIn, int FE = 0, int FM = 0, int QM = -1, int NTH = NT>
__global__ void __launch_bounds__(NTH, 1024 / NTH) k_lut_tables(const TIn* __restrict__ P, int64_t K, int64_t n,
                                                   int64_t sk, int64_t sj, int G, int gpc, int max_iters, int priv_ok,
                                                   const __grid_constant__ TableParams tp, float* __restrict__ T,
                                                   int* __restrict__ status, float* __restrict__ cmap,
                                                   float* __restrict__ out, const FusedArgs fa) {
  constexpr int NTK = NTH, NWK = NTH / 32;                  // threads and warps of a CTA
  // dynamic shared memory: counts [gpc][nv | 1] (this CTA's rows; then merged, its own groups), then the fits'
  // prefix sums [2][nfw][nv + 1] doubles for the nfw warps that fit a group; with `out`, the panel's code -> entry
  // maps [gpc][ncodes + 1] over the same bytes once the fits are done
  constexpr bool FUSED = QM >= 0;
  constexpr bool BYTES = sizeof(TIn) == 1 || FUSED;          // codes counted and looked up as OCP bytes
  extern __shared__ int counts[];
  __shared__ double scratch[NWK][LUT], fsum[NWK][LUT], fw[NWK][LUT];
  __shared__ __align__(16) float sgrid[MAXV];                // the format's tables, read with per-lane indices
  __shared__ double sgridd[MAXV], ssafed[MAXV];              // the same as float64: no conversion in the fits
  __shared__ __align__(16) float ssafe[MAXV];
  __shared__ __align__(16) float svals[MAXV];
  __shared__ __align__(16) uint8_t sorder[MAXV];
  __shared__ float stab[NWK][LUT];                            // each fitting warp's finished table
  __shared__ unsigned char member[NWK][MAXV];
  __shared__ __align__(16) uint8_t sbin[BYTES ? MAXV : KEYS];
  __shared__ int bad;
  cg::cluster_group cluster = cg::this_cluster();
  const int cs = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nv = tp.nv;
  const int nfw = fit_warps(gpc, cs, NWK);
  const unsigned lt = (1u << lane) - 1u;
  const int64_t ng = (n + ((int64_t)1 << G) - 1) >> G;
  const int64_t g0 = (int64_t)(blockIdx.x / cs) * gpc;       // the cluster's panel of groups
  const int64_t j0 = g0 << G, jend = (g0 + gpc) << G, j1 = jend < n ? jend : n;
  const int64_t W = j1 - j0;
  const int64_t kper = FUSED ? ((K / 32 + cs - 1) / cs) * 32 : (K + cs - 1) / cs;   // this CTA's rows of the panel
                                                             // (fused: whole blocks of 32)
  const int64_t kbeg = (int64_t)rank * kper < K ? (int64_t)rank * kper : K;
  const int64_t kend = kbeg + kper < K ? kbeg + kper : K;
  const int nvp = nv | 1;                                   // a group's histogram row, odd: a bin of 32 groups hits 32 banks
  double* const pw = reinterpret_cast<double*>(counts + ((gpc * nvp + 3) & ~3));   // [nfw][nv + 1]
  double* const pwx = pw + nfw * (nv + 1);
  for (int i = tid; i < gpc * nvp; i += NTK) counts[i] = 0;
  // the tables the fits index per lane, into shared memory once
  {
    const DevTables* dt = tp.dt;
    for (int i = tid; i < MAXV / 4; i += NTK) {
      reinterpret_cast<float4*>(sgrid)[i] = __ldg(reinterpret_cast<const float4*>(dt->grid) + i);
      reinterpret_cast<float4*>(ssafe)[i] = __ldg(reinterpret_cast<const float4*>(dt->safe) + i);
      if (cmap != nullptr) reinterpret_cast<float4*>(svals)[i] = __ldg(reinterpret_cast<const float4*>(dt->vals) + i);
    }
    for (int i = tid; i < MAXV / 16; i += NTK)
      reinterpret_cast<uint4*>(sorder)[i] = __ldg(reinterpret_cast<const uint4*>(dt->order) + i);
    const uint4* bsrc = reinterpret_cast<const uint4*>(BYTES ? dt->cbin : dt->bin);   // a code's grid rank
    for (int i = tid; i < (BYTES ? MAXV : KEYS) / 16; i += NTK) reinterpret_cast<uint4*>(sbin)[i] = __ldg(bsrc + i);
  }
  for (int i = tid; i < MAXV; i += NTK) {
    sgridd[i] = (double)__ldg(tp.dt->grid + i);
    ssafed[i] = (double)__ldg(tp.dt->safe + i);
  }
  if (tid == 0) bad = 0;
  __syncthreads();

  // 1. counts of each distinct code per group (kmeans.py:58-64); consecutive threads read consecutive memory
  const int64_t Kc = kend - kbeg;                           // rows of this CTA
  const int64_t total = Kc * W;
  const bool kfast = !BYTES && sk == 1;
  bool mybad = false;
  constexpr int BATCH = 8;                                  // loads in flight per thread
  constexpr int PBATCH = 8;                                 // the pair path's
  // the panel's first element and row stride (a panel never spans two 32-column runs of code bytes), and any
  // element's place
  const TIn* const pb = BYTES ? P + j0 * K : P + j0 * sj;
  const int64_t rs = BYTES ? 32 : sk, cst = BYTES ? 1 : sj;
  auto at = [&](int64_t k, int64_t j) -> int64_t { return BYTES ? ((j >> 5) * K + k) * 32 + (j & 31) : k * sk + j * sj; };
  const bool pairs = cst == 1 && W <= 32 && W % 2 == 0 && rs % 2 == 0 && ((uintptr_t)pb) % (2 * sizeof(TIn)) == 0;
  if constexpr (FUSED) {
    // A. block.mxgemmini of the CTA's rows of the panel (block.py, mxgemmini.py): lane l owns column j0 + l, warp w
    // blocks w, w + 8, ... of 32 rows. A lane loads its block's 32 values (a warp load is one 128-byte row
    // segment), takes the block max, the scale (X) and its reciprocal, quantizes the 32 values -- the short step when
    // the block is finite with a power-of-two scale, else the general one (the TMA quantizer's two element steps) --
    // and writes the 32 code bytes as two 16-byte stores to its column of codesT. Each code is counted as it is
    // made: 6-bit codes in the thread's own 16-bit counters (private_counts), 8-bit ones by shared atomics.
    const bool live = lane < W;
    const int64_t j = j0 + lane;
    const int grow = (lane >> G) * nvp;
    uint16_t* const mine = reinterpret_cast<uint16_t*>(pw) + tid;   // [64][NTK]
    const bool six = FE + FM == 5;
    if (six) {
      for (int i = tid; i < 64 * NTK / 8; i += NTK) reinterpret_cast<uint4*>(mine - tid)[i] = make_uint4(0u, 0u, 0u, 0u);
      __syncthreads();
    }
    uint32_t mxb = 0;                                        // 8-bit: the largest bin seen (0xFF: no code)
    // the thread's counter of code c at a 32-bit shared address (the increment is a load, an add and a store)
    const uint32_t mbase = (uint32_t)__cvta_generic_to_shared(mine);
    auto tally = [&](uint32_t c) {
      if (six) {
        const uint32_t at = mbase + c * (2 * NTK);
        unsigned short cnt;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(cnt) : "r"(at));
        asm volatile("st.shared.u16 [%0], %1;" ::"r"(at), "h"((unsigned short)(cnt + 1)) : "memory");
      } else {
        const uint32_t bn = sbin[c];
        mxb = max(mxb, bn);
        atomicAdd(&counts[grow + (int)bn], 1);
      }
    };
    const int64_t b0 = kbeg / 32, b1 = kend / 32;
    for (int64_t b = b0 + warp; b < b1 && live; b += NWK)
      if (quant_block<FE, FM, QM>(reinterpret_cast<const float*>(P) + b * 32 * n + j, n, fa.X + b * n + j,
                                  fa.codesT + j * K + b * 32, fa.scale_floor, fa.rounding, tally))
        mybad = true;
    if (!six && mxb == 0xFFu) mybad = true;
    if (six) {
      __syncthreads();
      // into the CTA's histogram: warp w sums code s over the 8 warps' counters, then over the 2^G lanes (columns)
      // of a group, and the group's first lane adds the total to the code's bin
      const int sh = G < 5 ? G : 5;
      for (int sl = warp; sl < 64; sl += NWK) {
        int sum = 0;
#pragma unroll
        for (int q = 0; q < NWK; q++) sum += mine[sl * NTK - tid + q * 32 + lane];
        for (int o = 1; o < (1 << sh); o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if ((lane & ((1 << sh) - 1)) == 0 && lane < W && sum > 0) {
          const uint32_t bin = sbin[sl];
          if (bin == 0xFFu) mybad = true;
          else atomicAdd(&counts[(lane >> sh) * nvp + (int)bin], sum);
        }
      }
    }
  } else {
  // a code's grid rank from its bit pattern: the key (sign, exponent, top m fraction bits) through the table; any
  // other fraction bit set, or a key that names no code (NaN, Inf, off-grid), is not a code
  // (code bytes: the byte's rank through its own table)
  auto count = [&](TIn v, int gc) {
    uint32_t b;
    bool ok;
    if constexpr (BYTES) {
      b = sbin[(uint32_t)v];
      ok = b != 0xFFu;
    } else {
      const uint32_t u = f2u(v);
      b = sbin[u >> tp.keyshift];
      ok = (u & tp.lowmask) == 0u && b != 0xFFu;
    }
    if (!ok) mybad = true;
    else atomicAdd(&counts[gc * nvp + (int)b], 1);
  };
  using V2 = typename std::conditional<BYTES, uchar2, float2>::type;
  bool counted = false;
  if constexpr (BYTES) {
    if (pairs && priv_ok && G >= 1 && tp.ncodes <= 64 && Kc <= 16 * 32767) {
      // 6-bit codes: every thread counts its bytes in its own column of [64][NTK] 16-bit counters (a thread's column
      // pair lies in one group at G >= 1, and it sees at most 2 ceil(Kc / 16) codes) with plain shared loads and
      // stores: no atomics, and the 32 counters of one code of a warp are 64 consecutive bytes, so lanes never meet
      // in a bank whatever their codes. A code past the format's (a byte >= ncodes) is remembered by the largest
      // byte seen and counted, masked, where it cannot hurt: the whole panel is refused.
      uint16_t* const priv = reinterpret_cast<uint16_t*>(pw);
      for (int i = tid; i < 64 * NTK / 8; i += NTK) reinterpret_cast<uint4*>(priv)[i] = make_uint4(0u, 0u, 0u, 0u);
      __syncthreads();
      const int c2 = lane & 15, ro = lane >> 4;
      uint32_t mx = 0;
      if (2 * c2 < W) {
        const int64_t r0 = 2 * warp + ro;                    // rows r0, r0 + 16, ... of the CTA's
        const int64_t nr = r0 < Kc ? (Kc - 1 - r0) / 16 + 1 : 0;
        const uint16_t* src = reinterpret_cast<const uint16_t*>(pb + (kbeg + r0) * rs) + c2;
        const int64_t rstep = 8 * rs;                          // 16 rows, in 2-byte units
        uint16_t* const mine = priv + tid;
        constexpr int PB = 16;
        auto add = [&](uint32_t v) {
          const uint32_t a = v & 0xffu, b = v >> 8;
          mx = max(mx, max(a, b));
          mine[(a & 63u) * NTK] += 1;
          mine[(b & 63u) * NTK] += 1;
        };
        int64_t r = 0;
        for (; r + PB <= nr; r += PB) {
          uint32_t v[PB];
#pragma unroll
          for (int u = 0; u < PB; u++) v[u] = src[u * rstep];
          src += PB * rstep;
#pragma unroll
          for (int u = 0; u < PB; u++) add(v[u]);
        }
        for (; r < nr; r++, src += rstep) add(*src);
      }
      if (mx >= (uint32_t)tp.ncodes) mybad = true;
      __syncthreads();
      // into the CTA's histogram: warp w sums code s over the 8 warps' counters, then over the lanes of a group (its
      // two rows and its 2^(G-1) column pairs), and one lane adds the total to the group's bin
      const int sh = G - 1 < 4 ? G - 1 : 4;
      for (int sl = warp; sl < tp.ncodes; sl += NWK) {
        int sum = 0;
#pragma unroll
        for (int j = 0; j < NWK; j++) sum += priv[sl * NTK + j * 32 + lane];
        sum += __shfl_xor_sync(0xffffffffu, sum, 16);
        for (int o = 1; o < (1 << sh); o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane < 16 && (c2 & ((1 << sh) - 1)) == 0 && 2 * c2 < W && sum > 0) {
          const uint32_t bin = sbin[sl];
          if (bin == 0xFFu) mybad = true;                    // a NaN / Inf code
          else atomicAdd(&counts[(c2 >> sh) * nvp + (int)bin], sum);
        }
      }
      counted = true;
    } else if (pairs && W % 4 == 0 && rs % 4 == 0 && ((uintptr_t)pb) % 4 == 0) {
      // 8-bit codes: 4-byte quads, lane l taking columns 4 (l % 8) .. 4 (l % 8) + 3 of row l / 8 of its warp's four
      // rows, one shared atomic per code into its group's bin. A byte that is no code has bin 0xFF: remembered by the
      // largest bin seen and counted where it cannot hurt (within the 256 spare counters after the histograms; the
      // whole panel is refused)
      const int q = lane & 7, ro = lane >> 3;
      uint32_t mxb = 0;
      if (4 * q < W) {
        int rb[4];
#pragma unroll
        for (int i = 0; i < 4; i++) rb[i] = ((4 * q + i) >> G) * nvp;
        const int64_t r0 = 4 * warp + ro;                    // rows r0, r0 + 32, ... of the CTA's
        const int64_t nr = r0 < Kc ? (Kc - 1 - r0) / 32 + 1 : 0;
        const uint32_t* src = reinterpret_cast<const uint32_t*>(pb + (kbeg + r0) * rs) + q;
        const int64_t rstep = 8 * rs;                          // 32 rows, in 4-byte units
        constexpr int QB = 16;
        auto add = [&](uint32_t v) {
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const uint32_t bn = sbin[(v >> (8 * i)) & 0xffu];
            mxb = max(mxb, bn);
            atomicAdd(&counts[rb[i] + (int)bn], 1);
          }
        };
        int64_t r = 0;
        for (; r + QB <= nr; r += QB) {
          uint32_t v[QB];
#pragma unroll
          for (int u = 0; u < QB; u++) v[u] = src[u * rstep];
          src += QB * rstep;
#pragma unroll
          for (int u = 0; u < QB; u++) add(v[u]);
        }
        for (; r < nr; r++, src += rstep) add(*src);
      }
      if (mxb == 0xFFu) mybad = true;
      counted = true;
    }
  }
  if (counted) {
  } else if (pairs) {
    // a panel of at most 32 columns as float2 pairs: lane l takes the pair of columns 2 (l % 16), 2 (l % 16) + 1 of
    // row (l / 16) of its warp's two rows, so a warp instruction's 32 lanes count into (at G = 1) 16 different
    // groups' rows and the 16-byte-per-lane-pair row segments are read whole; the CTA steps 2 x 8 rows
    const int c2 = lane & 15, ro = lane >> 4;
    if (2 * c2 < W) {
      const V2* src = reinterpret_cast<const V2*>(pb) + c2;
      const int ga = (2 * c2) >> G, gb = (2 * c2 + 1) >> G;
      const int64_t step = 2 * NWK;
      for (int64_t k0 = kbeg + 2 * warp + ro; k0 < kend; k0 += step * PBATCH) {
        V2 v[PBATCH];
#pragma unroll
        for (int u = 0; u < PBATCH; u++)
          v[u] = k0 + (int64_t)u * step < kend ? src[(k0 + (int64_t)u * step) * (rs / 2)] : V2{};
#pragma unroll
        for (int u = 0; u < PBATCH; u++) {
          if (k0 + (int64_t)u * step >= kend) break;
          count(v[u].x, ga);
          count(v[u].y, gb);
        }
      }
    }
  } else if (!BYTES && sj == 1 && W % 4 == 0 && W <= 4 * NTK && sk % 4 == 0 && ((uintptr_t)(P + j0)) % 16 == 0) {
    // rows of the panel as float4: thread (row r, quad q) of rows_per_pass rows at a time, pointers advanced by
    // whole rows (no index arithmetic per element)
    const int qpr = (int)(W / 4), rows_per_pass = NTK / qpr, r = tid / qpr, q = tid - r * qpr;
    if (r < rows_per_pass) {
      const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(P) + j0) + q;
      int gc[4];
#pragma unroll
      for (int i = 0; i < 4; i++) gc[i] = (4 * q + i) >> G;
      for (int64_t k0 = kbeg + r; k0 < kend; k0 += (int64_t)rows_per_pass * BATCH) {
        float4 v[BATCH];
#pragma unroll
        for (int u = 0; u < BATCH; u++)
          v[u] = k0 + (int64_t)u * rows_per_pass < kend ? src[(k0 + (int64_t)u * rows_per_pass) * (sk / 4)]
                                                        : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int u = 0; u < BATCH; u++) {
          if (k0 + (int64_t)u * rows_per_pass >= kend) break;
          count(v[u].x, gc[0]);
          count(v[u].y, gc[1]);
          count(v[u].z, gc[2]);
          count(v[u].w, gc[3]);
        }
      }
    }
  } else if (total > 0) {
  // element e = (kfast ? jj * Kc + k : k * W + jj) walked without a division per element: the position (major,
  // minor) advances by NTK elements as (NTK / R, NTK % R) with R the minor extent, plus a carry
  const int64_t R = kfast ? Kc : W, dmaj = NTK / R, dmin = NTK % R;
  int64_t maj = tid / R, mnr = tid % R;
  for (int64_t e0 = tid; e0 < total; e0 += (int64_t)NTK * BATCH) {
    TIn v[BATCH];
    int gcol[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; u++) {
      const int64_t e = e0 + (int64_t)u * NTK;
      const int64_t k = kfast ? mnr : maj, jj = kfast ? maj : mnr;
      gcol[u] = e < total ? (int)(jj >> G) : -1;
      v[u] = e < total ? P[at(kbeg + k, j0 + jj)] : TIn{};
      maj += dmaj;
      mnr += dmin;
      if (mnr >= R) {
        mnr -= R;
        maj++;
      }
    }
#pragma unroll
    for (int u = 0; u < BATCH; u++)
      if (gcol[u] >= 0) count(v[u], gcol[u]);
  }
  }
  }
  if (mybad) bad = 1;
  // the cluster's CTAs meet: every histogram of the panel is complete (cluster barriers order shared memory across
  // the cluster); CTA r merges groups r, r + cs, ... from all of them into its own rows, then they meet again so no
  // CTA leaves while another still reads its histograms. Every thread of every CTA reaches every barrier: a bad code
  // anywhere in the panel sends the whole cluster out after the second one.
  cluster.sync();
  if (bad && tid == 0) atomicExch(status, 1);
  int anybad = 0;
  for (int q = 0; q < cs; q++) anybad |= *cluster.map_shared_rank(&bad, q);
  if (cs > 1) {
    const int nown = (gpc - rank + cs - 1) / cs;             // this CTA's groups: rank, rank + cs, ...
    for (int i = tid; i < nown * nv; i += NTK) {
      const int gi = i / nv, b = i - gi * nv;
      const int idx = (rank + cs * gi) * nvp + b;
      int part[8];                                           // cs <= 8: every remote read in flight at once
#pragma unroll
      for (int q = 0; q < 8; q++) part[q] = q < cs ? cluster.map_shared_rank(counts, q)[idx] : 0;
      int sum = 0;
#pragma unroll
      for (int q = 0; q < 8; q++) sum += part[q];
      counts[idx] = sum;                                     // only this CTA reads row gl of its own histogram
    }
  }
  cluster.sync();
  if (anybad) return;

  for (int gl = rank + cs * warp; gl < gpc; gl += cs * NWK) {
    const int64_t g = g0 + gl;
    if (g >= ng) break;
    const int* cnt = counts + gl * nvp;
    double* PW = pw + warp * (nv + 1);                        // warp < nfw: gl = rank + cs * warp < gpc
    double* PWX = pwx + warp * (nv + 1);
    // 2. prefix sums over the sorted codes, and the number of distinct codes present: lane l sums its run of q
    // consecutive codes, one warp scan gives each run's offset, then the run's prefixes are written (the sums are
    // exact, so any order gives the same bits)
    const int q = (nv + 31) >> 5, b0 = lane * q, b1 = b0 + q < nv ? b0 + q : nv;
    double w = 0.0, wx = 0.0;
    int npres = 0;
    for (int b = b0; b < b1; b++) {
      const int cb = cnt[b];
      w = __dadd_rn(w, i2d(cb));
      wx = __dadd_rn(wx, __dmul_rn(i2d(cb), sgridd[b]));
      npres += cb > 0;
    }
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {                       // inclusive scans of the runs' sums
      const double ow = __shfl_up_sync(0xffffffffu, w, s), ox = __shfl_up_sync(0xffffffffu, wx, s);
      if (lane >= s) {
        w = __dadd_rn(w, ow);
        wx = __dadd_rn(wx, ox);
      }
      npres += __shfl_xor_sync(0xffffffffu, npres, s);
    }
    {
      double rw = __shfl_up_sync(0xffffffffu, w, 1), rx = __shfl_up_sync(0xffffffffu, wx, 1);
      if (lane == 0) {
        rw = 0.0;
        rx = 0.0;
        PW[0] = 0.0;
        PWX[0] = 0.0;
      }
      for (int b = b0; b < b1; b++) {
        const int cb = cnt[b];
        rw = __dadd_rn(rw, i2d(cb));
        rx = __dadd_rn(rx, __dmul_rn(i2d(cb), sgridd[b]));
        PW[b + 1] = rw;
        PWX[b + 1] = rx;
      }
    }
    __syncwarp();

    double c = INFINITY;                                     // lane t < 16: centre t
    if (npres <= LUT) {                                      // 2a: the present codes are the centres, ascending
      int base = 0;
      for (int b0 = 0; b0 < nv; b0 += 32) {
        const int b = b0 + lane;
        const bool pr = b < nv && cnt[b] > 0;
        const unsigned mask = __ballot_sync(0xffffffffu, pr);
        if (pr) scratch[warp][base + __popc(mask & lt)] = sgridd[b];
        base += __popc(mask);
      }
      __syncwarp();
      if (lane < npres) c = scratch[warp][lane];
      __syncwarp();
    } else {
      // 2b: quantile seeds: the first code whose cumulative weight share (rounded, so non-decreasing) reaches
      // p_t = (t + 0.5) / 16, i.e. seed_t = #{codes b : share_b < p_t}. Code b's count of probes at or below its
      // share, q_b = #{t : p_t <= share_b}, is floor(16 share_b - 0.5) + 1 clamped to [0, 16] (16 share_b - 0.5 is
      // exact; the floor is the round-down add of 2^52); then share_b < p_t exactly when q_b <= t, so seed_t is the
      // prefix sum up to t of a 17-bin histogram of the q_b, which every lane fills for its codes at once
      const double tot = PW[nv];
      int* const qh = reinterpret_cast<int*>(fsum[warp]);   // 17 counters (fsum's first use comes later)
      if (lane <= LUT) qh[lane] = 0;
      __syncwarp();
      for (int b = lane; b < nv; b += 32) {
        const double y = __dsub_rn(__dmul_rn(__ddiv_rn(PW[b + 1], tot), (double)LUT), 0.5);
        const int q = y < 0.0 ? 0 : min(__double2loint(__dadd_rd(y, 4503599627370496.0)) + 1, LUT);
        atomicAdd(&qh[q], 1);
      }
      __syncwarp();
      int seed = lane <= LUT ? qh[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {                     // inclusive prefix sums over lanes 0..16
        const int up = __shfl_up_sync(0xffffffffu, seed, o);
        if (lane >= o) seed += up;
      }
      __syncwarp();
      if (lane < LUT) c = sgridd[seed < nv - 1 ? seed : nv - 1];
      c = dedupe_lanes(c, scratch[warp]);
      // 2c: weighted Lloyd passes
      for (int it = 0; it < max_iters; it++) {
        const double cn = __shfl_down_sync(0xffffffffu, c, 1);          // centre t + 1
        const bool close = lane < LUT - 1 && finite_d(cn) && __dsub_rn(cn, c) < MIN_GAP;
        double nw;
        if (!__any_sync(0xffffffffu, close)) {
          int end = nv;                                                  // first code past centre t's run
          if (lane < LUT - 1 && finite_d(cn)) {
            // the first code strictly closer to centre t + 1 (monotone along the sorted codes, as the gap check
            // above guarantees): start at the codes around the midpoint of the two centres and walk to it
            auto closer = [&](int k) {
              const double x = sgridd[k];
              return fabs(__dsub_rn(x, cn)) < fabs(__dsub_rn(x, c));
            };
            int i = grid_rank((float)__dmul_rn(__dadd_rn(c, cn), 0.5), tp);
            if (closer(i)) {
              while (i > 0 && closer(i - 1)) i--;
            } else {
              while (i < nv && !closer(i)) i++;
            }
            end = i;
          }
          int begin = __shfl_up_sync(0xffffffffu, end, 1);
          if (lane == 0) begin = 0;
          double ws = 0.0, sm = 0.0;
          if (lane < LUT && begin < end) {
            ws = __dsub_rn(PW[end], PW[begin]);
            sm = __dsub_rn(PWX[end], PWX[begin]);
          }
          nw = ws > 0.0 ? __ddiv_rn(sm, ws) : c;
        } else {                                                         // code by code, as the reference's argmin
          if (lane < LUT) {
            fsum[warp][lane] = 0.0;
            fw[warp][lane] = 0.0;
          }
          double cc[LUT];
#pragma unroll
          for (int t = 0; t < LUT; t++) cc[t] = __shfl_sync(0xffffffffu, c, t);
          __syncwarp();
          for (int b = lane; b < nv; b += 32) {
            if (cnt[b] == 0) continue;
            const double x = sgridd[b];
            int best = 0;
            double bd = fabs(__dsub_rn(x, cc[0]));
#pragma unroll
            for (int t = 1; t < LUT; t++) {
              const double d = fabs(__dsub_rn(x, cc[t]));
              if (d < bd) {
                bd = d;
                best = t;
              }
            }
            atomicAdd(&fsum[warp][best], __dmul_rn(i2d(cnt[b]), x));
            atomicAdd(&fw[warp][best], i2d(cnt[b]));
          }
          __syncwarp();
          const double ws = lane < LUT ? fw[warp][lane] : 0.0, sm = lane < LUT ? fsum[warp][lane] : 0.0;
          nw = ws > 0.0 ? __ddiv_rn(sm, ws) : c;
          __syncwarp();
        }
        // _dedupe (sort, equal neighbours to +inf, sort) is the identity on centres that are already strictly
        // increasing with any +inf at the end, which the run-based pass produces: skip it then
        nw = lane < LUT ? nw : INFINITY;
        const double nx = __shfl_down_sync(0xffffffffu, nw, 1);
        const bool ordered = lane >= LUT - 1 || nw < nx || (nw == INFINITY && nx == INFINITY);
        if (!__all_sync(0xffffffffu, ordered)) nw = dedupe_lanes(nw, scratch[warp]);
        const bool valid = finite_d(c);
        const bool ok = lane >= LUT || (finite_d(nw) == valid &&
                                        (!valid || fabs(__dsub_rn(nw, c)) <= __dadd_rn(1e-8, __dmul_rn(1e-5, fabs(c)))));
        if (__all_sync(0xffffffffu, ok)) break;                          // converged: keep the current centres
        c = nw;
      }
    }
    // 3. each centre snapped to the nearest finder-safe value (safe is sorted: the nearest is a neighbour of the
    // insertion point), ties to the smaller
    for (int i = lane; i < tp.nsafe; i += 32) member[warp][i] = 0;
    __syncwarp();
    if (lane < LUT && finite_d(c)) {
      int lo = 0, hi = tp.nsafe;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (ssafed[mid] < c) lo = mid + 1;
        else hi = mid;
      }
      int best = lo < tp.nsafe ? lo : tp.nsafe - 1;
      if (lo > 0 && (lo == tp.nsafe || fabs(__dsub_rn(c, ssafed[lo - 1])) <= fabs(__dsub_rn(c, ssafed[lo]))))
        best = lo - 1;
      member[warp][best] = 1;
    }
    __syncwarp();
    // 4. pad with unused values, smallest magnitude first, then write the members in ascending order
    int nmem = 0;
    for (int i0 = 0; i0 < tp.nsafe; i0 += 32) {
      const int i = i0 + lane;
      nmem += __popc(__ballot_sync(0xffffffffu, i < tp.nsafe && member[warp][i]));
    }
    int need = LUT - nmem;
    for (int i0 = 0; i0 < tp.nsafe && need > 0; i0 += 32) {
      const int i = i0 + lane;
      const int sidx = i < tp.nsafe ? sorder[i] : 0;
      const bool fr = i < tp.nsafe && !member[warp][sidx];
      const unsigned mask = __ballot_sync(0xffffffffu, fr);
      __syncwarp();
      if (fr && __popc(mask & lt) < need) member[warp][sidx] = 1;
      need -= __popc(mask);
      __syncwarp();
    }
    int base = 0;
    for (int i0 = 0; i0 < tp.nsafe && base < LUT; i0 += 32) {
      const int i = i0 + lane;
      const bool mb = i < tp.nsafe && member[warp][i];
      const unsigned mask = __ballot_sync(0xffffffffu, mb);
      const int pos = base + __popc(mask & lt);
      if (mb && pos < LUT) {
        T[g * LUT + pos] = ssafe[i];
        stab[warp][pos] = ssafe[i];
      }
      base += __popc(mask);
    }
    if (lane >= base && lane < LUT) {
      T[g * LUT + lane] = INFINITY;
      stab[warp][lane] = INFINITY;
    }
    __syncwarp();
    if (cmap != nullptr) {
      // block.lut: the entry pick(P, T) chooses for each code's value (nearest of the two sorted entries around it,
      // ties to the lower index), so that the lookup of an element is one read
      const float* t = stab[warp];
      for (int c = lane; c < tp.ncodes; c += 32) {
        const float v = svals[c];
        int b = 0;
        b += t[b + 7] < v ? 8 : 0;
        b += t[b + 3] < v ? 4 : 0;
        b += t[b + 1] < v ? 2 : 0;
        b += t[b] < v ? 1 : 0;
        const int lb = b + (b == LUT - 1 && t[LUT - 1] < v ? 1 : 0);
        const int lo = lb < 1 ? 0 : (lb > LUT - 1 ? LUT - 2 : lb - 1);
        const float rl = t[lo], rh = t[lo + 1];
        cmap[g * tp.ncodes + c] = abs_f(__fsub_rn(v, rl)) <= abs_f(__fsub_rn(rh, v)) ? rl : rh;
      }
    }
  }
  if constexpr (BYTES) {
  if (out == nullptr) return;

  // 5. block.lut: every code of this CTA's rows replaced by its group's map entry. The panel's maps come from the
  // cluster's fits through global memory (ordered by the fence and the cluster barrier; every CTA of the cluster
  // reaches it) into padded shared rows over the dead histograms; the codes are read a second time (from L2).
  __threadfence();
  cluster.sync();
  float* const smap = reinterpret_cast<float*>(counts);      // [groups of the panel][ncodes + 1]
  const int nc = tp.ncodes, ncp = nc + 1;
  const int ngp = (int)((g0 + gpc < ng ? g0 + gpc : ng) - g0);
  for (int i = tid; i < ngp * nc; i += NTK) {
    const int gi = i / nc;
    smap[i + gi] = __ldcg(cmap + g0 * nc + i);
  }
  __syncthreads();
  if constexpr (FUSED) {
    // lane l: column j0 + l, its codes of each of the warp's blocks (two 16-byte loads, from L2), 32 coalesced rows
    if (lane < W) {
      const int64_t j = j0 + lane;
      const float* m = smap + (lane >> G) * ncp;
      for (int64_t b = kbeg / 32 + warp; b < kend / 32; b += NWK) {
        const uint4* src = reinterpret_cast<const uint4*>(fa.codesT + j * K + b * 32);
        const uint4 c0 = __ldcs(src), c1 = __ldcs(src + 1);
        const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        float* dst = out + b * 32 * n + j;
#pragma unroll
        for (int i = 0; i < 32; i++) __stcs(dst + i * n, m[(w[i >> 2] >> (8 * (i & 3))) & 0xffu]);
      }
    }
  } else if (pairs && W % 4 == 0 && rs % 4 == 0 && ((uintptr_t)pb) % 4 == 0 && n % 4 == 0 &&
      ((uintptr_t)(out + j0)) % 16 == 0) {
    // 4 codes (one 4-byte load, the histogram's quads) into one float4 store per lane
    const int q = lane & 7, ro = lane >> 3;
    if (4 * q < W) {
      int mo[4];
#pragma unroll
      for (int i = 0; i < 4; i++) mo[i] = ((4 * q + i) >> G) * ncp;
      const int64_t r0 = 4 * warp + ro;                      // rows r0, r0 + 32, ... of the CTA's
      const int64_t nr = r0 < Kc ? (Kc - 1 - r0) / 32 + 1 : 0;
      const uint32_t* src = reinterpret_cast<const uint32_t*>(pb + (kbeg + r0) * rs) + q;
      float4* dst = reinterpret_cast<float4*>(out + (kbeg + r0) * n + j0) + q;
      const int64_t rstep = 8 * rs, ostep = 8 * n;             // 32 rows of codes (4-byte units), of out (float4s)
      auto put = [&](uint32_t v, float4* o) {
        __stcs(o, make_float4(smap[mo[0] + (int)(v & 0xffu)], smap[mo[1] + (int)((v >> 8) & 0xffu)],
                              smap[mo[2] + (int)((v >> 16) & 0xffu)], smap[mo[3] + (int)(v >> 24)]));
      };
      constexpr int LB = 8;
      int64_t r = 0;
      for (; r + LB <= nr; r += LB) {
        uint32_t v[LB];
#pragma unroll
        for (int u = 0; u < LB; u++) v[u] = __ldcs(src + u * rstep);
#pragma unroll
        for (int u = 0; u < LB; u++) put(v[u], dst + u * ostep);
        src += LB * rstep;
        dst += LB * ostep;
      }
      for (; r < nr; r++, src += rstep, dst += ostep) put(__ldcs(src), dst);
    }
  } else {
    for (int64_t e = tid; e < total; e += NTK) {              // element (k, jj) of the CTA's rows
      const int64_t k = kbeg + e / W, jj = e % W;
      out[k * n + j0 + jj] = smap[(int)(jj >> G) * ncp + (int)P[at(k, j0 + jj)]];
    }
  }
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
    if (c < -ct.ncodes || c >= ct.ncodes) {              // torch indexing: a negative code counts from the end
      atomicOr(status, 1);
      out[i] = 0.0f;
    } else {
      out[i] = ct.vals[c < 0 ? c + ct.ncodes : c];
    }
  }
}

// finder (formats.py:140-159): fixed points of the code and of the 16 entries, masked |difference|, first minimum.
// status bits: 1 a code outside [-ncodes, ncodes) (negative codes count from the end, as torch indexes), 2 a table
// value that is no code; the caller raises for bit 1 first, as the reference indexes the codes first.
__global__ void k_lut_finder(const int64_t* __restrict__ codes, const float* __restrict__ T, int64_t K, int64_t n,
                             int G, long long mask, const __grid_constant__ CodeTables ct, int64_t* __restrict__ I,
                             int* __restrict__ status) {
  const int64_t total = K * n;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = e % n, c = codes[e];
    if (c < -ct.ncodes || c >= ct.ncodes) {
      atomicOr(status, 1);
      I[e] = 0;
      continue;
    }
    const long long f = ct.fx[c < 0 ? c + ct.ncodes : c];
    const float* row = T + (j >> G) * LUT;
    int best = 0;
    long long bd = 0;
    for (int t = 0; t < LUT; t++) {
      int tc = encode1(ct, __ldg(row + t));
      if (tc < 0) {
        atomicOr(status, 2);
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

// Column forms of pick and finder for a row-major K x n operand with 16-entry tables; consecutive threads take
// consecutive columns and walk rows, so every warp reads and writes whole row segments.
//   pick: a CTA owns a panel of CT = 256 columns (one per thread) and a slice of rows; the panel's tables are
//         staged once per CTA (a copy), the search runs on them in shared memory.
//   finder: a CTA owns a panel of PW = 32 columns (lane l of every warp is column l) and its 8 warps take the rows
//         in turn, because each CTA first evaluates the answer for every (group, code) pair of its panel: with
//         256-column panels that table work, repeated by every row slice, dominated the kernel.
constexpr int CT = 256, PW = 32, CW = CT / 32;               // threads, finder panel columns, warps per CTA

constexpr int ROWP = LUT + 1;                                // a table row in shared memory, padded (banks)

__global__ void __launch_bounds__(CT) k_lut_pick_cols(const float* __restrict__ P, const float* __restrict__ T,
                                                      int64_t K, int64_t n, int G, int64_t rows,
                                                      int64_t* __restrict__ I, float* __restrict__ out_vals) {
  __shared__ float st[CT * ROWP];                            // the panel's tables (at most one per column)
  const int64_t jp = (int64_t)blockIdx.x * CT, j = jp + threadIdx.x;
  const int64_t gfirst = jp >> G, glast = ((jp + CT < n ? jp + CT : n) - 1) >> G;
  const int ngp = (int)(glast - gfirst + 1);
  for (int i = threadIdx.x; i < ngp * LUT; i += CT) st[(i / LUT) * ROWP + i % LUT] = __ldg(T + gfirst * LUT + i);
  __syncthreads();
  if (j >= n) return;
  const int64_t k0 = (int64_t)blockIdx.y * rows, k1 = k0 + rows < K ? k0 + rows : K;
  const float* t = st + (int)((j >> G) - gfirst) * ROWP;
  constexpr int BATCH = 4;                                   // loads in flight per thread
  for (int64_t kb = k0; kb < k1; kb += BATCH) {
    float vb[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; u++) vb[u] = kb + u < k1 ? P[(kb + u) * n + j] : 0.0f;
#pragma unroll
    for (int u = 0; u < BATCH; u++) {
    const int64_t k = kb + u;
    if (k >= k1) break;
    const float v = vb[u];
    int base = 0;                                            // lower_bound over 16 sorted entries, branch-free
    base += t[base + 7] < v ? 8 : 0;
    base += t[base + 3] < v ? 4 : 0;
    base += t[base + 1] < v ? 2 : 0;
    base += t[base] < v ? 1 : 0;
    const int lb = base + (base == LUT - 1 && t[LUT - 1] < v ? 1 : 0);
    const int lo = lb < 1 ? 0 : (lb > LUT - 1 ? LUT - 2 : lb - 1);
    const float rl = t[lo], rh = t[lo + 1];
    const bool left = abs_f(__fsub_rn(v, rl)) <= abs_f(__fsub_rn(rh, v));
    if (out_vals) out_vals[k * n + j] = left ? rl : rh;
    else I[k * n + j] = lo + (left ? 0 : 1);
    }
  }
}

// finder: each CTA first tabulates the answer for every (group of its panel, code) pair -- 16 masked fixed-point
// distances, first minimum, as a packed (distance << 4 | index) minimum -- then an element is a shared-memory read.
template <typename F>                                        // F: int where every fixed point fits, else long long
__global__ void __launch_bounds__(CT) k_lut_finder_cols(const int64_t* __restrict__ codes, const float* __restrict__ T,
                                                        int64_t K, int64_t n, int G, int64_t rows, long long mask,
                                                        const __grid_constant__ CodeTables ct,
                                                        int64_t* __restrict__ I, int* __restrict__ status) {
  extern __shared__ unsigned char ans[];                     // [groups of the panel][ncodes]
  __shared__ F sfx[MAXV];
  __shared__ F sft[PW][LUT];                                 // the panel's tables as fixed points
  __shared__ uint32_t sbits[MAXV];                           // encode's map (value bits -> lowest code), staged
  __shared__ int16_t scode[MAXV];
  const int nc = ct.ncodes, ne = ct.nenc;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t jp = (int64_t)blockIdx.x * PW;
  const int64_t gfirst = jp >> G, glast = ((jp + PW < n ? jp + PW : n) - 1) >> G;
  const int ngp = (int)(glast - gfirst + 1);
  const int64_t k0 = (int64_t)blockIdx.y * rows, k1 = k0 + rows < K ? k0 + rows : K;
  for (int i = threadIdx.x; i < nc; i += CT) sfx[i] = (F)ct.fx[i];
  for (int i = threadIdx.x; i < ne; i += CT) {
    sbits[i] = ct.enc_bits[i];
    scode[i] = ct.enc_code[i];
  }
  __syncthreads();
  bool tbad = false;
  for (int i = threadIdx.x; i < ngp * LUT; i += CT) {
    const uint32_t b = f2u(__ldg(T + gfirst * LUT + i));
    int lo = 0, hi = ne;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (sbits[mid] < b) lo = mid + 1;
      else hi = mid;
    }
    int tc = (lo < ne && sbits[lo] == b) ? scode[lo] : -1;
    if (tc < 0) {
      tbad = true;
      tc = 0;
    }
    sft[i / LUT][i % LUT] = sfx[tc];
  }
  if (tbad && k1 > k0) atomicOr(status, 2);
  __syncthreads();
  const F fm = (F)mask;
  for (int i = threadIdx.x; i < ngp * nc; i += CT) {
    const int gl = i / nc;
    const F f = sfx[i % nc];
    long long key = 0;
#pragma unroll
    for (int t = 0; t < LUT; t++) {
      F d = f - sft[gl][t];
      d = d < 0 ? -d : d;
      if (mask) d &= fm;
      const long long kt = ((long long)d << 4) | t;          // the smaller distance, then the lower index
      key = (t == 0 || kt < key) ? kt : key;
    }
    ans[i] = (unsigned char)(key & 15);
  }
  __syncthreads();
  const int64_t j = jp + lane;
  if (j >= n) return;
  const unsigned char* a = ans + (int)((j >> G) - gfirst) * nc;
  constexpr int BATCH = 8;                                   // loads in flight per thread
  for (int64_t kb = k0 + warp; kb < k1; kb += (int64_t)CW * BATCH) {
    int64_t c[BATCH];
#pragma unroll
    for (int u = 0; u < BATCH; u++) {
      const int64_t k = kb + (int64_t)u * CW;
      c[u] = k < k1 ? (int64_t)__ldcs(reinterpret_cast<const long long*>(codes) + k * n + j) : 0;
    }
#pragma unroll
    for (int u = 0; u < BATCH; u++) {
      const int64_t k = kb + (int64_t)u * CW;
      if (k >= k1) break;
      int64_t r = 0;
      if (c[u] < -nc || c[u] >= nc) atomicOr(status, 1);
      else r = a[c[u] < 0 ? c[u] + nc : c[u]];
      __stcs(reinterpret_cast<long long*>(I) + k * n + j, (long long)r);
    }
  }
}

// the column kernels' grid: panels of `width` columns, and row slices so that about per_sm CTAs per SM are launched
dim3 cols_grid(int64_t K, int64_t n, int64_t width, int per_sm, int64_t* rows) {
  const int64_t panels = (n + width - 1) / width;
  const int64_t want = per_sm * (int64_t)sm_count();
  int64_t slices = (want + panels - 1) / panels;
  if (slices > K) slices = K;
  if (slices < 1) slices = 1;
  *rows = (K + slices - 1) / slices;
  return dim3((unsigned)panels, (unsigned)((K + *rows - 1) / *rows));
}

int fmt_slot_check(int e, int m, const char* what) {
  MXQ_REQUIRE(format_tables(e, m) != nullptr, MXQ_ERR_VALUE,
              "mxq.lut: (e=%d, m=%d) is not a LUT format; MX-Gemmini sends MXFP6_E3M2, MXFP6_E2M3, MXFP8_E5M2, "
              "MXFP8_E4M3 through LUTs (%s)",
              e, m, what);
  return MXQ_OK;
}

// The format's DevTables on the current device, uploaded on its first use there (a synchronous copy; again after the
// context changes, as cudaDeviceReset makes a new one with fresh module globals)
int device_tables(int e, int m, const DevTables** out) {
  static std::mutex mu;
  static unsigned long long loaded[64][4] = {};              // the context each slot was uploaded in
  const int slot = (e == 3 && m == 2) ? 0 : (e == 2 && m == 3) ? 1 : (e == 5 && m == 2) ? 2 : 3;
  const FormatTables* f = format_tables(e, m);
  int dev = 0;
  if (int r = check_cuda(cudaGetDevice(&dev), "lut tables: device")) return r;
  MXQ_REQUIRE(dev >= 0 && dev < 64, MXQ_ERR_UNSUPPORTED, "lut tables: device %d", dev);
  void* base = nullptr;
  if (int r = check_cuda(cudaGetSymbolAddress(&base, g_dev_tables), "lut tables: device tables")) return r;
  DevTables* mine = static_cast<DevTables*>(base) + slot;
  const unsigned long long ctx = context_id();
  std::lock_guard<std::mutex> lock(mu);
  if (ctx == 0 || loaded[dev][slot] != ctx) {
    std::unique_ptr<DevTables> h(new DevTables());
    for (int i = 0; i < MAXV; i++) {
      h->grid[i] = i < f->nv ? f->grid[i] : INFINITY;
      h->safe[i] = i < f->nsafe ? f->safe[i] : INFINITY;
      h->order[i] = i < f->nsafe ? f->order[i] : 0;
      h->vals[i] = i < f->ncodes ? f->vals[i] : NAN;
    }
    const int keyshift = 23 - m;
    for (int i = 0; i < KEYS; i++) h->bin[i] = 0xFF;
    for (int b = 0; b < f->nv; b++) h->bin[f2u(f->grid[b]) >> keyshift] = (uint8_t)b;
    for (int b = 0; b < f->nv; b++)                        // -0 counts as the zero code (the grid holds +0)
      if (f->grid[b] == 0.0f) h->bin[0x80000000u >> keyshift] = (uint8_t)b;
    for (int c = 0; c < MAXV; c++) {                       // a code byte's rank: its value's place in the grid
      h->cbin[c] = 0xFF;
      if (c < f->ncodes && !std::isnan(f->vals[c]) && !std::isinf(f->vals[c]))
        for (int b = 0; b < f->nv; b++)
          if (f->grid[b] == f->vals[c]) h->cbin[c] = (uint8_t)b;
    }
    if (int r = check_cuda(cudaMemcpy(mine, h.get(), sizeof(DevTables), cudaMemcpyHostToDevice), "lut tables: upload"))
      return r;
    loaded[dev][slot] = ctx;
  }
  *out = mine;
  return MXQ_OK;
}

template <typename TIn, int FE = 0, int FM = 0, int QM = -1>
int launch_tables(const TIn* P, float* T, int64_t K, int64_t n, int64_t sk, int64_t sj, int32_t group,
                   int32_t max_iters, int32_t e, int32_t m, int32_t* status, void* stream, bool zero_status = true,
                   float* cmap = nullptr, float* out = nullptr, const FusedArgs& fa = FusedArgs{}) {
  constexpr bool FUSED = QM >= 0;
  constexpr int NTH = NT;
  auto kernel = k_lut_tables<TIn, FE, FM, QM, NTH>;
  if (int r = fmt_slot_check(e, m, "tables")) return r;
  MXQ_REQUIRE(group >= 0 && group < 31, MXQ_ERR_VALUE, "mxq.lut: group %d must be a non-negative integer", group);
  MXQ_REQUIRE(max_iters >= 0, MXQ_ERR_VALUE, "mxq.lut: max_iters %d must be a non-negative integer", max_iters);
  MXQ_REQUIRE(status != nullptr, MXQ_ERR_VALUE, "mxq.lut.tables: no status word");
  const FormatTables* f = format_tables(e, m);
  MXQ_REQUIRE(f->nmag > 0, MXQ_ERR_UNSUPPORTED, "lut.tables: (e=%d, m=%d) has no sign-magnitude grid", e, m);
  cudaStream_t st = as_stream(stream);
  if (zero_status)
    if (int r = check_cuda(cudaMemsetAsync(status, 0, sizeof(int32_t), st), "lut.tables")) return r;
  const int64_t ng = (n + ((int64_t)1 << group) - 1) >> group;
  if (ng == 0) return MXQ_OK;
  TableParams tp;
  tp.nv = f->nv;
  tp.nsafe = f->nsafe;
  tp.ncodes = f->ncodes;
  tp.nmag = f->nmag;
  tp.bias = (1 << (e - 1)) - 1;
  tp.m = m;
  tp.keyshift = 23 - m;
  tp.lowmask = (1u << (23 - m)) - 1u;
  if (int r = device_tables(e, m, &tp.dt)) return r;
  // A cluster of cs CTAs per panel of gpc groups (32 columns, or one group when a group is wider): the CTAs split
  // the panel's rows (fused: whole blocks of 32) for the histogram and its groups for the fits; cs (1..8) makes about
  // three CTAs per SM. (Clusters of eight CTAs of 128 threads, eight to an SM, measured slower for the fused kernel:
  // more registers spilled, and the eight-CTA clusters did not spread more evenly over the SMs.)
  const int gpc = group >= 5 ? 1 : (32 >> group);
  const int64_t panels = (ng + gpc - 1) / gpc;
  int cs = 1;
  while (cs < 8 && panels * cs < 3 * (int64_t)sm_count() && 2 * cs <= (FUSED ? K / 32 : K)) cs *= 2;
  // dynamic shared memory: the histograms, then one region for the fits' prefix sums, the private counters of
  // 6-bit code bytes, and (code bytes) room for the spare counts of bytes that are no code; the panel's maps over all
  const int priv_ok = (FUSED || (sizeof(TIn) == 1 && group >= 1)) && f->ncodes <= 64;
  size_t region = 2 * (size_t)fit_warps(gpc, cs, NTH / 32) * (f->nv + 1) * sizeof(double);
  if (priv_ok) region = std::max(region, (size_t)64 * NTH * sizeof(uint16_t));
  if (FUSED || sizeof(TIn) == 1) region = std::max(region, (size_t)MAXV * sizeof(int));
  size_t smem = (((size_t)gpc * (f->nv | 1) + 3) & ~(size_t)3) * sizeof(int) + region;
  if (out != nullptr) smem = std::max(smem, (size_t)gpc * (f->ncodes + 1) * sizeof(float));
  // the histograms and the prefix sums (up to 33 KB) with the static tables (~10 KB) may pass the 48 KB default
  if (int r = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                         "lut.tables: shared memory attribute"))
    return r;
  // all of shared memory for the L1 / shared split, so four CTAs (with their static ~40 KB) fit on an SM
  if (int r = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100),
                         "lut.tables: shared memory carveout"))
    return r;
  MXQ_REQUIRE(panels * cs < (1ll << 31), MXQ_ERR_UNSUPPORTED, "lut.tables: %lld column groups", (long long)ng);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(panels * cs));
  cfg.blockDim = dim3(NTH);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (int r = check_cuda(cudaLaunchKernelEx(&cfg, kernel, P, K, n, sk, sj, (int)group, gpc, (int)max_iters,
                                            priv_ok, tp, T, status, cmap, out, fa),
                         "lut.tables"))
    return r;
  return MXQ_LAUNCH_CHECK("lut.tables");
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

namespace mxq {
// block.lut from code bytes (K x n, stored by 32-column panels as the quantizer's OutCodes writes them): the tables of the codes (status not zeroed: the quantizer's bits stay),
// every group's code -> entry map (cmap, groups x ncodes, the entry pick would choose for the code's value), and every
// code replaced by its entry in `out`, in one launch
int lut_tables_codes_lookup(const uint8_t* codes, float* T, float* cmap, float* out, int64_t K, int64_t n,
                            int32_t group, int32_t max_iters, int32_t e, int32_t m, int32_t* status, void* stream) {
  return launch_tables(codes, T, K, n, n, 1, group, max_iters, e, m, status, stream, false, cmap, out);
}

// block.lut in one launch (axis 0, block.mxgemmini without via, blocks of 32): V (row-major K x n) quantized, its
// scales to X, its code bytes to codesT (n x K), the tables to T, each group's code -> entry map to cmap and the
// looked-up values to out. MXQ_ERR_UNSUPPORTED unless K is a multiple of 32, group <= 5 and the buffers are aligned
// (status is not zeroed).
int block_lut_fused(const float* V, float* out, float* X, float* T, float* cmap, uint8_t* codesT, int64_t K, int64_t n,
                    int32_t group, int32_t max_iters, int32_t e, int32_t m, int32_t rounding, float scale_floor,
                    int32_t* status, void* stream) {
  if (K % 32 || K == 0 || n == 0 || group > 5 || rounding < 0 || rounding > 2 || (uintptr_t)codesT % 16 ||
      K >= (1ll << 31) || n >= (1ll << 31))
    return MXQ_ERR_UNSUPPORTED;
  const FusedArgs fa{X, codesT, scale_floor, rounding};
  auto go = [&](auto fe, auto fm) -> int {
    constexpr int E = decltype(fe)::value, M = decltype(fm)::value;
    if (rounding == 0)
      return launch_tables<float, E, M, 0>(V, T, K, n, n, 1, group, max_iters, e, m, status, stream, false, cmap, out, fa);
    if (rounding == 1)
      return launch_tables<float, E, M, 1>(V, T, K, n, n, 1, group, max_iters, e, m, status, stream, false, cmap, out, fa);
    return launch_tables<float, E, M, 2>(V, T, K, n, n, 1, group, max_iters, e, m, status, stream, false, cmap, out, fa);
  };
  if (e == 3 && m == 2) return go(std::integral_constant<int, 3>{}, std::integral_constant<int, 2>{});
  if (e == 2 && m == 3) return go(std::integral_constant<int, 2>{}, std::integral_constant<int, 3>{});
  if (e == 4 && m == 3) return go(std::integral_constant<int, 4>{}, std::integral_constant<int, 3>{});
  if (e == 5 && m == 2) return go(std::integral_constant<int, 5>{}, std::integral_constant<int, 2>{});
  return MXQ_ERR_UNSUPPORTED;
}
}  // namespace mxq

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
  return launch_tables(P, T, K, n, sk, sj, group, max_iters, e, m, status, stream);
}

int mxq_lut_pick(const float* P, const float* T, int64_t* I, int64_t K, int64_t n, int64_t sk, int64_t sj,
                 int32_t group, int32_t width, void* stream) {
  MXQ_REQUIRE(width >= 2, MXQ_ERR_VALUE, "mxq.lut.pick: tables need width >= 2");
  if (K * n == 0) return MXQ_OK;
  if (sj == 1 && sk == n && width == LUT && (uintptr_t)T % 16 == 0 && K < (1ll << 31)) {
    int64_t rows;
    const dim3 grid = cols_grid(K, n, CT, 16, &rows);
    k_lut_pick_cols<<<grid, CT, 0, as_stream(stream)>>>(P, T, K, n, group, rows, I, nullptr);
    return MXQ_LAUNCH_CHECK("lut.pick");
  }
  k_lut_pick<<<grid_for(K * n, 256), 256, 0, as_stream(stream)>>>(P, T, K, n, sk, sj, group, width, I, nullptr);
  return MXQ_LAUNCH_CHECK("lut.pick");
}

int mxq_lut_pick_lookup(const float* P, const float* T, float* out, int64_t K, int64_t n, int64_t sk, int64_t sj,
                        int32_t group, int32_t width, void* stream) {
  MXQ_REQUIRE(width >= 2, MXQ_ERR_VALUE, "mxq.lut.pick: tables need width >= 2");
  if (K * n == 0) return MXQ_OK;
  if (sj == 1 && sk == n && width == LUT && (uintptr_t)T % 16 == 0 && K < (1ll << 31)) {
    int64_t rows;
    const dim3 grid = cols_grid(K, n, CT, 16, &rows);
    k_lut_pick_cols<<<grid, CT, 0, as_stream(stream)>>>(P, T, K, n, group, rows, nullptr, out);
    return MXQ_LAUNCH_CHECK("lut.pick_lookup");
  }
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
  if ((uintptr_t)T % 16 == 0 && K < (1ll << 31)) {
    int64_t rows;
    const FormatTables* f = format_tables(e, m);
    const dim3 grid = cols_grid(K, n, PW, 8, &rows);
    bool narrow = true;                                       // every fixed point and difference fits in an int
    for (int i = 0; i < f->ncodes; i++) narrow = narrow && f->fx[i] > -(1ll << 30) && f->fx[i] < (1ll << 30);
    const size_t smem = (size_t)PW * f->ncodes;               // answers: at most one group per column
    int r;
    if (narrow) {
      r = check_cuda(cudaFuncSetAttribute(k_lut_finder_cols<int>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem), "lut.finder: shared memory attribute");
      if (r == MXQ_OK)
        k_lut_finder_cols<int><<<grid, CT, smem, st>>>(codes, T, K, n, group, rows, (long long)fx_mask(e, m),
                                                       code_tables(f), I, status);
    } else {
      r = check_cuda(cudaFuncSetAttribute(k_lut_finder_cols<long long>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                     "lut.finder: shared memory attribute");
      if (r == MXQ_OK)
        k_lut_finder_cols<long long><<<grid, CT, smem, st>>>(codes, T, K, n, group, rows,
                                                             (long long)fx_mask(e, m), code_tables(f), I, status);
    }
    if (r) return r;
    return MXQ_LAUNCH_CHECK("lut.finder");
  }
  k_lut_finder<<<grid_for(K * n, 256), 256, 0, st>>>(codes, T, K, n, group, (long long)fx_mask(e, m),
                                                     code_tables(format_tables(e, m)), I, status);
  return MXQ_LAUNCH_CHECK("lut.finder");
}

}  // extern "C"
