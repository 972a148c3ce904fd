// Block quantizers: mxq/block/_driver.py compose with the named quantizers' two steps fused into one pass over
// HBM (read V once, write P once, write X once per block). A tensor is viewed as [outer, len, inner] with blocks of
// `block` along len.
//
// Kernels (each templated on the quantizer family so the element step is inlined). The TMA-staged kernel of
// quantize_tma.cu takes every layout it can map; these register kernels cover the rest:
//   k_rows<QB> inner == 1, block a power of two from 4 to 128, len % block == 0, 16-byte aligned: one float4 per
//              thread, QB = block / 4 lanes per block, the block max by log2(QB) xor-shuffles; fully coalesced
//              128-bit loads and stores.
//   k_cols_tile  inner % 4 == 0, block == 32, 16-byte aligned: one CTA per 32-row block x 256 columns; each thread
//              keeps 8 float4 of 4 columns in registers, the four row groups' column maxima meet in shared memory,
//              and every load and store is a coalesced 128-bit access along the rows.
//   k_cols32   inner > 1 otherwise, block == 32: one thread per (block, column run of VEC columns); the 32 rows of a
//              block are loaded into registers, so consecutive threads read consecutive columns (coalesced rows).
//   k_generic  any block size or alignment: one thread per (outer, block, column), two passes over the block.
#include "common.cuh"
#include "numerics.cuh"

using namespace mxq;

namespace mxq {
int quantize_tma(const float* V, float* P, float* X, int64_t outer, int64_t len, int64_t inner, int64_t block,
                 const mxq_quant_spec& s, cudaStream_t st);
}

namespace {

struct QParams {
  int e, m, rounding, placement, via_e, via_m, bits;
  float scale_floor, scale_emax, max_norm;
};

QParams make_params(const mxq_quant_spec& s) {
  QParams q;
  q.e = s.e;
  q.m = s.m;
  q.rounding = s.rounding;
  q.placement = s.placement;
  q.via_e = s.via_e;
  q.via_m = s.via_m;
  q.bits = s.m + 2;                                   // microxcaling mbits: sign + implicit + m
  q.scale_floor = s.scale_floor;
  q.scale_emax = s.scale_emax;
  q.max_norm = ocp_max_norm(s.e, s.m);
  return q;
}

// step 1: the scale of a block from its max |value| (scale_factor.py:40-81)
template <int FAM>
__device__ __forceinline__ float block_scale(float amax, const QParams& q) {
  if (FAM == MXQ_FAMILY_MXQUANT || FAM == MXQ_FAMILY_MXGEMMINI) return scale_mxquant(amax, q.scale_floor);
  if (q.placement == 0) return scale_ocp(amax, ocp_emax(q.e, q.m), q.scale_emax);
  if (q.placement == 1) return scale_ocp(amax, ocp_emax(q.e, q.m) - 1, q.scale_emax);
  return scale_ocp_no_clip(amax, q.e, q.m, q.rounding, q.scale_emax);
}

// step 2: the code of one scaled value (mxquant.py:28, mxgemmini.py:50-55, ocp.py:46)
template <int FAM>
__device__ __forceinline__ float elem(float z, const QParams& q) {
  if (FAM == MXQ_FAMILY_MXQUANT) return q_qtorch(z, q.e, q.m, RM_TIES_AWAY);
  if (FAM == MXQ_FAMILY_MXGEMMINI) {
    if (q.via_e) z = q_ieee(z, q.via_e, q.via_m, q.rounding);
    return q_ocp_bits(z, q.e, q.m, q.rounding, q.max_norm);
  }
  if (FAM == MXQ_FAMILY_OCP) return q_microsoft_sat(z, q.bits, q.e, q.max_norm, q.rounding);
  return z;
}

// z = v / X (_driver.py:64). X is a power of two in all but the floor/overflow cases; then its reciprocal is exact
// and the division is a multiply. The qtorch family keeps the host's NaN propagation (the sign reaches the code).
struct Divider {
  float X, r;
  bool fast;
  __device__ __forceinline__ explicit Divider(float x) : X(x) {
    uint32_t u = f2u(x);
    bool pow2_normal = (u & 0x807fffffu) == 0u && u >= 0x00800000u && u < 0x7f800000u;
    fast = pow2_normal || u == 0x00400000u;           // 2^-127: its reciprocal 2^127 is still finite
    r = fast ? pow2f(-ilogb_f(x)) : 0.0f;
  }
  template <int FAM>
  __device__ __forceinline__ float operator()(float v) const {
    if (FAM == MXQ_FAMILY_MXQUANT) {
      if (!fast) return x86_div(v, X);
      return isnan_f(v) ? u2f(f2u(v) | 0x00400000u) : mul_rn(v, r);
    }
    return fast ? mul_rn(v, r) : div_rn(v, X);
  }
};

// max |v| of a block; NaN anywhere gives the canonical +NaN (torch's amax)
struct AbsMax {
  float m = 0.0f;
  bool nan = false;
  __device__ __forceinline__ void add(float v) {
    float a = abs_f(v);
    nan |= isnan_f(a);
    m = fmaxf(m, a);
  }
  __device__ __forceinline__ float value() const { return nan ? qnan_f() : m; }
};

constexpr int kThreads = 256;

template <int FAM, int QB>
__global__ void __launch_bounds__(kThreads) k_rows(const float4* __restrict__ V, float4* __restrict__ P,
                                                   float* __restrict__ X, int64_t nquads, QParams q) {
  // a quad is 4 consecutive values; QB quads (QB = 1..32, a power of two) make a block; a warp covers 32 / QB blocks
  // per step. The loop runs per warp (every lane takes every trip, so the full-mask shuffles always see 32 lanes);
  // nquads is a multiple of QB, so a block is either wholly inside or wholly past the end.
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int lane = threadIdx.x & 31;
  for (int64_t w = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31); w < nquads; w += stride) {
    const int64_t t = w + lane;
    const bool live = t < nquads;
    float4 v = live ? __ldcs(V + t) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);   // streamed once: evict-first
    float a = fmaxf(fmaxf(abs_f(v.x), abs_f(v.y)), fmaxf(abs_f(v.z), abs_f(v.w)));
    unsigned nan = isnan_f(v.x) | isnan_f(v.y) | isnan_f(v.z) | isnan_f(v.w);
#pragma unroll
    for (int s = 1; s < QB; s <<= 1) {
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, s));
      nan |= __shfl_xor_sync(0xffffffffu, nan, s);
    }
    float amax = nan ? qnan_f() : a;
    float x = (FAM == MXQ_FAMILY_FP32) ? 1.0f : block_scale<FAM>(amax, q);
    if (!live) continue;
    if ((lane & (QB - 1)) == 0) X[t / QB] = x;
    float4 o;
    if (FAM == MXQ_FAMILY_FP32) {
      o = v;
    } else {
      Divider d(x);
      o.x = elem<FAM>(d.template operator()<FAM>(v.x), q);
      o.y = elem<FAM>(d.template operator()<FAM>(v.y), q);
      o.z = elem<FAM>(d.template operator()<FAM>(v.z), q);
      o.w = elem<FAM>(d.template operator()<FAM>(v.w), q);
    }
    __stcs(P + t, o);
  }
}

template <int FAM, int VEC>
__global__ void __launch_bounds__(kThreads) k_cols32(const float* __restrict__ V, float* __restrict__ P,
                                                     float* __restrict__ X, int64_t outer, int64_t len, int64_t inner,
                                                     int64_t nb, QParams q) {
  using VT = typename std::conditional<VEC == 4, float4, typename std::conditional<VEC == 2, float2, float>::type>::type;
  const int64_t runs = inner / VEC;
  const int64_t total = outer * nb * runs;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    int64_t run = t % runs, ob = t / runs, b = ob % nb, o = ob / nb;
    int64_t l0 = b * 32;
    int rows = (int)((len - l0) < 32 ? (len - l0) : 32);
    const float* src = V + (o * len + l0) * inner + run * VEC;
    float* dst = P + (o * len + l0) * inner + run * VEC;
    float v[32][VEC];
#pragma unroll
    for (int r = 0; r < 32; r++) {
      if (r < rows) {
        VT w = __ldcs(reinterpret_cast<const VT*>(src + (int64_t)r * inner));
        const float* wf = reinterpret_cast<const float*>(&w);
#pragma unroll
        for (int c = 0; c < VEC; c++) v[r][c] = wf[c];
      } else {
#pragma unroll
        for (int c = 0; c < VEC; c++) v[r][c] = 0.0f;
      }
    }
#pragma unroll
    for (int c = 0; c < VEC; c++) {
      AbsMax am;
#pragma unroll
      for (int r = 0; r < 32; r++) am.add(v[r][c]);
      float x = (FAM == MXQ_FAMILY_FP32) ? 1.0f : block_scale<FAM>(am.value(), q);
      X[(o * nb + b) * inner + run * VEC + c] = x;
      if (FAM != MXQ_FAMILY_FP32) {
        Divider d(x);
#pragma unroll
        for (int r = 0; r < 32; r++) v[r][c] = elem<FAM>(d.template operator()<FAM>(v[r][c]), q);
      }
    }
#pragma unroll
    for (int r = 0; r < 32; r++) {
      if (r < rows) {
        VT w;
        float* wf = reinterpret_cast<float*>(&w);
#pragma unroll
        for (int c = 0; c < VEC; c++) wf[c] = v[r][c];
        __stcs(reinterpret_cast<VT*>(dst + (int64_t)r * inner), w);
      }
    }
  }
}

template <int FAM>
__global__ void __launch_bounds__(kThreads) k_cols_tile(const float* __restrict__ V, float* __restrict__ P,
                                                        float* __restrict__ X, int64_t outer, int64_t len,
                                                        int64_t inner, int64_t nb, QParams q) {
  __shared__ float part[4][256];                      // column maxima of the four row groups (NaN: a NaN was seen)
  const int tid = threadIdx.x, c4 = tid & 63, rg = tid >> 6;   // float4 column in the tile, row group 0..3
  const int64_t inner4 = inner >> 2, ctiles = (inner4 + 63) >> 6, tiles = outer * nb * ctiles;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t ct = tile % ctiles, ob = tile / ctiles, b = ob % nb, o = ob / nb;
    const int64_t col4 = ct * 64 + c4, l0 = b * 32;
    const bool colok = col4 < inner4;
    const int rows = (int)((len - l0) < 32 ? (len - l0) : 32);
    const float4* src = reinterpret_cast<const float4*>(V + (o * len + l0) * inner) + col4;
    float4* dst = reinterpret_cast<float4*>(P + (o * len + l0) * inner) + col4;
    float4 v[8];
    float mx[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    bool nan[4] = {false, false, false, false};
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int r = rg + 4 * i;
      v[i] = (colok && r < rows) ? __ldcs(src + (int64_t)r * inner4) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      const float c[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int j = 0; j < 4; j++) {
        nan[j] |= isnan_f(c[j]);
        mx[j] = fmaxf(mx[j], abs_f(c[j]));
      }
    }
#pragma unroll
    for (int j = 0; j < 4; j++) part[rg][c4 * 4 + j] = nan[j] ? qnan_f() : mx[j];
    __syncthreads();
    float x[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float a = 0.0f;
      bool n = false;
#pragma unroll
      for (int g = 0; g < 4; g++) {
        float p = part[g][c4 * 4 + j];
        n |= isnan_f(p);
        a = fmaxf(a, p);
      }
      x[j] = (FAM == MXQ_FAMILY_FP32) ? 1.0f : block_scale<FAM>(n ? qnan_f() : a, q);
    }
    if (rg == 0 && colok)
      *reinterpret_cast<float4*>(X + (o * nb + b) * inner + col4 * 4) = make_float4(x[0], x[1], x[2], x[3]);
    if (FAM != MXQ_FAMILY_FP32) {
      const Divider d0(x[0]), d1(x[1]), d2(x[2]), d3(x[3]);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        v[i].x = elem<FAM>(d0.template operator()<FAM>(v[i].x), q);
        v[i].y = elem<FAM>(d1.template operator()<FAM>(v[i].y), q);
        v[i].z = elem<FAM>(d2.template operator()<FAM>(v[i].z), q);
        v[i].w = elem<FAM>(d3.template operator()<FAM>(v[i].w), q);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const int r = rg + 4 * i;
      if (colok && r < rows) __stcs(dst + (int64_t)r * inner4, v[i]);
    }
    __syncthreads();                                   // part[] is rewritten by the next tile
  }
}

template <int FAM>
__global__ void __launch_bounds__(kThreads) k_generic(const float* __restrict__ V, float* __restrict__ P,
                                                      float* __restrict__ X, int64_t outer, int64_t len, int64_t inner,
                                                      int64_t block, int64_t nb, QParams q) {
  const int64_t total = outer * nb * inner;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    int64_t j = t % inner, ob = t / inner, b = ob % nb, o = ob / nb;
    int64_t l0 = b * block, l1 = l0 + block < len ? l0 + block : len;
    const float* src = V + o * len * inner + j;
    float* dst = P + o * len * inner + j;
    AbsMax am;
    for (int64_t l = l0; l < l1; l++) am.add(src[l * inner]);
    float x = (FAM == MXQ_FAMILY_FP32) ? 1.0f : block_scale<FAM>(am.value(), q);
    X[(o * nb + b) * inner + j] = x;
    Divider d(x);
    for (int64_t l = l0; l < l1; l++) {
      float v = src[l * inner];
      dst[l * inner] = (FAM == MXQ_FAMILY_FP32) ? v : elem<FAM>(d.template operator()<FAM>(v), q);
    }
  }
}

template <int FAM>
int launch_quant(const float* V, float* P, float* X, int64_t outer, int64_t len, int64_t inner, int64_t block,
                 const QParams& q, const mxq_quant_spec& spec, cudaStream_t st) {
  int r = quantize_tma(V, P, X, outer, len, inner, block, spec, st);
  if (r != MXQ_ERR_UNSUPPORTED) return r;
  int64_t nb = (len + block - 1) / block;
  bool al16 = ((uintptr_t)V % 16 == 0) && ((uintptr_t)P % 16 == 0);
  const bool pow2 = block >= 4 && block <= 128 && (block & (block - 1)) == 0;
  if (pow2 && inner == 1 && len % block == 0 && al16) {
    // rows of whole blocks of 4..128 values: a block is QB = block / 4 lanes' float4
    const int64_t nquads = outer * len / 4;
    const unsigned grid = grid_for(nquads, kThreads, 16);
    auto V4 = reinterpret_cast<const float4*>(V);
    auto P4 = reinterpret_cast<float4*>(P);
    switch (block) {
      case 4: k_rows<FAM, 1><<<grid, kThreads, 0, st>>>(V4, P4, X, nquads, q); break;
      case 8: k_rows<FAM, 2><<<grid, kThreads, 0, st>>>(V4, P4, X, nquads, q); break;
      case 16: k_rows<FAM, 4><<<grid, kThreads, 0, st>>>(V4, P4, X, nquads, q); break;
      case 32: k_rows<FAM, 8><<<grid, kThreads, 0, st>>>(V4, P4, X, nquads, q); break;
      case 64: k_rows<FAM, 16><<<grid, kThreads, 0, st>>>(V4, P4, X, nquads, q); break;
      default: k_rows<FAM, 32><<<grid, kThreads, 0, st>>>(V4, P4, X, nquads, q); break;
    }
  } else if (block == 32 && inner > 1) {
    if (inner % 4 == 0 && al16 && (uintptr_t)X % 16 == 0) {
      int64_t tiles = outer * nb * ((inner / 4 + 63) / 64);
      unsigned grid = (unsigned)(tiles < (int64_t)sm_count() * 6 ? tiles : (int64_t)sm_count() * 6);
      k_cols_tile<FAM><<<grid, kThreads, 0, st>>>(V, P, X, outer, len, inner, nb, q);
    } else if (inner % 2 == 0 && (uintptr_t)V % 8 == 0 && (uintptr_t)P % 8 == 0) {
      int64_t n = outer * nb * (inner / 2);
      k_cols32<FAM, 2><<<grid_for(n, kThreads, 8), kThreads, 0, st>>>(V, P, X, outer, len, inner, nb, q);
    } else {
      int64_t n = outer * nb * inner;
      k_cols32<FAM, 1><<<grid_for(n, kThreads, 8), kThreads, 0, st>>>(V, P, X, outer, len, inner, nb, q);
    }
  } else {
    int64_t n = outer * nb * inner;
    k_generic<FAM><<<grid_for(n, kThreads, 8), kThreads, 0, st>>>(V, P, X, outer, len, inner, block, nb, q);
  }
  return MXQ_LAUNCH_CHECK("block_quantize");
}

// ------------------------------------------------------------------------------------ compose pieces
__global__ void k_block_amax(const float* __restrict__ V, float* __restrict__ amax, int64_t outer, int64_t len,
                             int64_t inner, int64_t block, int64_t nb) {
  // output in the blocked layout [outer, inner, nb]; consecutive threads take consecutive columns j
  const int64_t total = outer * nb * inner;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t j = t % inner, ob = t / inner, b = ob % nb, o = ob / nb;
    int64_t l0 = b * block, l1 = l0 + block < len ? l0 + block : len;
    AbsMax am;
    for (int64_t l = l0; l < l1; l++) am.add(V[(o * len + l) * inner + j]);
    amax[(o * inner + j) * nb + b] = am.value();
  }
}

__global__ void k_to_blocks(const float* __restrict__ V, const float* __restrict__ X, float* __restrict__ Z,
                            int64_t outer, int64_t len, int64_t inner, int64_t block, int64_t nb) {
  // Z [outer, inner, nb * block] = pad(V moved to the last axis) / X; iterate in V's order for coalesced reads
  const int64_t padded = nb * block;
  const int64_t total = outer * padded * inner;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t j = t % inner, ol = t / inner, l = ol % padded, o = ol / padded;
    float v = l < len ? V[(o * len + l) * inner + j] : 0.0f;
    int64_t zi = (o * inner + j) * padded + l;
    Z[zi] = X ? x86_div(v, X[(o * inner + j) * nb + l / block]) : v;
  }
}

__global__ void k_from_blocks(const float* __restrict__ Zb, float* __restrict__ P, int64_t outer, int64_t len,
                              int64_t inner, int64_t padded) {
  const int64_t total = outer * len * inner;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t j = t % inner, ol = t / inner, l = ol % len, o = ol / len;
    P[t] = Zb[(o * inner + j) * padded + l];
  }
}

__global__ void k_dequantize(const float* __restrict__ P, const float* __restrict__ X, float* __restrict__ out,
                             int64_t outer, int64_t len, int64_t inner, int64_t block, int64_t nb) {
  const int64_t total = outer * len * inner;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t j = t % inner, ol = t / inner, l = ol % len, o = ol / len;
    out[t] = x86_mul(P[t], X[(o * nb + l / block) * inner + j]);
  }
}

// dequantize on float4: one float4 per thread (one-shot grid), 32-bit index arithmetic. Preconditions (checked by
// the launcher): 16-byte aligned P and out, fewer than 2^32 elements, and either inner % 4 == 0 (the float4 runs along
// inner, its scales are a float4 of X, 16-byte aligned) or inner == 1 with len % 4 == 0 and block % 4 == 0 (the
// float4 lies in one block of one row: one scale).
template <bool COLS>
__global__ void __launch_bounds__(256) k_dequantize4(const float4* __restrict__ P, const float* __restrict__ X,
                                                     float4* __restrict__ out, uint32_t n4, uint32_t len,
                                                     uint32_t inner, uint32_t block, uint32_t nb) {
  const uint32_t q = blockIdx.x * 256u + threadIdx.x;
  if (q >= n4) return;
  const uint32_t e = q * 4u;
  const float4 p = P[q];
  float4 x;
  if (COLS) {
    const uint32_t ol = e / inner, j = e - ol * inner, o = ol / len, l = ol - o * len;
    x = reinterpret_cast<const float4*>(X)[((o * nb + l / block) * inner + j) / 4u];
  } else {
    const uint32_t o = e / len, l = e - o * len;
    const float s = X[o * nb + l / block];
    x = make_float4(s, s, s, s);
  }
  out[q] = make_float4(x86_mul(p.x, x.x), x86_mul(p.y, x.y), x86_mul(p.z, x.z), x86_mul(p.w, x.w));
}

int check_layout(int64_t outer, int64_t len, int64_t inner, int64_t block, const char* what) {
  MXQ_REQUIRE(outer >= 0 && len >= 0 && inner >= 0, MXQ_ERR_VALUE, "%s: negative extent", what);
  MXQ_REQUIRE(block >= 1, MXQ_ERR_VALUE, "%s: block_size must be >= 1, got %lld", what, (long long)block);
  return MXQ_OK;
}

}  // namespace

extern "C" {

int mxq_block_quantize(const float* V, float* P, float* X, int64_t outer, int64_t len, int64_t inner, int64_t block,
                       const mxq_quant_spec* spec, void* stream) {
  if (int r = check_layout(outer, len, inner, block, "block_quantize")) return r;
  MXQ_REQUIRE(spec != nullptr, MXQ_ERR_VALUE, "block_quantize: no spec");
  const mxq_quant_spec& s = *spec;
  if (s.family != MXQ_FAMILY_FP32) {
    MXQ_REQUIRE(ocp_max_norm(s.e, s.m) > 0.0f, MXQ_ERR_VALUE, "block_quantize: (e=%d, m=%d) is not an OCP format",
                s.e, s.m);
  }
  switch (s.family) {
    case MXQ_FAMILY_FP32: break;
    case MXQ_FAMILY_MXQUANT: break;
    case MXQ_FAMILY_MXGEMMINI:
      MXQ_REQUIRE(s.rounding >= 0 && s.rounding <= 2, MXQ_ERR_VALUE, "rounding_mode %d unknown", s.rounding);
      MXQ_REQUIRE(s.via_e == 0 || (s.via_e == 8 && s.via_m == 23) ||
                      (s.via_e >= 1 && s.via_e <= 8 && s.via_m >= 1 && s.via_m <= 22),
                  MXQ_ERR_VALUE, "unsupported widths e=%d, m=%d", s.via_e, s.via_m);
      break;
    case MXQ_FAMILY_OCP:
      MXQ_REQUIRE(s.rounding >= 0 && s.rounding <= 2, MXQ_ERR_VALUE, "Unrecognized round method %d", s.rounding);
      MXQ_REQUIRE(s.placement >= 0 && s.placement <= 2, MXQ_ERR_VALUE, "placement %d unknown", s.placement);
      break;
    default: return set_error(MXQ_ERR_VALUE, "block_quantize: unknown family %d", s.family);
  }
  if (outer * len * inner == 0) return MXQ_OK;
  QParams q = make_params(s);
  cudaStream_t st = as_stream(stream);
  switch (s.family) {
    case MXQ_FAMILY_FP32: return launch_quant<MXQ_FAMILY_FP32>(V, P, X, outer, len, inner, block, q, s, st);
    case MXQ_FAMILY_MXQUANT: return launch_quant<MXQ_FAMILY_MXQUANT>(V, P, X, outer, len, inner, block, q, s, st);
    case MXQ_FAMILY_MXGEMMINI: return launch_quant<MXQ_FAMILY_MXGEMMINI>(V, P, X, outer, len, inner, block, q, s, st);
    default: return launch_quant<MXQ_FAMILY_OCP>(V, P, X, outer, len, inner, block, q, s, st);
  }
}

int mxq_block_amax(const float* V, float* amax, int64_t outer, int64_t len, int64_t inner, int64_t block,
                   void* stream) {
  if (int r = check_layout(outer, len, inner, block, "block_amax")) return r;
  int64_t nb = (len + block - 1) / block, n = outer * nb * inner;
  if (n == 0) return MXQ_OK;
  k_block_amax<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(V, amax, outer, len, inner, block, nb);
  return MXQ_LAUNCH_CHECK("block_amax");
}

int mxq_to_blocks(const float* V, const float* X, float* Z, int64_t outer, int64_t len, int64_t inner, int64_t block,
                  void* stream) {
  if (int r = check_layout(outer, len, inner, block, "to_blocks")) return r;
  int64_t nb = (len + block - 1) / block, n = outer * nb * block * inner;
  if (n == 0) return MXQ_OK;
  k_to_blocks<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(V, X, Z, outer, len, inner, block, nb);
  return MXQ_LAUNCH_CHECK("to_blocks");
}

int mxq_from_blocks(const float* Zb, float* P, int64_t outer, int64_t len, int64_t inner, int64_t block,
                    void* stream) {
  if (int r = check_layout(outer, len, inner, block, "from_blocks")) return r;
  int64_t nb = (len + block - 1) / block, n = outer * len * inner;
  if (n == 0) return MXQ_OK;
  k_from_blocks<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(Zb, P, outer, len, inner, nb * block);
  return MXQ_LAUNCH_CHECK("from_blocks");
}

int mxq_dequantize(const float* P, const float* X, float* out, int64_t outer, int64_t len, int64_t inner,
                   int64_t block, void* stream) {
  if (int r = check_layout(outer, len, inner, block, "dequantize")) return r;
  int64_t nb = (len + block - 1) / block, n = outer * len * inner;
  if (n == 0) return MXQ_OK;
  const bool al = (uintptr_t)P % 16 == 0 && (uintptr_t)out % 16 == 0 && n < (1ll << 32) && outer * nb * inner < (1ll << 32);
  const bool cols = inner % 4 == 0 && (uintptr_t)X % 16 == 0, rows = inner == 1 && len % 4 == 0 && block % 4 == 0;
  if (al && (cols || rows)) {
    const uint32_t n4 = (uint32_t)(n / 4), grid = (n4 + 255) / 256;
    auto kern = cols ? k_dequantize4<true> : k_dequantize4<false>;
    kern<<<grid, 256, 0, as_stream(stream)>>>(reinterpret_cast<const float4*>(P), X, reinterpret_cast<float4*>(out),
                                              n4, (uint32_t)len, (uint32_t)inner, (uint32_t)block, (uint32_t)nb);
    return MXQ_LAUNCH_CHECK("dequantize");
  }
  k_dequantize<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(P, X, out, outer, len, inner, block, nb);
  return MXQ_LAUNCH_CHECK("dequantize");
}

}  // extern "C"
