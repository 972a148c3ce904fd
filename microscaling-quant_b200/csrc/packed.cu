// The compact operand form (no reference counterpart; the wire format MX-Gemmini's 4-bit LUT indices imply,
// mxq/lut/__init__.py:3-6): a block quantizer's codes as the element format's OCP bit patterns and its scales as
// E8M0 bytes, in the float32 outputs' own layouts. One byte per FP8 / FP6 element (FP6 in the low six bits), two
// FP4 elements per byte (the even one in the low nibble); a scale byte b is 2^(b - 127), 0xFF NaN. The quantizer is
// the fused TMA kernel with a packing output stage (quantize_tma.cu); unpacking decodes a byte arithmetically.
#include <type_traits>

#include "common.cuh"
#include "numerics.cuh"

using namespace mxq;

namespace mxq {
int quantize_tma_packed(const float* V, uint8_t* Pc, uint8_t* Xc, int* status, int64_t outer, int64_t len,
                        int64_t inner, int64_t block, const mxq_quant_spec& s, cudaStream_t st);
}

namespace {

bool ocp_format(int e, int m) {
  return (e == 4 && m == 3) || (e == 5 && m == 2) || (e == 3 && m == 2) || (e == 2 && m == 3) || (e == 2 && m == 1);
}

// the value of an OCP element code (E4M3: S.1111.111 is NaN; E5M2: exponent 31 is Inf / NaN; FP6 / FP4 all finite)
__device__ __forceinline__ float ocp_value(uint32_t c, int e, int m) {
  const int bias = (1 << (e - 1)) - 1;
  const uint32_t s = (c >> (e + m)) & 1u, ex = (c >> m) & ((1u << e) - 1u), man = c & ((1u << m) - 1u);
  uint32_t bits;
  if (e == 4 && m == 3 && ex == 15u && man == 7u) {
    bits = 0x7fc00000u;
  } else if (e == 5 && m == 2 && ex == 31u) {
    bits = man ? 0x7fc00000u : 0x7f800000u;
  } else if (ex == 0u) {                                       // man x 2^(1 - bias - m), exact
    bits = f2u(__fmul_rn((float)man, u2f((uint32_t)(128 - bias - m) << 23)));
  } else {
    bits = ((ex + 127u - (uint32_t)bias) << 23) | (man << (23 - m));
  }
  return u2f(bits | (s << 31));
}

__device__ __forceinline__ float e8m0_value(uint32_t b) {
  return b == 0xffu ? u2f(0x7fc00000u) : (b == 0u ? u2f(0x00400000u) : u2f(b << 23));
}

__device__ __forceinline__ uint32_t code_at(const uint8_t* codes, int64_t i, bool nibble) {
  const uint32_t byte = codes[nibble ? i >> 1 : i];
  return nibble ? ((i & 1) ? byte >> 4 : byte & 15u) : byte;
}

__global__ void k_unpack(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales, float* __restrict__ P,
                         float* __restrict__ X, int64_t nc, int64_t ns, int e, int m) {
  const bool nibble = e + m == 3;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nc; i += stride)
    P[i] = ocp_value(code_at(codes, i, nibble), e, m);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < ns; i += stride) X[i] = e8m0_value(scales[i]);
}

// dequantize (mxq/block/_driver.py:69-72) straight from the compact form: code value x its block's scale
__global__ void k_dequantize_packed(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                                    float* __restrict__ out, int64_t outer, int64_t len, int64_t inner, int64_t block,
                                    int e, int m) {
  const bool nibble = e + m == 3;
  const int64_t nb = (len + block - 1) / block, n = outer * len * inner;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t c = i % inner, l = (i / inner) % len, o = i / (inner * len);
    out[i] = __fmul_rn(ocp_value(code_at(codes, i, nibble), e, m), e8m0_value(scales[(o * nb + l / block) * inner + c]));
  }
}

// unpack on vectors, the format as template arguments (the decode folds to a few integer ops): a thread turns 4 codes
// (one 32-bit word of FP8 / FP6 bytes, or one 16-bit word of FP4 nibbles) into a float4 of P, and 4 scale bytes
// into a float4 of X. Preconditions: n_codes and n_scales multiples of 4, 16-byte aligned P and X, codes aligned to
// the word, fewer than 2^32 codes.
template <int E, int M>
__global__ void __launch_bounds__(256) k_unpack4(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scales,
                                                 float4* __restrict__ P, float4* __restrict__ X, uint32_t nc4,
                                                 uint32_t ns4) {
  // a grid of a few CTAs per SM striding over the words, four words' loads in flight per thread before their
  // decodes and stores
  const uint32_t stride = gridDim.x * 256u;
  constexpr int U = 4;
  for (uint32_t q0 = blockIdx.x * 256u + threadIdx.x; q0 < nc4; q0 += U * stride) {
    uint32_t w[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint32_t q = q0 + u * stride;
      w[u] = q < nc4 ? (E + M == 3 ? (uint32_t)reinterpret_cast<const uint16_t*>(codes)[q]
                                   : reinterpret_cast<const uint32_t*>(codes)[q])
                     : 0u;
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint32_t q = q0 + u * stride;
      if (q >= nc4) break;
      if (E + M == 3)
        __stcs(P + q, make_float4(ocp_value(w[u] & 15u, E, M), ocp_value((w[u] >> 4) & 15u, E, M),
                                  ocp_value((w[u] >> 8) & 15u, E, M), ocp_value((w[u] >> 12) & 15u, E, M)));
      else
        __stcs(P + q, make_float4(ocp_value(w[u] & 255u, E, M), ocp_value((w[u] >> 8) & 255u, E, M),
                                  ocp_value((w[u] >> 16) & 255u, E, M), ocp_value(w[u] >> 24, E, M)));
    }
  }
  for (uint32_t q = blockIdx.x * 256u + threadIdx.x; q < ns4; q += stride) {
    const uint32_t w = reinterpret_cast<const uint32_t*>(scales)[q];
    X[q] = make_float4(e8m0_value(w & 255u), e8m0_value((w >> 8) & 255u), e8m0_value((w >> 16) & 255u),
                       e8m0_value(w >> 24));
  }
}

// dequantize_packed on vectors with blocks along the row (inner 1): a thread decodes 4 codes and multiplies by their
// block's scale (one E8M0 byte), striding over the float4s with four words' and scale bytes' loads in flight.
// bsh >= 0 when block = 2^bsh divides len: the scale of element e is then byte e >> bsh, no division. Preconditions as
// k_dequantize4 (quantize.cu), codes aligned to the word.
template <int E, int M>
__global__ void __launch_bounds__(256) k_dequantize_packed4(const uint8_t* __restrict__ codes,
                                                            const uint8_t* __restrict__ scales,
                                                            float4* __restrict__ out, uint32_t n4, uint32_t len,
                                                            uint32_t block, uint32_t nb, int bsh) {
  const uint32_t stride = gridDim.x * 256u;
  constexpr int U = 4;
  for (uint32_t q0 = blockIdx.x * 256u + threadIdx.x; q0 < n4; q0 += U * stride) {
    uint32_t w[U], sb[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint32_t q = q0 + u * stride;
      w[u] = sb[u] = 0u;
      if (q < n4) {
        w[u] = E + M == 3 ? (uint32_t)reinterpret_cast<const uint16_t*>(codes)[q]
                          : reinterpret_cast<const uint32_t*>(codes)[q];
        const uint32_t e = q * 4u;
        uint32_t si;
        if (bsh >= 0) {
          si = e >> bsh;
        } else {
          const uint32_t o = e / len, l = e - o * len;
          si = o * nb + l / block;
        }
        sb[u] = scales[si];
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint32_t q = q0 + u * stride;
      if (q >= n4) break;
      float4 v;
      if (E + M == 3)
        v = make_float4(ocp_value(w[u] & 15u, E, M), ocp_value((w[u] >> 4) & 15u, E, M),
                        ocp_value((w[u] >> 8) & 15u, E, M), ocp_value((w[u] >> 12) & 15u, E, M));
      else
        v = make_float4(ocp_value(w[u] & 255u, E, M), ocp_value((w[u] >> 8) & 255u, E, M),
                        ocp_value((w[u] >> 16) & 255u, E, M), ocp_value(w[u] >> 24, E, M));
      const float s = e8m0_value(sb[u]);
      __stcs(out + q, make_float4(__fmul_rn(v.x, s), __fmul_rn(v.y, s), __fmul_rn(v.z, s), __fmul_rn(v.w, s)));
    }
  }
}

// dequantize_packed with blocks along len and inner a multiple of 4 (axis 0 of a matrix): a thread owns 4 adjacent
// columns of one block of rows, reads their 4 scale bytes once and walks the block's rows, one 4-code word in and one
// float4 out per row (a warp's loads and stores are consecutive across its lanes' columns). Threads: outer x nb x
// inner / 4, fewer than 2^32; one index split per thread instead of three divisions per float4.
template <int E, int M>
__global__ void __launch_bounds__(256) k_dequantize_packed_cols(const uint8_t* __restrict__ codes,
                                                                const uint8_t* __restrict__ scales,
                                                                float4* __restrict__ out, uint32_t nthreads,
                                                                uint32_t len, uint32_t inner, uint32_t block,
                                                                uint32_t nb) {
  const uint32_t t = blockIdx.x * 256u + threadIdx.x;
  if (t >= nthreads) return;
  const uint32_t iq = inner / 4u, jq = t % iq, rest = t / iq, b = rest % nb, o = rest / nb;
  const uint32_t w = reinterpret_cast<const uint32_t*>(scales)[(o * nb + b) * iq + jq];
  const float x0 = e8m0_value(w & 255u), x1 = e8m0_value((w >> 8) & 255u), x2 = e8m0_value((w >> 16) & 255u),
              x3 = e8m0_value(w >> 24);
  const uint32_t l0 = b * block, l1 = l0 + block < len ? l0 + block : len;
  uint32_t q = (o * len + l0) * iq + jq;                   // float4 index of (row l0, columns 4 jq ..)
  constexpr int U = 4;                                     // rows whose code words are loaded before any decode
  for (uint32_t l = l0; l < l1; l += U, q += U * iq) {
    uint32_t c[U];
#pragma unroll
    for (int u = 0; u < U; u++)
      c[u] = l + u < l1 ? (E + M == 3 ? (uint32_t)reinterpret_cast<const uint16_t*>(codes)[q + u * iq]
                                      : reinterpret_cast<const uint32_t*>(codes)[q + u * iq])
                        : 0u;
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (l + u >= l1) break;
      float4 v;
      if (E + M == 3)
        v = make_float4(ocp_value(c[u] & 15u, E, M), ocp_value((c[u] >> 4) & 15u, E, M),
                        ocp_value((c[u] >> 8) & 15u, E, M), ocp_value((c[u] >> 12) & 15u, E, M));
      else
        v = make_float4(ocp_value(c[u] & 255u, E, M), ocp_value((c[u] >> 8) & 255u, E, M),
                        ocp_value((c[u] >> 16) & 255u, E, M), ocp_value(c[u] >> 24, E, M));
      __stcs(out + q + u * iq,
             make_float4(__fmul_rn(v.x, x0), __fmul_rn(v.y, x1), __fmul_rn(v.z, x2), __fmul_rn(v.w, x3)));
    }
  }
}

// the (e, m) of an MX element format as template arguments: f(std::integral_constant<int, E>, ...<int, M>)
template <class F>
int by_format(int e, int m, F f) {
  if (e == 4 && m == 3) return f(std::integral_constant<int, 4>(), std::integral_constant<int, 3>());
  if (e == 5 && m == 2) return f(std::integral_constant<int, 5>(), std::integral_constant<int, 2>());
  if (e == 3 && m == 2) return f(std::integral_constant<int, 3>(), std::integral_constant<int, 2>());
  if (e == 2 && m == 3) return f(std::integral_constant<int, 2>(), std::integral_constant<int, 3>());
  return f(std::integral_constant<int, 2>(), std::integral_constant<int, 1>());
}

}  // namespace

extern "C" {

int mxq_block_quantize_packed(const float* V, uint8_t* codes, uint8_t* scales, int64_t outer, int64_t len,
                              int64_t inner, int64_t block, const mxq_quant_spec* spec, int32_t* status,
                              void* stream) {
  MXQ_REQUIRE(spec != nullptr && status != nullptr, MXQ_ERR_VALUE, "block_quantize_packed: no spec or status word");
  const mxq_quant_spec& s = *spec;
  MXQ_REQUIRE((s.family == MXQ_FAMILY_MXGEMMINI && s.via_e == 0) || s.family == MXQ_FAMILY_OCP, MXQ_ERR_VALUE,
              "block_quantize_packed: the compact form holds OCP-grid codes: block.mxgemmini (without via) or "
              "block.ocp, not family %d", s.family);
  MXQ_REQUIRE(ocp_format(s.e, s.m), MXQ_ERR_VALUE, "block_quantize_packed: (e=%d, m=%d) is not an MX element format",
              s.e, s.m);
  MXQ_REQUIRE(outer >= 0 && len >= 0 && inner >= 0 && block >= 1, MXQ_ERR_VALUE, "block_quantize_packed: bad layout");
  MXQ_REQUIRE(s.rounding >= 0 && s.rounding <= 2, MXQ_ERR_VALUE, "block_quantize_packed: rounding %d", s.rounding);
  MXQ_REQUIRE(s.family != MXQ_FAMILY_OCP || (s.placement >= 0 && s.placement <= 2), MXQ_ERR_VALUE,
              "block_quantize_packed: placement %d", s.placement);
  cudaStream_t st = as_stream(stream);
  if (int r = check_cuda(cudaMemsetAsync(status, 0, sizeof(int32_t), st), "block_quantize_packed")) return r;
  if (outer * len * inner == 0) return MXQ_OK;
  const int r = quantize_tma_packed(V, codes, scales, status, outer, len, inner, block, s, st);
  MXQ_REQUIRE(r != MXQ_ERR_UNSUPPORTED, MXQ_ERR_UNSUPPORTED,
              "block_quantize_packed: blocks of 32, rows a multiple of 4 elements, 16-byte aligned buffers");
  return r;
}

int mxq_unpack(const uint8_t* codes, const uint8_t* scales, float* P, float* X, int64_t n_codes, int64_t n_scales,
               int32_t e, int32_t m, void* stream) {
  MXQ_REQUIRE(ocp_format(e, m), MXQ_ERR_VALUE, "unpack: (e=%d, m=%d) is not an MX element format", e, m);
  MXQ_REQUIRE(n_codes >= 0 && n_scales >= 0, MXQ_ERR_VALUE, "unpack: negative size");
  const int64_t n = n_codes > n_scales ? n_codes : n_scales;
  if (n == 0) return MXQ_OK;
  const int word = e + m == 3 ? 2 : 4;                      // code bytes per 4 codes
  if (n_codes % 4 == 0 && n_scales % 4 == 0 && n < (1ll << 32) && (uintptr_t)codes % word == 0 &&
      (uintptr_t)scales % 4 == 0 && (uintptr_t)P % 16 == 0 && (uintptr_t)X % 16 == 0) {
    const uint32_t nc4 = (uint32_t)(n_codes / 4), ns4 = (uint32_t)(n_scales / 4);
    const uint32_t grid = grid_for((int64_t)(nc4 > ns4 ? nc4 : ns4), 256, 8);
    cudaStream_t st = as_stream(stream);
    by_format(e, m, [&](auto E, auto M) {
      k_unpack4<decltype(E)::value, decltype(M)::value><<<grid, 256, 0, st>>>(
          codes, scales, reinterpret_cast<float4*>(P), reinterpret_cast<float4*>(X), nc4, ns4);
      return 0;
    });
    return MXQ_LAUNCH_CHECK("unpack");
  }
  k_unpack<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(codes, scales, P, X, n_codes, n_scales, e, m);
  return MXQ_LAUNCH_CHECK("unpack");
}

int mxq_dequantize_packed(const uint8_t* codes, const uint8_t* scales, float* out, int64_t outer, int64_t len,
                          int64_t inner, int64_t block, int32_t e, int32_t m, void* stream) {
  MXQ_REQUIRE(ocp_format(e, m), MXQ_ERR_VALUE, "dequantize_packed: (e=%d, m=%d) is not an MX element format", e, m);
  MXQ_REQUIRE(outer >= 0 && len >= 0 && inner >= 0 && block >= 1, MXQ_ERR_VALUE, "dequantize_packed: bad layout");
  const int64_t n = outer * len * inner, nb = (len + block - 1) / block;
  if (n == 0) return MXQ_OK;
  const int word = e + m == 3 ? 2 : 4;
  const bool al = (uintptr_t)codes % word == 0 && (uintptr_t)out % 16 == 0 && n < (1ll << 32) &&
                  outer * nb * inner < (1ll << 32);
  const bool cols = inner % 4 == 0 && (uintptr_t)scales % 4 == 0, rows = inner == 1 && len % 4 == 0 && block % 4 == 0;
  if (al && cols) {
    const uint32_t nthreads = (uint32_t)(outer * nb * (inner / 4)), grid = (nthreads + 255) / 256;
    cudaStream_t st = as_stream(stream);
    by_format(e, m, [&](auto E, auto M) {
      k_dequantize_packed_cols<decltype(E)::value, decltype(M)::value><<<grid, 256, 0, st>>>(
          codes, scales, reinterpret_cast<float4*>(out), nthreads, (uint32_t)len, (uint32_t)inner, (uint32_t)block,
          (uint32_t)nb);
      return 0;
    });
    return MXQ_LAUNCH_CHECK("dequantize_packed");
  }
  if (al && rows) {
    const uint32_t n4 = (uint32_t)(n / 4), grid = grid_for(n4, 256, 8);
    int bsh = -1;
    if ((block & (block - 1)) == 0 && len % block == 0)
      for (bsh = 0; (1ll << bsh) < block; bsh++) {
      }
    cudaStream_t st = as_stream(stream);
    by_format(e, m, [&](auto E, auto M) {
      k_dequantize_packed4<decltype(E)::value, decltype(M)::value><<<grid, 256, 0, st>>>(
          codes, scales, reinterpret_cast<float4*>(out), n4, (uint32_t)len, (uint32_t)block, (uint32_t)nb, bsh);
      return 0;
    });
    return MXQ_LAUNCH_CHECK("dequantize_packed");
  }
  k_dequantize_packed<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(codes, scales, out, outer, len, inner, block,
                                                                       e, m);
  return MXQ_LAUNCH_CHECK("dequantize_packed");
}

}  // extern "C"
