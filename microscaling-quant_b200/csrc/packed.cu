// The compact operand form (no reference counterpart; the wire format MX-Gemmini's 4-bit LUT indices imply,
// mxq/lut/__init__.py:3-6): a block quantizer's codes as the element format's OCP bit patterns and its scales as
// E8M0 bytes, in the float32 outputs' own layouts. One byte per FP8 / FP6 element (FP6 in the low six bits), two
// FP4 elements per byte (the even one in the low nibble); a scale byte b is 2^(b - 127), 0xFF NaN. The quantizer is
// the fused TMA kernel with a packing output stage (quantize_tma.cu); unpacking decodes a byte arithmetically.
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
  k_unpack<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(codes, scales, P, X, n_codes, n_scales, e, m);
  return MXQ_LAUNCH_CHECK("unpack");
}

int mxq_dequantize_packed(const uint8_t* codes, const uint8_t* scales, float* out, int64_t outer, int64_t len,
                          int64_t inner, int64_t block, int32_t e, int32_t m, void* stream) {
  MXQ_REQUIRE(ocp_format(e, m), MXQ_ERR_VALUE, "dequantize_packed: (e=%d, m=%d) is not an MX element format", e, m);
  MXQ_REQUIRE(outer >= 0 && len >= 0 && inner >= 0 && block >= 1, MXQ_ERR_VALUE, "dequantize_packed: bad layout");
  const int64_t n = outer * len * inner;
  if (n == 0) return MXQ_OK;
  k_dequantize_packed<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(codes, scales, out, outer, len, inner, block,
                                                                       e, m);
  return MXQ_LAUNCH_CHECK("dequantize_packed");
}

}  // extern "C"
