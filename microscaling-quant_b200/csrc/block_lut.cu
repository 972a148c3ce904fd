// block.lut.quantize (mxq/block/lut.py:23-34) as one C-ABI call on one stream, allocating nothing and never waiting
// on the host. Axis 0, blocks of 32: one launch (the tables kernel's fused mode) that quantizes V, fits the tables
// and writes every entry (rows a multiple of 32), else the TMA quantizer's code bytes and one launch that fits and
// looks up from them. Otherwise: the fused mxgemmini quantizer writes V's float codes into the workspace, the table
// fit reads them as the K x n operand (axis 1: V read transposed in place) and writes its tables into the same
// workspace, and pick with lookup replaces every code by its table entry in V's layout.
#include "common.cuh"

#include <mutex>

using namespace mxq;

// The scratch of mxq_block_lut_quantize_static: one array per device, shared by every call on that device.
constexpr int64_t kStaticScratchBytes = (int64_t)16 << 20;
static __device__ __align__(256) unsigned char g_block_lut_scratch[kStaticScratchBytes];

namespace {

constexpr int64_t kAlign = 256;
constexpr int kTableWidth = 16;        // mxq/lut/__init__.py SIZE

int64_t round_up(int64_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

bool lut_format(int e, int m) { return (e == 3 && m == 2) || (e == 2 && m == 3) || (e == 5 && m == 2) || (e == 4 && m == 3); }

constexpr int kMaxDevices = 64;

}  // namespace

namespace mxq {
int quantize_tma_codes(const float* V, uint8_t* codes, float* X, int* status, int64_t outer, int64_t len,
                       int64_t inner, const mxq_quant_spec& s, cudaStream_t st);
int lut_tables_codes_lookup(const uint8_t* codes, float* T, float* cmap, float* out, int64_t K, int64_t n,
                            int32_t group, int32_t max_iters, int32_t e, int32_t m, int32_t* status, void* stream);
int block_lut_fused(const float* V, float* out, float* X, float* T, float* cmap, uint8_t* codesT, int64_t K, int64_t n,
                    int32_t group, int32_t max_iters, int32_t e, int32_t m, int32_t rounding, float scale_floor,
                    int32_t* status, void* stream);
}  // namespace mxq

namespace {
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};

// The current device's address of g_block_lut_scratch, looked up with that device current once per context (a
// context made after cudaDeviceReset loads the module again, and the array may move)
int static_scratch(void** out) {
  int dev = 0;
  if (int r = check_cuda(cudaGetDevice(&dev), "block.lut static scratch: current device")) return r;
  MXQ_REQUIRE(dev >= 0 && dev < kMaxDevices, MXQ_ERR_UNSUPPORTED, "block.lut static scratch: device %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  const unsigned long long ctx = mxq::context_id();
  if (g_scratch_ptr[dev] == nullptr || ctx == 0 || g_scratch_ctx[dev] != ctx) {
    void* p = nullptr;
    if (int r = check_cuda(cudaGetSymbolAddress(&p, g_block_lut_scratch), "block.lut static scratch: address"))
      return r;
    g_scratch_ptr[dev] = p;
    g_scratch_ctx[dev] = mxq::context_id();                 // the lookup made the context current if it was not
  }
  *out = g_scratch_ptr[dev];
  return MXQ_OK;
}

}  // namespace

extern "C" {

int64_t mxq_block_lut_workspace(int64_t rows, int64_t cols, int32_t axis, int32_t group) {
  if (rows < 0 || cols < 0 || group < 0 || group >= 31) return -1;
  const int64_t n = (axis % 2 == 0) ? cols : rows;
  const int64_t ng = (n + ((int64_t)1 << group) - 1) >> group;
  return round_up(rows * cols * (int64_t)sizeof(float)) + round_up(ng * kTableWidth * (int64_t)sizeof(float));
}

int mxq_block_lut_quantize(const float* V, float* P_lut, float* X, int64_t rows, int64_t cols, int32_t axis,
                           int64_t block, const mxq_quant_spec* spec, int32_t group, int32_t max_iters,
                           void* workspace, int64_t workspace_bytes, int32_t* status, void* stream) {
  MXQ_REQUIRE(spec != nullptr, MXQ_ERR_VALUE, "block.lut: no spec");
  MXQ_REQUIRE(axis >= -2 && axis <= 1, MXQ_ERR_VALUE, "block.lut: V must be 2-D with axis 0 or 1, got axis %d", axis);
  MXQ_REQUIRE(spec->family == MXQ_FAMILY_MXGEMMINI && spec->via_e == 0, MXQ_ERR_VALUE,
              "block.lut: the codes come from block.mxgemmini without via");
  MXQ_REQUIRE(lut_format(spec->e, spec->m), MXQ_ERR_VALUE, "mxq.lut: no LUT format (e=%d, m=%d)", spec->e, spec->m);
  MXQ_REQUIRE(status != nullptr, MXQ_ERR_VALUE, "block.lut: no status word");
  const int64_t need = mxq_block_lut_workspace(rows, cols, axis, group);
  MXQ_REQUIRE(need >= 0, MXQ_ERR_VALUE, "block.lut: bad sizes (%lld x %lld, group %d)", (long long)rows,
              (long long)cols, group);
  MXQ_REQUIRE(need == 0 || (workspace != nullptr && workspace_bytes >= need && (uintptr_t)workspace % kAlign == 0),
              MXQ_ERR_VALUE,
              "block.lut: the workspace needs %lld bytes, 256-byte aligned (got %lld)", (long long)need,
              (long long)workspace_bytes);
  const bool ax0 = axis % 2 == 0;
  // Axis 0 (the K x n operand is V's own row-major layout) with blocks of 32: one launch that quantizes V, fits the
  // tables and writes the looked-up values (block_lut_fused: rows a multiple of 32, groups of at most 32 columns);
  // else the codes as bytes (their OCP bit patterns) from the fused quantizer, then one launch that fits the tables
  // from the bytes, leaves each group's code -> entry map and reads one map entry per element. The workspace holds
  // the bytes, the tables and the maps (less than the float codes of the general path below).
  if (ax0 && block == 32 && rows * cols > 0) {
    const int64_t ng = (cols + ((int64_t)1 << group) - 1) >> group;
    const int64_t nc = (int64_t)1 << (1 + spec->e + spec->m);
    uint8_t* codesT = static_cast<uint8_t*>(workspace);        // column-major: cols x rows
    float* Tb = reinterpret_cast<float*>(codesT + round_up(rows * cols));
    float* cmap = Tb + round_up(ng * kTableWidth * (int64_t)sizeof(float)) / (int64_t)sizeof(float);
    const int64_t used = round_up(rows * cols) + round_up(ng * kTableWidth * (int64_t)sizeof(float)) +
                         ng * nc * (int64_t)sizeof(float);
    if (used <= workspace_bytes) {
      cudaStream_t st = as_stream(stream);
      if (int r = check_cuda(cudaMemsetAsync(status, 0, sizeof(int32_t), st), "block.lut")) return r;
      const int q = mxq::block_lut_fused(V, P_lut, X, Tb, cmap, codesT, rows, cols, group, max_iters, spec->e, spec->m,
                                         spec->rounding, spec->scale_floor, status, stream);
      if (q != MXQ_ERR_UNSUPPORTED) return q;
    }
  }
  if (ax0 && block == 32 && rows * cols > 0 && cols % 4 == 0 && (uintptr_t)V % 16 == 0 &&
      (uintptr_t)P_lut % 16 == 0) {
    const int64_t ng = (cols + ((int64_t)1 << group) - 1) >> group;
    const int64_t nc = (int64_t)1 << (1 + spec->e + spec->m);
    uint8_t* codes = static_cast<uint8_t*>(workspace);         // by 32-column panels: rows x (cols rounded up to 32)
    const int64_t code_bytes = round_up(rows * ((cols + 31) / 32 * 32));
    float* Tb = reinterpret_cast<float*>(codes + code_bytes);
    float* cmap = Tb + round_up(ng * kTableWidth * (int64_t)sizeof(float)) / (int64_t)sizeof(float);
    const int64_t used = code_bytes + round_up(ng * kTableWidth * (int64_t)sizeof(float)) +
                         ng * nc * (int64_t)sizeof(float);
    cudaStream_t st = as_stream(stream);
    if (used <= workspace_bytes) {
      if (int r = check_cuda(cudaMemsetAsync(status, 0, sizeof(int32_t), st), "block.lut")) return r;
      const int q = mxq::quantize_tma_codes(V, codes, X, status, 1, rows, cols, *spec, st);
      if (q != MXQ_ERR_UNSUPPORTED) {
        if (q) return q;
        return mxq::lut_tables_codes_lookup(codes, Tb, cmap, P_lut, rows, cols, group, max_iters, spec->e, spec->m,
                                            status, stream);
      }
    }
  }
  float* P = static_cast<float*>(workspace);
  float* T = reinterpret_cast<float*>(static_cast<char*>(workspace) + round_up(rows * cols * (int64_t)sizeof(float)));
  // the codes: V viewed as [outer, len, inner] with blocks along `axis`
  const int64_t outer = ax0 ? 1 : rows, len = ax0 ? rows : cols, inner = ax0 ? cols : 1;
  if (int r = mxq_block_quantize(V, P, X, outer, len, inner, block, spec, stream)) return r;
  // the K x n operand: axis 0 is V's own layout; axis 1 reads V's transpose in place
  const int64_t K = ax0 ? rows : cols, n = ax0 ? cols : rows, sk = ax0 ? cols : 1, sj = ax0 ? 1 : cols;
  if (int r = mxq_lut_tables(P, T, K, n, sk, sj, group, max_iters, spec->e, spec->m, status, stream)) return r;
  return mxq_lut_pick_lookup(P, T, P_lut, K, n, sk, sj, group, kTableWidth, stream);
}

int mxq_block_lut_quantize_static(const float* V, float* P_lut, float* X, int64_t rows, int64_t cols, int32_t axis,
                                  int64_t block, const mxq_quant_spec* spec, int32_t group, int32_t max_iters,
                                  int32_t* status, void* stream) {
  const int64_t need = mxq_block_lut_workspace(rows, cols, axis, group);
  MXQ_REQUIRE(need >= 0, MXQ_ERR_VALUE, "block.lut: bad sizes (%lld x %lld, group %d)", (long long)rows,
              (long long)cols, group);
  MXQ_REQUIRE(need <= kStaticScratchBytes, MXQ_ERR_VALUE,
              "block.lut static scratch: %lld x %lld at group %d needs %lld bytes of scratch, above the %lld-byte "
              "maximum (call mxq_block_lut_quantize with a workspace instead)",
              (long long)rows, (long long)cols, group, (long long)need, (long long)kStaticScratchBytes);
  void* scratch = nullptr;
  if (int r = static_scratch(&scratch)) return r;
  return mxq_block_lut_quantize(V, P_lut, X, rows, cols, axis, block, spec, group, max_iters, scratch,
                                kStaticScratchBytes, status, stream);
}

}  // extern "C"
