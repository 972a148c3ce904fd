/* mxq_b200 — C ABI of the B200 (sm_100a) implementation of mxq's quantize-and-emulated-matmul hot path.
 *
 * Every entry point replaces one function of the reference Python package (chloe-wong/microscaling-quant,
 * paths below are mxq/...:line) and computes bit-identical results on the device. Conventions:
 *   - all array arguments are DEVICE pointers to contiguous row-major data; sizes are element counts;
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream); calls are asynchronous unless stated;
 *   - the return value is MXQ_OK (0) or an MXQ_ERR_* code; mxq_last_error() returns this thread's message;
 *   - kernels never trap on data: NaN and Inf are values, and results follow the reference's rules for them.
 * Thread safety: the library's mutable global state is the per-thread error message, caches filled once under a
 * lock (per-device SM counts, the driver's tensor-map entry point, the static scratch's per-device address, each LUT
 * format's tables in device memory: uploaded by a synchronous copy at the first LUT call on a device, and again when
 * that device's context has changed), and the wait-status word (mxq_wait_status_word), which kernels only increment.
 */
#ifndef MXQ_B200_H
#define MXQ_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------------------------ status */
#define MXQ_OK 0
#define MXQ_ERR_VALUE 1      /* an argument the reference rejects with ValueError */
#define MXQ_ERR_INDEX 2      /* an axis out of range (IndexError in the reference) */
#define MXQ_ERR_UNSUPPORTED 3 /* a configuration this build has no kernel for */
#define MXQ_ERR_CUDA 4       /* the CUDA runtime reported an error */

/* rounding modes: mxq/rounding/__init__.py:25 MODES */
#define MXQ_RM_TIES_AWAY 0
#define MXQ_RM_RNE 1
#define MXQ_RM_TRUNCATE 2
/* microxcaling rounding names: mxq/microxcaling/elemwise.py:29-60 */
#define MXQ_MS_NEAREST 0
#define MXQ_MS_FLOOR 1
#define MXQ_MS_EVEN 2
/* float_em grids: mxq/element_quant/float_em.py:41 GRIDS */
#define MXQ_GRID_QTORCH 0
#define MXQ_GRID_IEEE 1
#define MXQ_GRID_OCP 2

const char* mxq_version(void);
const char* mxq_last_error(void);

/* ------------------------------------------------------------------------------ elementwise (n values) */
/* mxq/rounding/__init__.py:51-55 round_bits: int64 bit patterns rounded to `keep` fraction bits. keep == NULL
 * uses keep_scalar for every element; otherwise keep[i] per element (each in [0, 22]). */
int mxq_round_bits(const int64_t* bits, const int64_t* keep, int32_t keep_scalar, int64_t* out, int64_t n,
                   int32_t mode, void* stream);
/* mxq/rounding/ties_away.py:5-6, rne.py:6-8, truncate.py:5-6 bits(bits, drop, mask, half): one mode's rounding of
 * int64 patterns with the caller's drop / mask / half, each an array of n values or (NULL) its scalar; the int64
 * result is not reduced to 32 bits (round_bits does that). A drop outside [0, 63] shifts by 63, as torch's >>. */
int mxq_round_pattern(const int64_t* bits, const int64_t* drop, int64_t drop_s, const int64_t* mask, int64_t mask_s,
                      const int64_t* half, int64_t half_s, int64_t* out, int64_t n, int32_t mode, void* stream);
/* mxq/rounding/__init__.py:58-61 round_int */
int mxq_round_int_f32(const float* k, float* out, int64_t n, int32_t mode, void* stream);
int mxq_round_int_f64(const double* k, double* out, int64_t n, int32_t mode, void* stream);
/* mxq/rounding/__init__.py:64-85 bf16 */
int mxq_bf16(const float* x, float* out, int64_t n, void* stream);
/* mxq/element_quant/float_em.py:50-61 quantize, float32 or float64 input, float32 output */
int mxq_float_em_f32(const float* z, float* out, int64_t n, int32_t e, int32_t m, int32_t mode, int32_t grid,
                     void* stream);
int mxq_float_em_f64(const double* z, float* out, int64_t n, int32_t e, int32_t m, int32_t mode, int32_t grid,
                     void* stream);
/* mxq/microxcaling/elemwise.py:63-151 _quantize_elemwise_core (allow_denorm=True), as
 * mxq/element_quant/microsoft.py:18-23 calls it. bits includes sign and implicit bit; exp_bits 0 = integer. */
int mxq_microsoft(const float* A, float* out, int64_t n, int32_t bits, int32_t exp_bits, float max_norm,
                  int32_t round, int32_t saturate_normals, void* stream);
/* mxq/scale_factor.py:40-44 mxquant; floor = float32(floor) */
int mxq_scale_mxquant(const float* amax, float* X, int64_t n, float floor, void* stream);
/* mxq/scale_factor.py:47-59 ocp (and :62-65 ocp_below_top with emax - 1); scale_emax = float32(2^(bits-1) - 1) */
int mxq_scale_ocp(const float* amax, float* X, int64_t n, int32_t emax, float scale_emax, void* stream);
/* mxq/scale_factor.py:68-81 ocp_no_clip for the OCP element format (e, m) */
int mxq_scale_ocp_no_clip(const float* amax, float* X, int64_t n, int32_t e, int32_t m, int32_t round,
                          float scale_emax, void* stream);
/* mxq/arith.py:68-103 exact_add */
int mxq_exact_add(const float* a, const float* b, float* out, int64_t n, int32_t e, int32_t m, int32_t mode,
                  int32_t grid, void* stream);
/* mxq/arith.py:106-117 truncate_significand */
int mxq_truncate_significand(const float* x, float* out, int64_t n, int32_t m, void* stream);
/* mxq/arith.py:120-124 flush_product; thr = float32(2^floor_exp) */
int mxq_flush_product(const float* x, float* out, int64_t n, float thr, void* stream);
/* mxq/arith.py:127-137 saturate */
int mxq_saturate(const float* x, float* out, int64_t n, float limit, float value, void* stream);

/* ---------------------------------------------------------------------------- Arithmetic datapaths */
/* An Arithmetic of mxq/matmul/_arithmetic.py: MXQUANT(prod_e, prod_m) (:64-73) or MXGEMMINI(prod_e, prod_m,
 * prod_floor) (:111-134) with spike's saturation pair (:88-102). */
#define MXQ_ARITH_MXQUANT 0
#define MXQ_ARITH_MXGEMMINI 1
typedef struct mxq_arith {
  int32_t kind;
  int32_t prod_e, prod_m;
  int32_t has_floor;      /* MXGEMMINI: prod_floor is not None */
  float floor_thr;        /* float32(2^prod_floor) */
  float sat_limit, sat_value;
} mxq_arith;
/* Arithmetic.product / acc_add / tile_add as elementwise operations (the reducers inline the same code) */
int mxq_arith_product(const float* a, const float* b, float* out, int64_t n, const mxq_arith* arith, void* stream);
int mxq_arith_acc_add(const float* S, const float* p, float* out, int64_t n, const mxq_arith* arith, int32_t e,
                      int32_t m, void* stream);
int mxq_arith_tile_add(const float* C, const float* t, float* out, int64_t n, const mxq_arith* arith, void* stream);

/* ------------------------------------------------------------------------------------ block quantizers */
/* A tensor is viewed as [outer, len, inner] with blocks of `block` along len (mxq/block/_driver.py:23-32); the
 * codes P have V's layout and the scales X are [outer, ceil(len / block), inner]. */
#define MXQ_FAMILY_FP32 0        /* format "FP32": X = 1, P = V */
#define MXQ_FAMILY_MXQUANT 1     /* mxq/block/mxquant.py:26-32 */
#define MXQ_FAMILY_MXGEMMINI 2   /* mxq/block/mxgemmini.py:37-59 */
#define MXQ_FAMILY_OCP 3         /* mxq/block/ocp.py:35-49 */
typedef struct mxq_quant_spec {
  int32_t family;
  int32_t e, m;            /* element format */
  int32_t rounding;        /* MXQ_RM_* (mxquant: ties away; mxgemmini: its rounding_mode) or MXQ_MS_* (ocp) */
  float scale_floor;       /* mxquant / mxgemmini: float32(scale_floor) */
  int32_t placement;       /* ocp: 0 top, 1 below_top, 2 no_clip (mxq/block/ocp.py:32) */
  float scale_emax;        /* ocp: float32(2^(scale_bits - 1) - 1) */
  int32_t via_e, via_m;    /* mxgemmini `via`: ieee pre-rounding format, 0 = none */
} mxq_quant_spec;
/* mxq/block/_driver.py:45-66 compose with a named quantizer's two steps, fused: block amax, scale, divide and
 * element rounding in one pass. */
int mxq_block_quantize(const float* V, float* P, float* X, int64_t outer, int64_t len, int64_t inner, int64_t block,
                       const mxq_quant_spec* spec, void* stream);
/* No reference counterpart: the compact operand form (the wire format of MX-Gemmini's LUT indices,
 * mxq/lut/__init__.py:3-6). mxq_block_quantize for the OCP-grid families (mxgemmini without `via`, and ocp) writing
 * each code as its element format's OCP bit pattern -- a byte per FP8 / FP6 element (FP6 in the low six bits), two
 * FP4 elements per byte (the even element in the low nibble) -- in P's layout, and each scale as an E8M0 byte
 * (2^(b - 127), 0xFF NaN) in X's layout. status bits: 1 a code the format cannot hold (Inf in E4M3 / FP6 / FP4,
 * NaN in FP6 / FP4), 2 a scale that is not a power of two in [2^-127, 2^127] (mxgemmini's floor for an all-zero
 * block, below it). Blocks of 32, rows (the innermost extent) a multiple of 4, 16-byte aligned V and codes. */
int mxq_block_quantize_packed(const float* V, uint8_t* codes, uint8_t* scales, int64_t outer, int64_t len,
                              int64_t inner, int64_t block, const mxq_quant_spec* spec, int32_t* status,
                              void* stream);
/* No reference counterpart: mxq_block_quantize writing its codes and scales to ndst (1..8) destinations at once,
 * P[i] / X[i] each a DEVICE pointer to a [outer, len, inner] / [outer, ceil(len/block), inner] buffer (a HOST array
 * of ndst pointers). With peer mappings of the other ranks' buffers (CUDA IPC or symmetric memory over NVLink) the
 * quantizer of a rank's slice of rows is also the all-gather of its outputs: mxq/shard.py quantize_gathered. The
 * caller orders the ranks' writes before anyone reads (a barrier after the call). Blocks of 32; the TMA kernel's
 * layouts (rows a multiple of 4 elements, 16-byte aligned V and destinations); MXQ_ERR_UNSUPPORTED otherwise. */
int mxq_block_quantize_multi(const float* V, float* const* P, float* const* X, int32_t ndst, int64_t outer,
                             int64_t len, int64_t inner, int64_t block, const mxq_quant_spec* spec, void* stream);
/* No reference counterpart: float32 codes and scales from the compact form (n_codes elements, n_scales scales) */
int mxq_unpack(const uint8_t* codes, const uint8_t* scales, float* P, float* X, int64_t n_codes, int64_t n_scales,
               int32_t e, int32_t m, void* stream);
/* No reference counterpart: mxq_dequantize from the compact form */
int mxq_dequantize_packed(const uint8_t* codes, const uint8_t* scales, float* out, int64_t outer, int64_t len,
                          int64_t inner, int64_t block, int32_t e, int32_t m, void* stream);
/* The pieces of compose with caller-supplied steps (mxq/block/_driver.py:23-42, :63-64): the blocked layout is
 * [outer, inner, nblocks, block] (the block axis moved last, zero-padded). */
int mxq_block_amax(const float* V, float* amax, int64_t outer, int64_t len, int64_t inner, int64_t block,
                   void* stream);
/* Z = pad(V) / X in the blocked layout; X is [outer, inner, nblocks] (NULL: a copy) */
int mxq_to_blocks(const float* V, const float* X, float* Z, int64_t outer, int64_t len, int64_t inner, int64_t block,
                  void* stream);
/* blocked [outer, inner, nblocks, block] -> [outer, len, inner], padding dropped (codes_from_blocks, :35-37;
 * with block = 1 and len = nblocks it is scales_from_blocks, :40-42) */
int mxq_from_blocks(const float* Zb, float* P, int64_t outer, int64_t len, int64_t inner, int64_t block,
                    void* stream);
/* mxq/block/_driver.py:69-72 dequantize: P * expand(X) along len */
int mxq_dequantize(const float* P, const float* X, float* out, int64_t outer, int64_t len, int64_t inner,
                   int64_t block, void* stream);

/* ------------------------------------------------------------------------------------------ reducers */
/* Y (M x N) = A^T B from codes P_A (K x M), P_B (K x N) and scales X_A (ceil(K/block) x M), X_B (.. x N).
 * The schedule is `size` lane formats (sched_e[i], sched_m[i]), host arrays. */
/* mxq/matmul/_systolic.py:23-62 systolic */
int mxq_systolic(const float* PA, const float* XA, const float* PB, const float* XB, float* Y, int64_t K, int64_t M,
                 int64_t N, int64_t block, int64_t size, const mxq_arith* arith, const int32_t* sched_e,
                 const int32_t* sched_m, void* stream);
/* No reference counterpart: mxq_systolic over `batch` independent problems stacked contiguously (PA batch x K x M,
 * XA batch x ceil(K/block) x M, PB batch x K x N, XB batch x ceil(K/block) x N, Y batch x M x N), each result
 * bit-identical to mxq_systolic on that problem alone; one launch for many small problems (attend's heads,
 * mxq/nn/_attention.py:102-141). */
int mxq_systolic_batched(const float* PA, const float* XA, const float* PB, const float* XB, float* Y,
                         int64_t batch, int64_t K, int64_t M, int64_t N, int64_t block, int64_t size,
                         const mxq_arith* arith, const int32_t* sched_e, const int32_t* sched_m, void* stream);
/* mxq/matmul/_adder.py:42-71 adder_tree: log2(size) levels, level formats (level_e[l], level_m[l]) */
int mxq_adder_tree(const float* PA, const float* XA, const float* PB, const float* XB, float* Y, int64_t K, int64_t M,
                   int64_t N, int64_t block, int64_t size, const mxq_arith* arith, const int32_t* level_e,
                   const int32_t* level_m, void* stream);
/* mxq/matmul/_anchor.py:95-138 anchor_tree; tree_bits is [size / width][nbits] level widths per tree */
typedef struct mxq_anchor_spec {
  int32_t width, nbits, drop_rne, headroom, has_emin, emin;
} mxq_anchor_spec;
int mxq_anchor_tree(const float* PA, const float* XA, const float* PB, const float* XB, float* Y, int64_t K,
                    int64_t M, int64_t N, int64_t block, int64_t size, const mxq_arith* arith, const int32_t* tree_e,
                    const int32_t* tree_m, const mxq_anchor_spec* anchor, const int32_t* tree_bits, void* stream);
/* mxq/_fp64_accum.py:24-29 fp64_accum: dequantized operands, float64 products and sums in K order, float32 out */
int mxq_fp64_accum(const float* PA, const float* XA, const float* PB, const float* XB, float* Y, int64_t K, int64_t M,
                   int64_t N, int64_t block, void* stream);

/* ------------------------------------------------------------------------------------------- LUTs */
/* MX-Gemmini's look-up tables for the LUT formats (e, m) in {(3,2), (2,3), (5,2), (4,3)}. An operand is K x n,
 * element (k, j) at P[k * sk + j * sj] (row-major: sk = n, sj = 1; transposed in place: sk = 1, sj = K); one table
 * of 16 ascending values per 2^group columns. `status` is a device int32 the call zeroes and a kernel sets when an
 * input is not what the reference accepts (the caller reads it to raise the reference's error). */
/* mxq/lut/formats.py:83-122 _tables / values: every code's value and fixed point, the finder-safe values (HOST
 * pointers, any may be NULL; vals/fx hold 2^(1+e+m) entries, safe up to 256); synchronous, no device work */
int mxq_lut_format_tables(int32_t e, int32_t m, float* vals, int64_t* fx, float* safe, int32_t* nsafe);
/* mxq/lut/kmeans.py:46-122 tables: T is ceil(n / 2^group) x 16; status 1: a value of P is not a code */
int mxq_lut_tables(const float* P, float* T, int64_t K, int64_t n, int64_t sk, int64_t sj, int32_t group,
                   int32_t max_iters, int32_t e, int32_t m, int32_t* status, void* stream);
/* mxq/lut/kmeans.py:125-138 pick: I is K x n int64 row-major; T rows of `width` ascending entries */
int mxq_lut_pick(const float* P, const float* T, int64_t* I, int64_t K, int64_t n, int64_t sk, int64_t sj,
                 int32_t group, int32_t width, void* stream);
/* mxq/block/lut.py:33 lookup(pick(P, T), T) in one pass, written in P's own layout */
int mxq_lut_pick_lookup(const float* P, const float* T, float* out, int64_t K, int64_t n, int64_t sk, int64_t sj,
                        int32_t group, int32_t width, void* stream);
/* mxq/lut/kmeans.py:141-146 lookup */
int mxq_lut_lookup(const int64_t* I, const float* T, float* out, int64_t K, int64_t n, int32_t group, int32_t width,
                   void* stream);
/* mxq/lut/formats.py:125-137 encode (status 1: a value is not a code) and :114-117 decode (status 1: bad code) */
int mxq_lut_encode(const float* V, int64_t* codes, int64_t n, int32_t e, int32_t m, int32_t* status, void* stream);
int mxq_lut_decode(const int64_t* codes, float* out, int64_t n, int32_t e, int32_t m, int32_t* status, void* stream);
/* mxq/lut/formats.py:140-159 finder: I is K x n int64 (status 1: bad code, 2: a table value is not a code) */
int mxq_lut_finder(const int64_t* codes, const float* T, int64_t* I, int64_t K, int64_t n, int32_t group, int32_t e,
                   int32_t m, int32_t* status, void* stream);

/* mxq/block/lut.py:23-34 quantize in one call: block.mxgemmini codes of the 2-D V (rows x cols, blocks along
 * `axis`), the tables of the K x n operand (axis 0: V itself; axis 1: V's transpose, read in place), every code
 * replaced by its table entry. P_lut has V's layout; X is the scales (as mxq_block_quantize writes them). spec must be
 * the mxgemmini family without `via` and a LUT format. The codes and the tables live in `workspace`, at least
 * mxq_block_lut_workspace(rows, cols, axis, group) bytes, 256-byte aligned (-1 for bad sizes). `status` as for
 * mxq_lut_tables (1: a code is not on the format's grid, e.g. from a NaN or Inf in V). Asynchronous. */
int64_t mxq_block_lut_workspace(int64_t rows, int64_t cols, int32_t axis, int32_t group);
int mxq_block_lut_quantize(const float* V, float* P_lut, float* X, int64_t rows, int64_t cols, int32_t axis,
                           int64_t block, const mxq_quant_spec* spec, int32_t group, int32_t max_iters,
                           void* workspace, int64_t workspace_bytes, int32_t* status, void* stream);
/* No counterpart in the reference: mxq_block_lut_quantize with its workspace taken from a static device array of
 * 16 MiB (one per device) instead of the caller, so the call allocates nothing. Sizes whose workspace
 * (mxq_block_lut_workspace) exceeds 16 MiB are rejected with MXQ_ERR_VALUE. Every call on a device shares the
 * array: calls whose work overlaps on the GPU (other streams, or other host threads, without ordering between
 * them) race on it. Nothing in the array needs to start at zero. The array's device address is looked up again
 * whenever the device's current context has changed (cudaDeviceReset makes a new one, and the module's arrays with
 * it). */
int mxq_block_lut_quantize_static(const float* V, float* P_lut, float* X, int64_t rows, int64_t cols, int32_t axis,
                                  int64_t block, const mxq_quant_spec* spec, int32_t group, int32_t max_iters,
                                  int32_t* status, void* stream);

/* ------------------------------------------------------------------------------------------ diagnostics */
/* No reference counterpart: the number of bounded shared-memory waits (mbarrier) that gave up in the TMA-staged
 * kernels on the current device since the library was loaded. Always 0 in a correct run; synchronous. */
int mxq_device_timeouts(uint32_t* out);
/* No reference counterpart: the address of the wait-status word, a 32-bit counter in pinned, mapped host memory
 * (allocated on first use, shared by every device) that a TMA-staged kernel increments when a bounded wait gives up
 * -- the tile it was loading is then written as NaN codes and NaN scales (the compact form sets status bit 4
 * instead). The host reads it with a plain load and no synchronisation; it counts the kernels that have finished.
 * A caller checks it after its calls and clears it (stores 0) once it has handled the event. A cudaDeviceReset of the
 * device whose context allocated the word frees it; the library then allocates a new one at its next use on that
 * device, so a caller that keeps the address fetches it again after such a reset. */
int mxq_wait_status_word(uint32_t** out);
/* No reference counterpart; for tests of the timeout path only: mxq_block_quantize of a rows x cols V (blocks of 32
 * along rows, mxgemmini MXFP8_E4M3) through the TMA kernel with its loads never issued and waits of wait_rounds
 * (1..65536) rounds, so every tile's wait runs out with nothing in flight; P and X come out NaN and the wait-status
 * word and the device counter rise by one per 32 x 256 tile. cols a multiple of 32, V and P 16-byte aligned. */
int mxq_testing_wait_timeout(const float* V, float* P, float* X, int64_t rows, int64_t cols, uint32_t wait_rounds,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MXQ_B200_H */
