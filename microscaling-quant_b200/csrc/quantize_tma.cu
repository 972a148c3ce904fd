// The block quantizers' main kernel on sm_100a: one CTA per 32 x TC float32 tile of V (TC = 256). A CTA loads its
// tile into shared memory with one TMA copy (cp.async.bulk.tensor, mbarrier-tracked, bounded wait), quantizes it and
// exits; the block scheduler keeps several such CTAs resident per SM, so one CTA's load overlaps the others'
// arithmetic and stores, and one pass over HBM reads V once and writes P and X once. (Persistent CTAs cycling
// through tiles with a two- or three-stage pipeline measured 11-12% slower on the same sweep: fewer loads in
// flight per SM, and each launch ended on a partial round of 32 KB tiles.)
//
// Two layouts of the [outer, len, inner] view (blocks of BS along len; BS = 32, or 16 / 64 with float outputs):
//   ROWS (inner == 1): a tile is 32 rows x TC consecutive values of a row, i.e. TC / BS blocks per row (blocks of
//                      BS = 16, 32 or 64);
//   COLS (inner > 1):  a tile is one block of BS rows (along len; BS = 16 or 32) x TC columns (along inner).
// Per tile: (1) one thread per block takes the block max from shared memory and computes the block's scale and
// reciprocal (ROWS: a thread reads its block's BS / 4 float4 in a rotated order, so a quarter-warp hits distinct
// banks; COLS: a thread walks its column), and the CTA votes whether every block is clean (finite, with a
// power-of-two scale); (2) every thread quantizes its float4 of the tile, reading values and scales from shared
// memory and writing P with coalesced 128-bit streaming stores -- a clean tile with the short element step.
// The element format is a template parameter, so the grid constants of each format fold into immediates.
#include "common.cuh"
#include "numerics.cuh"
#include "tma.cuh"
#include "quant_elem.cuh"

using namespace mxq;

namespace {

constexpr int TR = 32, TC = 256, NT = 256;
constexpr int C4 = TC / 4;              // float4 per tile row
constexpr int RPI = NT / C4;            // tile rows per pass of the CTA in the element step
static_assert(TC % 32 == 0 && TC <= NT && NT % C4 == 0 && TR % RPI == 0, "tile shape");
// a tile is at most TR x TC floats: 32 KB, below the 48 KB default, no shared-memory attribute needed

struct TParams {
  int rounding, placement, via_e, via_m;
  float scale_floor, scale_emax;
  unsigned* status_word;   // the host-mapped wait-status word (wait_status_word())
  unsigned wait_rounds;    // try_wait rounds before the tile's wait gives up (kWaitLimit)
  int skip_load;           // 1 only in mxq_testing_wait_timeout: the load is never issued, so the wait runs out
};

// float_em._qtorch ties away (mxq/element_quant/float_em.py:64-84), constants folded
template <int E, int M>
__device__ __forceinline__ float qtorch_ties_away(float z) {
  constexpr uint32_t drop = 23 - M, half = 1u << (drop - 1), mask = ~((1u << drop) - 1u);
  constexpr uint32_t L = (1u << (E - 1)) - 1u, mins = 127u - L, maxs = 127u + L;
  constexpr uint32_t MAXMAG = (maxs << 23) | (0x007fffffu & mask), MINMAG = mins << 23;
  constexpr uint32_t MID = (mins - 1u) << 23, OVF = (maxs + 1u) << 23;
  const uint32_t u = f2u(z), q = (u + half) & mask, qm = q & 0x7fffffffu, s = u & 0x80000000u;
  uint32_t r = q;
  if (qm >= OVF) r = s | MAXMAG;
  if (qm < MINMAG) r = qm > MID ? (s | MINMAG) : 0u;
  return u2f(r);
}

template <int FAM, int E, int M>
__device__ __forceinline__ float element(float z, const TParams& p) {
  if (FAM == MXQ_FAMILY_MXQUANT) return qtorch_ties_away<E, M>(z);
  if (FAM == MXQ_FAMILY_MXGEMMINI) {
    if (p.via_e) z = q_ieee(z, p.via_e, p.via_m, p.rounding);          // mxgemmini.py:50-55: the via pre-rounding
    return ocp_grid<E, M>(z, p.rounding);
  }
  return q_microsoft_ocp(z, M + 2, E, Fmt<E, M>::MAX_NORM, p.rounding);
}

// The element step of a clean tile (every block finite, every scale a power of two with an exact reciprocal): z is
// then finite and |z| < 2^17, so the Inf / NaN / huge-value branches cannot be taken, the rounding is one float add
// at the step's magic constant (q_ocp_small, q_microsoft_ocp_small), and the rounding mode is a template argument.
// VIA: block.mxgemmini's pre-rounding onto float(via_e, via_m) (mxgemmini.py:50-55), for via_e <= 7 and via_m <= 21
// (q_ieee_small's range).
template <int FAM, int E, int M, int MODE, bool VIA>
__device__ __forceinline__ float element_clean(float z, int via_e, int via_m) {
  if (FAM == MXQ_FAMILY_MXQUANT) return qtorch_ties_away<E, M>(z);
  if (FAM == MXQ_FAMILY_MXGEMMINI) {
    if (VIA) z = q_ieee_small(z, via_e, via_m, MODE);
    return q_ocp_small(z, E, M, MODE, Fmt<E, M>::MAX_NORM);
  }
  return q_microsoft_ocp_small(z, M + 2, E, Fmt<E, M>::MAX_NORM, MODE);
}

template <int FAM, int E, int M>
__device__ __forceinline__ float block_scale(float amax, const TParams& p) {
  if (FAM == MXQ_FAMILY_MXQUANT || FAM == MXQ_FAMILY_MXGEMMINI) return scale_mxquant(amax, p.scale_floor);
  if (p.placement == 0) return scale_ocp(amax, Fmt<E, M>::EMAX, p.scale_emax);
  if (p.placement == 1) return scale_ocp(amax, Fmt<E, M>::EMAX - 1, p.scale_emax);
  return scale_ocp_no_clip(amax, E, M, p.rounding, p.scale_emax);
}

template <int FAM>
__device__ __forceinline__ float divide(float v, float x, float r) {
  if (r != 0.0f) return __fmul_rn(v, r);
  return FAM == MXQ_FAMILY_MXQUANT ? x86_div(v, x) : div_rn(v, x);
}

// Where a kernel puts its results. OutF: float32 codes and scales (the reference's outputs). OutPack: the compact
// form -- each code as its OCP bit pattern (a byte; FP4: a nibble, two per byte, the even element low) and each
// scale as an E8M0 byte -- with a flag for any value the form cannot hold. Element index idx is a multiple of 4.
struct OutF {
  static constexpr bool kPanels = false;   // codes at their element index (the others but OutCodes alike)
  float* P;
  float* X;
  template <bool FINITE = false>
  __device__ __forceinline__ void codes(int64_t idx, float4 v) { __stcs(reinterpret_cast<float4*>(P + idx), v); }
  __device__ __forceinline__ void scale(int64_t idx, float x) { X[idx] = x; }
  __device__ __forceinline__ void finish() {}
  __device__ __forceinline__ void lost() {}                // the tile's NaN codes and scales say it
};

// The float32 outputs written to up to kMaxDst destinations at once: this GPU's buffers and, through peer (NVLink)
// mappings, the same slice of every other rank's buffers, so the quantizer is also the all-gather of its outputs.
// Destination 0 takes streaming stores; the others plain stores (remote writes over NVLink).
constexpr int kMaxDst = 8;
struct OutMulti {
  static constexpr bool kPanels = false;
  float* P[kMaxDst];
  float* X[kMaxDst];
  int n;
  template <bool FINITE = false>
  __device__ __forceinline__ void codes(int64_t idx, float4 v) {
    __stcs(reinterpret_cast<float4*>(P[0] + idx), v);
#pragma unroll
    for (int d = 1; d < kMaxDst; d++)
      if (d < n) *reinterpret_cast<float4*>(P[d] + idx) = v;
  }
  __device__ __forceinline__ void scale(int64_t idx, float x) {
#pragma unroll
    for (int d = 0; d < kMaxDst; d++)
      if (d < n) X[d][idx] = x;
  }
  __device__ __forceinline__ void finish() {}
  __device__ __forceinline__ void lost() {}                // the tile's NaN codes and scales say it
};

__device__ __forceinline__ uint32_t e8m0(float x, bool& bad) {     // 2^(b - 127); 0xFF NaN
  const uint32_t u = f2u(x);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0xffu;
  if (u == 0x00400000u) return 0u;                                  // 2^-127
  if ((u & 0x807fffffu) == 0u && u >= 0x00800000u && u < 0x7f800000u) return u >> 23;
  bad = true;                                                       // not a power of two the byte can hold
  return 0u;
}

template <int E, int M>
struct OutPack {
  static constexpr bool kPanels = false;
  uint8_t* P;
  uint8_t* X;
  int* status;
  bool bad_code = false, bad_scale = false;
  template <bool FINITE = false>
  __device__ __forceinline__ void codes(int64_t idx, float4 v) {
    uint32_t c0, c1, c2, c3;
    if (FINITE) {
      c0 = ocp_code_finite<E, M>(v.x);
      c1 = ocp_code_finite<E, M>(v.y);
      c2 = ocp_code_finite<E, M>(v.z);
      c3 = ocp_code_finite<E, M>(v.w);
    } else {
      c0 = ocp_code<E, M>(v.x, bad_code);
      c1 = ocp_code<E, M>(v.y, bad_code);
      c2 = ocp_code<E, M>(v.z, bad_code);
      c3 = ocp_code<E, M>(v.w, bad_code);
    }
    if (E + M == 3) __stcs(reinterpret_cast<unsigned short*>(P + idx / 2),
                           (unsigned short)(c0 | (c1 << 4) | (c2 << 8) | (c3 << 12)));
    else __stcs(reinterpret_cast<unsigned int*>(P + idx), c0 | (c1 << 8) | (c2 << 16) | (c3 << 24));
  }
  __device__ __forceinline__ void scale(int64_t idx, float x) { X[idx] = (uint8_t)e8m0(x, bad_scale); }
  __device__ __forceinline__ void finish() {
    const int bits = (bad_code ? 1 : 0) | (bad_scale ? 2 : 0);
    if (bits) atomicOr(status, bits);
  }
  __device__ __forceinline__ void lost() {
    if (threadIdx.x == 0) atomicOr(status, 4);
  }
};

// block.lut's codes: each code as a byte (lut_code; the 6- and 8-bit LUT formats) and each scale as float32; status
// bit 1 for a code the format cannot hold (as OutPack), 4 for a lost tile. The bytes of a blocks-along-rows operand
// (len rows x inner columns) are stored by 32-column panels: panel p holds its rows one after another, 32 bytes each
// (byte (l, col) at ((col / 32) len + l) 32 + col % 32), so the table fit reads each panel as one contiguous run.
template <int E, int M>
struct OutCodes {
  static constexpr bool kPanels = true;
  uint8_t* P;
  float* X;
  int* status;
  int64_t len;
  bool bad_code = false;
  template <bool FINITE = false>
  __device__ __forceinline__ void codes(int64_t idx, float4 v) {
    uint32_t c0, c1, c2, c3;
    if (FINITE) {
      c0 = ocp_code_finite<E, M>(v.x);
      c1 = ocp_code_finite<E, M>(v.y);
      c2 = ocp_code_finite<E, M>(v.z);
      c3 = ocp_code_finite<E, M>(v.w);
    } else {
      c0 = lut_code<E, M>(v.x, bad_code);
      c1 = lut_code<E, M>(v.y, bad_code);
      c2 = lut_code<E, M>(v.z, bad_code);
      c3 = lut_code<E, M>(v.w, bad_code);
    }
    *reinterpret_cast<unsigned int*>(P + idx) = c0 | (c1 << 8) | (c2 << 16) | (c3 << 24);
  }
  __device__ __forceinline__ void scale(int64_t idx, float x) { X[idx] = x; }
  __device__ __forceinline__ void finish() {
    if (bad_code) atomicOr(status, 1);
  }
  __device__ __forceinline__ void lost() {
    if (threadIdx.x == 0) atomicOr(status, 4);
  }
};

// A tile's coordinates, from its index by 32-bit division once per tile: column tile ct, and rest = the row tile
// (ROWS) or (o, b) = the outer slice and block (COLS). Tile counts stay below 2^31 (the launch checks).
struct TileAt {
  int64_t ct, rest, b, o;
};
template <bool COLS>
__device__ __forceinline__ TileAt tile_at(int64_t tile, uint32_t ctiles, uint32_t nb) {
  TileAt t;
  const uint32_t i = (uint32_t)tile, rest = i / ctiles;
  t.ct = i - rest * ctiles;
  t.rest = rest;
  if (COLS) {
    const uint32_t o = rest / nb;
    t.o = o;
    t.b = rest - o * nb;
  } else {
    t.o = t.b = 0;
  }
  return t;
}

// the store of the 4 codes at (l, col) .. (l, col + 3) of a blocks-along-rows tile, at their element index idx or, for an
// output stored by 32-column panels, at their place in the panel
template <bool FINITE, class Out>
__device__ __forceinline__ void put_codes(Out& out, int64_t l, int64_t col, int64_t idx, float4 v) {
  if constexpr (Out::kPanels) out.template codes<FINITE>(((col >> 5) * out.len + l) * 32 + (col & 31), v);
  else out.template codes<FINITE>(idx, v);
}

// (2) for a clean tile: every thread quantizes TR / RPI float4 (float4 q = tid + NT i: row q / C4, column q % C4)
template <int FAM, int E, int M, bool COLS, int BS, int MODE, bool VIA, class Out>
__device__ __forceinline__ void pass_clean(const float* T, const float* s_r, Out& out, const TileAt& at,
                                           int64_t outer, int64_t len, int64_t inner, int via_e, int via_m) {
  const int tid = threadIdx.x, c4 = tid % C4;
  float4 rs;
  if (COLS) rs = *reinterpret_cast<const float4*>(s_r + c4 * 4);
#pragma unroll 2
  for (int i = 0; i < (COLS ? BS : TR) / RPI; i++) {
    const int row = tid / C4 + RPI * i;
    float4 v = reinterpret_cast<const float4*>(T + row * TC)[c4];
    if (!COLS) {
      const float r = s_r[row * (TC / BS) + (int)((unsigned)c4 / (BS / 4))];
      rs = make_float4(r, r, r, r);
    }
    v.x = element_clean<FAM, E, M, MODE, VIA>(__fmul_rn(v.x, rs.x), via_e, via_m);
    v.y = element_clean<FAM, E, M, MODE, VIA>(__fmul_rn(v.y, rs.y), via_e, via_m);
    v.z = element_clean<FAM, E, M, MODE, VIA>(__fmul_rn(v.z, rs.z), via_e, via_m);
    v.w = element_clean<FAM, E, M, MODE, VIA>(__fmul_rn(v.w, rs.w), via_e, via_m);
    if (COLS) {
      const int64_t l = at.b * BS + row, col = at.ct * TC + c4 * 4;
      if (l < len && col < inner) put_codes<true>(out, l, col, (at.o * len + l) * inner + col, v);
    } else {
      const int64_t grow = at.rest * TR + row, col = at.ct * TC + c4 * 4;
      if (grow < outer && col < len) out.template codes<true>(grow * len + col, v);
    }
  }
}

// A tile whose load never arrived: NaN for each of its codes and scales (the same index arithmetic as the normal
// path, no shared-memory reads), then the output's own mark of a lost tile
template <bool COLS, int BS, class Out>
__device__ __forceinline__ void lose_tile(Out& out, const TileAt& at, int64_t outer, int64_t len, int64_t inner,
                                          int64_t nb) {
  const int tid = threadIdx.x, c4 = tid % C4;
  const float q = qnan_f();
  const float4 q4 = make_float4(q, q, q, q);
  for (int i = 0; i < (COLS ? BS : TR) / RPI; i++) {
    const int row = tid / C4 + RPI * i;
    if (COLS) {
      const int64_t l = at.b * BS + row, col = at.ct * TC + c4 * 4;
      if (l < len && col < inner) put_codes<false>(out, l, col, (at.o * len + l) * inner + col, q4);
    } else {
      const int64_t grow = at.rest * TR + row, col = at.ct * TC + c4 * 4;
      if (grow < outer && col < len) out.codes(grow * len + col, q4);
    }
  }
  if (COLS) {
    const int64_t col = at.ct * TC + tid;
    if (tid < TC && col < inner) out.scale((at.o * nb + at.b) * inner + col, q);
  } else {
    constexpr int BPR = TC / BS;
    for (int bi = tid; bi < TR * BPR; bi += NT) {
      const int64_t grow = at.rest * TR + bi / BPR, gblk = at.ct * BPR + bi % BPR;
      if (grow < outer && gblk < nb) out.scale(grow * nb + gblk, q);
    }
  }
  out.finish();
  out.lost();
}

// BS: the block length: 16 or 32 for COLS (a tile is one block of BS rows), 16, 32 or 64 for ROWS
template <int FAM, int E, int M, bool COLS, int BS, class Out>
__global__ void __launch_bounds__(NT) k_quant_tma(const __grid_constant__ CUtensorMap tmap, Out out, int64_t outer,
                                                  int64_t len, int64_t inner, TParams prm) {
  extern __shared__ __align__(128) float T[];               // [TRB][TC]: this CTA's tile
  __shared__ __align__(8) uint64_t bar;
  constexpr int TRB = COLS ? BS : TR;                       // tile rows
  static_assert(BS >= 4 && TC % BS == 0, "ROWS blocks tile the tile row");
  constexpr int BPR = TC / BS;                              // blocks per tile row (ROWS)
  constexpr int NBT = COLS ? TC : TR * BPR;                 // blocks per tile
  __shared__ __align__(16) float s_x[NBT];                  // read as float4 (COLS): 16-byte aligned
  __shared__ __align__(16) float s_r[NBT];

  const int tid = threadIdx.x;
  // tile grid: ROWS -> (row tiles, column tiles) of the [outer, len] matrix; COLS -> (outer, blocks, column tiles)
  const int64_t nb = (len + BS - 1) / BS;                  // blocks along len
  const int64_t ctiles = COLS ? (inner + TC - 1) / TC : (len + TC - 1) / TC;
  const TileAt at = tile_at<COLS>(blockIdx.x, (uint32_t)ctiles, (uint32_t)nb);
  const int64_t ct = at.ct, rest = at.rest;

  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  // launched as a programmatic dependent of the kernel before it on the stream: everything above overlaps that
  // kernel's last CTAs; no global memory is read or written before it has completed and flushed
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __syncthreads();
  if (tid == 0) {
    fence_proxy_async();
    mbar_expect_tx(&bar, (unsigned)(TRB * TC * sizeof(float)));
    if (!prm.skip_load) {
      if (COLS) tma_load_3d(T, &tmap, (int)(ct * TC), (int)(at.b * BS), (int)at.o, &bar);
      else tma_load_2d(T, &tmap, (int)(ct * TC), (int)(rest * TR), &bar);
    }
  }
  // every thread waits (bounded); if the wait gave up anywhere the tile is lost: the event is counted once, a load
  // that was issued gets a second bounded wait so that the CTA does not leave with a copy into its shared memory in
  // flight, and the tile's codes and scales are written as NaN (the compact form also sets status bit 4), so a
  // lost tile cannot pass for a quantized one
  if (!__syncthreads_and(mbar_try_wait_rounds(&bar, 0u, prm.wait_rounds))) {
    if (tid == 0) {
      note_wait_timeout(prm.status_word);
      if (!prm.skip_load) mbar_try_wait_rounds(&bar, 0u, prm.wait_rounds);
    }
    __syncthreads();
    lose_tile<COLS, BS>(out, at, outer, len, inner, nb);
    return;
  }

  // (1) block scales: one thread per block of the tile (TC of them)
  bool bad = false;
  if (tid >= TC) {
  } else if (COLS) {
    const int64_t col = ct * TC + tid;
    uint32_t mbits = 0u;                                    // max |v| as bits: a NaN pattern tops every number
#pragma unroll 8
    for (int r = 0; r < TRB; r++) mbits = max(mbits, f2u(T[r * TC + tid]) & 0x7fffffffu);
    const bool nan = mbits > 0x7f800000u;
    const float x = block_scale<FAM, E, M>(nan ? qnan_f() : u2f(mbits), prm);
    const float r = reciprocal_of<FAM>(x, nan);
    s_x[tid] = x;
    s_r[tid] = r;
    bad = col < inner && (mbits >= 0x7f800000u || r == 0.0f);       // padding columns do not vote
    if (col < inner) out.scale((at.o * nb + at.b) * inner + col, x);
  } else {
    constexpr int QB = BS / 4;                              // float4 per block
    auto one = [&](int bi) {                                // block bi of the tile: row bi / BPR, block bi % BPR
      const int row = bi / BPR, blk = bi % BPR;
      const float4* src = reinterpret_cast<const float4*>(T + row * TC + blk * BS);
      uint32_t mbits = 0u;                                  // max |v| as bits: a NaN pattern tops every number
#pragma unroll
      for (int i = 0; i < QB; i++) {
        const float4 v = src[(i + bi) & (QB - 1)];           // rotated: a quarter-warp spreads over the banks
        mbits = max(max(mbits, f2u(v.x) & 0x7fffffffu), max(f2u(v.y) & 0x7fffffffu, f2u(v.z) & 0x7fffffffu));
        mbits = max(mbits, f2u(v.w) & 0x7fffffffu);
      }
      const bool nan = mbits > 0x7f800000u;
      const float x = block_scale<FAM, E, M>(nan ? qnan_f() : u2f(mbits), prm);
      const float r = reciprocal_of<FAM>(x, nan);
      s_x[bi] = x;
      s_r[bi] = r;
      const int64_t grow = rest * TR + row, gblk = ct * BPR + blk;
      bad |= grow < outer && gblk < nb && (mbits >= 0x7f800000u || r == 0.0f);  // padding blocks do not vote
      if (grow < outer && gblk < nb) out.scale(grow * nb + gblk, x);
    };
    if constexpr (NBT == NT) {                              // blocks of 32: one per thread
      one(tid);
    } else {
      for (int bi = tid; bi < NBT; bi += NT) one(bi);
    }
  }
  // the whole tile takes the short element step (with a via pre-rounding in q_ieee_small's range)
  const bool via = FAM == MXQ_FAMILY_MXGEMMINI && prm.via_e != 0;
  const bool clean = !__syncthreads_or(bad) && (!via || (prm.via_e <= 7 && prm.via_m <= 21));

  if (clean) {
    if constexpr (FAM == MXQ_FAMILY_MXGEMMINI) {
      if (via) {
        if (prm.rounding == 0)
          pass_clean<FAM, E, M, COLS, BS, 0, true>(T, s_r, out, at, outer, len, inner, prm.via_e, prm.via_m);
        else if (prm.rounding == 1)
          pass_clean<FAM, E, M, COLS, BS, 1, true>(T, s_r, out, at, outer, len, inner, prm.via_e, prm.via_m);
        else
          pass_clean<FAM, E, M, COLS, BS, 2, true>(T, s_r, out, at, outer, len, inner, prm.via_e, prm.via_m);
        out.finish();
        return;
      }
    }
    if (FAM == MXQ_FAMILY_MXQUANT || prm.rounding == 0)
      pass_clean<FAM, E, M, COLS, BS, 0, false>(T, s_r, out, at, outer, len, inner, 0, 0);
    else if (prm.rounding == 1)
      pass_clean<FAM, E, M, COLS, BS, 1, false>(T, s_r, out, at, outer, len, inner, 0, 0);
    else
      pass_clean<FAM, E, M, COLS, BS, 2, false>(T, s_r, out, at, outer, len, inner, 0, 0);
    out.finish();
    return;
  }

  // (2) elements: float4 q = tid + NT i of the tile (row q / C4, float4 column q % C4)
  const int c4 = tid % C4;
  float4 xs, rs;
  if (COLS) {
    xs = *reinterpret_cast<const float4*>(s_x + c4 * 4);
    rs = *reinterpret_cast<const float4*>(s_r + c4 * 4);
  }
#pragma unroll 2
  for (int i = 0; i < TRB / RPI; i++) {
    const int row = tid / C4 + RPI * i;
    float4 v = reinterpret_cast<const float4*>(T + row * TC)[c4];
    if (!COLS) {
      const int b = row * BPR + (int)((unsigned)c4 / (BS / 4));
      const float x = s_x[b], r = s_r[b];
      xs = make_float4(x, x, x, x);
      rs = make_float4(r, r, r, r);
    }
    v.x = element<FAM, E, M>(divide<FAM>(v.x, xs.x, rs.x), prm);
    v.y = element<FAM, E, M>(divide<FAM>(v.y, xs.y, rs.y), prm);
    v.z = element<FAM, E, M>(divide<FAM>(v.z, xs.z, rs.z), prm);
    v.w = element<FAM, E, M>(divide<FAM>(v.w, xs.w, rs.w), prm);
    if (COLS) {
      const int64_t l = at.b * BS + row, col = ct * TC + c4 * 4;
      if (l < len && col < inner) put_codes<false>(out, l, col, (at.o * len + l) * inner + col, v);
    } else {
      const int64_t grow = rest * TR + row, col = ct * TC + c4 * 4;
      if (grow < outer && col < len) out.codes(grow * len + col, v);
    }
  }
  out.finish();
}

// One CTA per tile: the hardware's block scheduler streams the tiles, so every SM keeps several tiles' loads in
// flight (one 32 KB TMA load per resident CTA) while other CTAs quantize and store, and the last tiles of a launch
// spread over the SMs a CTA at a time. Launched as a programmatic dependent (PDL) of the kernel before it.
template <int FAM, int E, int M, int BS, class Out>
int launch(const CUtensorMap& map, bool cols, Out out, int64_t outer, int64_t len, int64_t inner,
           const TParams& prm, cudaStream_t st) {
  if (cols && BS > TR) return MXQ_ERR_UNSUPPORTED;         // a COLS tile is one block of at most TR rows
  const int64_t nb = (len + BS - 1) / BS;                  // COLS: blocks of BS rows, one per tile row band
  const int64_t ntiles = cols ? outer * nb * ((inner + TC - 1) / TC) : ((outer + TR - 1) / TR) * ((len + TC - 1) / TC);
  if (ntiles >= (1ll << 31)) return MXQ_ERR_UNSUPPORTED;   // one CTA per tile; 32-bit tile coordinates
  void (*kern)(const CUtensorMap, Out, int64_t, int64_t, int64_t, TParams) = k_quant_tma<FAM, E, M, false, BS, Out>;
  if constexpr (BS <= TR) {                                // only blocks that fit a COLS tile instantiate one
    if (cols) kern = k_quant_tma<FAM, E, M, true, BS, Out>;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ntiles);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = (size_t)(cols ? BS : TR) * TC * sizeof(float);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;     // may start while the previous kernel drains
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (int r = check_cuda(cudaLaunchKernelEx(&cfg, kern, map, out, outer, len, inner, prm), "block_quantize"))
    return r;
  return MXQ_LAUNCH_CHECK("block_quantize");
}

// the float32 outputs (packed == nullptr) or the compact ones, or (multi != nullptr) float32 outputs to several
// destinations
struct Dest {
  float* P;
  float* X;
  uint8_t* Pc;
  uint8_t* Xc;
  int* status;
  const OutMulti* multi = nullptr;
  bool codes8 = false;     // Pc: byte codes, X: float32 scales (block.lut's codes)
};

// block: 32 for every layout and output; 16 or 64 for ROWS with float outputs (the launcher checks)
template <int FAM, int E, int M>
int launch_dest(const CUtensorMap& map, bool cols, const Dest& d, int64_t outer, int64_t len, int64_t inner,
                int64_t block, const TParams& prm, cudaStream_t st) {
  if (d.multi != nullptr) return launch<FAM, E, M, 32>(map, cols, *d.multi, outer, len, inner, prm, st);
  if (d.codes8) {
    if constexpr (FAM == MXQ_FAMILY_MXGEMMINI && E + M >= 5)
      return cols && outer == 1 ? launch<FAM, E, M, 32>(map, cols, OutCodes<E, M>{d.Pc, d.X, d.status, len}, outer, len,
                                                        inner, prm, st)
                                : MXQ_ERR_UNSUPPORTED;
    else
      return MXQ_ERR_UNSUPPORTED;
  }
  if (d.Pc == nullptr) {
    const OutF o{d.P, d.X};
    if (block == 16) return launch<FAM, E, M, 16>(map, cols, o, outer, len, inner, prm, st);
    if (block == 64) return launch<FAM, E, M, 64>(map, cols, o, outer, len, inner, prm, st);
    return launch<FAM, E, M, 32>(map, cols, o, outer, len, inner, prm, st);
  }
  if (FAM == MXQ_FAMILY_MXQUANT) return MXQ_ERR_UNSUPPORTED;          // the qtorch grid is not the OCP one
  return launch<FAM, E, M, 32>(map, cols, OutPack<E, M>{d.Pc, d.Xc, d.status}, outer, len, inner, prm, st);
}

template <int FAM>
int launch_fmt(int e, int m, const CUtensorMap& map, bool cols, const Dest& d, int64_t outer, int64_t len,
               int64_t inner, int64_t block, const TParams& prm, cudaStream_t st) {
  if (e == 4 && m == 3) return launch_dest<FAM, 4, 3>(map, cols, d, outer, len, inner, block, prm, st);
  if (e == 5 && m == 2) return launch_dest<FAM, 5, 2>(map, cols, d, outer, len, inner, block, prm, st);
  if (e == 3 && m == 2) return launch_dest<FAM, 3, 2>(map, cols, d, outer, len, inner, block, prm, st);
  if (e == 2 && m == 3) return launch_dest<FAM, 2, 3>(map, cols, d, outer, len, inner, block, prm, st);
  if (e == 2 && m == 1) return launch_dest<FAM, 2, 1>(map, cols, d, outer, len, inner, block, prm, st);
  return MXQ_ERR_UNSUPPORTED;
}

}  // namespace

namespace mxq {

// The TMA kernel for blocks of 32 (with float outputs also 16, and 64 along rows) when the layout allows a tensor map (16-byte aligned base, rows a multiple of 16
// bytes, extents below 2^31); MXQ_ERR_UNSUPPORTED otherwise (the caller then takes the register kernels).
int quantize_tma_dest(const float* V, const Dest& d, int64_t outer, int64_t len, int64_t inner, int64_t block,
                      const mxq_quant_spec& s, cudaStream_t st, int test_skip_load = 0,
                      unsigned wait_rounds = kWaitLimit) {
  const bool cols = inner > 1;
  // blocks of 32 in every layout; with float outputs also blocks of 16 (tiles of 16 rows across rows) and of 64
  // along rows (ROWS tiles hold any block dividing 256)
  const bool other = d.Pc == nullptr && (block == 16 || (block == 64 && !cols));
  if ((block != 32 && !other) || s.family == MXQ_FAMILY_FP32) return MXQ_ERR_UNSUPPORTED;
  const int64_t rowlen = cols ? inner : len;
  uintptr_t out_base = d.Pc ? (uintptr_t)d.Pc : (uintptr_t)d.P;
  if (d.codes8 && (block != 32 || (uintptr_t)d.X % 4)) return MXQ_ERR_UNSUPPORTED;
  if (d.multi != nullptr) {
    if (block != 32) return MXQ_ERR_UNSUPPORTED;
    out_base = 0;
    for (int i = 0; i < d.multi->n; i++) out_base |= (uintptr_t)d.multi->P[i];   // every destination 16-byte aligned
  }
  if ((uintptr_t)V % 16 || out_base % 16 || rowlen % 4 || outer >= (1ll << 31) || len >= (1ll << 31) ||
      inner >= (1ll << 31))
    return MXQ_ERR_UNSUPPORTED;
  CUtensorMap map;
  if (cols) {
    const uint64_t dims[3] = {(uint64_t)inner, (uint64_t)len, (uint64_t)outer};
    const uint64_t strides[2] = {(uint64_t)inner * 4, (uint64_t)(len * inner) * 4};
    const uint32_t box[3] = {TC, (uint32_t)block, 1};
    if (encode_tmap_f32(&map, V, 3, dims, strides, box) != MXQ_OK) return MXQ_ERR_UNSUPPORTED;
  } else {
    const uint64_t dims[2] = {(uint64_t)len, (uint64_t)outer};
    const uint64_t strides[1] = {(uint64_t)len * 4};
    const uint32_t box[2] = {TC, TR};
    if (encode_tmap_f32(&map, V, 2, dims, strides, box) != MXQ_OK) return MXQ_ERR_UNSUPPORTED;
  }
  unsigned* word = wait_status_word();
  if (word == nullptr) return MXQ_ERR_CUDA;                 // the reason is recorded
  TParams prm{s.rounding, s.placement, s.via_e, s.via_m, s.scale_floor, s.scale_emax, word, wait_rounds,
              test_skip_load};
  switch (s.family) {
    case MXQ_FAMILY_MXQUANT: return launch_fmt<MXQ_FAMILY_MXQUANT>(s.e, s.m, map, cols, d, outer, len, inner, block, prm, st);
    case MXQ_FAMILY_MXGEMMINI:
      return launch_fmt<MXQ_FAMILY_MXGEMMINI>(s.e, s.m, map, cols, d, outer, len, inner, block, prm, st);
    default: return launch_fmt<MXQ_FAMILY_OCP>(s.e, s.m, map, cols, d, outer, len, inner, block, prm, st);
  }
}

int quantize_tma(const float* V, float* P, float* X, int64_t outer, int64_t len, int64_t inner, int64_t block,
                 const mxq_quant_spec& s, cudaStream_t st) {
  return quantize_tma_dest(V, Dest{P, X, nullptr, nullptr, nullptr}, outer, len, inner, block, s, st);
}

int quantize_tma_packed(const float* V, uint8_t* Pc, uint8_t* Xc, int* status, int64_t outer, int64_t len,
                        int64_t inner, int64_t block, const mxq_quant_spec& s, cudaStream_t st) {
  return quantize_tma_dest(V, Dest{nullptr, nullptr, Pc, Xc, status}, outer, len, inner, block, s, st);
}

}  // namespace mxq

namespace mxq {
// block.lut's codes: block.mxgemmini (no via) of V (blocks along rows: outer 1, len rows, inner columns) as byte
// codes stored by 32-column panels (OutCodes) and float32 scales; status bit 1 for a code the format cannot hold.
// MXQ_ERR_UNSUPPORTED for layouts the TMA kernel does not take.
int quantize_tma_codes(const float* V, uint8_t* codes, float* X, int* status, int64_t outer, int64_t len,
                       int64_t inner, const mxq_quant_spec& s, cudaStream_t st) {
  if (s.family != MXQ_FAMILY_MXGEMMINI || s.via_e != 0) return MXQ_ERR_UNSUPPORTED;
  Dest d{nullptr, X, codes, nullptr, status};
  d.codes8 = true;
  return quantize_tma_dest(V, d, outer, len, inner, 32, s, st);
}
}  // namespace mxq

extern "C" int mxq_block_quantize_multi(const float* V, float* const* P, float* const* X, int32_t ndst,
                                        int64_t outer, int64_t len, int64_t inner, int64_t block,
                                        const mxq_quant_spec* spec, void* stream) {
  MXQ_REQUIRE(spec != nullptr && P != nullptr && X != nullptr, MXQ_ERR_VALUE, "block_quantize_multi: null argument");
  MXQ_REQUIRE(ndst >= 1 && ndst <= kMaxDst, MXQ_ERR_VALUE, "block_quantize_multi: %d destinations (1..%d)", ndst,
              kMaxDst);
  MXQ_REQUIRE(outer >= 0 && len >= 0 && inner >= 0, MXQ_ERR_VALUE, "block_quantize_multi: bad layout");
  MXQ_REQUIRE(spec->family != MXQ_FAMILY_FP32, MXQ_ERR_VALUE, "block_quantize_multi: format FP32 has no kernel");
  if (outer * len * inner == 0) return MXQ_OK;
  OutMulti o{};
  o.n = ndst;
  for (int i = 0; i < ndst; i++) {
    MXQ_REQUIRE(P[i] != nullptr && X[i] != nullptr, MXQ_ERR_VALUE, "block_quantize_multi: destination %d is null", i);
    o.P[i] = P[i];
    o.X[i] = X[i];
  }
  Dest d{nullptr, nullptr, nullptr, nullptr, nullptr, &o};
  const int r = mxq::quantize_tma_dest(V, d, outer, len, inner, block, *spec, mxq::as_stream(stream));
  MXQ_REQUIRE(r != MXQ_ERR_UNSUPPORTED, MXQ_ERR_UNSUPPORTED,
              "block_quantize_multi: blocks of 32, rows (the innermost extent) a multiple of 4, 16-byte aligned buffers");
  return r;
}

// Test-only: block.mxgemmini MXFP8_E4M3 along the rows of a rows x cols V through the TMA kernel with its loads never
// issued and waits of `wait_rounds` rounds, so every tile's wait runs out (nothing is in flight when the CTAs
// leave). The tiles come out as NaN and the wait-status word and the device counter rise by one per tile.
extern "C" int mxq_testing_wait_timeout(const float* V, float* P, float* X, int64_t rows, int64_t cols,
                                        uint32_t wait_rounds, void* stream) {
  MXQ_REQUIRE(rows > 0 && cols > 0 && cols % 32 == 0, MXQ_ERR_VALUE, "testing_wait_timeout: bad sizes");
  MXQ_REQUIRE(wait_rounds >= 1 && wait_rounds <= (1u << 16), MXQ_ERR_VALUE, "testing_wait_timeout: wait_rounds");
  mxq_quant_spec s{};
  s.family = MXQ_FAMILY_MXGEMMINI;
  s.e = 4;
  s.m = 3;
  s.rounding = MXQ_RM_TIES_AWAY;
  s.scale_floor = 1e-38f;
  const int r = mxq::quantize_tma_dest(V, Dest{P, X, nullptr, nullptr, nullptr}, rows, cols, 1, 32, s,
                                       mxq::as_stream(stream), 1, wait_rounds);
  MXQ_REQUIRE(r != MXQ_ERR_UNSUPPORTED, MXQ_ERR_VALUE, "testing_wait_timeout: the layout has no TMA path");
  return r;
}

// Number of bounded shared-memory waits that gave up in the staged kernels since the library was loaded on the
// current device (0 in every correct run); synchronous.
extern "C" int mxq_device_timeouts(uint32_t* out) {
  if (!out) return mxq::set_error(MXQ_ERR_VALUE, "device_timeouts: null output");
  *out = mxq::read_wait_timeouts();
  return MXQ_OK;
}
