// kernels.cuh -- the sm_100a kernels of libenvgemm:
//
//   k1_gemm      large-M GEMM: persistent, warp-specialised (TMA warp / UMMA warp / 4 epilogue
//                warps), 128 x BN x 64 tiles in a STAGES-deep shared-memory ring, fp32
//                accumulators double-buffered in TMEM so the epilogue of tile i overlaps the
//                main loop of tile i+1.  The B operand is either a plain K-major matrix (2D TMA)
//                or, for convolutions, an implicit im2col tile fetched straight from an NHWC
//                activation with a 4D TMA box (no col buffer is ever written).
//   k2_skinny    M <= 64: swap-AB (D^T = W . X^T, W rows on the 128-lane M side of the MMA,
//                tokens on N), split-K across CTAs with a deterministic last-CTA reduction.
//   k_cast_rows  fp32 -> bf16 (round-to-nearest-even) row copy with zero K padding.
//   k_transpose_cast  fp32 [R][C] -> bf16 [C][Rp]: NCHW -> NHWC for convolutions, and the
//                transposed operands of envg_sgemm.
//   k_im2col_nhwc  explicit bf16 im2col, only for strided convolutions.
//
// Arithmetic of every GEMM: bf16 x bf16 products accumulated in fp32 by tcgen05.mma; the
// epilogue applies bias / SiLU / SiLU-gate / gated residual in fp32.  Envision's CPU path
// (src/quicknncpu.pas:1241-1337) accumulates fp32 x fp32 in fp32; the tests bound the
// difference.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

#include "ptx.cuh"

namespace envg {

constexpr int BM = 128;                       // rows of a UMMA tile (TMEM lanes)
constexpr int BK = 64;                        // bf16 per 128-byte swizzled row
constexpr int TILE_A_BYTES = BM * BK * 2;     // 16 KB
constexpr int K1_THREADS = 192;               // warp 0 TMA, warp 1 UMMA, warps 2-5 epilogue

enum EpiMode : int { EPI_PLAIN = 0, EPI_SILU_GATE = 1, EPI_GATED_RES = 2, EPI_ALPHA_BETA = 3 };

struct EpiArgs {
  float* Y;           // output base
  int64_t ldy;        // row stride of Y (floats)
  const float* bias;  // fp32 or null
  int bias_mode;      // 0 none, 1 per output column, 2 per output row
  int act;            // 1: SiLU after the bias
  int mode;           // EpiMode
  const float* gate;  // EPI_GATED_RES: per-column gate (convolutions: no gate, Y += conv + bias)
  float alpha, beta;  // EPI_ALPHA_BETA: Y = alpha*acc + beta*Y
  int n_out;          // valid output columns
  int m_valid;        // valid output rows
  int half_n;         // EPI_SILU_GATE: gate rows of the original W (up bias at half_n + col)
  int vec_ok;         // Y 16-byte aligned and ldy % 4 == 0
  int store_mode;     // k1_gemm: STORE_DIRECT, STORE_TMA or STORE_TMA_ADD
  // N-split output (envg_linear_nsplit): every value goes to the same offset of each rank's copy
  // of Y.  nremote = 0: Y only; > 0: P2P stores to remote[0 .. nremote); -1: one multimem store
  // through the multicast address remote[0].  Column indices are shard-relative; col_off places
  // them in the full Y (row stride ldy).  Reads of Y (residual) use the local copy Y.
  float* remote[8];
  int nremote;
  int col_off;
  // Optional bf16 copy of the finished output (row stride ldyb elements, ldyb % 8 == 0): the
  // activation operand of a following linear that reads this Y, written here instead of by a
  // separate cast (row-major linears on the TMA / coalesced store paths, the split reduces and
  // the skinny k2_set path).
  __nv_bfloat16* yb;
  int64_t ldyb;
};

// Write one value / four consecutive values (16-byte aligned) at element offset idx of Y, on
// every copy the epilogue targets.
ENVG_DEV void out_store1(const EpiArgs& e, int64_t idx, float v) {
  if (e.nremote == 0) {
    e.Y[idx] = v;
  } else if (e.nremote < 0) {
    multimem_st_f32(e.remote[0] + idx, v);
  } else {
    for (int r = 0; r < e.nremote; ++r) e.remote[r][idx] = v;
  }
}
ENVG_DEV void out_store4(const EpiArgs& e, int64_t idx, float4 v) {
  if (e.nremote == 0) {
    *reinterpret_cast<float4*>(e.Y + idx) = v;
  } else if (e.nremote < 0) {
    multimem_st_v4(e.remote[0] + idx, v);
  } else {
    for (int r = 0; r < e.nremote; ++r) *reinterpret_cast<float4*>(e.remote[r] + idx) = v;
  }
}

// How k1_gemm writes Y: per-thread global stores (one row per thread); 32x32 tiles staged in
// shared memory and written by a TMA bulk store (clipped at the tensor edges) or added into Y by a
// TMA bulk reduce (Y += tile); or (STORE_COALESCED, the default) the staged tile read back
// transposed so that every warp store writes whole 128-byte rows, keeping the output off the
// SM's TMA unit, which the operand loads keep busy.
enum StoreMode : int {
  STORE_DIRECT = 0,
  STORE_TMA = 1,
  STORE_TMA_ADD = 2,
  STORE_COALESCED = 3,
  STORE_TMA_PEERS = 4,      // N-split: one TMA bulk store per rank's copy of Y (GemmArgs::pm)
  STORE_TMA_ADD_PEERS = 5,  // the same with bulk reduce-add (gated residual)
};

// Tensor maps over each rank's copy of Y for STORE_TMA_PEERS, each based at this rank's column
// shard (so the shard edge clips the tile like the local map does).
struct PeerMaps {
  CUtensorMap m[8];
};

struct ConvGeom {
  int tileW, tileH;   // pixel tile, tileW * tileH == BN
  int outH, outW;
  int tiles_w, tiles_h;
  int KW, pad, cblocks;
  int64_t img_stride; // floats between images of Y
  int64_t plane;      // outH * outW
};

struct GemmArgs {
  int num_kb;
  int tiles_m, tiles_n, num_tiles;
  int group_m;
  EpiArgs epi;
  ConvGeom conv;
  int* status;
  uint64_t wait_cap_ns;
  PeerMaps pm;  // STORE_TMA_PEERS only
  // Split-K (k1_gemm_pair, splits > 1): num_tiles counts units (split, tile), split-major, with
  // tiles_per_split tiles in each split; split s covers K blocks [s * kb_per_split, ...) and
  // stores its raw fp32 tile at row offset s * split_rows of the partial buffer the Y map covers.
  int splits, kb_per_split, tiles_per_split, split_rows;
  // k1_gemm_pair, STORE_TMA / STORE_TMA_ADD: the same output as the Y map with 32-column x
  // 128-row boxes, one box per chunk for the CTA's 128 rows (ybig_ok = 1 when built).
  CUtensorMap ybig;
  int ybig_ok;
};

// Unit -> (split, tile, K-block range) of a k1_gemm_pair launch; without split-K the unit is
// the tile and the range is all of K.
template <typename Args>
ENVG_DEV void unit_split(int unit, const Args& a, int& tile, int& split, int& kb0, int& kb1) {
  if (a.splits > 1) {
    split = unit / a.tiles_per_split;
    tile = unit - split * a.tiles_per_split;
    kb0 = split * a.kb_per_split;
    kb1 = min(kb0 + a.kb_per_split, a.num_kb);
  } else {
    split = 0;
    tile = unit;
    kb0 = 0;
    kb1 = a.num_kb;
  }
}

constexpr int PSET_MAX = 4;

// One linear of a k1_gemm_pair launch (fields as in GemmArgs).
struct PairLin {
  int num_kb, tiles_m, tiles_n, group_m;
  int splits, kb_per_split, tiles_per_split, split_rows;
  int ybig_ok;
  EpiArgs epi;
};

// A k1_gemm_pair launch: up to PSET_MAX linears that share the A operand (one activation
// matrix), walked as one persistent sequence of units; units [base[i], base[i + 1]) belong to
// linear i.  A convolution is a set of one, with A = its weights and B = the NHWC activations.
struct PairSet {
  CUtensorMap tmB[PSET_MAX];   // B operand of each linear
  CUtensorMap tmY[PSET_MAX];   // output, 32 x 32 boxes (TMA store modes)
  CUtensorMap ybig[PSET_MAX];  // output, 32 x 128 boxes (last-unit stores, PairLin::ybig_ok)
  PairLin lin[PSET_MAX];
  int n, total;
  int base[PSET_MAX + 1];
  ConvGeom conv;
  int* status;
  uint64_t wait_cap_ns;
  int l2_hints;  // activation loads evict_last, local output stores evict_first
  // Dynamic unit order (NULL: static, pair p takes units p, p + pairs, ...): [0] the next unit
  // to hand out, [1] pairs done.  Both are zero at launch; the last pair to finish zeroes them.
  int* sched;
  PeerMaps pm;  // STORE_TMA_PEERS (a set of one)
};

// Linear of a set that owns `unit`.
ENVG_DEV int set_linear(const PairSet& set, int unit) {
  int li = 0;
  while (li + 1 < set.n && unit >= set.base[li + 1]) ++li;
  return li;
}

struct SkinnyArgs {
  int n_tiles, splits, kb_per_split, num_kb;
  EpiArgs epi;
  float* partial;
  int* counters;
  int* status;
  uint64_t wait_cap_ns;
};

ENVG_DEV float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// One output element of a GEMM-shaped epilogue.  GATED_RES restates QNNGatedAdd
// (quicknncpu.pas:853-859): y + (gate * proj), product and sum rounded separately.
ENVG_DEV float epi_value(const EpiArgs& e, float acc, int row, int col, const float* yp) {
  float v = acc;
  if (e.bias_mode == 1) v = __fadd_rn(v, __ldg(e.bias + col));
  else if (e.bias_mode == 2) v = __fadd_rn(v, __ldg(e.bias + row));
  if (e.act) v = silu_f(v);
  if (e.mode == EPI_GATED_RES) {
    v = __fadd_rn(*yp, __fmul_rn(__ldg(e.gate + col), v));
  } else if (e.mode == EPI_ALPHA_BETA) {
    v = (e.beta == 0.0f) ? __fmul_rn(e.alpha, v) : __fadd_rn(__fmul_rn(e.alpha, v), __fmul_rn(e.beta, *yp));
  }
  return v;
}

// Value handed to a TMA store / reduce: everything but the read of Y.
ENVG_DEV float epi_pre(const EpiArgs& e, float acc, int row, int col) {
  float v = acc;
  const bool cok = col < e.n_out, rok = row < e.m_valid;
  if (e.bias_mode == 1) v = __fadd_rn(v, cok ? __ldg(e.bias + col) : 0.0f);
  else if (e.bias_mode == 2) v = __fadd_rn(v, rok ? __ldg(e.bias + row) : 0.0f);
  if (e.act) v = silu_f(v);
  if (e.mode == EPI_GATED_RES) v = __fmul_rn(cok ? __ldg(e.gate + col) : 0.0f, v);
  else if (e.mode == EPI_ALPHA_BETA) v = __fmul_rn(e.alpha, v);
  return v;
}

// Per-column vector (bias or gate) for the 32 columns [col0, col0+32): eight 16-byte loads when
// the chunk is whole and aligned, guarded scalar loads at the ragged edge.
ENVG_DEV void load_col32(const float* p, int col0, int n_out, float (&c)[32]) {
  if (col0 + 32 <= n_out && (reinterpret_cast<uintptr_t>(p + col0) & 15) == 0) {
    const float4* p4 = reinterpret_cast<const float4*>(p + col0);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 t = __ldg(p4 + q);
      c[4 * q] = t.x;
      c[4 * q + 1] = t.y;
      c[4 * q + 2] = t.z;
      c[4 * q + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) c[j] = (col0 + j < n_out) ? __ldg(p + col0 + j) : 0.0f;
  }
}

// epi_pre for a whole 32-column chunk of one row, with the mode tests taken once per chunk.
// `e` is the kernel's EpiArgs, read in place from its grid-constant parameters.
ENVG_DEV void epi_pre_chunk(const EpiArgs& e, float (&v)[32], int row, int col0) {
  if (e.bias_mode == 1) {
    float b[32];
    load_col32(e.bias, col0, e.n_out, b);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], b[j]);
  } else if (e.bias_mode == 2) {
    const float bv = row < e.m_valid ? __ldg(e.bias + row) : 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], bv);
  }
  if (e.act) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = silu_f(v[j]);
  }
  if (e.mode == EPI_GATED_RES) {
    float g[32];
    load_col32(e.gate, col0, e.n_out, g);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(g[j], v[j]);
  } else if (e.mode == EPI_ALPHA_BETA) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(e.alpha, v[j]);
  }
}

// SiLU-gate of a 32-column chunk: v = silu(g + bias_g) * (u + bias_u).
ENVG_DEV void silu_gate_chunk(const EpiArgs& e, const uint32_t (&g)[32], const uint32_t (&u)[32], int col0,
                              float (&v)[32]) {
  if (e.bias_mode == 1) {
    float bg[32], bu[32];
    load_col32(e.bias, col0, e.n_out, bg);
    load_col32(e.bias + e.half_n, col0, e.n_out, bu);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      v[j] = __fmul_rn(silu_f(__fadd_rn(__uint_as_float(g[j]), bg[j])), __fadd_rn(__uint_as_float(u[j]), bu[j]));
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(silu_f(__uint_as_float(g[j])), __uint_as_float(u[j]));
  }
}

// Write row `lane` of a 32 x 32 fp32 tile into a 128-byte-swizzled staging buffer (16-byte chunk
// j of row r lands at chunk j ^ (r % 8), the layout the TMA store reads).
ENVG_DEV void stage_row32(uint8_t* buf, int lane, const float (&v)[32]) {
  float4* rowp = reinterpret_cast<float4*>(buf + lane * 128);
#pragma unroll
  for (int j = 0; j < 8; ++j) rowp[j ^ (lane & 7)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

// Write a staged 32 x 32 tile (rows row0.., columns col0..) of a row-major Y with coalesced
// stores: lane l moves 16-byte chunk (l % 8) of rows (l / 8) + 4i, so each store instruction
// covers four full 128-byte rows.  `v` already holds everything but the read of Y
// (epi_pre); GATED_RES adds the old Y, ALPHA_BETA adds beta * old Y.
ENVG_DEV void store_tile32_rows(const EpiArgs& e, const uint8_t* buf, int lane, int row0, int col0) {
  const int ch = lane & 7;
  const bool rmw = e.mode == EPI_GATED_RES || (e.mode == EPI_ALPHA_BETA && e.beta != 0.0f);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = (lane >> 3) + 4 * i;
    const int grow = row0 + r;
    if (grow >= e.m_valid) continue;
    const float4 t = *reinterpret_cast<const float4*>(buf + r * 128 + ((ch ^ (r & 7)) * 16));
    const int gcol = col0 + ch * 4;
    const int64_t idx = (int64_t)grow * e.ldy + e.col_off + gcol;
    const float* yp = e.Y + idx;
    float tv[4] = {t.x, t.y, t.z, t.w};
    if (e.vec_ok && gcol + 3 < e.n_out) {
      if (rmw) {
        const float4 o = *reinterpret_cast<const float4*>(yp);
        const float ov[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tv[j] = (e.mode == EPI_GATED_RES) ? __fadd_rn(ov[j], tv[j]) : __fadd_rn(tv[j], __fmul_rn(e.beta, ov[j]));
      }
      out_store4(e, idx, make_float4(tv[0], tv[1], tv[2], tv[3]));
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (gcol + j >= e.n_out) break;
        float v = tv[j];
        if (rmw) v = (e.mode == EPI_GATED_RES) ? __fadd_rn(yp[j], v) : __fadd_rn(v, __fmul_rn(e.beta, yp[j]));
        out_store1(e, idx + j, v);
      }
    }
  }
}

// Coalesced store of a staged 32 x 32 conv tile: rows are output channels row0.., the 32
// columns are consecutive pixels starting at (h, w) of image b.
ENVG_DEV void store_tile32_conv(const EpiArgs& e, const ConvGeom& g, const uint8_t* buf, int lane, int row0, int b,
                                int h, int w) {
  if (h >= g.outH) return;
  const int ch = lane & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = (lane >> 3) + 4 * i;
    const int oc = row0 + r;
    if (oc >= e.m_valid) continue;
    const float4 t = *reinterpret_cast<const float4*>(buf + r * 128 + ((ch ^ (r & 7)) * 16));
    const int wc = w + ch * 4;
    float* yp = e.Y + (int64_t)b * g.img_stride + (int64_t)oc * g.plane + (int64_t)h * g.outW + wc;
    if (e.vec_ok && wc + 3 < g.outW) {
      float4 o = t;
      if (e.mode == EPI_GATED_RES) {
        const float4 old = *reinterpret_cast<const float4*>(yp);
        o = make_float4(__fadd_rn(old.x, t.x), __fadd_rn(old.y, t.y), __fadd_rn(old.z, t.z), __fadd_rn(old.w, t.w));
      }
      *reinterpret_cast<float4*>(yp) = o;
    } else {
      const float tv[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (wc + j < g.outW) yp[j] = (e.mode == EPI_GATED_RES) ? __fadd_rn(yp[j], tv[j]) : tv[j];
    }
  }
}

// bf16 (RNE) copy of the finished 32-column chunk [col0, col0+32) of row `row` into e.yb.
ENVG_DEV void store_bf16_row32(const EpiArgs& e, int row, int col0, const float (&v)[32]) {
  if (row >= e.m_valid) return;
  __nv_bfloat16* p = e.yb + (int64_t)row * e.ldyb + col0;
  if (col0 + 32 <= e.n_out) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      uint4 o;
      __nv_bfloat162 h0 = __float22bfloat162_rn(make_float2(v[j + 0], v[j + 1]));
      __nv_bfloat162 h1 = __float22bfloat162_rn(make_float2(v[j + 2], v[j + 3]));
      __nv_bfloat162 h2 = __float22bfloat162_rn(make_float2(v[j + 4], v[j + 5]));
      __nv_bfloat162 h3 = __float22bfloat162_rn(make_float2(v[j + 6], v[j + 7]));
      o.x = *reinterpret_cast<uint32_t*>(&h0);
      o.y = *reinterpret_cast<uint32_t*>(&h1);
      o.z = *reinterpret_cast<uint32_t*>(&h2);
      o.w = *reinterpret_cast<uint32_t*>(&h3);
      *reinterpret_cast<uint4*>(p + j) = o;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < e.n_out) p[j] = __float2bfloat16_rn(v[j]);
  }
}

// Store 32 consecutive output columns [col0, col0+32) of one row.
ENVG_DEV void epi_store_row32(const EpiArgs& e, int row, int col0, const float (&v)[32]) {
  if (row >= e.m_valid) return;
  float* yrow = e.Y + (int64_t)row * e.ldy;
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const int col = col0 + j;
    if (e.vec_ok && col + 3 < e.n_out) {
      float4 o;
      const float* yp = yrow + col;
      float4 old = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e.mode == EPI_GATED_RES || (e.mode == EPI_ALPHA_BETA && e.beta != 0.0f))
        old = *reinterpret_cast<const float4*>(yp);
      o.x = epi_value(e, v[j + 0], row, col + 0, &old.x);
      o.y = epi_value(e, v[j + 1], row, col + 1, &old.y);
      o.z = epi_value(e, v[j + 2], row, col + 2, &old.z);
      o.w = epi_value(e, v[j + 3], row, col + 3, &old.w);
      *reinterpret_cast<float4*>(yrow + col) = o;
    } else {
#pragma unroll
      for (int t = 0; t < 4; ++t)
        if (col + t < e.n_out) yrow[col + t] = epi_value(e, v[j + t], row, col + t, yrow + col + t);
    }
  }
}

// Store 32 accumulator columns of a convolution tile: column jj -> pixel (h0 + jj / tileW,
// w0 + jj % tileW) of image b; Y is NCHW, row = output channel.
ENVG_DEV void epi_store_conv32(const EpiArgs& e, const ConvGeom& g, int b, int oc, int h0, int w0, int jj0,
                               const float (&v)[32]) {
  if (oc >= e.m_valid) return;
  float* yplane = e.Y + (int64_t)b * g.img_stride + (int64_t)oc * g.plane;
  const float bv = (e.bias_mode == 2) ? __ldg(e.bias + oc) : 0.0f;
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const int jj = jj0 + j;
    const int h = h0 + jj / g.tileW;
    const int w = w0 + jj % g.tileW;
    if (h >= g.outH) continue;
    float o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      float x = __fadd_rn(v[j + t], bv);
      o[t] = e.act ? silu_f(x) : x;
    }
    float* yp = yplane + (int64_t)h * g.outW + w;
    if (e.vec_ok && (g.tileW % 4) == 0 && w + 3 < g.outW) {
      if (e.mode == EPI_GATED_RES) {
        const float4 old = *reinterpret_cast<const float4*>(yp);
        o[0] = __fadd_rn(old.x, o[0]);
        o[1] = __fadd_rn(old.y, o[1]);
        o[2] = __fadd_rn(old.z, o[2]);
        o[3] = __fadd_rn(old.w, o[3]);
      }
      *reinterpret_cast<float4*>(yp) = make_float4(o[0], o[1], o[2], o[3]);
    } else {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int jt = jj + t;
        const int ht = h0 + jt / g.tileW, wt = w0 + jt % g.tileW;
        if (ht < g.outH && wt < g.outW) {
          float* q = yplane + (int64_t)ht * g.outW + wt;
          *q = (e.mode == EPI_GATED_RES) ? __fadd_rn(*q, o[t]) : o[t];
        }
      }
    }
  }
}

// Tile order: groups of `group_m` M-tiles sweep all N-tiles, so CTAs that run together share
// A rows and B rows in L2.
template <typename Args>
ENVG_DEV void map_tile(int tile, const Args& a, int& m_blk, int& n_blk) {
  const int group = a.group_m * a.tiles_n;
  const int g = tile / group;
  const int first_m = g * a.group_m;
  const int gm = min(a.tiles_m - first_m, a.group_m);
  const int r = tile - g * group;
  m_blk = first_m + r % gm;
  n_blk = r / gm;
}

template <int BN, int STAGES>
struct K1Smem {
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = TILE_A_BYTES + B_BYTES;
  static constexpr int STAGING_BYTES = 4 * 2 * 32 * 128;  // 4 epilogue warps x 2 buffers x 32x32 fp32
  static constexpr int BAR_BYTES = (2 * STAGES + 5) * 8 + 16;
  static constexpr int TOTAL = 1024 /*alignment slack*/ + STAGES * STAGE_BYTES + STAGING_BYTES + BAR_BYTES;
  static constexpr uint32_t TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
};

// ------------------------------------------------------------------------------------------
// K1: persistent tcgen05 GEMM.  D[128 x BN] tiles of A[M, K] . B[N, K]^T.
// ------------------------------------------------------------------------------------------
template <int BN, int STAGES, bool CONV_B, bool SILU_GATE>
__global__ void __launch_bounds__(K1_THREADS, 1)
    k1_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmY, const __grid_constant__ GemmArgs args) {
  using L = K1Smem<BN, STAGES>;
  constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN);
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN");
  static_assert(!SILU_GATE || BN == 256, "SiLU-gate tiles hold 128 gate + 128 up columns");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * TILE_A_BYTES;
  uint8_t* sStage = sB + STAGES * L::B_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStage + L::STAGING_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + 8 * STAGES;
  const uint32_t tfull0 = empty0 + 8 * STAGES;
  const uint32_t tempty0 = tfull0 + 16;
  const uint32_t drain = tempty0 + 16;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, 4);
    }
    mbar_init(drain, 1);
    *abort_s = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (args.epi.store_mode == STORE_TMA || args.epi.store_mode == STORE_TMA_ADD) tma_prefetch_desc(&tmY);
    if (args.epi.store_mode >= STORE_TMA_PEERS)
      for (int r = 0; r < args.epi.nremote; ++r) tma_prefetch_desc(&args.pm.m[r]);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtl wc{args.wait_cap_ns, args.status, abort_s, 0};

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      uint32_t pending = 0;   // stages whose last load may still be in flight
      uint32_t issue_ph = 0;  // parity of that load's phase, per stage
      for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x) {
        int m_blk, n_blk;
        int b = 0, h0 = 0, w0 = 0;
        if (CONV_B) {
          m_blk = tile % args.tiles_m;  // output-channel blocks of one pixel tile run together
          n_blk = tile / args.tiles_m;
          const int per_img = args.conv.tiles_w * args.conv.tiles_h;
          b = n_blk / per_img;
          const int r = n_blk - b * per_img;
          h0 = (r / args.conv.tiles_w) * args.conv.tileH;
          w0 = (r % args.conv.tiles_w) * args.conv.tileW;
        } else {
          map_tile(tile, args, m_blk, n_blk);
        }
        const int m0 = m_blk * BM;
        const int n0 = n_blk * BN;
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!wait_bounded(empty0 + 8 * stage, ph ^ 1, wc, 1)) goto producer_done;
          const uint32_t fb = full0 + 8 * stage;
          mbar_arrive_expect_tx(fb, L::STAGE_BYTES);
          tma_load_2d(smem_u32(sA + stage * TILE_A_BYTES), &tmA, fb, kb * BK, m0);
          if (CONV_B) {
            const int kpos = kb / args.conv.cblocks;
            const int cb = kb - kpos * args.conv.cblocks;
            const int kh = kpos / args.conv.KW;
            const int kw = kpos - kh * args.conv.KW;
            tma_load_4d(smem_u32(sB + stage * L::B_BYTES), &tmB, fb, cb * BK, w0 + kw - args.conv.pad,
                        h0 + kh - args.conv.pad, b);
          } else {
            tma_load_2d(smem_u32(sB + stage * L::B_BYTES), &tmB, fb, kb * BK, n0);
          }
          pending |= 1u << stage;
          issue_ph = (issue_ph & ~(1u << stage)) | (ph << stage);
          if (++stage == STAGES) {
            stage = 0;
            ph ^= 1;
          }
        }
      }
    producer_done:
      if (*abort_s) {
        // Let every copy this thread started land before the CTA's shared memory is released.
        for (int s = 0; s < STAGES; ++s)
          if (pending & (1u << s)) wait_drain(full0 + 8 * s, (issue_ph >> s) & 1u, args.wait_cap_ns);
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x) {
        if (!wait_bounded(tempty0 + 8 * acc, aph ^ 1, wc, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!wait_bounded(full0 + 8 * stage, ph, wc, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_kmajor_desc(smem_u32(sA + stage * TILE_A_BYTES));
          const uint64_t bd = sw128_kmajor_desc(smem_u32(sB + stage * L::B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(d_tmem, ad + 2 * k, bd + 2 * k, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(empty0 + 8 * stage);
          if (++stage == STAGES) {
            stage = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(tfull0 + 8 * acc);
        acc ^= 1;
        if (acc == 0) aph ^= 1;
      }
      if (*abort_s) {
        // Every UMMA issued so far must finish before TMEM is released.
        umma_commit(drain);
        wait_drain(drain, 0, args.wait_cap_ns);
      }
    }
  } else {
    // ---------------- epilogue: 4 warps, one TMEM lane quadrant each ----------------
    const int q = warp & 3;
    const int smode = args.epi.store_mode;
    // A reference into the (grid-constant) parameter space: a local copy would be placed in local
    // memory, because the peer stores index ep.remote[] at run time.
    const EpiArgs& ep = args.epi;
    uint8_t* stg = sStage + (warp - 2) * 8192;  // this warp's two 4 KB staging tiles
    int sb = 0;
    int acc = 0;
    uint32_t aph = 0;
    for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x) {
      int m_blk, n_blk;
      int b = 0, h0 = 0, w0 = 0;
      if (CONV_B) {
        m_blk = tile % args.tiles_m;
        n_blk = tile / args.tiles_m;
        const int per_img = args.conv.tiles_w * args.conv.tiles_h;
        b = n_blk / per_img;
        const int r = n_blk - b * per_img;
        h0 = (r / args.conv.tiles_w) * args.conv.tileH;
        w0 = (r % args.conv.tiles_w) * args.conv.tileW;
      } else {
        map_tile(tile, args, m_blk, n_blk);
      }
      if (!wait_bounded_warp(tfull0 + 8 * acc, aph, wc, 4)) break;
      tc_fence_after();
      const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      const int row0 = m_blk * BM + q * 32;
      const int row = row0 + lane;
      constexpr int NCHUNK = SILU_GATE ? BN / 64 : BN / 32;
#pragma unroll 1
      for (int c = 0; c < NCHUNK; ++c) {
        float v[32];
        int col0;
        if (SILU_GATE) {
          uint32_t g[32], u[32];
          tmem_ld32(trow + c * 32, g);
          tmem_ld32(trow + BN / 2 + c * 32, u);
          col0 = n_blk * (BN / 2) + c * 32;
          silu_gate_chunk(ep, g, u, col0, v);
        } else {
          uint32_t r[32];
          tmem_ld32(trow + c * 32, r);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          col0 = n_blk * BN + c * 32;
        }
        if (smode == STORE_DIRECT) {
          if (SILU_GATE) {
            EpiArgs e2 = ep;
            e2.bias_mode = 0;
            e2.act = 0;
            epi_store_row32(e2, row, col0, v);
          } else if (CONV_B) {
            epi_store_conv32(ep, args.conv, b, row, h0, w0, c * 32, v);
          } else {
            epi_store_row32(ep, row, col0, v);
          }
          continue;
        }
        // ---- TMA store path ----
        int x = col0, y = row0;
        if (CONV_B) {
          const int jj = c * 32;
          const int w = w0 + jj % args.conv.tileW;
          const int h = h0 + jj / args.conv.tileW;
          if (w >= args.conv.outW) continue;  // tile overhang past the image row (uniform per warp)
          x = h * args.conv.outW + w;          // h >= outH lands past the plane and is clipped
          const float bv = (ep.bias_mode == 2 && row < ep.m_valid) ? __ldg(ep.bias + row) : 0.0f;
          if (ep.act) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = silu_f(__fadd_rn(v[j], bv));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], bv);
          }
        } else if (!SILU_GATE) {
          epi_pre_chunk(ep, v, row, col0);
        }
        if (!CONV_B && ep.yb) store_bf16_row32(ep, row, col0, v);
        uint8_t* buf = stg + sb * 4096;
        if (smode == STORE_COALESCED) {
          stage_row32(buf, lane, v);
          __syncwarp();
          if (CONV_B) {
            const int jj = c * 32;
            store_tile32_conv(ep, args.conv, buf, lane, row0, b, h0 + jj / args.conv.tileW,
                              w0 + jj % args.conv.tileW);
          } else {
            store_tile32_rows(ep, buf, lane, row0, col0);
          }
          sb ^= 1;  // the other buffer is written next, so no wait before this one is reused
          continue;
        }
        if (lane == 0) bulk_wait_read<1>();  // the store that last read this buffer is done with it
        __syncwarp();
        stage_row32(buf, lane, v);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (CONV_B) {
            if (smode == STORE_TMA_ADD) tma_reduce_add_3d(&tmY, smem_u32(buf), x, y, b);
            else tma_store_3d(&tmY, smem_u32(buf), x, y, b);
          }
          else if (smode == STORE_TMA_PEERS) {
            for (int r = 0; r < ep.nremote; ++r) tma_store_2d(&args.pm.m[r], smem_u32(buf), x, y);
          } else if (smode == STORE_TMA_ADD_PEERS) {
            for (int r = 0; r < ep.nremote; ++r) tma_reduce_add_2d(&args.pm.m[r], smem_u32(buf), x, y);
          }
          else if (smode == STORE_TMA_ADD) tma_reduce_add_2d(&tmY, smem_u32(buf), x, y);
          else tma_store_2d(&tmY, smem_u32(buf), x, y);
          bulk_commit();
        }
        sb ^= 1;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty0 + 8 * acc);
      acc ^= 1;
      if (acc == 0) aph ^= 1;
    }
    if (lane == 0) bulk_wait_all();
    if (ep.nremote != 0) __threadfence_system();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------
// K1 pair: the same GEMM on 256 x 256 tiles computed by a CTA pair (cluster of 2) with
// tcgen05.mma.cta_group::2.  Each CTA loads its own 128 rows of A and its own 128 rows of B
// (no multicast loads); the even CTA issues the UMMAs, which read both CTAs' shared memory and
// write each CTA's 128 accumulator rows into its own TMEM.  Per SM this halves the B bytes read
// from L2 and from shared memory relative to k1_gemm.
//   full[s]   (even CTA)  : its producer's expect_tx of both CTAs' bytes + both CTAs' TMA
//   empty[s]  (both)      : UMMA commit multicast to the pair
//   tfull[a]  (both)      : UMMA commit multicast after a tile's last k-block
//   tempty[a] (even CTA)  : 4 epilogue warps x 2 CTAs arrive
// ------------------------------------------------------------------------------------------
template <int STAGES>
struct KPairSmem {
  static constexpr int HALF_B_BYTES = 128 * BK * 2;
  static constexpr int STAGE_BYTES = TILE_A_BYTES + HALF_B_BYTES;  // this CTA's share of a stage
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;            // A stages, then B stages
  static constexpr int STAGING_BYTES = 4 * 2 * 32 * 128;
  static constexpr int UNIT_RING = 4;  // units handed out ahead (dynamic unit order)
  static constexpr int BAR_BYTES = (2 * STAGES + 6 + 2 * UNIT_RING) * 8 + 16 + 4 * UNIT_RING;
  static constexpr int TOTAL = 1024 + STAGES * STAGE_BYTES + STAGING_BYTES + BAR_BYTES;
  static constexpr uint32_t TMEM_COLS = 512;
};

template <int STAGES, bool CONV_B, bool SILU_GATE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(K1_THREADS, 1)
    k1_gemm_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ PairSet set) {
  using L = KPairSmem<STAGES>;
  constexpr int BN = 256;
  constexpr uint32_t IDESC = idesc_bf16_f32(2 * BM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * TILE_A_BYTES;
  uint8_t* sStage = sB + STAGES * L::HALF_B_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStage + L::STAGING_BYTES);
  uint64_t* ubars = bars + 2 * STAGES + 6;  // unit_full[UNIT_RING], unit_empty[UNIT_RING]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ubars + 2 * L::UNIT_RING);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* uring = reinterpret_cast<volatile int*>(tmem_slot + 2);  // the units handed out

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + 8 * STAGES;
  const uint32_t tfull0 = empty0 + 8 * STAGES;
  const uint32_t tempty0 = tfull0 + 16;
  const uint32_t drain = tempty0 + 16;
  const uint32_t staged = drain + 8;  // the four epilogue warps have staged the last unit
  const uint32_t full0_leader = mapa_shared(full0, 0);
  const uint32_t tempty0_leader = mapa_shared(tempty0, 0);
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  // Dynamic unit order: the even CTA's producer takes each next unit from set.sched[0] (after the
  // pair's first, its index) and writes it into slot it % UNIT_RING of both CTAs' rings (ufull); the consumers (the UMMA thread and the
  // four epilogue warps of the even CTA, the producer and the four epilogue warps of the odd one:
  // 10 arrivals) release the slot on the even CTA's uempty.  Consecutive units then run on
  // whichever pairs are free, so the pairs at work always hold a contiguous run of the raster and
  // its A panels are read while they are still in L2.
  constexpr int UR = L::UNIT_RING;
  const bool dyn = set.sched != nullptr;
  const uint32_t ufull0 = smem_u32(ubars);
  const uint32_t uempty0 = ufull0 + 8 * UR;
  const uint32_t uempty0_leader = mapa_shared(uempty0, 0);
  const uint32_t ufull0_peer = mapa_shared(ufull0, 1);
  const uint32_t uring_peer = mapa_shared(smem_u32(const_cast<int*>(uring)), 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, 8);
    }
    mbar_init(drain, 1);
    mbar_init(staged, 4);
    for (int s = 0; s < UR; ++s) {
      mbar_init(ufull0 + 8 * s, 1);
      mbar_init(uempty0 + 8 * s, 10);
    }
    *abort_s = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    for (int i = 0; i < set.n; ++i) {
      const EpiArgs& e = set.lin[i].epi;
      tma_prefetch_desc(&set.tmB[i]);
      if (e.store_mode == STORE_TMA || e.store_mode == STORE_TMA_ADD) {
        tma_prefetch_desc(&set.tmY[i]);
        if (set.lin[i].ybig_ok) tma_prefetch_desc(&set.ybig[i]);
      }
      if (e.store_mode >= STORE_TMA_PEERS)
        for (int r = 0; r < e.nremote; ++r) tma_prefetch_desc(&set.pm.m[r]);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), L::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtl wc{set.wait_cap_ns, set.status, abort_s, 0};
  // everything above (barriers, TMEM, descriptor prefetch) overlaps the previous kernel's tail
  griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();

  // The it-th unit of this pair (set.total ends the sequence).  publish_unit: the even CTA's
  // producer; take_unit: every other role (one thread each); peek_unit reads a slot without
  // releasing it.  false: a bounded wait gave up.  Dynamic order: a pair's first unit is its
  // index; the counter hands out the units from npairs on, and the producer asks it for the
  // pair's next unit as soon as it publishes one, so the atomic's round trip overlaps the
  // current unit's loads instead of delaying the next unit's first one.
  int next_raw = -1;  // the counter's value for the next unit; -1: the pair's first unit
  auto publish_unit = [&](int it, int& unit) -> bool {
    if (!dyn) {
      unit = min(pair + it * npairs, set.total);
      return true;
    }
    const int slot = it % UR;
    if (!wait_bounded_cluster(uempty0 + 8 * slot, ((it / UR) & 1) ^ 1, wc, 26)) return false;
    const int u = min(next_raw < 0 ? pair : npairs + next_raw, set.total);
    uring[slot] = u;
    st_shared_cluster_u32(uring_peer + 4 * slot, (uint32_t)u);
    mbar_arrive(ufull0 + 8 * slot);
    mbar_arrive_cluster(ufull0_peer + 8 * slot);
    if (u < set.total) next_raw = atomicAdd(set.sched, 1);  // read at the next publish_unit
    unit = u;
    return true;
  };
  auto peek_unit = [&](int it, int& unit) -> bool {
    if (!dyn) {
      unit = min(pair + it * npairs, set.total);
      return true;
    }
    const int slot = it % UR;
    if (!wait_bounded_cluster(ufull0 + 8 * slot, (it / UR) & 1, wc, 27)) return false;
    unit = uring[slot];
    return true;
  };
  auto take_unit = [&](int it, int& unit) -> bool {
    if (!peek_unit(it, unit)) return false;
    if (dyn) mbar_arrive_cluster(uempty0_leader + 8 * (it % UR));
    return true;
  };

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      uint32_t pending = 0, issue_ph = 0;
      const uint64_t pol_a = l2_policy_evict_last();
      for (int it = 0;; ++it) {
        int unit;
        if (!(leader ? publish_unit(it, unit) : take_unit(it, unit))) goto producer_done;
        if (unit >= set.total) break;
        const int li = set_linear(set, unit);
        const PairLin& P = set.lin[li];
        int tile, split, kb0, kb1;
        unit_split(unit - set.base[li], P, tile, split, kb0, kb1);
        int m_blk, n_blk;
        int b = 0, h0 = 0, w0 = 0;
        if (CONV_B) {
          m_blk = tile % P.tiles_m;
          n_blk = tile / P.tiles_m;
          const int per_img = set.conv.tiles_w * set.conv.tiles_h;
          b = n_blk / per_img;
          const int r = n_blk - b * per_img;
          h0 = (r / set.conv.tiles_w) * set.conv.tileH;
          w0 = (r % set.conv.tiles_w) * set.conv.tileW;
          // this CTA's half of the pixel tile: half the rows, or half the row when one row
          if (set.conv.tileH >= 2) h0 += (int)rank * (set.conv.tileH / 2);
          else w0 += (int)rank * (set.conv.tileW / 2);
        } else {
          map_tile(tile, P, m_blk, n_blk);
        }
        const int m0 = m_blk * 2 * BM + (int)rank * BM;
        const int n0 = n_blk * BN + (int)rank * 128;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bounded(empty0 + 8 * stage, ph ^ 1, wc, 21)) goto producer_done;
          const uint32_t fb = full0_leader + 8 * stage;
          if (leader) mbar_arrive_expect_tx(full0 + 8 * stage, 2 * L::STAGE_BYTES);
          if (!CONV_B && set.l2_hints)
            tma_load_2d_pair_hint(smem_u32(sA + stage * TILE_A_BYTES), &tmA, fb, kb * BK, m0, pol_a);
          else
            tma_load_2d_pair(smem_u32(sA + stage * TILE_A_BYTES), &tmA, fb, kb * BK, m0);
          if (CONV_B) {
            const int kpos = kb / set.conv.cblocks;
            const int cb = kb - kpos * set.conv.cblocks;
            const int kh = kpos / set.conv.KW;
            const int kw = kpos - kh * set.conv.KW;
            tma_load_4d_pair(smem_u32(sB + stage * L::HALF_B_BYTES), &set.tmB[li], fb, cb * BK,
                             w0 + kw - set.conv.pad, h0 + kh - set.conv.pad, b);
          } else {
            tma_load_2d_pair(smem_u32(sB + stage * L::HALF_B_BYTES), &set.tmB[li], fb, kb * BK, n0);
          }
          pending |= 1u << stage;
          issue_ph = (issue_ph & ~(1u << stage)) | (ph << stage);
          if (++stage == STAGES) {
            stage = 0;
            ph ^= 1;
          }
        }
      }
    producer_done:
      if (dyn && leader && !*abort_s) {
        // every unit this pair took has been fetched: count the pair done; the last pair zeroes
        // the schedule for the next launch (a stream-ordered launch reads it only after
        // griddep_wait, once this grid has finished)
        __threadfence();
        if (atomicAdd(set.sched + 1, 1) == npairs - 1) {
          set.sched[0] = 0;
          set.sched[1] = 0;
          __threadfence();
        }
      }
      if (*abort_s && pending) {
        if (leader) {
          for (int s = 0; s < STAGES; ++s)
            if (pending & (1u << s)) wait_drain(full0 + 8 * s, (issue_ph >> s) & 1u, set.wait_cap_ns);
        } else {
          // The odd CTA's copies signal the even CTA's barriers; give them time to land.
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 2000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      for (int it = 0;; ++it) {
        int unit;
        if (!take_unit(it, unit) || unit >= set.total) break;
        const int li = set_linear(set, unit);
        int tile, split, kb0, kb1;
        unit_split(unit - set.base[li], set.lin[li], tile, split, kb0, kb1);
        if (!wait_bounded(tempty0 + 8 * acc, aph ^ 1, wc, 22)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bounded(full0 + 8 * stage, ph, wc, 23)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_kmajor_desc(smem_u32(sA + stage * TILE_A_BYTES));
          const uint64_t bd = sw128_kmajor_desc(smem_u32(sB + stage * L::HALF_B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16_pair(d_tmem, ad + 2 * k, bd + 2 * k, IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
          umma_commit_pair_mc(empty0 + 8 * stage, 0x3);
          if (++stage == STAGES) {
            stage = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair_mc(tfull0 + 8 * acc, 0x3);
        acc ^= 1;
        if (acc == 0) aph ^= 1;
      }
      if (*abort_s) {
        umma_commit_pair(drain);
        wait_drain(drain, 0, set.wait_cap_ns);
      }
    }
  } else {
    const int q = warp & 3;
    bool any_remote = false;
    uint8_t* stg = sStage + (warp - 2) * 8192;
    int sb = 0;
    int acc = 0;
    uint32_t aph = 0;
    const uint64_t pol_y = l2_policy_evict_first();
    for (int it = 0;; ++it) {
      int unit = 0, next = 0;
      int ok = 1;
      if (lane == 0) ok = take_unit(it, unit) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      unit = __shfl_sync(0xffffffffu, unit, 0);
      if (!ok || unit >= set.total) break;
      const int li = set_linear(set, unit);
      const PairLin& P = set.lin[li];
      // A reference into the (grid-constant) parameter space: a local copy would be placed in
      // local memory, because the peer stores index ep.remote[] at run time.
      const EpiArgs& ep = P.epi;
      const int smode = ep.store_mode;
      any_remote = any_remote || ep.nremote != 0;
      int tile, split, kb0, kb1;
      unit_split(unit - set.base[li], P, tile, split, kb0, kb1);
      int m_blk, n_blk;
      int b = 0, h0 = 0, w0 = 0;
      if (CONV_B) {
        m_blk = tile % P.tiles_m;
        n_blk = tile / P.tiles_m;
        const int per_img = set.conv.tiles_w * set.conv.tiles_h;
        b = n_blk / per_img;
        const int r = n_blk - b * per_img;
        h0 = (r / set.conv.tiles_w) * set.conv.tileH;
        w0 = (r % set.conv.tiles_w) * set.conv.tileW;
      } else {
        map_tile(tile, P, m_blk, n_blk);
      }
      if (!wait_bounded_warp(tfull0 + 8 * acc, aph, wc, 24)) break;
      tc_fence_after();
      const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      const int row0 = m_blk * 2 * BM + (int)rank * BM + q * 32;
      const int row = row0 + lane;
      constexpr int NCHUNK = SILU_GATE ? BN / 64 : BN / 32;
      // On the CTA's last unit no operand load is in flight or still to come, and the UMMAs have
      // read their operands (the accumulator is complete), so each epilogue warp stages all its
      // chunks in its own quarter of the idle operand ring, then makes them visible to the TMA
      // unit with one proxy fence and issues every store back to back: the tail of the launch
      // is one pass over TMEM and the store drain, with no per-chunk fence or buffer wait.
      static_assert(L::RING_BYTES / 4 >= NCHUNK * 4096 && (L::RING_BYTES / 4) % 1024 == 0, "ring staging");
      // the CTA's last unit: the next one this pair gets is the end of the sequence
      if (lane == 0) ok = peek_unit(it + 1, next) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      next = __shfl_sync(0xffffffffu, next, 0);
      const bool ring_mode = ok && next >= set.total && smode != STORE_COALESCED && smode != STORE_DIRECT;
      // With the 128-row map, the four warps' 32 x 32 tiles of chunk c sit one above the other
      // (rows q * 32 ..) in a 16 KB box, and one thread stores each chunk of the CTA's 128 rows:
      // a quarter of the TMA stores, each four times larger.
      const bool big = ring_mode && P.ybig_ok && (smode == STORE_TMA || smode == STORE_TMA_ADD);
      static_assert(L::RING_BYTES >= NCHUNK * 16384, "ring staging, 128-row boxes");
      uint8_t* ring = big ? smem + q * 4096 : smem + (warp - 2) * (L::RING_BYTES / 4);
      const int ring_stride = big ? 16384 : 4096;
      // Y coordinates of chunk c's 32 x 32 box; false when a conv chunk lies past the row end.
      auto chunk_xy = [&](int c, int& x, int& y) -> bool {
        if (CONV_B) {
          const int jj = c * 32;
          const int w = w0 + jj % set.conv.tileW;
          const int h = h0 + jj / set.conv.tileW;
          x = h * set.conv.outW + w;
          y = row0;
          return w < set.conv.outW;
        }
        x = n_blk * (SILU_GATE ? BN / 2 : BN) + c * 32;
        y = row0 + split * P.split_rows;
        return true;
      };
      auto issue_store = [&](const uint8_t* buf, int x, int y) {
        if (CONV_B) {
          if (smode == STORE_TMA_ADD) tma_reduce_add_3d(&set.tmY[li], smem_u32(buf), x, y, b);
          else tma_store_3d(&set.tmY[li], smem_u32(buf), x, y, b);
        } else if (smode == STORE_TMA_PEERS) {
          for (int r = 0; r < ep.nremote; ++r) tma_store_2d(&set.pm.m[r], smem_u32(buf), x, y);
        } else if (smode == STORE_TMA_ADD_PEERS) {
          for (int r = 0; r < ep.nremote; ++r) tma_reduce_add_2d(&set.pm.m[r], smem_u32(buf), x, y);
        } else if (smode == STORE_TMA_ADD) {
          tma_reduce_add_2d(&set.tmY[li], smem_u32(buf), x, y);
        } else if (set.l2_hints) {
          tma_store_2d_hint(&set.tmY[li], smem_u32(buf), x, y, pol_y);
        } else {
          tma_store_2d(&set.tmY[li], smem_u32(buf), x, y);
        }
      };
#pragma unroll 1
      for (int c = 0; c < NCHUNK; ++c) {
        float v[32];
        int col0;
        if (SILU_GATE) {
          uint32_t g[32], u[32];
          tmem_ld32(trow + c * 32, g);
          tmem_ld32(trow + BN / 2 + c * 32, u);
          col0 = n_blk * (BN / 2) + c * 32;
          silu_gate_chunk(ep, g, u, col0, v);
        } else {
          uint32_t r[32];
          tmem_ld32(trow + c * 32, r);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          col0 = n_blk * BN + c * 32;
        }
        if (smode == STORE_DIRECT) {
          if (SILU_GATE) {
            EpiArgs e2 = ep;
            e2.bias_mode = 0;
            e2.act = 0;
            epi_store_row32(e2, row, col0, v);
          } else if (CONV_B) {
            epi_store_conv32(ep, set.conv, b, row, h0, w0, c * 32, v);
          } else {
            epi_store_row32(ep, row, col0, v);
          }
          continue;
        }
        int x, y;
        if (!chunk_xy(c, x, y)) continue;
        if (CONV_B) {
          const float bv = (ep.bias_mode == 2 && row < ep.m_valid) ? __ldg(ep.bias + row) : 0.0f;
          if (ep.act) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = silu_f(__fadd_rn(v[j], bv));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], bv);
          }
        } else if (!SILU_GATE) {
          epi_pre_chunk(ep, v, row, col0);
        }
        if (!CONV_B && ep.yb) store_bf16_row32(ep, row, col0, v);
        uint8_t* buf = stg + sb * 4096;
        if (smode == STORE_COALESCED) {
          stage_row32(buf, lane, v);
          __syncwarp();
          if (CONV_B) {
            const int jj = c * 32;
            store_tile32_conv(ep, set.conv, buf, lane, row0, b, h0 + jj / set.conv.tileW,
                              w0 + jj % set.conv.tileW);
          } else {
            store_tile32_rows(ep, buf, lane, row0, col0);
          }
          sb ^= 1;  // the other buffer is written next, so no wait before this one is reused
          continue;
        }
        if (ring_mode) {
          stage_row32(ring + c * ring_stride, lane, v);  // stored after the loop
          continue;
        }
        if (lane == 0) bulk_wait_read<1>();  // the store that last read this buffer is done with it
        __syncwarp();
        stage_row32(buf, lane, v);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          issue_store(buf, x, y);
          bulk_commit();
        }
        sb ^= 1;
      }
      if (ring_mode) {
        fence_proxy_async_smem();
        __syncwarp();
        if (big) {
          if (lane == 0) mbar_arrive(staged);
          if (warp == 2 && lane == 0 && wait_bounded(staged, 0, wc, 25)) {
            for (int c = 0; c < NCHUNK; ++c) {
              int x, y;
              if (!chunk_xy(c, x, y)) continue;
              y -= q * 32;  // the CTA's first row
              const uint32_t src = smem_u32(smem + c * 16384);
              if (CONV_B) {
                if (smode == STORE_TMA_ADD) tma_reduce_add_3d(&set.ybig[li], src, x, y, b);
                else tma_store_3d(&set.ybig[li], src, x, y, b);
              } else if (smode == STORE_TMA_ADD) {
                tma_reduce_add_2d(&set.ybig[li], src, x, y);
              } else if (set.l2_hints) {
                tma_store_2d_hint(&set.ybig[li], src, x, y, pol_y);
              } else {
                tma_store_2d(&set.ybig[li], src, x, y);
              }
            }
            bulk_commit();
          }
        } else if (lane == 0) {
          for (int c = 0; c < NCHUNK; ++c) {
            int x, y;
            if (chunk_xy(c, x, y)) issue_store(ring + c * 4096, x, y);
          }
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0_leader + 8 * acc);
      acc ^= 1;
      if (acc == 0) aph ^= 1;
    }
    if (lane == 0) bulk_wait_all();
    if (any_remote) __threadfence_system();  // peer / multicast stores ordered before the caller's barrier
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, L::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------
// Split-K reduction of k1_gemm_pair: Y = epilogue(sum of the raw fp32 partial tiles, added in
// split order, so the result does not depend on which split finished first).  part holds
// [splits][split_rows][ldp] accumulators over the device weight's rows; with SILU_GATE those
// rows interleave 128 gate rows with their 128 up rows, so output column j pairs partial
// columns 256 (j / 128) + j % 128 (gate) and that + 128 (up).  The epilogue is the one the
// unsplit kernel applies: bias / SiLU / gated residual / alpha-beta (epi_value) or the SiLU gate,
// the stores to each rank's copy of Y, and the optional bf16 side output.
// ------------------------------------------------------------------------------------------
ENVG_DEV float4 add4(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// Sum of the partials at offset `off` of every split, added in split order; four loads are in
// flight at a time.
ENVG_DEV float4 split_sum4(const float* __restrict__ part, int64_t off, int64_t split_elems, int splits) {
  float4 a = __ldcs(reinterpret_cast<const float4*>(part + off));
  int sp = 1;
  for (; sp + 3 < splits; sp += 4) {
    const float* p = part + sp * split_elems + off;
    const float4 p1 = __ldcs(reinterpret_cast<const float4*>(p));
    const float4 p2 = __ldcs(reinterpret_cast<const float4*>(p + split_elems));
    const float4 p3 = __ldcs(reinterpret_cast<const float4*>(p + 2 * split_elems));
    const float4 p4 = __ldcs(reinterpret_cast<const float4*>(p + 3 * split_elems));
    a = add4(add4(add4(add4(a, p1), p2), p3), p4);
  }
  for (; sp < splits; ++sp) a = add4(a, __ldcs(reinterpret_cast<const float4*>(part + sp * split_elems + off)));
  return a;
}

// The split linears of one launch_pair_set call, reduced by one launch: work items (one row and
// four output columns each) [base[i], base[i + 1]) belong to linear i.
struct SplitReduceSet {
  const float* part[PSET_MAX];
  int64_t ldp[PSET_MAX], split_elems[PSET_MAX];
  int splits[PSET_MAX];
  int silu_gate[PSET_MAX];
  EpiArgs e[PSET_MAX];
  int64_t base[PSET_MAX + 1];
  int n;
};

__global__ void __launch_bounds__(256) k_split_reduce(const __grid_constant__ SplitReduceSet rs) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t total = rs.base[rs.n];
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    int li = 0;
    while (li + 1 < rs.n && t >= rs.base[li + 1]) ++li;
    const EpiArgs& e = rs.e[li];
    const float* part = rs.part[li];
    const int64_t ldp = rs.ldp[li], split_elems = rs.split_elems[li];
    const int splits = rs.splits[li];
    const int quads = (e.n_out + 3) >> 2;
    const int64_t u = t - rs.base[li];
    const int row = (int)(u / quads);
    const int col = (int)(u - (int64_t)row * quads) * 4;
    const bool silu_gate = rs.silu_gate[li] != 0;
    float v[4];
    if (silu_gate) {
      const int64_t pg = (int64_t)row * ldp + (col >> 7) * 256 + (col & 127);
      const float4 g = split_sum4(part, pg, split_elems, splits);
      const float4 up = split_sum4(part, pg + 128, split_elems, splits);
      const float gv[4] = {g.x, g.y, g.z, g.w}, uv[4] = {up.x, up.y, up.z, up.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = min(col + j, e.n_out - 1);
        v[j] = (e.bias_mode == 1)
                   ? __fmul_rn(silu_f(__fadd_rn(gv[j], __ldg(e.bias + c))), __fadd_rn(uv[j], __ldg(e.bias + e.half_n + c)))
                   : __fmul_rn(silu_f(gv[j]), uv[j]);
      }
    } else {
      const float4 a = split_sum4(part, (int64_t)row * ldp + col, split_elems, splits);
      v[0] = a.x;
      v[1] = a.y;
      v[2] = a.z;
      v[3] = a.w;
    }
    const int64_t idx = (int64_t)row * e.ldy + e.col_off + col;
    const bool rmw = e.mode == EPI_GATED_RES || (e.mode == EPI_ALPHA_BETA && e.beta != 0.0f);
    // the SiLU gate already holds its bias; epi_value then adds nothing (mode SILU_GATE)
    const bool plain = silu_gate;
    if (e.vec_ok && col + 3 < e.n_out) {
      float4 old = make_float4(0.f, 0.f, 0.f, 0.f);
      if (rmw) old = *reinterpret_cast<const float4*>(e.Y + idx);
      if (!plain) {
        v[0] = epi_value(e, v[0], row, col + 0, &old.x);
        v[1] = epi_value(e, v[1], row, col + 1, &old.y);
        v[2] = epi_value(e, v[2], row, col + 2, &old.z);
        v[3] = epi_value(e, v[3], row, col + 3, &old.w);
      }
      out_store4(e, idx, make_float4(v[0], v[1], v[2], v[3]));
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (col + j >= e.n_out) break;
        if (!plain) v[j] = epi_value(e, v[j], row, col + j, e.Y + idx + j);
        out_store1(e, idx + j, v[j]);
      }
    }
    if (e.yb) {
      __nv_bfloat16* p = e.yb + (int64_t)row * e.ldyb + col;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (col + j < e.n_out) p[j] = __float2bfloat16_rn(v[j]);
    }
  }
}

template <int MPAD, int R, int STAGES>
struct K2Smem {
  static constexpr int W_BYTES = R * TILE_A_BYTES;
  static constexpr int X_BYTES = MPAD * BK * 2;
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
  static constexpr int BAR_BYTES = (2 * STAGES + 3) * 8 + 32;
  static constexpr int TOTAL = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
  static constexpr uint32_t TMEM_COLS = (R * MPAD <= 32) ? 32 : (R * MPAD <= 64) ? 64 : 128;
};

// ------------------------------------------------------------------------------------------
// K2: skinny-M GEMM (M <= 64), HBM-bound on W.  CTA (tile, split) multiplies R*128 rows of W
// by all M tokens over one contiguous K range; R = 2 pairs a gate tile with its up tile.
// ------------------------------------------------------------------------------------------
template <int MPAD, int R, int STAGES>
__global__ void __launch_bounds__(K1_THREADS, 1)
    k2_skinny(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
              const __grid_constant__ SkinnyArgs args) {
  using L = K2Smem<MPAD, R, STAGES>;
  constexpr uint32_t IDESC = idesc_bf16_f32(BM, MPAD);
  static_assert(MPAD % 16 == 0 && MPAD >= 16 && MPAD <= 64, "MPAD");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sX = smem + STAGES * L::W_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sX + STAGES * L::X_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 3);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_s = reinterpret_cast<volatile int*>(tmem_slot + 2);
  volatile int* ok_s = reinterpret_cast<volatile int*>(tmem_slot + 3);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + 8 * STAGES;
  const uint32_t tfull = empty0 + 8 * STAGES;
  const uint32_t drain = tfull + 8;

  const int tile = blockIdx.x / args.splits;
  const int split = blockIdx.x - tile * args.splits;
  const int kb0 = split * args.kb_per_split;
  const int kb1 = min(kb0 + args.kb_per_split, args.num_kb);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    *abort_s = 0;
    *last_s = 0;
    *ok_s = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtl wc{args.wait_cap_ns, args.status, abort_s, 0};

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      uint32_t pending = 0, issue_ph = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!wait_bounded(empty0 + 8 * stage, ph ^ 1, wc, 11)) break;
        const uint32_t fb = full0 + 8 * stage;
        mbar_arrive_expect_tx(fb, L::STAGE_BYTES);
#pragma unroll
        for (int r = 0; r < R; ++r)
          tma_load_2d(smem_u32(sW + stage * L::W_BYTES + r * TILE_A_BYTES), &tmW, fb, kb * BK,
                      (tile * R + r) * BM);
        tma_load_2d(smem_u32(sX + stage * L::X_BYTES), &tmX, fb, kb * BK, 0);
        pending |= 1u << stage;
        issue_ph = (issue_ph & ~(1u << stage)) | (ph << stage);
        if (++stage == STAGES) {
          stage = 0;
          ph ^= 1;
        }
      }
      if (*abort_s)
        for (int s = 0; s < STAGES; ++s)
          if (pending & (1u << s)) wait_drain(full0 + 8 * s, (issue_ph >> s) & 1u, args.wait_cap_ns);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!wait_bounded(full0 + 8 * stage, ph, wc, 12)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t xd = sw128_kmajor_desc(smem_u32(sX + stage * L::X_BYTES));
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const uint64_t wd = sw128_kmajor_desc(smem_u32(sW + stage * L::W_BYTES + r * TILE_A_BYTES));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(tmem_base + (uint32_t)(r * MPAD), wd + 2 * k, xd + 2 * k, IDESC,
                      (kb > kb0 || k > 0) ? 1u : 0u);
        }
        umma_commit(empty0 + 8 * stage);
        if (++stage == STAGES) {
          stage = 0;
          ph ^= 1;
        }
      }
      if (ok) umma_commit(tfull);
      if (*abort_s) {
        umma_commit(drain);
        wait_drain(drain, 0, args.wait_cap_ns);
      }
    }
  } else {
    const int q = warp & 3;
    const int rowin = q * 32 + lane;  // W row within a 128-row tile
    const int et = threadIdx.x - 64;  // 0..127
    if (et == 0) *ok_s = wait_bounded(tfull, 0, wc, 13) ? 1 : 0;
    named_bar_sync(1, 128);
    if (*ok_s) {
      tc_fence_after();
      float acc[R][MPAD];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t ta = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(r * MPAD);
#pragma unroll
        for (int c = 0; c < MPAD / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(ta + c * 32, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[r][c * 32 + j] = __uint_as_float(v[j]);
        }
        if (MPAD % 32) {
          uint32_t v[16];
          tmem_ld16(ta + (MPAD / 32) * 32, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[r][(MPAD / 32) * 32 + j] = __uint_as_float(v[j]);
        }
      }
      bool finalize = true;
      if (args.splits > 1) {
        // Deterministic split-K: every split stores its partial; the CTA that arrives last sums
        // the partials in split order 0..S-1 and runs the epilogue.
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float* p = args.partial + ((((int64_t)tile * args.splits + split) * R + r) * BM + rowin) * MPAD;
#pragma unroll
          for (int m = 0; m < MPAD; m += 4)
            __stcg(reinterpret_cast<float4*>(p + m), make_float4(acc[r][m], acc[r][m + 1], acc[r][m + 2], acc[r][m + 3]));
        }
        named_bar_sync(1, 128);
        if (et == 0) {
          const int old = atom_add_acq_rel_gpu(args.counters + tile, 1);
          *last_s = (old == args.splits - 1) ? 1 : 0;
        }
        named_bar_sync(1, 128);
        finalize = (*last_s != 0);
        if (finalize) {
#pragma unroll
          for (int r = 0; r < R; ++r) {
#pragma unroll
            for (int m = 0; m < MPAD; ++m) acc[r][m] = 0.0f;
            // unrolled so that the loads of several splits are in flight together; the adds
            // still run in split order
#pragma unroll 4
            for (int s = 0; s < args.splits; ++s) {
              const float* p = args.partial + ((((int64_t)tile * args.splits + s) * R + r) * BM + rowin) * MPAD;
#pragma unroll
              for (int m = 0; m < MPAD; m += 4) {
                const float4 t = __ldcg(reinterpret_cast<const float4*>(p + m));
                acc[r][m] += t.x;
                acc[r][m + 1] += t.y;
                acc[r][m + 2] += t.z;
                acc[r][m + 3] += t.w;
              }
            }
          }
          if (et == 0) args.counters[tile] = 0;  // re-arm for the next launch
        }
      }
      if (finalize) {
        const EpiArgs& e = args.epi;  // in parameter space (a local copy would go to local memory)
        const int col = tile * BM + rowin;  // output column (shard-relative)
        if (col < e.n_out) {
#pragma unroll
          for (int m = 0; m < MPAD; ++m) {
            if (m >= e.m_valid) break;
            const int64_t idx = (int64_t)m * e.ldy + e.col_off + col;
            float* yp = e.Y + idx;
            float v;
            if (R == 2) {
              float gv = acc[0][m], uv = acc[R - 1][m];
              if (e.bias_mode == 1) {
                gv = __fadd_rn(gv, __ldg(e.bias + col));
                uv = __fadd_rn(uv, __ldg(e.bias + e.half_n + col));
              }
              v = __fmul_rn(silu_f(gv), uv);
            } else {
              v = epi_value(e, acc[0][m], m, col, yp);
            }
            out_store1(e, idx, v);
          }
        }
        if (e.nremote != 0) __threadfence_system();
      }
    }
    tc_fence_before();
  }
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------
// K2 set: the skinny GEMM of k2_skinny, persistent over the units (linear, tile, split) of up to
// K2S_MAX_LIN linears in one launch.  The producer, the UMMA thread and the epilogue warps walk
// the same unit sequence (blockIdx.x, +gridDim.x, ...); the accumulator is double-buffered in
// TMEM so the epilogue of one unit overlaps the main loop of the next, and the launch cost, the
// TMEM allocation and the pipeline fill are paid once for all the weights of the set.  Each unit
// issues the same UMMAs in the same order as k2_skinny does for that (tile, split); a unit of a
// split linear stores its partial and k_skinny_reduce sums a tile's partials in split order, so
// results do not depend on the set a linear is launched in.
// ------------------------------------------------------------------------------------------
constexpr int K2S_MAX_LIN = 4;

struct K2Lin {
  SkinnyArgs s;  // n_tiles, splits, kb_per_split, num_kb, epi, partial (counters unused here)
  int R;         // 2: the unit pairs a gate tile with its up tile (SiLU-gate); one R per set
};

struct K2Set {
  CUtensorMap tmW[K2S_MAX_LIN];  // W, box 64 x 128 rows
  CUtensorMap tmX[K2S_MAX_LIN];  // X (bf16), box 64 x MPAD rows
  K2Lin lin[K2S_MAX_LIN];
  int n, total;
  int base[K2S_MAX_LIN + 1];
  int* status;
  uint64_t wait_cap_ns;
};
static_assert(sizeof(K2Set) <= 4096, "K2Set is a kernel parameter");

template <int MPAD, int R, int STAGES>
struct K2SetSmem {
  static constexpr int W_BYTES = R * TILE_A_BYTES;
  static constexpr int X_BYTES = MPAD * BK * 2;
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
  static constexpr int NBARS = 2 * STAGES + 5;       // full/empty, tfull[2], tempty[2], drain
  static constexpr int TOTAL = 1024 + STAGES * STAGE_BYTES + NBARS * 8 + 32;
  static constexpr uint32_t ACC_COLS = R * MPAD;      // R accumulators of MPAD columns
  static constexpr uint32_t TMEM_COLS = (2 * ACC_COLS <= 32) ? 32 : (2 * ACC_COLS <= 64) ? 64
                                        : (2 * ACC_COLS <= 128) ? 128 : 256;
};

ENVG_DEV void k2_unit(const K2Set& S, int u, int& l, int& tile, int& split) {
  l = 0;
  while (l + 1 < S.n && u >= S.base[l + 1]) ++l;
  const int v = u - S.base[l];
  tile = v / S.lin[l].s.splits;
  split = v - tile * S.lin[l].s.splits;
}

template <int MPAD, int R, int STAGES>
__global__ void __launch_bounds__(K1_THREADS, 1) k2_set(const __grid_constant__ K2Set S) {
  using L = K2SetSmem<MPAD, R, STAGES>;
  constexpr uint32_t IDESC = idesc_bf16_f32(BM, MPAD);
  static_assert(MPAD % 16 == 0 && MPAD >= 16 && MPAD <= 64, "MPAD");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sX = smem + STAGES * L::W_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sX + STAGES * L::X_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::NBARS);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = full0 + 8 * STAGES;
  const uint32_t tfull0 = empty0 + 8 * STAGES;
  const uint32_t tempty0 = tfull0 + 16;
  const uint32_t drain = tempty0 + 16;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, 4);
    }
    mbar_init(drain, 1);
    *abort_s = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane < S.n) {
    tma_prefetch_desc(&S.tmW[lane]);
    tma_prefetch_desc(&S.tmX[lane]);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtl wc{S.wait_cap_ns, S.status, abort_s, 0};
  griddep_wait();  // the prologue above overlaps the previous kernel's tail
  if (threadIdx.x == 0) griddep_launch_dependents();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      uint32_t pending = 0, issue_ph = 0;
      for (int u = blockIdx.x; u < S.total; u += gridDim.x) {
        int l, tile, split;
        k2_unit(S, u, l, tile, split);
        const SkinnyArgs& a = S.lin[l].s;
        const int kb0 = split * a.kb_per_split;
        const int kb1 = min(kb0 + a.kb_per_split, a.num_kb);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bounded(empty0 + 8 * stage, ph ^ 1, wc, 41)) goto producer_done;
          const uint32_t fb = full0 + 8 * stage;
          mbar_arrive_expect_tx(fb, R * TILE_A_BYTES + L::X_BYTES);
          for (int r = 0; r < R; ++r)
            tma_load_2d(smem_u32(sW + stage * L::W_BYTES + r * TILE_A_BYTES), &S.tmW[l], fb, kb * BK,
                        (tile * R + r) * BM);
          tma_load_2d(smem_u32(sX + stage * L::X_BYTES), &S.tmX[l], fb, kb * BK, 0);
          pending |= 1u << stage;
          issue_ph = (issue_ph & ~(1u << stage)) | (ph << stage);
          if (++stage == STAGES) {
            stage = 0;
            ph ^= 1;
          }
        }
      }
    producer_done:
      if (*abort_s)
        for (int s = 0; s < STAGES; ++s)
          if (pending & (1u << s)) wait_drain(full0 + 8 * s, (issue_ph >> s) & 1u, S.wait_cap_ns);
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      for (int u = blockIdx.x; u < S.total; u += gridDim.x) {
        int l, tile, split;
        k2_unit(S, u, l, tile, split);
        const SkinnyArgs& a = S.lin[l].s;
        const int kb0 = split * a.kb_per_split;
        const int kb1 = min(kb0 + a.kb_per_split, a.num_kb);
        if (!wait_bounded(tempty0 + 8 * acc, aph ^ 1, wc, 42)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)acc * L::ACC_COLS;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bounded(full0 + 8 * stage, ph, wc, 43)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t xd = sw128_kmajor_desc(smem_u32(sX + stage * L::X_BYTES));
          for (int r = 0; r < R; ++r) {
            const uint64_t wd = sw128_kmajor_desc(smem_u32(sW + stage * L::W_BYTES + r * TILE_A_BYTES));
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_bf16(d_tmem + (uint32_t)(r * MPAD), wd + 2 * k, xd + 2 * k, IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(empty0 + 8 * stage);
          if (++stage == STAGES) {
            stage = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(tfull0 + 8 * acc);
        acc ^= 1;
        if (acc == 0) aph ^= 1;
      }
      if (*abort_s) {
        umma_commit(drain);
        wait_drain(drain, 0, S.wait_cap_ns);
      }
    }
  } else {
    // ---------------- epilogue: 4 warps, one TMEM lane quadrant each ----------------
    const int q = warp & 3;
    const int rowin = q * 32 + lane;  // W row within a 128-row tile
    int acc = 0;
    uint32_t aph = 0;
    for (int u = blockIdx.x; u < S.total; u += gridDim.x) {
      int l, tile, split;
      k2_unit(S, u, l, tile, split);
      const SkinnyArgs& a = S.lin[l].s;
      if (!wait_bounded_warp(tfull0 + 8 * acc, aph, wc, 44)) break;
      tc_fence_after();
      float accv[R][MPAD];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t ta = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)acc * L::ACC_COLS + (uint32_t)(r * MPAD);
#pragma unroll
        for (int c = 0; c < MPAD / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(ta + c * 32, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) accv[r][c * 32 + j] = __uint_as_float(v[j]);
        }
        if (MPAD % 32) {
          uint32_t v[16];
          tmem_ld16(ta + (MPAD / 32) * 32, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) accv[r][(MPAD / 32) * 32 + j] = __uint_as_float(v[j]);
        }
      }
      // the accumulator is in registers: hand the TMEM buffer back to the UMMA thread
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty0 + 8 * acc);
      acc ^= 1;
      if (acc == 0) aph ^= 1;
      if (a.splits > 1) {
        // a split stores its partial; k_skinny_reduce sums a tile's partials in split order
        for (int r = 0; r < R; ++r) {
          float* p = a.partial + ((((int64_t)tile * a.splits + split) * R + r) * BM + rowin) * MPAD;
#pragma unroll
          for (int m = 0; m < MPAD; m += 4)
            __stcg(reinterpret_cast<float4*>(p + m),
                   make_float4(accv[r][m], accv[r][m + 1], accv[r][m + 2], accv[r][m + 3]));
        }
        continue;
      }
      {
        const EpiArgs& e = a.epi;
        const int col = tile * BM + rowin;  // output column (shard-relative)
        if (col < e.n_out) {
#pragma unroll
          for (int m = 0; m < MPAD; ++m) {
            if (m >= e.m_valid) break;
            const int64_t idx = (int64_t)m * e.ldy + e.col_off + col;
            float* yp = e.Y + idx;
            float v;
            if (R == 2) {
              float gv = accv[0][m], uv = accv[R - 1][m];
              if (e.bias_mode == 1) {
                gv = __fadd_rn(gv, __ldg(e.bias + col));
                uv = __fadd_rn(uv, __ldg(e.bias + e.half_n + col));
              }
              v = __fmul_rn(silu_f(gv), uv);
            } else {
              v = epi_value(e, accv[0][m], m, col, yp);
            }
            out_store1(e, idx, v);
            if (e.yb) e.yb[(int64_t)m * e.ldyb + col] = __float2bfloat16_rn(v);
          }
        }
        if (e.nremote != 0) __threadfence_system();
      }
    }
    tc_fence_before();
  }
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

// Split-K finish of a k2_set launch: one thread per four outputs (four tokens m of one output
// column, i.e. of one W row of a 128-row tile) of each split linear.  It loads up to eight
// splits' partials at once and adds them in split order, from 0, as one CTA would, then applies
// the linear's epilogue.  Work items [base[i], base[i + 1]) belong to linear i:
// n_tiles * 128 * MPAD / 4 of them, the four tokens fastest (the partials' layout).
struct SkinnyReduceSet {
  const float* partial[K2S_MAX_LIN];  // [tile][split][R][128][MPAD]
  int splits[K2S_MAX_LIN];
  EpiArgs e[K2S_MAX_LIN];
  int base[K2S_MAX_LIN + 1];
  int n;
};
static_assert(sizeof(SkinnyReduceSet) <= 4096, "SkinnyReduceSet is a kernel parameter");

template <int MPAD, int R>
__global__ void __launch_bounds__(256) k_skinny_reduce(const __grid_constant__ SkinnyReduceSet rs) {
  griddep_wait();
  griddep_launch_dependents();
  constexpr int Q = MPAD / 4;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= rs.base[rs.n]) return;
  int li = 0;
  while (li + 1 < rs.n && t >= rs.base[li + 1]) ++li;
  const int v = t - rs.base[li];
  const int quad = v % Q, rv = v / Q;
  const int tile = rv / BM, rowin = rv - tile * BM;
  const EpiArgs& e = rs.e[li];
  const int col = tile * BM + rowin;  // output column (shard-relative)
  const int m0 = quad * 4;
  if (col >= e.n_out || m0 >= e.m_valid) return;
  const int splits = rs.splits[li];
  const float* base = rs.partial[li] + ((int64_t)tile * splits * R * BM + rowin) * MPAD + m0;
  const int64_t sstride = (int64_t)R * BM * MPAD;  // floats between splits
  float4 acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = 0; s0 < splits; s0 += 8) {
    float4 p[8][R];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (s0 + j < splits)
#pragma unroll
        for (int r = 0; r < R; ++r)
          p[j][r] = __ldcs(reinterpret_cast<const float4*>(base + (s0 + j) * sstride + r * BM * MPAD));
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (s0 + j < splits)
#pragma unroll
        for (int r = 0; r < R; ++r) {
          acc[r].x += p[j][r].x;
          acc[r].y += p[j][r].y;
          acc[r].z += p[j][r].z;
          acc[r].w += p[j][r].w;
        }
  }
  const float g4[4] = {acc[0].x, acc[0].y, acc[0].z, acc[0].w};
  const float u4[4] = {acc[R - 1].x, acc[R - 1].y, acc[R - 1].z, acc[R - 1].w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int m = m0 + j;
    if (m >= e.m_valid) break;
    const int64_t idx = (int64_t)m * e.ldy + e.col_off + col;
    float val;
    if (R == 2) {
      float gv = g4[j], uv = u4[j];
      if (e.bias_mode == 1) {
        gv = __fadd_rn(gv, __ldg(e.bias + col));
        uv = __fadd_rn(uv, __ldg(e.bias + e.half_n + col));
      }
      val = __fmul_rn(silu_f(gv), uv);
    } else {
      val = epi_value(e, g4[j], m, col, e.Y + idx);
    }
    out_store1(e, idx, val);
    if (e.yb) e.yb[(int64_t)m * e.ldyb + col] = __float2bfloat16_rn(val);
  }
  if (e.nremote != 0) __threadfence_system();
}

// ------------------------------------------------------------------------------------------
// k_gemv: linears with M <= 8 on CUDA cores.  X stays fp32 (products are exact fp32 x bf16, sums
// in fp32, as in the reference), so no activation cast runs.  Each warp streams 8 rows of W with
// 16-byte loads (one load instruction = 512 contiguous bytes of a row) and keeps the 8 x M dot
// products in registers; a warp-wide xor reduction finishes them.  Blocks of 8 warps cover 64 W
// rows (32 gate + 32 up output pairs for the GATE_UP layout); split-K across blocks reduces
// deterministically: the last block of a row group sums the partials in split order.
// ------------------------------------------------------------------------------------------
constexpr int GEMV_MAX_M = 8;
constexpr int GEMV_PART = GEMV_MAX_M * 64;  // floats per (row group, split) partial

struct GemvArgs {
  const float* X;
  int64_t ldx;
  int M, K;
  const uint16_t* W;
  int64_t Kp;
  int rows;       // W rows stored on the device
  int gate_up;    // interleaved GATE_UP layout: 128 gate rows then their 128 up rows
  int groups;     // row groups of 64 device rows
  int splits, kchunk;  // split-K: K elements per split (multiple of 256)
  int xvec;       // X rows 16-byte aligned and K % 8 == 0
  EpiArgs epi;
  float* partial;  // [groups][splits][GEMV_PART]
  int* counters;   // [groups]
  // In-launch chaining (a linear whose X is the output of an earlier linear of the same set):
  //   done:     this linear's completion count, when a later linear reads its output:
  //             [0] row groups whose outputs are stored, [1] units of the reader past their wait;
  //   wait_on:  the producer's `done`; this linear's units start once [0] reaches wait_groups,
  //             and read X through L2 (it was written during this launch), not the
  //             non-coherent read-only path.  The reader's last unit past the wait zeroes both.
  int* done;
  int* wait_on;
  int wait_groups;
};

ENVG_DEV uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Several skinny linears in one persistent launch: unit u of the set is (linear l, row group,
// K split); block b takes units b, b + gridDim.x, ...  The host sizes the units (about one per
// resident block, by bytes) and the launch streams every weight of the set back to back.
constexpr int GEMV_MAX_LIN = 6;
struct GemvSet {
  int n;                        // linears in the set
  int total;                    // units over all of them
  int base[GEMV_MAX_LIN + 1];   // first unit of each linear
  int* status;                  // device status word (a chained unit's wait that ran out)
  uint64_t wait_cap_ns;
  GemvArgs lin[GEMV_MAX_LIN];
};
static_assert(sizeof(GemvSet) <= 4096, "GemvSet is a kernel parameter");

template <int MT>
__global__ void __launch_bounds__(256) k_gemv(const __grid_constant__ GemvSet set) {
  __shared__ float s_sum[MT][64];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();
  for (int u = blockIdx.x; u < set.total; u += gridDim.x) {
  int l = 0;
  while (l + 1 < set.n && u >= set.base[l + 1]) ++l;
  const GemvArgs& a = set.lin[l];
  const int v = u - set.base[l];
  const int group = v / a.splits;
  const int split = v - group * a.splits;
  // the 8 device rows of this warp
  int drow[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (a.gate_up) {
      const int c = group * 32 + warp * 4 + (j & 3);  // output column of the pair
      drow[j] = 256 * (c >> 7) + (c & 127) + (j >= 4 ? 128 : 0);
    } else {
      drow[j] = group * 64 + warp * 8 + j;
    }
  }
  if (a.wait_on) {
    // X is an earlier linear's output from this launch: wait (bounded) until all its row groups
    // are stored.  Units run in increasing order on every block and the producer's units all come
    // first, so every unit waited for is running or done.
    if (threadIdx.x == 0) {
      int ok = 1;
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_gpu(a.wait_on) < a.wait_groups) {
        if (globaltimer_ns() - t0 > set.wait_cap_ns) {
          ok = 0;
          if (set.status) {
            atomicExch(set.status, -5);  // ENVG_ERR_TIMEOUT
            atomicExch(set.status + 1, 61);
          }
          break;
        }
      }
      if (ok && atomicAdd(a.wait_on + 1, 1) == set.base[l + 1] - set.base[l] - 1) {
        a.wait_on[0] = 0;  // the last unit past the wait re-arms the counters for the next launch
        a.wait_on[1] = 0;
      }
      s_last = ok;
    }
    __syncthreads();
    if (!s_last) continue;
  }
  float acc[MT][8];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[m][j] = 0.0f;
  const int kb = split * a.kchunk;
  const int ke = min(a.K, kb + a.kchunk);
#pragma unroll 2
  for (int k0 = kb + lane * 8; k0 < ke; k0 += 256) {
    uint4 wv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      wv[j] = (drow[j] < a.rows) ? ld_nc_v4(a.W + (int64_t)drow[j] * a.Kp + k0) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m >= a.M) break;
      float xv[8];
      const float* xp = a.X + (int64_t)m * a.ldx + k0;
      if (a.wait_on && k0 + 8 <= a.K && a.xvec) {
        const float4 x0 = __ldcg(reinterpret_cast<const float4*>(xp));
        const float4 x1 = __ldcg(reinterpret_cast<const float4*>(xp + 4));
        xv[0] = x0.x; xv[1] = x0.y; xv[2] = x0.z; xv[3] = x0.w;
        xv[4] = x1.x; xv[5] = x1.y; xv[6] = x1.z; xv[7] = x1.w;
      } else if (a.wait_on) {
#pragma unroll
        for (int e = 0; e < 8; ++e) xv[e] = (k0 + e < a.K) ? __ldcg(xp + e) : 0.0f;
      } else if (a.xvec && k0 + 8 <= a.K) {
        const float4 x0 = __ldg(reinterpret_cast<const float4*>(xp));
        const float4 x1 = __ldg(reinterpret_cast<const float4*>(xp + 4));
        xv[0] = x0.x; xv[1] = x0.y; xv[2] = x0.z; xv[3] = x0.w;
        xv[4] = x1.x; xv[5] = x1.y; xv[6] = x1.z; xv[7] = x1.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) xv[e] = (k0 + e < a.K) ? __ldg(xp + e) : 0.0f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t w4[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
        float t = acc[m][j];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          t = fmaf(xv[2 * q], __uint_as_float(w4[q] << 16), t);
          t = fmaf(xv[2 * q + 1], __uint_as_float(w4[q] & 0xFFFF0000u), t);
        }
        acc[m][j] = t;
      }
    }
  }
  // warp reduction; afterwards lane (m * 8 + j) % 32 owns sum (m, j)
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v = acc[m][j];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      acc[m][j] = v;
    }
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int j = 0; j < 8; ++j) s_sum[m][warp * 8 + j] = acc[m][j];
  }
  __syncthreads();
  if (a.splits > 1) {
    float* part = a.partial + ((int64_t)group * a.splits + split) * GEMV_PART;
    for (int t = threadIdx.x; t < MT * 64; t += blockDim.x) __stcg(part + t, s_sum[t / 64][t % 64]);
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atom_add_acq_rel_gpu(a.counters + group, 1) == a.splits - 1) ? 1 : 0;
    __syncthreads();
    if (!s_last) continue;  // uniform across the block; s_sum is rewritten only after the next
                            // unit's __syncthreads
    for (int t = threadIdx.x; t < MT * 64; t += blockDim.x) {
      float v = 0.0f;
#pragma unroll 8
      for (int sp = 0; sp < a.splits; ++sp) v += __ldcg(a.partial + ((int64_t)group * a.splits + sp) * GEMV_PART + t);
      s_sum[t / 64][t % 64] = v;
    }
    if (threadIdx.x == 0) a.counters[group] = 0;  // re-arm for the next launch
    __syncthreads();
  }
  const EpiArgs& e = a.epi;  // in parameter space (a local copy would go to local memory)
  if (a.gate_up) {
    for (int t = threadIdx.x; t < MT * 32; t += blockDim.x) {
      const int m = t / 32, c = t % 32;
      if (m >= a.M) continue;
      const int col = group * 32 + c;
      if (col >= e.n_out) continue;
      float g = s_sum[m][(c >> 2) * 8 + (c & 3)], u = s_sum[m][(c >> 2) * 8 + 4 + (c & 3)];
      if (e.bias_mode == 1) {
        g = __fadd_rn(g, __ldg(e.bias + col));
        u = __fadd_rn(u, __ldg(e.bias + e.half_n + col));
      }
      out_store1(e, (int64_t)m * e.ldy + e.col_off + col, __fmul_rn(silu_f(g), u));
    }
  } else {
    for (int t = threadIdx.x; t < MT * 64; t += blockDim.x) {
      const int m = t / 64, r = t % 64;
      if (m >= a.M) continue;
      const int col = group * 64 + r;
      if (col >= e.n_out) continue;
      const int64_t idx = (int64_t)m * e.ldy + e.col_off + col;
      out_store1(e, idx, epi_value(e, s_sum[m][r], m, col, e.Y + idx));
    }
  }
  if (e.nremote != 0) __threadfence_system();
  // every thread is done with s_sum before the next unit writes it, and (a.done) this group's
  // outputs are ordered before the release that counts it
  __syncthreads();
  if (a.done && threadIdx.x == 0) red_release_gpu_add(a.done, 1);
  }
}

// ------------------------------------------------------------------------------------------
// Casts
// ------------------------------------------------------------------------------------------

// X fp32 [rows][K] (row stride ldx) -> Xb bf16 [rows][Kp] with zeros in [K, Kp).  RNE.
__global__ void k_cast_rows(const float* __restrict__ X, int64_t ldx, int rows, int K, int Kp,
                            __nv_bfloat16* __restrict__ Xb, int vec8) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (vec8 == 2) {
    // Contiguous rows (ldx == K == Kp, K % 8 == 0, 16-byte aligned): one flat run of 8-float
    // groups, four groups in flight per thread (all loads issued before the first store).
    const int64_t total = (int64_t)rows * (K / 8);
    const float4* src = reinterpret_cast<const float4*>(X);
    uint4* dst = reinterpret_cast<uint4*>(Xb);
    for (int64_t i0 = tid; i0 < total; i0 += 4 * stride) {
      float4 a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t i = i0 + u * stride;
        if (i < total) {
          a[u] = __ldcs(src + 2 * i);
          b[u] = __ldcs(src + 2 * i + 1);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t i = i0 + u * stride;
        if (i < total) {
          __nv_bfloat162 p0 = __float22bfloat162_rn(make_float2(a[u].x, a[u].y));
          __nv_bfloat162 p1 = __float22bfloat162_rn(make_float2(a[u].z, a[u].w));
          __nv_bfloat162 p2 = __float22bfloat162_rn(make_float2(b[u].x, b[u].y));
          __nv_bfloat162 p3 = __float22bfloat162_rn(make_float2(b[u].z, b[u].w));
          uint4 o;
          o.x = *reinterpret_cast<uint32_t*>(&p0);
          o.y = *reinterpret_cast<uint32_t*>(&p1);
          o.z = *reinterpret_cast<uint32_t*>(&p2);
          o.w = *reinterpret_cast<uint32_t*>(&p3);
          dst[i] = o;
        }
      }
    }
  } else if (vec8) {
    // K == Kp, K % 8 == 0, ldx % 4 == 0, 16-byte aligned rows.
    const int kv = K / 8;
    const int64_t total = (int64_t)rows * kv;
    for (int64_t i = tid; i < total; i += stride) {
      const int64_t r = i / kv;
      const int c = (int)(i - r * kv) * 8;
      const float4 a = __ldcs(reinterpret_cast<const float4*>(X + r * ldx + c));
      const float4 b = __ldcs(reinterpret_cast<const float4*>(X + r * ldx + c + 4));
      __nv_bfloat162 p0 = __float22bfloat162_rn(make_float2(a.x, a.y));
      __nv_bfloat162 p1 = __float22bfloat162_rn(make_float2(a.z, a.w));
      __nv_bfloat162 p2 = __float22bfloat162_rn(make_float2(b.x, b.y));
      __nv_bfloat162 p3 = __float22bfloat162_rn(make_float2(b.z, b.w));
      uint4 o;
      o.x = *reinterpret_cast<uint32_t*>(&p0);
      o.y = *reinterpret_cast<uint32_t*>(&p1);
      o.z = *reinterpret_cast<uint32_t*>(&p2);
      o.w = *reinterpret_cast<uint32_t*>(&p3);
      *reinterpret_cast<uint4*>(Xb + r * Kp + c) = o;
    }
  } else {
    const int64_t total = (int64_t)rows * Kp;
    for (int64_t i = tid; i < total; i += stride) {
      const int64_t r = i / Kp;
      const int c = (int)(i - r * Kp);
      const float v = (c < K) ? X[r * ldx + c] : 0.0f;
      Xb[i] = __float2bfloat16_rn(v);
    }
  }
}

// src fp32 [batch][R][C] (row stride lds, batch stride sbs) -> dst bf16 [batch][C][Rp]
// (row stride ldd, batch stride dbs), zeros for R <= r < Rp.  Rp must be even.
// With aff set, each value first becomes x * aff[b*R + r].x + aff[b*R + r].y (the per-channel
// form of a GroupNorm), then SiLU when act != 0: the GroupNorm + SiLU prologue of a conv.
__global__ void __launch_bounds__(256) k_transpose_cast(const float* __restrict__ src, int64_t lds, int64_t sbs, int R,
                                                        int C, __nv_bfloat16* __restrict__ dst, int64_t ldd,
                                                        int64_t dbs, int Rp, const float2* __restrict__ aff,
                                                        int act) {
  __shared__ float t[64][33];
  griddep_wait();
  griddep_launch_dependents();
  const int c0 = blockIdx.x * 32;
  const int r0 = blockIdx.y * 64;
  const int b = blockIdx.z;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const float* s = src + (int64_t)b * sbs;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int rr = ty + i * 8;
    const int r = r0 + rr, c = c0 + tx;
    float v = 0.0f;
    if (r < R && c < C) {
      v = __ldcs(s + (int64_t)r * lds + c);
      if (aff) {
        const float2 a = __ldg(aff + (int64_t)b * R + r);
        v = __fmaf_rn(v, a.x, a.y);
      }
      if (act) v = silu_f(v);
    }
    t[rr][tx] = v;
  }
  __syncthreads();
  __nv_bfloat16* d = dst + (int64_t)b * dbs;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = threadIdx.x + i * 256;
    const int cc = idx >> 5, rp = idx & 31;
    const int c = c0 + cc, r = r0 + 2 * rp;
    if (c < C && r < Rp) {
      __nv_bfloat162 p = __float22bfloat162_rn(make_float2(t[2 * rp][cc], t[2 * rp + 1][cc]));
      *reinterpret_cast<__nv_bfloat162*>(d + (int64_t)c * ldd + r) = p;
    }
  }
}

// The same transpose for aligned operands (C % 4 == 0, lds % 4 == 0, Rp % 8 == 0, ldd % 8 == 0,
// 16-byte aligned bases and batch strides): a 64 x 64 tile per CTA, 16-byte loads of 4 floats
// along C and 16-byte stores of 8 bf16 along R.
__global__ void __launch_bounds__(256) k_transpose_cast_v(const float* __restrict__ src, int64_t lds, int64_t sbs,
                                                          int R, int C, __nv_bfloat16* __restrict__ dst, int64_t ldd,
                                                          int64_t dbs, int Rp, const float2* __restrict__ aff, int act) {
  __shared__ float t[64][65];
  griddep_wait();
  griddep_launch_dependents();
  const int c0 = blockIdx.x * 64;
  const int r0 = blockIdx.y * 64;
  const int b = blockIdx.z;
  const float* s = src + (int64_t)b * sbs;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = threadIdx.x + 256 * i;
    const int rr = idx >> 4, c4 = (idx & 15) * 4;
    const int r = r0 + rr, c = c0 + c4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < R && c < C) {
      v = __ldcs(reinterpret_cast<const float4*>(s + (int64_t)r * lds + c));
      if (aff) {
        const float2 a = __ldg(aff + (int64_t)b * R + r);
        v.x = __fmaf_rn(v.x, a.x, a.y);
        v.y = __fmaf_rn(v.y, a.x, a.y);
        v.z = __fmaf_rn(v.z, a.x, a.y);
        v.w = __fmaf_rn(v.w, a.x, a.y);
      }
      if (act) {
        v.x = silu_f(v.x);
        v.y = silu_f(v.y);
        v.z = silu_f(v.z);
        v.w = silu_f(v.w);
      }
    }
    t[rr][c4] = v.x;
    t[rr][c4 + 1] = v.y;
    t[rr][c4 + 2] = v.z;
    t[rr][c4 + 3] = v.w;
  }
  __syncthreads();
  __nv_bfloat16* d = dst + (int64_t)b * dbs;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int idx = threadIdx.x + 256 * i;
    const int px = idx >> 3, ch = (idx & 7) * 8;
    const int c = c0 + px, r = r0 + ch;
    if (c < C && r < Rp) {
      uint4 o;
      __nv_bfloat162 h0 = __float22bfloat162_rn(make_float2(t[ch][px], t[ch + 1][px]));
      __nv_bfloat162 h1 = __float22bfloat162_rn(make_float2(t[ch + 2][px], t[ch + 3][px]));
      __nv_bfloat162 h2 = __float22bfloat162_rn(make_float2(t[ch + 4][px], t[ch + 5][px]));
      __nv_bfloat162 h3 = __float22bfloat162_rn(make_float2(t[ch + 6][px], t[ch + 7][px]));
      o.x = *reinterpret_cast<uint32_t*>(&h0);
      o.y = *reinterpret_cast<uint32_t*>(&h1);
      o.z = *reinterpret_cast<uint32_t*>(&h2);
      o.w = *reinterpret_cast<uint32_t*>(&h3);
      *reinterpret_cast<uint4*>(d + (int64_t)c * ldd + r) = o;
    }
  }
}

// ---- bf16x3 operands for fp32 inputs ----------------------------------------------------------
// An fp32 value v is held as two bf16 parts, hi = bf16_rn(v) and lo = bf16_rn(v - hi); hi + lo
// equals v to about 2^-17 relative (v - hi is exact in fp32).  An operand row of K values becomes
// three K-segments of Ks = K rounded up to 8 (zeros in [K, Ks)), each holding the hi or the lo
// parts; bit s of lo_mask marks segment s as lo.  One bf16 GEMM over the 3 * Ks columns of an
// activation laid out hi|hi|lo (mask 4) and a weight laid out hi|lo|hi (mask 2) accumulates
//   x_hi w_hi + x_hi w_lo + x_lo w_hi
// in fp32: the bf16x3 product of Henry, Tang and Heinecke ("Leveraging the bfloat16 Artificial
// Intelligence Datatype For Higher-Precision Computations", ARITH 2019).  The dropped x_lo w_lo
// term and the two residuals are each about 2^-16 of the product, so the GEMM matches an fp32
// GEMM to fp32-accumulation accuracy instead of carrying the 2^-9 rounding of bf16 operands.
// (An infinite hi, from an infinite v or one that rounds up past the bf16 range, takes lo = 0 so
// that the sum stays infinite instead of becoming inf - inf.)
ENVG_DEV void split_bf16(float v, __nv_bfloat16& hi, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(v);
  const float h = __bfloat162float(hi);
  lo = __float2bfloat16_rn(isinf(h) ? 0.0f : v - h);
}

// X fp32 [rows][K] (row stride ldx) -> Xs bf16 [rows][3 * Ks], segments per lo_mask.  One thread
// per pair of columns (Ks is even).
__global__ void __launch_bounds__(256) k_cast_x3(const float* __restrict__ X, int64_t ldx, int rows, int K,
                                                    int Ks, __nv_bfloat16* __restrict__ Xs, int lo_mask) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t pairs = (int64_t)rows * (Ks / 2);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < pairs; i += stride) {
    const int64_t r = i / (Ks / 2);
    const int c = (int)(i - r * (Ks / 2)) * 2;
    const float v0 = c < K ? X[r * ldx + c] : 0.0f;
    const float v1 = c + 1 < K ? X[r * ldx + c + 1] : 0.0f;
    __nv_bfloat162 hi, lo;
    split_bf16(v0, hi.x, lo.x);
    split_bf16(v1, hi.y, lo.y);
    __nv_bfloat16* row = Xs + r * 3 * (int64_t)Ks + c;
#pragma unroll
    for (int s = 0; s < 3; ++s)
      *reinterpret_cast<__nv_bfloat162*>(row + (int64_t)s * Ks) = ((lo_mask >> s) & 1) ? lo : hi;
  }
}

// src fp32 [R][C] (row stride lds) -> dst bf16 [C][3 * Rs] (the transpose, split as k_cast_x3;
// zeros for R <= r < Rs).  Rs must be even.  64 x 32 tiles through shared memory.
__global__ void __launch_bounds__(256) k_transpose_cast_x3(const float* __restrict__ src, int64_t lds, int R, int C,
                                                         __nv_bfloat16* __restrict__ dst, int Rs, int lo_mask) {
  __shared__ float t[64][33];
  griddep_wait();
  griddep_launch_dependents();
  const int c0 = blockIdx.x * 32;
  const int r0 = blockIdx.y * 64;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int rr = ty + i * 8;
    const int r = r0 + rr, c = c0 + tx;
    t[rr][tx] = (r < R && c < C) ? src[(int64_t)r * lds + c] : 0.0f;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = threadIdx.x + i * 256;
    const int cc = idx >> 5, rp = idx & 31;
    const int c = c0 + cc, r = r0 + 2 * rp;
    if (c < C && r < Rs) {
      __nv_bfloat162 hi, lo;
      split_bf16(t[2 * rp][cc], hi.x, lo.x);
      split_bf16(t[2 * rp + 1][cc], hi.y, lo.y);
      __nv_bfloat16* row = dst + (int64_t)c * 3 * Rs + r;
#pragma unroll
      for (int s = 0; s < 3; ++s)
        *reinterpret_cast<__nv_bfloat162*>(row + (int64_t)s * Rs) = ((lo_mask >> s) & 1) ? lo : hi;
    }
  }
}

// Explicit im2col for strided convolutions: NHWC bf16 [B][H][W][Cp] -> col bf16
// [B][outH*outW][KH*KW*Cp] in (kh, kw, c) order, zeros outside the image.  8 channels/thread.
__global__ void k_im2col_nhwc(const __nv_bfloat16* __restrict__ in, int B, int H, int W, int Cp, int KH, int KW,
                              int stride, int pad, int outH, int outW, __nv_bfloat16* __restrict__ col) {
  const int c8n = Cp / 8;
  const int64_t total = (int64_t)B * outH * outW * KH * KW * c8n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = i;
    const int c8 = (int)(t % c8n); t /= c8n;
    const int kw = (int)(t % KW); t /= KW;
    const int kh = (int)(t % KH); t /= KH;
    const int ow = (int)(t % outW); t /= outW;
    const int oh = (int)(t % outH); t /= outH;
    const int b = (int)t;
    const int ih = oh * stride - pad + kh, iw = ow * stride - pad + kw;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (ih >= 0 && ih < H && iw >= 0 && iw < W)
      v = *reinterpret_cast<const uint4*>(in + (((int64_t)b * H + ih) * W + iw) * Cp + c8 * 8);
    const int64_t pix = ((int64_t)b * outH + oh) * outW + ow;
    *reinterpret_cast<uint4*>(col + (pix * (KH * KW) + kh * KW + kw) * (int64_t)Cp + c8 * 8) = v;
  }
}

// Adaptive layer norm fused with the activation cast (QNNAdaLN, quicknncpu.pas:3042-3060, then
// the linear's bf16 rounding): per row r, mean and population variance in fp32, then
//   out[r][k] = (1 + scale[k]) * ((x[r][k] - mean) * rsqrt-free 1/sqrt(var + eps)) + shift[k]
// written as bf16 (RNE) into [rows][Kp] with zero padding for the tensor-core paths, or as fp32
// into [rows][K] for k_gemv.  One block per row; the row is re-read from L1 by the later passes.
ENVG_DEV float block_sum256(float v, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (threadIdx.x < 8) ? red[threadIdx.x] : 0.0f;
  if (w == 0) {
#pragma unroll
    for (int off = 4; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
    if (l == 0) red[8] = t;
  }
  __syncthreads();
  return red[8];
}

__global__ void __launch_bounds__(256) k_adaln(const float* __restrict__ X, int64_t ldx, int K, int Kp,
                                               const float* __restrict__ shift, const float* __restrict__ scale,
                                               float eps, void* out, int out_bf16) {
  __shared__ float red[9];
  griddep_wait();
  griddep_launch_dependents();
  const int64_t r = blockIdx.x;
  const float* xr = X + r * ldx;
  float s = 0.0f;
  for (int k = threadIdx.x; k < K; k += 256) s += xr[k];
  const float mean = block_sum256(s, red) / (float)K;
  float q = 0.0f;
  for (int k = threadIdx.x; k < K; k += 256) {
    const float dlt = xr[k] - mean;
    q = fmaf(dlt, dlt, q);
  }
  const float var = block_sum256(q, red) / (float)K;
  const float inv = 1.0f / sqrtf(var + eps);
  if (out_bf16) {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out) + r * Kp;
    for (int k = threadIdx.x; k < Kp; k += 256) {
      float v = 0.0f;
      if (k < K) {
        const float norm = __fmul_rn(__fsub_rn(xr[k], mean), inv);
        v = __fadd_rn(__fmul_rn(__fadd_rn(1.0f, __ldg(scale + k)), norm), __ldg(shift + k));
      }
      o[k] = __float2bfloat16_rn(v);
    }
  } else {
    float* o = reinterpret_cast<float*>(out) + r * K;
    for (int k = threadIdx.x; k < K; k += 256) {
      const float norm = __fmul_rn(__fsub_rn(xr[k], mean), inv);
      o[k] = __fadd_rn(__fmul_rn(__fadd_rn(1.0f, __ldg(scale + k)), norm), __ldg(shift + k));
    }
  }
}

// QNNRMSNorm per row (src/quicknncpu.pas:2159-2185), fused with the activation cast: one CTA per
// row; inv = 1 / sqrt(sum(x^2) / K + eps), out = (x * weight) * inv, or x * inv when weight is
// NULL.  bf16 output is zero-padded to Kp columns (the GEMM operand), fp32 output has K columns.
__global__ void __launch_bounds__(256) k_rmsnorm(const float* __restrict__ X, int64_t ldx, int K, int Kp,
                                                 const float* __restrict__ weight, float eps, void* out, int out_bf16) {
  __shared__ float red[9];
  griddep_wait();
  griddep_launch_dependents();
  const int64_t r = blockIdx.x;
  const float* xr = X + r * ldx;
  float q = 0.0f;
  for (int k = threadIdx.x; k < K; k += 256) q = fmaf(xr[k], xr[k], q);
  const float ms = block_sum256(q, red) / (float)K;
  const float inv = 1.0f / sqrtf(ms + eps);
  if (out_bf16) {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out) + r * Kp;
    for (int k = threadIdx.x; k < Kp; k += 256) {
      float v = 0.0f;
      if (k < K) v = weight ? __fmul_rn(__fmul_rn(xr[k], __ldg(weight + k)), inv) : __fmul_rn(xr[k], inv);
      o[k] = __float2bfloat16_rn(v);
    }
  } else {
    float* o = reinterpret_cast<float*>(out) + r * K;
    for (int k = threadIdx.x; k < K; k += 256)
      o[k] = weight ? __fmul_rn(__fmul_rn(xr[k], __ldg(weight + k)), inv) : __fmul_rn(xr[k], inv);
  }
}

// ---- GroupNorm (QNNGroupNorm, src/quicknncpu.pas:2259-2313) --------------------------------
// Group (b, g) of an NCHW tensor is the contiguous run of cpg * HW floats starting at
// (b*C + g*cpg) * HW.  Statistics are taken in two launches:
//   k_group_stats   grid (chunks, B*G): each CTA takes GN_CHUNK consecutive floats of one group
//                   and writes {count, mean, M2} of its chunk (two passes over registers);
//   k_group_affine  one warp per (b, g): merges its group's chunks (Chan et al.'s pairwise
//                   update, fp64, fixed order), then var = M2 / n (population, as QNNVariance),
//                   std_inv = 1 / sqrt(var + eps) and the per-channel affine
//                   a = gamma_c * std_inv, s = beta_c - mean * gamma_c * std_inv (QNNFusedScaleBias).
constexpr int GN_THREADS = 256;
constexpr int GN_PER_THREAD = 32;
constexpr int GN_CHUNK = GN_THREADS * GN_PER_THREAD;  // 8192 floats

ENVG_DEV double block_sum256_d(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < GN_THREADS / 32; ++i) t += red[i];
    red[8] = t;
  }
  __syncthreads();
  return red[8];
}

ENVG_DEV void group_stats_block(const float* __restrict__ X, int C, int64_t HW, int cpg, int groups,
                                double* __restrict__ part, int chunks) {
  __shared__ double red[9];
  const int bg = blockIdx.y;
  const int b = bg / groups, g = bg - b * groups;
  const int64_t n = (int64_t)cpg * HW;
  const int64_t c0 = (int64_t)blockIdx.x * GN_CHUNK;
  const int64_t cn = min((int64_t)GN_CHUNK, n - c0);
  const float* src = X + ((int64_t)b * C + (int64_t)g * cpg) * HW + c0;
  float v[GN_PER_THREAD];
  float s = 0.0f;
  if ((HW & 3) == 0 && (reinterpret_cast<uintptr_t>(X) & 15) == 0) {
    // 16-byte loads: thread t takes float4 t, t + 256, ... (cn is a multiple of 4 here)
#pragma unroll
    for (int i = 0; i < GN_PER_THREAD / 4; ++i) {
      const int64_t k = 4 * ((int64_t)threadIdx.x + (int64_t)i * GN_THREADS);
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k < cn) x = __ldg(reinterpret_cast<const float4*>(src + k));
      v[4 * i] = x.x, v[4 * i + 1] = x.y, v[4 * i + 2] = x.z, v[4 * i + 3] = x.w;
      s += (x.x + x.y) + (x.z + x.w);
    }
  } else {
#pragma unroll
    for (int i = 0; i < GN_PER_THREAD; ++i) {
      const int64_t k = threadIdx.x + (int64_t)i * GN_THREADS;
      v[i] = k < cn ? __ldg(src + k) : 0.0f;
      s += v[i];
    }
  }
  const double mean = block_sum256_d((double)s, red) / (double)cn;
  const float mf = (float)mean;
  // padding slots hold 0 and must not count: they sit beyond cn in both layouts
  float q = 0.0f;
  const bool vec = (HW & 3) == 0 && (reinterpret_cast<uintptr_t>(X) & 15) == 0;
#pragma unroll
  for (int i = 0; i < GN_PER_THREAD; ++i) {
    const int64_t k = vec ? 4 * ((int64_t)threadIdx.x + (int64_t)(i >> 2) * GN_THREADS) + (i & 3)
                          : threadIdx.x + (int64_t)i * GN_THREADS;
    const float dl = v[i] - mf;
    if (k < cn) q = __fmaf_rn(dl, dl, q);
  }
  const double m2 = block_sum256_d((double)q, red);
  if (threadIdx.x == 0) {
    // M2 about the chunk mean: shift the fp32 deviations' sum back from mf to mean
    const double dm = mean - (double)mf;
    double* o = part + ((int64_t)bg * chunks + blockIdx.x) * 3;
    o[0] = (double)cn;
    o[1] = mean;
    o[2] = m2 - (double)cn * dm * dm;
  }
}

__global__ void __launch_bounds__(GN_THREADS) k_group_stats(const float* __restrict__ X, int C, int64_t HW, int cpg,
                                                            int groups, double* __restrict__ part, int chunks) {
  group_stats_block(X, C, HW, cpg, groups, part, chunks);
}

// Chan et al.'s pairwise update: (n, mean, m2) <- (n, mean, m2) merged with (nb, mb, qb).
ENVG_DEV void chan_merge(double& n, double& mean, double& m2, double nb, double mb, double qb) {
  if (nb == 0.0) return;
  if (n == 0.0) {
    n = nb, mean = mb, m2 = qb;
    return;
  }
  const double nn = n + nb, dl = mb - mean;
  mean += dl * (nb / nn);
  m2 += qb + dl * dl * (n * nb / nn);
  n = nn;
}

// Group wid = (b, g) by one warp: lane l merges chunks l, l + 32, ... in order, then a fixed
// shuffle tree merges the lanes (deterministic); the warp writes the group's per-channel affine.
ENVG_DEV void group_affine_warp(int wid, int lane, const double* __restrict__ part, int chunks, int C, int cpg,
                                int groups, const float* __restrict__ gamma, const float* __restrict__ beta,
                                float eps, float2* __restrict__ aff) {
  const int b = wid / groups, g = wid - b * groups;
  const double* p = part + (int64_t)wid * chunks * 3;
  double n = 0.0, mean = 0.0, m2 = 0.0;
  for (int k = lane; k < chunks; k += 32) chan_merge(n, mean, m2, p[3 * k], p[3 * k + 1], p[3 * k + 2]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double nb = __shfl_down_sync(0xffffffffu, n, o);
    const double mb = __shfl_down_sync(0xffffffffu, mean, o);
    const double qb = __shfl_down_sync(0xffffffffu, m2, o);
    if (lane < o) chan_merge(n, mean, m2, nb, mb, qb);
  }
  n = __shfl_sync(0xffffffffu, n, 0);
  mean = __shfl_sync(0xffffffffu, mean, 0);
  m2 = __shfl_sync(0xffffffffu, m2, 0);
  const float var = (float)(m2 / n);
  const float std_inv = 1.0f / sqrtf(var + eps);
  const float mf = (float)mean;
  for (int c = g * cpg + lane; c < (g + 1) * cpg; c += 32) {
    const float ga = gamma ? __ldg(gamma + c) : 1.0f;
    const float be = beta ? __ldg(beta + c) : 0.0f;
    const float a = __fmul_rn(ga, std_inv);
    aff[(int64_t)b * C + c] = make_float2(a, __fsub_rn(be, __fmul_rn(__fmul_rn(mf, ga), std_inv)));
  }
}

__global__ void __launch_bounds__(256) k_group_affine(const double* __restrict__ part, int chunks, int batch, int C,
                                                      int cpg, int groups, const float* __restrict__ gamma,
                                                      const float* __restrict__ beta, float eps,
                                                      float2* __restrict__ aff) {
  const int wid = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  if (wid >= batch * groups) return;
  group_affine_warp(wid, threadIdx.x & 31, part, chunks, C, cpg, groups, gamma, beta, eps, aff);
}

// dst[b][c][i] = act(src[b][c][i] * aff[b*C + c].x + aff[b*C + c].y), fp32 NCHW (in place allowed).
__global__ void __launch_bounds__(256) k_group_apply(const float* src, float* dst, int64_t HW, int BC,
                                                     const float2* __restrict__ aff, int act) {
  const int64_t total = (int64_t)BC * HW;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const float2 a = __ldg(aff + i / HW);
    float v = __fmaf_rn(src[i], a.x, a.y);
    if (act) v = silu_f(v);
    dst[i] = v;
  }
}

// Self-test of the bounded wait: one CTA waits on a barrier nothing arrives at.
__global__ void k_wait_selftest(int* status, uint64_t cap_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const WaitCtl wc{cap_ns, status, &abort_flag, 0};
    wait_bounded(smem_u32(&bar), 0, wc, 99);
  }
}

}  // namespace envg
