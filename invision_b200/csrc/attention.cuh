// attention.cuh -- multi-head attention forward on tcgen05 (flash-attention schedule).
//
// Replaces, per head, the reference's cblas_gemm(Q, K^T) -> QNNSoftmaxRows -> cblas_gemm(P, V)
// (src/quicknn_transformers.pas:1150-1200 TTransformerFlux.multiHeadForward, :1202-1270
// jointAttentionForward; src/quicknn_qwen3.pas:726-768 with GQA and the causal
// QNNMatTriangularFill).  The [seq_q, seq_k] score matrix never leaves the SM:
//
//   k_attention, one CTA per (128 query rows, head), 192 threads:
//     warp 0      TMA producer: the Q tile once, then (K_j, V_j) blocks of 128 keys through a
//                 2-stage ring (64 KB per stage);
//     warp 1      one thread issues the UMMAs: S_j = Q K_j^T into one of two TMEM score buffers,
//                 and O += P_j V_j into the TMEM output accumulator;
//     warps 2-5   softmax, one query row per thread (TMEM lane quadrant = warp % 4): row max,
//                 p = 2^(s * scale * log2e - m), the running sum, P_j as fp16 into shared memory
//                 in the 128-byte-swizzled K-major layout the next UMMA reads; at the end
//                 O / sum goes to the fp32 output.
//   The running max is only moved (and O rescaled in TMEM) when a row's maximum grows by more
//   than 2^8; between moves p <= 2^8, well inside the fp16 range, and the final O / sum is
//   unchanged by the choice of reference point.
//   S_{j+1} is computed while the softmax works on S_j.
//
// Operands (written by the prep kernels below, launched from envgemm.cu):
//   Qh [heads][sq_pad][128] fp16, Kh [kv_heads][sk_pad][128] fp16, Vt [kv_heads][128][sk_pad]
//   fp16 (V transposed so that both UMMAs read K-major operands), key bits [sk_pad / 32]:
//   bit c set when key c exists (c < seq_k) and is not masked.
// Precision: all three UMMA operands are fp16 (kind::f16, fp32 accumulation).  fp16 carries 11
// significant bits against bf16's 8, so the rounding of Q and K -- which dominates the error of
// a bf16 attention -- shrinks 8x.  Range is kept safe by an exact power-of-two scale per head and
// tensor (fa_pow2_scale of the head's max |x|, from k_absmax_heads): scaled values stay below
// 2^14, and the kernel divides the scales back out (scores by sq * sk, the output by sv).
// P = 2^(s - m) <= 2^8 fits fp16 as it is.
#pragma once
#include <cuda_fp16.h>

#include "kernels.cuh"

namespace envg {

constexpr int FA_D = 128;                 // head dimension
constexpr int FA_BQ = 128;                // query rows per CTA (TMEM lanes)
constexpr int FA_BKV = 128;               // keys per block
constexpr int FA_THREADS = 192;
constexpr int FA_SUB = 128 * 64 * 2;      // one 128-row x 64-column fp16 swizzled sub-tile (16 KB)
constexpr int FA_TILE = 2 * FA_SUB;       // a 128 x 128 fp16 tile (32 KB)
constexpr int FA_STAGES = 2;
constexpr int FA_TMEM_COLS = 512;         // S0 [0,128), S1 [128,256), O [256,384)
constexpr float FA_RESCALE_LOG2 = 8.0f;   // move the reference max only beyond 2^8 growth

struct FaSmem {
  static constexpr int Q = 0;
  static constexpr int KV = FA_TILE;                           // stage s: K, then V
  static constexpr int P = KV + FA_STAGES * 2 * FA_TILE;
  static constexpr int BARS = P + FA_TILE;
  static constexpr int NBARS = 1 + 2 * FA_STAGES + 2 + 1 + 1 + 1;
  static constexpr int END = BARS + NBARS * 8 + 16;
  static constexpr int TOTAL = END + 1024;                     // + slack for 1024-byte alignment
};

struct FaArgs {
  int seq_q, seq_k, heads, kv_heads;
  int sq_pad, sk_pad;
  int causal;
  float sl2;                 // scale * log2(e)
  const uint32_t* kbits;     // key validity bits
  int full_blocks;           // leading key blocks whose keys are all valid (no mask, inside seq_k)
  const float* amax;         // max |x| per head: Q [heads], then K [kv_heads], then V [kv_heads]
  float* out;                // fp32 [seq_q][ldo], head h at column h * 128
  int64_t ldo;
  int* status;
  uint64_t wait_cap_ns;
};

// Three-input max and packed fp32 pairs (sm_100): each lane of fma/add.rn.f32x2 rounds exactly
// as the scalar instruction does.
ENVG_DEV float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
ENVG_DEV uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
ENVG_DEV void f2_unpack(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
ENVG_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
ENVG_DEV uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// D[tmem] <- 32 registers per thread (32 lanes x 32 columns); completion by tmem_st_wait.
ENVG_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
ENVG_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 64 consecutive 32-bit columns -> 64 registers per thread, without the wait: the
// caller issues tmem_ld_wait() before any use of r.
ENVG_DEV void tmem_ld64_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
}
ENVG_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Instruction descriptor, kind::f16 with fp16 A and B (type fields 0), fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// 2^e such that amax * 2^e lies in [2^13, 2^14) (1 for zero or non-finite amax).
ENVG_DEV float fa_pow2_scale(float amax) {
  if (!(amax > 0.0f) || !isfinite(amax)) return 1.0f;
  int ex;
  frexpf(amax, &ex);  // amax = m * 2^ex, 0.5 <= m < 1
  return ldexpf(1.0f, max(-120, min(120, 14 - ex)));
}

// 2^x with the hardware approximation (PTX ex2.approx.ftz.f32; 2^-inf = 0).
ENVG_DEV float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Eight floats -> eight fp16 (RNE) in one 16-byte word.
ENVG_DEV uint4 pack_half8(const float* v) {
  uint4 o;
  __half2 h0 = __floats2half2_rn(v[0], v[1]);
  __half2 h1 = __floats2half2_rn(v[2], v[3]);
  __half2 h2 = __floats2half2_rn(v[4], v[5]);
  __half2 h3 = __floats2half2_rn(v[6], v[7]);
  o.x = *reinterpret_cast<uint32_t*>(&h0);
  o.y = *reinterpret_cast<uint32_t*>(&h1);
  o.z = *reinterpret_cast<uint32_t*>(&h2);
  o.w = *reinterpret_cast<uint32_t*>(&h3);
  return o;
}

__global__ void __launch_bounds__(FA_THREADS, 1)
    k_attention(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const FaArgs a) {
  constexpr uint32_t IDESC = idesc_f16_f32(FA_BQ, 128);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm + FaSmem::Q;
  uint8_t* sKV = sm + FaSmem::KV;
  uint8_t* sP = sm + FaSmem::P;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + FaSmem::BARS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + FaSmem::NBARS);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t q_full = smem_u32(bars);
  const uint32_t kv_full0 = q_full + 8;
  const uint32_t kv_empty0 = kv_full0 + 8 * FA_STAGES;
  const uint32_t s_full0 = kv_empty0 + 8 * FA_STAGES;
  const uint32_t p_full = s_full0 + 16;
  const uint32_t o_done = p_full + 8;
  const uint32_t drain = o_done + 8;

  const int h = blockIdx.y;
  const int kvh = h / (a.heads / a.kv_heads);
  const int q0 = blockIdx.x * FA_BQ;
  const int64_t coff = (int64_t)a.seq_k - a.seq_q;  // causal: key c visible to row r if c <= r + coff
  int nb = (a.seq_k + FA_BKV - 1) / FA_BKV;
  if (a.causal) {
    const int64_t last = (int64_t)q0 + FA_BQ - 1 + coff;  // last key any row of this tile sees
    nb = (int)min((int64_t)nb, last / FA_BKV + 1);
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < FA_STAGES; ++s) {
      mbar_init(kv_full0 + 8 * s, 1);
      mbar_init(kv_empty0 + 8 * s, 1);
    }
    mbar_init(s_full0, 1);
    mbar_init(s_full0 + 8, 1);
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_s = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), FA_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtl wc{a.wait_cap_ns, a.status, abort_s, 0};

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t pending = 0, issue_ph = 0;
      mbar_arrive_expect_tx(q_full, FA_TILE);
      tma_load_2d(smem_u32(sQ), &tmQ, q_full, 0, h * a.sq_pad + q0);
      tma_load_2d(smem_u32(sQ + FA_SUB), &tmQ, q_full, 64, h * a.sq_pad + q0);
      for (int j = 0; j < nb; ++j) {
        const int stage = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!wait_bounded(kv_empty0 + 8 * stage, ph ^ 1u, wc, 21)) break;
        const uint32_t fb = kv_full0 + 8 * stage;
        uint8_t* sK = sKV + stage * 2 * FA_TILE;
        uint8_t* sV = sK + FA_TILE;
        mbar_arrive_expect_tx(fb, 2 * FA_TILE);
        tma_load_2d(smem_u32(sK), &tmK, fb, 0, kvh * a.sk_pad + j * FA_BKV);
        tma_load_2d(smem_u32(sK + FA_SUB), &tmK, fb, 64, kvh * a.sk_pad + j * FA_BKV);
        tma_load_2d(smem_u32(sV), &tmV, fb, j * FA_BKV, kvh * FA_D);
        tma_load_2d(smem_u32(sV + FA_SUB), &tmV, fb, j * FA_BKV + 64, kvh * FA_D);
        pending |= 1u << stage;
        issue_ph = (issue_ph & ~(1u << stage)) | (ph << stage);
      }
      if (*abort_s) {
        // every copy this thread started lands before the CTA's shared memory is released
        wait_drain(q_full, 0, a.wait_cap_ns);
        for (int s = 0; s < FA_STAGES; ++s)
          if (pending & (1u << s)) wait_drain(kv_full0 + 8 * s, (issue_ph >> s) & 1u, a.wait_cap_ns);
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer ----------------
    if (lane == 0) {
      bool ok = wait_bounded(q_full, 0, wc, 22);
      tc_fence_after();
      const uint64_t qd0 = sw128_kmajor_desc(smem_u32(sQ));
      const uint64_t qd1 = sw128_kmajor_desc(smem_u32(sQ + FA_SUB));
      const uint64_t pd0 = sw128_kmajor_desc(smem_u32(sP));
      const uint64_t pd1 = sw128_kmajor_desc(smem_u32(sP + FA_SUB));
      for (int j = 0; ok && j <= nb; ++j) {
        if (j < nb) {
          const int stage = j & 1;
          if (!wait_bounded(kv_full0 + 8 * stage, (uint32_t)(j >> 1) & 1u, wc, 23)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* sK = sKV + stage * 2 * FA_TILE;
          const uint64_t kd0 = sw128_kmajor_desc(smem_u32(sK));
          const uint64_t kd1 = sw128_kmajor_desc(smem_u32(sK + FA_SUB));
          const uint32_t d = tmem_base + (uint32_t)((j & 1) * 128);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint64_t ad = (k < 4 ? qd0 : qd1) + 2 * (k & 3);
            const uint64_t bd = (k < 4 ? kd0 : kd1) + 2 * (k & 3);
            umma_bf16(d, ad, bd, IDESC, k > 0 ? 1u : 0u);
          }
          umma_commit(s_full0 + 8 * (j & 1));
        }
        if (j >= 1) {
          const int i = j - 1;
          if (!wait_bounded(p_full, (uint32_t)i & 1u, wc, 24)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int stage = i & 1;
          const uint8_t* sV = sKV + stage * 2 * FA_TILE + FA_TILE;
          const uint64_t vd0 = sw128_kmajor_desc(smem_u32(sV));
          const uint64_t vd1 = sw128_kmajor_desc(smem_u32(sV + FA_SUB));
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint64_t ad = (k < 4 ? pd0 : pd1) + 2 * (k & 3);
            const uint64_t bd = (k < 4 ? vd0 : vd1) + 2 * (k & 3);
            umma_bf16(tmem_base + 256, ad, bd, IDESC, (i > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(o_done);
          umma_commit(kv_empty0 + 8 * stage);
        }
      }
      if (*abort_s) {
        umma_commit(drain);
        wait_drain(drain, 0, a.wait_cap_ns);
      }
    }
  } else {
    // ---------------- softmax: 4 warps, one query row per thread ----------------
    const int qd = warp & 3;
    const int prow = qd * 32 + lane;           // row inside the tile
    const int row = q0 + prow;                 // query row
    const uint32_t tl = tmem_base + ((uint32_t)(qd * 32) << 16);
    const int64_t climit = a.causal ? (int64_t)row + coff : INT64_MAX;
    // undo the operand scales: scores by sq * sk, the output by sv (powers of two: exact)
    const float sq = fa_pow2_scale(__ldg(a.amax + h));
    const float sk = fa_pow2_scale(__ldg(a.amax + a.heads + kvh));
    const float sv = fa_pow2_scale(__ldg(a.amax + a.heads + a.kv_heads + kvh));
    const float sl2 = a.sl2 / (sq * sk);
    float m_use = -INFINITY, lsum = 0.0f;
    bool ok = true;
    for (int j = 0; j < nb; ++j) {
      if (!wait_bounded_warp(s_full0 + 8 * (j & 1), (uint32_t)(j >> 1) & 1u, wc, 25)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sb = tl + (uint32_t)((j & 1) * 128);
      const int kc0 = j * FA_BKV;
      // the whole score row of this block in registers (one TMEM round trip)
      uint32_t r[128];
      tmem_ld64_nowait(sb, r);
      tmem_ld64_nowait(sb + 64, r + 64);
      tmem_ld_wait();
      // masks only where the block is not fully visible to every row of the warp; blocks before
      // full_blocks need no validity bits (no key mask, inside seq_k)
      const bool full = j < a.full_blocks && (int64_t)kc0 + FA_BKV - 1 <= climit;
      if (!__all_sync(0xffffffffu, full)) {
        const uint32_t w0 = __ldg(a.kbits + (kc0 >> 5)), w1 = __ldg(a.kbits + (kc0 >> 5) + 1);
        const uint32_t w2 = __ldg(a.kbits + (kc0 >> 5) + 2), w3 = __ldg(a.kbits + (kc0 >> 5) + 3);
        const uint32_t wd[4] = {w0, w1, w2, w3};
#pragma unroll
        for (int t = 0; t < 128; ++t) {
          const bool vis = ((wd[t >> 5] >> (t & 31)) & 1u) && (int64_t)(kc0 + t) <= climit;
          if (!vis) r[t] = 0xff800000u;  // -inf
        }
      }
      // row maximum: four chains of three-input maxima
      float mx4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) mx4[u] = __uint_as_float(r[u]);
#pragma unroll
      for (int t = 4; t < 124; t += 8)
#pragma unroll
        for (int u = 0; u < 4; ++u)
          mx4[u] = fmax3(mx4[u], __uint_as_float(r[t + 2 * u]), __uint_as_float(r[t + 2 * u + 1]));
      const float mx = fmax3(fmax3(mx4[0], mx4[1], mx4[2]), mx4[3],
                             fmax3(__uint_as_float(r[124]), __uint_as_float(r[125]),
                                   fmaxf(__uint_as_float(r[126]), __uint_as_float(r[127]))));
      const float m_cand = mx * sl2;
      float factor = 1.0f;
      bool rescale = false;
      if (j == 0) {
        m_use = m_cand;
      } else {
        rescale = __any_sync(0xffffffffu, m_cand > m_use + FA_RESCALE_LOG2);
        if (rescale) {
          const float m_new = fmaxf(m_use, m_cand);
          factor = (m_new == -INFINITY) ? 1.0f : ex2_approx(m_use - m_new);
          m_use = m_new;
          lsum *= factor;
        }
      }
      // p = 2^(s * sl2 - m) in place, a pair of columns per step: one packed FMA, two ex2, one
      // packed add into four pair accumulators (lane-wise the same sums as eight scalar ones)
      const float msub = (m_use == -INFINITY) ? 0.0f : m_use;
      const uint64_t sl2_2 = f2_pack(sl2, sl2), nm_2 = f2_pack(-msub, -msub);
      uint64_t ps2[4] = {0, 0, 0, 0};
#pragma unroll
      for (int t = 0; t < 128; t += 2) {
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(__uint_as_float(r[t]), __uint_as_float(r[t + 1])), sl2_2, nm_2), x0, x1);
        const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
        ps2[(t >> 1) & 3] = f2_add(ps2[(t >> 1) & 3], f2_pack(p0, p1));
        r[t] = __float_as_uint(p0);
        r[t + 1] = __float_as_uint(p1);
      }
      float ps8[8];
#pragma unroll
      for (int u = 0; u < 4; ++u) f2_unpack(ps2[u], ps8[2 * u], ps8[2 * u + 1]);
      lsum += ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
      if (j > 0) {
        // P and O are free once PV_{j-1} is complete
        if (!wait_bounded_warp(o_done, (uint32_t)(j - 1) & 1u, wc, 26)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (rescale) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tl + 256 + c * 32, o);
#pragma unroll
            for (int t = 0; t < 32; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * factor);
            tmem_st32(tl + 256 + c * 32, o);
          }
          tmem_st_wait();
        }
      }
      // P (fp16) into shared memory, 128-byte swizzled K-major rows
#pragma unroll
      for (int ch = 0; ch < 16; ++ch) {
        uint8_t* rowp = sP + (ch >> 3) * FA_SUB + prow * 128;
        *reinterpret_cast<uint4*>(rowp + (((ch & 7) ^ (prow & 7)) << 4)) =
            pack_half8(reinterpret_cast<const float*>(r) + 8 * ch);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // O / sum -> fp32 output
    if (ok && nb > 0 && wait_bounded_warp(o_done, (uint32_t)(nb - 1) & 1u, wc, 27)) {
      tc_fence_after();
      const float inv = lsum > 0.0f ? 1.0f / (lsum * sv) : 0.0f;
      float* orow = a.out + (int64_t)row * a.ldo + (int64_t)h * FA_D;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tl + 256 + c * 32, r);
        if (row < a.seq_q) {
#pragma unroll
          for (int t = 0; t < 32; t += 4)
            *reinterpret_cast<float4*>(orow + c * 32 + t) =
                make_float4(__uint_as_float(r[t]) * inv, __uint_as_float(r[t + 1]) * inv,
                            __uint_as_float(r[t + 2]) * inv, __uint_as_float(r[t + 3]) * inv);
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, FA_TMEM_COLS);
  }
}

// ---- two query tiles per CTA ------------------------------------------------------------------
// k_attention2: 256 query rows (tiles 0 and 1) of one head per CTA, 320 threads: warp 0 TMA,
// warp 1 UMMA issuer, warps 2-5 softmax of tile 0, warps 6-9 softmax of tile 1 (two softmax warps
// per SM sub-partition).  K and V blocks are loaded once for both tiles.  TMEM: S_t at columns
// [128t, 128t+128), O_t at [256 + 128t, ...).  The softmax writes P_t (fp16, packed two per
// column) over the first 64 columns of S_t, and the PV product reads it from there as its A
// operand (tcgen05.mma with A in tensor memory).  The UMMA thread issues S_t(j+1) only after the
// commit of PV_t(j) has arrived, so the overwrite of P_t is ordered after its last read; O_t is
// quiescent while softmax t works (PV_t(j-1) completed before S_t(j) was issued), which is when
// the softmax may rescale it.
constexpr int FA2_THREADS = 320;

struct Fa2Smem {
  static constexpr int Q = 0;                                  // tile t: Q at t * FA_TILE
  static constexpr int KV = 2 * FA_TILE;                       // stage s: K, then V
  static constexpr int BARS = KV + FA_STAGES * 2 * FA_TILE;
  static constexpr int NBARS = 1 + 2 * FA_STAGES + 2 + 2 + 2 + 1;  // q, kv full/empty, s, p, pv, drain
  static constexpr int END = BARS + NBARS * 8 + 16;
  static constexpr int TOTAL = END + 1024;
};

// D[tmem] += A[tmem] . B[smem]^T (A: 128 lanes x 16 fp16 packed in 8 columns), one thread.
ENVG_DEV void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 64 registers per thread -> 32 lanes x 64 consecutive columns; completion by tmem_st_wait.
ENVG_DEV void tmem_st64(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,"
      "%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,"
      "%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]), "r"(r[32]),
      "r"(r[33]), "r"(r[34]), "r"(r[35]), "r"(r[36]), "r"(r[37]), "r"(r[38]), "r"(r[39]), "r"(r[40]),
      "r"(r[41]), "r"(r[42]), "r"(r[43]), "r"(r[44]), "r"(r[45]), "r"(r[46]), "r"(r[47]), "r"(r[48]),
      "r"(r[49]), "r"(r[50]), "r"(r[51]), "r"(r[52]), "r"(r[53]), "r"(r[54]), "r"(r[55]), "r"(r[56]),
      "r"(r[57]), "r"(r[58]), "r"(r[59]), "r"(r[60]), "r"(r[61]), "r"(r[62]), "r"(r[63])
      : "memory");
}

__global__ void __launch_bounds__(FA2_THREADS, 1)
    k_attention2(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const FaArgs a) {
  constexpr uint32_t IDESC = idesc_f16_f32(FA_BQ, 128);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm + Fa2Smem::Q;
  uint8_t* sKV = sm + Fa2Smem::KV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Fa2Smem::BARS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Fa2Smem::NBARS);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t q_full = smem_u32(bars);
  const uint32_t kv_full0 = q_full + 8;
  const uint32_t kv_empty0 = kv_full0 + 8 * FA_STAGES;
  const uint32_t s_full0 = kv_empty0 + 8 * FA_STAGES;  // [t]
  const uint32_t p_full0 = s_full0 + 16;               // [t]
  const uint32_t pv_done0 = p_full0 + 16;              // [t]
  const uint32_t drain = pv_done0 + 16;

  const int h = blockIdx.y;
  const int kvh = h / (a.heads / a.kv_heads);
  const int q0 = blockIdx.x * 2 * FA_BQ;
  const int64_t coff = (int64_t)a.seq_k - a.seq_q;
  int nb = (a.seq_k + FA_BKV - 1) / FA_BKV;
  if (a.causal) {
    const int64_t last = (int64_t)q0 + 2 * FA_BQ - 1 + coff;
    nb = (int)min((int64_t)nb, last / FA_BKV + 1);
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < FA_STAGES; ++s) {
      mbar_init(kv_full0 + 8 * s, 1);
      mbar_init(kv_empty0 + 8 * s, 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full0 + 8 * t, 1);
      mbar_init(p_full0 + 8 * t, 4);
      mbar_init(pv_done0 + 8 * t, 1);
    }
    mbar_init(drain, 1);
    *abort_s = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), FA_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtl wc{a.wait_cap_ns, a.status, abort_s, 0};

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t pending = 0, issue_ph = 0;
      mbar_arrive_expect_tx(q_full, 2 * FA_TILE);
      for (int t = 0; t < 2; ++t) {
        tma_load_2d(smem_u32(sQ + t * FA_TILE), &tmQ, q_full, 0, h * a.sq_pad + q0 + t * FA_BQ);
        tma_load_2d(smem_u32(sQ + t * FA_TILE + FA_SUB), &tmQ, q_full, 64, h * a.sq_pad + q0 + t * FA_BQ);
      }
      for (int j = 0; j < nb; ++j) {
        const int stage = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!wait_bounded(kv_empty0 + 8 * stage, ph ^ 1u, wc, 31)) break;
        const uint32_t fb = kv_full0 + 8 * stage;
        uint8_t* sK = sKV + stage * 2 * FA_TILE;
        uint8_t* sV = sK + FA_TILE;
        mbar_arrive_expect_tx(fb, 2 * FA_TILE);
        tma_load_2d(smem_u32(sK), &tmK, fb, 0, kvh * a.sk_pad + j * FA_BKV);
        tma_load_2d(smem_u32(sK + FA_SUB), &tmK, fb, 64, kvh * a.sk_pad + j * FA_BKV);
        tma_load_2d(smem_u32(sV), &tmV, fb, j * FA_BKV, kvh * FA_D);
        tma_load_2d(smem_u32(sV + FA_SUB), &tmV, fb, j * FA_BKV + 64, kvh * FA_D);
        pending |= 1u << stage;
        issue_ph = (issue_ph & ~(1u << stage)) | (ph << stage);
      }
      if (*abort_s) {
        wait_drain(q_full, 0, a.wait_cap_ns);
        for (int s = 0; s < FA_STAGES; ++s)
          if (pending & (1u << s)) wait_drain(kv_full0 + 8 * s, (issue_ph >> s) & 1u, a.wait_cap_ns);
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer ----------------
    if (lane == 0) {
      bool ok = wait_bounded(q_full, 0, wc, 32) && wait_bounded(kv_full0, 0, wc, 33);
      tc_fence_after();
      uint64_t qd[2][2];
      for (int t = 0; t < 2; ++t) {
        qd[t][0] = sw128_kmajor_desc(smem_u32(sQ + t * FA_TILE));
        qd[t][1] = sw128_kmajor_desc(smem_u32(sQ + t * FA_TILE + FA_SUB));
      }
      auto issue_s = [&](int t, int j) {
        const uint8_t* sK = sKV + (j & 1) * 2 * FA_TILE;
        const uint64_t kd0 = sw128_kmajor_desc(smem_u32(sK));
        const uint64_t kd1 = sw128_kmajor_desc(smem_u32(sK + FA_SUB));
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_bf16(tmem_base + (uint32_t)(t * 128), qd[t][k >> 2] + 2 * (k & 3), (k < 4 ? kd0 : kd1) + 2 * (k & 3),
                    IDESC, k > 0 ? 1u : 0u);
        umma_commit(s_full0 + 8 * t);
      };
      // Tile 1 starts one softmax behind tile 0 (its first S is issued with tile 0's first PV),
      // so the two softmax warpgroups alternate instead of running in lock-step.
      if (ok) issue_s(0, 0);
      bool s1_started = false;
      // Per block j and tile t: PV_t(j) as soon as P_t(j) is ready, then S_t(j+1) once PV_t(j) has
      // read P_t; tile 0 never waits for tile 1's softmax, so the two softmax warpgroups drift
      // apart and each runs while the tensor pipe works for the other.
      for (int j = 0; ok && j < nb; ++j) {
        const int stage = j & 1;
        const uint8_t* sV = sKV + stage * 2 * FA_TILE + FA_TILE;
        const uint64_t vd0 = sw128_kmajor_desc(smem_u32(sV));
        const uint64_t vd1 = sw128_kmajor_desc(smem_u32(sV + FA_SUB));
        const bool more = j + 1 < nb;
        for (int t = 0; t < 2; ++t) {
          if (t == 1 && !s1_started) {
            issue_s(1, 0);
            s1_started = true;
          }
          if (!wait_bounded(p_full0 + 8 * t, (uint32_t)j & 1u, wc, 34)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 8; ++k)
            umma_f16_ts(tmem_base + 256 + (uint32_t)(t * 128), tmem_base + (uint32_t)(t * 128 + 8 * k),
                        (k < 4 ? vd0 : vd1) + 2 * (k & 3), IDESC, (j > 0 || k > 0) ? 1u : 0u);
          umma_commit(pv_done0 + 8 * t);
          if (t == 1) umma_commit(kv_empty0 + 8 * stage);
          if (!more) continue;
          if (t == 0 && !wait_bounded(kv_full0 + 8 * ((j + 1) & 1), (uint32_t)((j + 1) >> 1) & 1u, wc, 35)) {
            ok = false;
            break;
          }
          // P_t(j) (in S_t's columns) must be consumed before S_t(j+1) overwrites them
          if (!wait_bounded(pv_done0 + 8 * t, (uint32_t)j & 1u, wc, 36)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(t, j + 1);
        }
      }
      if (*abort_s) {
        umma_commit(drain);
        wait_drain(drain, 0, a.wait_cap_ns);
      }
    }
  } else {
    // ---------------- softmax: warpgroup t = tile t, one query row per thread ----------------
    const int t = (warp - 2) >> 2;
    const int qd = warp & 3;
    const int prow = qd * 32 + lane;
    const int row = q0 + t * FA_BQ + prow;
    const uint32_t tl = tmem_base + ((uint32_t)(qd * 32) << 16);
    const uint32_t s_addr = tl + (uint32_t)(t * 128);
    const uint32_t o_addr = tl + 256 + (uint32_t)(t * 128);
    const int64_t climit = a.causal ? (int64_t)row + coff : INT64_MAX;
    const float sq = fa_pow2_scale(__ldg(a.amax + h));
    const float sk = fa_pow2_scale(__ldg(a.amax + a.heads + kvh));
    const float sv = fa_pow2_scale(__ldg(a.amax + a.heads + a.kv_heads + kvh));
    const float sl2 = a.sl2 / (sq * sk);
    float m_use = -INFINITY, lsum = 0.0f;
    bool ok = true;
    for (int j = 0; j < nb; ++j) {
      if (!wait_bounded_warp(s_full0 + 8 * t, (uint32_t)j & 1u, wc, 37)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int kc0 = j * FA_BKV;
      uint32_t r[128];
      tmem_ld64_nowait(s_addr, r);
      tmem_ld64_nowait(s_addr + 64, r + 64);
      tmem_ld_wait();
      // blocks before full_blocks need no validity bits (no key mask, inside seq_k)
      bool full = j < a.full_blocks && (int64_t)kc0 + FA_BKV - 1 <= climit;
      if (!__all_sync(0xffffffffu, full)) {
        const uint32_t w0 = __ldg(a.kbits + (kc0 >> 5)), w1 = __ldg(a.kbits + (kc0 >> 5) + 1);
        const uint32_t w2 = __ldg(a.kbits + (kc0 >> 5) + 2), w3 = __ldg(a.kbits + (kc0 >> 5) + 3);
        const uint32_t wd[4] = {w0, w1, w2, w3};
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const bool vis = ((wd[c >> 5] >> (c & 31)) & 1u) && (int64_t)(kc0 + c) <= climit;
          if (!vis) r[c] = 0xff800000u;
        }
      }
      // row max: four chains of three-input maxima
      float mx4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) mx4[u] = __uint_as_float(r[u]);
#pragma unroll
      for (int c = 4; c < 124; c += 8)
#pragma unroll
        for (int u = 0; u < 4; ++u)
          mx4[u] = fmax3(mx4[u], __uint_as_float(r[c + 2 * u]), __uint_as_float(r[c + 2 * u + 1]));
      const float mx = fmax3(fmax3(mx4[0], mx4[1], mx4[2]), mx4[3],
                             fmax3(__uint_as_float(r[124]), __uint_as_float(r[125]),
                                   fmaxf(__uint_as_float(r[126]), __uint_as_float(r[127]))));
      const float m_cand = mx * sl2;
      if (j == 0) {
        m_use = m_cand;
      } else if (__any_sync(0xffffffffu, m_cand > m_use + FA_RESCALE_LOG2)) {
        // O_t is quiescent here: PV_t(j-1) completed before S_t(j) was issued
        const float m_new = fmaxf(m_use, m_cand);
        const float factor = (m_new == -INFINITY) ? 1.0f : ex2_approx(m_use - m_new);
        m_use = m_new;
        lsum *= factor;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + c * 32, o);
#pragma unroll
          for (int u = 0; u < 32; ++u) o[u] = __float_as_uint(__uint_as_float(o[u]) * factor);
          tmem_st32(o_addr + c * 32, o);
        }
      }
      const float msub = (m_use == -INFINITY) ? 0.0f : m_use;
      // p = 2^(s * sl2 - msub) for a pair of columns per step: one packed FMA, two ex2, one
      // packed add into four pair accumulators (lane-wise the same sums as eight scalar ones)
      const uint64_t sl2_2 = f2_pack(sl2, sl2), nm_2 = f2_pack(-msub, -msub);
      uint64_t ps2[4] = {0, 0, 0, 0};
      uint32_t ph[64];
#pragma unroll
      for (int c = 0; c < 128; c += 2) {
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(__uint_as_float(r[c]), __uint_as_float(r[c + 1])), sl2_2, nm_2), x0, x1);
        const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
        ps2[(c >> 1) & 3] = f2_add(ps2[(c >> 1) & 3], f2_pack(p0, p1));
        __half2 hp = __floats2half2_rn(p0, p1);
        ph[c >> 1] = *reinterpret_cast<uint32_t*>(&hp);
      }
      float ps8[8];
#pragma unroll
      for (int u = 0; u < 4; ++u) f2_unpack(ps2[u], ps8[2 * u], ps8[2 * u + 1]);
      lsum += ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
      tmem_st64(s_addr, ph);  // P_t over the first 64 columns of S_t
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full0 + 8 * t);
    }
    if (ok && nb > 0 && wait_bounded_warp(pv_done0 + 8 * t, (uint32_t)(nb - 1) & 1u, wc, 38)) {
      tc_fence_after();
      const float inv = lsum > 0.0f ? 1.0f / (lsum * sv) : 0.0f;
      float* orow = a.out + (int64_t)row * a.ldo + (int64_t)h * FA_D;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(o_addr + c * 32, o);
        if (row < a.seq_q) {
#pragma unroll
          for (int u = 0; u < 32; u += 4)
            *reinterpret_cast<float4*>(orow + c * 32 + u) =
                make_float4(__uint_as_float(o[u]) * inv, __uint_as_float(o[u + 1]) * inv,
                            __uint_as_float(o[u + 2]) * inv, __uint_as_float(o[u + 3]) * inv);
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, FA_TMEM_COLS);
  }
}

// Max |x| per head of the fp32 Q, K and V ([seq][ld], head h at column h * 128) into amax
// (Q heads, then K heads, then V heads; atomicMax on the float bits, amax zeroed beforehand).
// Grid (row blocks of 64, max(heads, kv_heads), 3): z picks the tensor; each warp reads whole
// 512-byte head rows with 16-byte loads (scalar loads when a row is not 16-byte aligned).
struct AbsmaxArgs {
  const float* X[3];
  int64_t ld[3];
  int seq[3];
  int heads[3];
  int base[3];  // first amax slot of each tensor
  int vec[3];
};

__global__ void __launch_bounds__(256) k_absmax_heads(const __grid_constant__ AbsmaxArgs a, float* __restrict__ amax) {
  __shared__ float red[8];
  const int z = blockIdx.z, h = blockIdx.y;
  if (h >= a.heads[z]) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* X = a.X[z] + (int64_t)h * FA_D;
  float m = 0.0f;
  const int r0 = blockIdx.x * 64;
#pragma unroll 4
  for (int rr = warp; rr < 64; rr += 8) {
    const int r = r0 + rr;
    if (r < a.seq[z]) {
      const float* p = X + (int64_t)r * a.ld[z] + lane * 4;
      if (a.vec[z]) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(p));
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      } else {
#pragma unroll
        for (int t = 0; t < 4; ++t) m = fmaxf(m, fabsf(__ldg(p + t)));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
    atomicMax(reinterpret_cast<unsigned int*>(amax + a.base[z] + h), __float_as_uint(m));  // NaN sorts above inf
  }
}

// Q or K fp32 [seq][ld] (head h at column h * 128) -> fp16 [heads][seq_pad][128] scaled by
// fa_pow2_scale(amax[h]), zero rows for seq <= r < seq_pad.  One thread per 8 elements.
__global__ void __launch_bounds__(256) k_cast_heads(const float* __restrict__ X, int64_t ld, int seq, int seq_pad,
                                                    const float* __restrict__ amax, __half* __restrict__ dst,
                                                    int vec) {
  const int h = blockIdx.y;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // 8-element group
  if (i >= (int64_t)seq_pad * 16) return;
  const int r = (int)(i >> 4), c = (int)(i & 15) * 8;
  const float sc = fa_pow2_scale(__ldg(amax + h));
  float v[8];
  if (r < seq) {
    const float* s = X + (int64_t)r * ld + (int64_t)h * FA_D + c;
    if (vec) {
      const float4 x0 = __ldg(reinterpret_cast<const float4*>(s));
      const float4 x1 = __ldg(reinterpret_cast<const float4*>(s + 4));
      v[0] = x0.x, v[1] = x0.y, v[2] = x0.z, v[3] = x0.w, v[4] = x1.x, v[5] = x1.y, v[6] = x1.z, v[7] = x1.w;
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) v[t] = __ldg(s + t);
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] *= sc;
  } else {
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = 0.0f;
  }
  *reinterpret_cast<uint4*>(dst + ((int64_t)h * seq_pad + r) * FA_D + c) = pack_half8(v);
}

// V fp32 [seq][ld] (head h at column h * 128) -> fp16 [heads][128][seq_pad] (transposed),
// scaled by fa_pow2_scale(amax[h]), zero columns for seq <= r < seq_pad.
// Grid (seq_pad / 64, 128 / 32, heads): a 64-row x 32-column tile through shared memory.
__global__ void __launch_bounds__(256) k_v_transpose(const float* __restrict__ X, int64_t ld, int seq, int seq_pad,
                                                     const float* __restrict__ amax, __half* __restrict__ dst) {
  __shared__ float t[32][65];
  const int h = blockIdx.z;
  const int r0 = blockIdx.x * 64, c0 = blockIdx.y * 32;
  const float sc = fa_pow2_scale(__ldg(amax + h));
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int rr = ty + 8 * i, r = r0 + rr;
    t[tx][rr] = r < seq ? __ldg(X + (int64_t)r * ld + (int64_t)h * FA_D + c0 + tx) * sc : 0.0f;
  }
  __syncthreads();
  // each thread writes two consecutive rows of one column as a half2
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = threadIdx.x + 256 * i;  // 32 columns x 32 row pairs
    const int cc = idx >> 5, rp = idx & 31;
    const __half2 v = __floats2half2_rn(t[cc][2 * rp], t[cc][2 * rp + 1]);
    *reinterpret_cast<__half2*>(dst + ((int64_t)h * FA_D + c0 + cc) * seq_pad + r0 + 2 * rp) = v;
  }
}

// Key validity bits: bit c of word c / 32 = (c < seq_k) && (mask == null || mask[c] != 0).
__global__ void k_key_bits(const int32_t* __restrict__ mask, int seq_k, int words, uint32_t* __restrict__ bits) {
  const int w = blockIdx.x * blockDim.x + threadIdx.x;
  if (w >= words) return;
  uint32_t b = 0;
  for (int t = 0; t < 32; ++t) {
    const int c = w * 32 + t;
    if (c < seq_k && (!mask || mask[c] != 0)) b |= 1u << t;
  }
  bits[w] = b;
}

}  // namespace envg
