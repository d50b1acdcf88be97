// envg_oracle.cpp -- TEST INFRASTRUCTURE ONLY.
//
// CPU restatement ("O1") of Envision's dense-linear hot path, used as the parity
// checker for the CUDA library and as the CPU timing baseline ("port").  Nothing in
// the product library links or calls this file; only tests/, the smoke check in
// __graft_entry__.py and bench.py's CPU-baseline leg load it.
//
// What is restated, and from where (paths relative to the Envision source tree):
//   * BF16ToSingle          src/quicknn_common.pas:1991-2008  (bits << 16, exact)
//   * SingleToBF16          src/quicknn_common.pas:2010-2027  (bits >> 16, truncation)
//   * sdot_avx2             src/ops_avx2.inc:757-837          (4x8-lane accumulators over
//                                                              32-blocks, 8-blocks into acc0,
//                                                              masked tail, extract+hadd x2)
//   * sDot_x4_avx2          src/ops_avx2.inc:1407-1508        (1 A load, 4 B FMAs per 8 k;
//                                                              reduction extract+add+hadd x2;
//                                                              C = dot*alpha + C fused)
//   * saxpy_avx2            src/ops_avx2.inc:839-907          (y = a*x + y, fused)
//   * qscale/qdot/qaxpy     src/quicknncpu.pas:1067-1126
//   * gemm_nt / gemm_nn / gemm_tn / qgemm
//                           src/quicknncpu.pas:1176-1496      (8-row M tiles, 8-col N tiles)
//   * QNNLinear bias        src/quicknncpu.pas:1807-1820      (QNNAddInplace per row, :704-709)
//   * QNNLinearNoBias_BF16  src/quicknncpu.pas:1830-1847      (widen W, then NT GEMM)
//   * fast_exp, QNNSiluMul  src/quicknncpu.pas:305-330, 2404-2419 (scalar build)
//   * QNNGatedAdd           src/quicknncpu.pas:853-859, 1752-1758
//   * QNNConv2d             src/quicknncpu.pas:1958-2132      (row-tiled im2col, NN GEMM,
//                                                              per-channel bias)
//   * QNNAdaLN              src/quicknncpu.pas:3042-3060      (QNNMean :679-685, QNNVariance
//                                                              :687-695, EPSILON quicknn_common.pas:51)
//
// Two builds of the reference are restated, selected by `path`:
//   ENVO_PATH_AVX2   (0) -- the shipped configuration (USE_AVX2 defined in
//                           Examples/FPC/EnvisionCLI/Envision.lpi).  Bit-exact restatement of
//                           the AVX2 lane order, including a quirk: the K%8 remainder block of
//                           sDot_x4_avx2 (ops_avx2.inc:1442-1460) loads B into the accumulator
//                           registers and then computes acc = A*acc + acc, so for K%8 != 0 the
//                           main-loop sum is discarded.  All model K values are multiples of 8.
//   ENVO_PATH_SCALAR (1) -- the build without USE_AVX2: sequential, unfused x*y + acc loops.
//
// Threading: like the reference pool (src/steroids.pas:773-807) the M dimension is cut into
// 8-row tiles handed out to threads; every output element is computed by one thread in one
// fixed order, so results do not depend on the thread count.

#include <stdint.h>
#include <string.h>
#include <math.h>
#include <stdlib.h>
#include <vector>
#include <thread>
#include <atomic>
#include <algorithm>

#ifdef __AVX2__
#include <immintrin.h>
#endif

#define ENVO_PATH_AVX2 0
#define ENVO_PATH_SCALAR 1

namespace {

int g_threads = 0;

int num_threads() {
  if (g_threads > 0) return g_threads;
  unsigned n = std::thread::hardware_concurrency();
  return n ? (int)n : 1;
}

// Parallel-for over tile starts 0, step, 2*step, ... < end (strided hand-out like MP.&For).
template <class F>
void parallel_tiles(int64_t end, int64_t step, F&& f) {
  int64_t ntiles = (end + step - 1) / step;
  int nt = (int)std::min<int64_t>(num_threads(), ntiles);
  if (nt <= 1) {
    for (int64_t t = 0; t < ntiles; ++t) f(t * step);
    return;
  }
  std::atomic<int64_t> next(0);
  std::vector<std::thread> pool;
  for (int i = 0; i < nt; ++i)
    pool.emplace_back([&]() {
      for (;;) {
        int64_t t = next.fetch_add(1);
        if (t >= ntiles) break;
        f(t * step);
      }
    });
  for (auto& th : pool) th.join();
}

inline float bf16_bits_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// ---- 8-lane vector helpers: portable, bit-identical to the AVX2 instructions ----------------
struct V8 {
  float l[8];
};

inline void v8_zero(V8& v) { for (int i = 0; i < 8; ++i) v.l[i] = 0.0f; }
// vfmadd231ps acc, a, b  : acc = a*b + acc (single rounding)
inline void v8_fma(V8& acc, const float* a, const float* b) {
  for (int i = 0; i < 8; ++i) acc.l[i] = fmaf(a[i], b[i], acc.l[i]);
}
// vextractf128 + addps + haddps + haddps: ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7))
inline float v8_reduce(const V8& v) {
  float s0 = v.l[0] + v.l[4], s1 = v.l[1] + v.l[5], s2 = v.l[2] + v.l[6], s3 = v.l[3] + v.l[7];
  float h0 = s0 + s1, h1 = s2 + s3;  // first haddps
  return h0 + h1;                    // second haddps
}

// sdot_avx2 (ops_avx2.inc:757-837)
float sdot_avx2(int64_t n, const float* a, const float* b) {
  V8 acc[4];
  for (int i = 0; i < 4; ++i) v8_zero(acc[i]);
  int64_t blocks32 = n >> 5;
  const float* A = a;
  const float* B = b;
#if defined(__AVX2__) && defined(__FMA__)
  {
    __m256 c[4];
    for (int r = 0; r < 4; ++r) c[r] = _mm256_setzero_ps();
    for (int64_t i = 0; i < blocks32; ++i) {
      for (int r = 0; r < 4; ++r) c[r] = _mm256_fmadd_ps(_mm256_loadu_ps(A + 8 * r), _mm256_loadu_ps(B + 8 * r), c[r]);
      A += 32;
      B += 32;
    }
    for (int r = 0; r < 4; ++r) _mm256_storeu_ps(acc[r].l, c[r]);
  }
#else
  for (int64_t i = 0; i < blocks32; ++i) {
    for (int r = 0; r < 4; ++r) v8_fma(acc[r], A + 8 * r, B + 8 * r);
    A += 32;
    B += 32;
  }
#endif
  V8 acc0 = acc[0];
  if (blocks32) {
    // vaddps ymm0,ymm0,ymm1 ; vaddps ymm2,ymm2,ymm3 ; vaddps ymm0,ymm0,ymm2
    for (int i = 0; i < 8; ++i) {
      float t01 = acc[0].l[i] + acc[1].l[i];
      float t23 = acc[2].l[i] + acc[3].l[i];
      acc0.l[i] = t01 + t23;
    }
  }
  int64_t blocks8 = (n & 31) >> 3;
  for (int64_t i = 0; i < blocks8; ++i) {
    v8_fma(acc0, A, B);
    A += 8;
    B += 8;
  }
  int64_t rem = n & 7;
  if (rem) {
    float ta[8] = {0}, tb[8] = {0};
    for (int64_t i = 0; i < rem; ++i) { ta[i] = A[i]; tb[i] = B[i]; }
    v8_fma(acc0, ta, tb);
  }
  return v8_reduce(acc0);
}

// sDot_x4_avx2 (ops_avx2.inc:1407-1508): C[0..3] = alpha*dot(A, B_j) + C[j]  (fused)
void sdot_x4_avx2(const float* A, const float* B, float* C, int64_t K, int64_t ldb, float alpha) {
  V8 acc[4];
  for (int j = 0; j < 4; ++j) v8_zero(acc[j]);
  int64_t kb = K >> 3;
  int64_t r10 = 0;
#if defined(__AVX2__) && defined(__FMA__)
  // The same lane-wise vfmadd231ps chain with the instructions themselves (identical bits to
  // v8_fma, whose per-lane fmaf the compiler may not vectorise), so the O1 timing is the
  // reference's instruction mix rather than a scalar emulation of it.
  {
    __m256 c0 = _mm256_setzero_ps(), c1 = c0, c2 = c0, c3 = c0;
    for (int64_t i = 0; i < kb; ++i) {
      const __m256 a = _mm256_loadu_ps(A + r10);
      c0 = _mm256_fmadd_ps(a, _mm256_loadu_ps(B + r10), c0);
      c1 = _mm256_fmadd_ps(a, _mm256_loadu_ps(B + r10 + ldb), c1);
      c2 = _mm256_fmadd_ps(a, _mm256_loadu_ps(B + r10 + 2 * ldb), c2);
      c3 = _mm256_fmadd_ps(a, _mm256_loadu_ps(B + r10 + 3 * ldb), c3);
      r10 += 8;
    }
    _mm256_storeu_ps(acc[0].l, c0);
    _mm256_storeu_ps(acc[1].l, c1);
    _mm256_storeu_ps(acc[2].l, c2);
    _mm256_storeu_ps(acc[3].l, c3);
  }
#else
  for (int64_t i = 0; i < kb; ++i) {
    for (int j = 0; j < 4; ++j) v8_fma(acc[j], A + r10, B + r10 + j * ldb);
    r10 += 8;
  }
#endif
  int64_t rem = K & 7;
  if (rem) {
    // Restated literally: vmaskmovps ymm1..4 <- B tails (overwriting the accumulators),
    // then vfmadd231ps ymmj, ymm0, ymmj  ->  acc = A_tail * B_tail + B_tail.
    float ta[8] = {0};
    for (int64_t i = 0; i < rem; ++i) ta[i] = A[r10 + i];
    for (int j = 0; j < 4; ++j) {
      float tb[8] = {0};
      for (int64_t i = 0; i < rem; ++i) tb[i] = B[r10 + j * ldb + i];
      for (int l = 0; l < 8; ++l) acc[j].l[l] = fmaf(ta[l], tb[l], tb[l]);
    }
  }
  for (int j = 0; j < 4; ++j) C[j] = fmaf(v8_reduce(acc[j]), alpha, C[j]);
}

// saxpy_avx2 (ops_avx2.inc:839-907): y = a*x + y, fused in every lane and in the scalar tail
inline void saxpy_fused(int64_t n, float a, const float* x, float* y) {
  for (int64_t i = 0; i < n; ++i) y[i] = fmaf(a, x[i], y[i]);
}

inline float qdot(int path, int64_t n, const float* x, const float* y) {
  if (path == ENVO_PATH_AVX2) return sdot_avx2(n, x, y);
  float r = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    float p = x[i] * y[i];
    r = r + p;
  }
  return r;
}

inline void qaxpy(int path, int64_t n, float a, const float* x, float* y) {
  if (path == ENVO_PATH_AVX2) {
    saxpy_fused(n, a, x, y);
    return;
  }
  for (int64_t i = 0; i < n; ++i) {
    float p = a * x[i];
    y[i] = p + y[i];
  }
}

inline void qscale(int64_t n, float beta, float* x) {
  for (int64_t i = 0; i < n; ++i) x[i] = x[i] * beta;
}

const int64_t TILE_M = 8, TILE_N = 8, TILE_K = 8;

// gemm_nt (quicknncpu.pas:1241-1337)
void gemm_nt(int path, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
             const float* B, int64_t ldb, float beta, float* C, int64_t ldc) {
  parallel_tiles(((M + TILE_M - 1) / TILE_M) * TILE_M, TILE_M, [&](int64_t tm_start) {
    int64_t tm_finish = std::min(tm_start + TILE_M, M);
    for (int64_t tm = tm_start; tm < tm_finish; ++tm) qscale(N, beta, C + tm * ldc);
    for (int64_t tn_start = 0; tn_start < N; tn_start += TILE_N) {
      int64_t tn_finish = std::min(tn_start + TILE_N, N);
      for (int64_t tm = tm_start; tm < tm_finish; ++tm) {
        float* CC = C + tm * ldc;
        int64_t tn = tn_start;
        if (path == ENVO_PATH_AVX2) {
          while (tn + 4 <= tn_finish) {
            sdot_x4_avx2(A + tm * lda, B + tn * ldb, CC + tn, K, ldb, alpha);
            tn += 4;
          }
        }
        while (tn < tn_finish) {
          float a_part = alpha * qdot(path, K, A + tm * lda, B + tn * ldb);
          CC[tn] = CC[tn] + a_part;
          ++tn;
        }
      }
    }
  });
}

// gemm_nn (quicknncpu.pas:1182-1239)
void gemm_nn(int path, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
             const float* B, int64_t ldb, float beta, float* C, int64_t ldc) {
  parallel_tiles(((M + TILE_M - 1) / TILE_M) * TILE_M, TILE_M, [&](int64_t tm_start) {
    int64_t tm_finish = std::min(tm_start + TILE_M, M);
    for (int64_t tm = tm_start; tm < tm_finish; ++tm) qscale(N, beta, C + tm * ldc);
    for (int64_t tk_start = 0; tk_start < K; tk_start += TILE_K) {
      int64_t tk_finish = std::min(tk_start + TILE_K, K);
      for (int64_t tm = tm_start; tm < tm_finish; ++tm)
        for (int64_t tk = tk_start; tk < tk_finish; ++tk)
          qaxpy(path, N, alpha * A[tm * lda + tk], B + tk * ldb, C + tm * ldc);
    }
  });
}

// gemm_tn (quicknncpu.pas:1339-1395)
void gemm_tn(int path, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
             const float* B, int64_t ldb, float beta, float* C, int64_t ldc) {
  parallel_tiles(((M + TILE_M - 1) / TILE_M) * TILE_M, TILE_M, [&](int64_t tm_start) {
    int64_t tm_finish = std::min(tm_start + TILE_M, M);
    for (int64_t tm = tm_start; tm < tm_finish; ++tm) qscale(N, beta, C + tm * ldc);
    for (int64_t tk_start = 0; tk_start < K; tk_start += TILE_K) {
      int64_t tk_finish = std::min(tk_start + TILE_K, K);
      for (int64_t tk = tk_start; tk < tk_finish; ++tk) {
        const float* AA = A + tk * lda;
        for (int64_t tm = tm_start; tm < tm_finish; ++tm)
          qaxpy(path, N, alpha * AA[tm], B + tk * ldb, C + tm * ldc);
      }
    }
  });
}

// fast_exp (quicknncpu.pas:305-330)
float fast_exp(float x) {
  if (x < -87.33f) return 0.0f;
  if (x > 88.72f) return 1e38f;
  float n = (float)floor((double)x * 1.4426950408889634 + 0.5);
  float r = (float)((double)x - (double)n * 0.6931471805599453);
  float p = (float)(1.0 + r * (1.0 + r * (0.5 + r * (0.16666667 + r * (0.04166667 + r * 0.00833333)))));
  int32_t bits;
  memcpy(&bits, &p, 4);
  bits += ((int32_t)n) << 23;
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

}  // namespace

extern "C" {

int envo_set_threads(int n) {
  g_threads = n;
  return num_threads();
}

int envo_get_threads(void) { return num_threads(); }

// BF16ToSingle (quicknn_common.pas:1991-2008)
void envo_bf16_to_f32(int64_t n, const uint16_t* src, float* dst) {
  for (int64_t i = 0; i < n; ++i) dst[i] = bf16_bits_to_f32(src[i]);
}

// SingleToBF16 (quicknn_common.pas:2010-2027): truncation
void envo_f32_to_bf16_trunc(int64_t n, const float* src, uint16_t* dst) {
  for (int64_t i = 0; i < n; ++i) {
    uint32_t u;
    memcpy(&u, &src[i], 4);
    dst[i] = (uint16_t)(u >> 16);
  }
}

float envo_sdot(int path, int64_t n, const float* x, const float* y) { return qdot(path, n, x, y); }

// TQNNSingleOPS.qgemm (quicknncpu.pas:1398-1496); RowMajor only, TT unsupported (returns -1).
int envo_qgemm(int path, int order, int transA, int transB, int64_t M, int64_t N, int64_t K,
               float alpha, const float* A, int64_t lda, const float* B, int64_t ldb, float beta,
               float* C, int64_t ldc) {
  const int RowMajor = 101, NoTrans = 111, Trans = 112;
  if (order != RowMajor) return -1;
  if (transA == NoTrans && transB == NoTrans)
    gemm_nn(path, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
  else if (transA == NoTrans && transB == Trans)
    gemm_nt(path, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
  else if (transA == Trans && transB == NoTrans)
    gemm_tn(path, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc);
  else
    return -1;
  return 0;
}

// QNNLinear / QNNLinearNoBias (quicknncpu.pas:1807-1828), fp32 weights.
void envo_linear_f32(int path, float* dst, const float* x, const float* W, const float* bias,
                     int64_t seqLen, int64_t inDIM, int64_t outDIM) {
  gemm_nt(path, seqLen, outDIM, inDIM, 1.0f, x, inDIM, W, inDIM, 0.0f, dst, outDIM);
  if (bias)
    for (int64_t i = 0; i < seqLen; ++i) {
      float* row = dst + i * outDIM;
      for (int64_t j = 0; j < outDIM; ++j) row[j] = row[j] + bias[j];  // QNNAddInplace
    }
}

// QNNLinearNoBias_BF16 (quicknncpu.pas:1830-1847) plus the optional QNNLinear bias:
// W widened to fp32 into a workspace on every call, then the fp32 NT GEMM.
void envo_linear_bf16(int path, float* dst, const float* x, const uint16_t* W, const float* bias,
                      int64_t seqLen, int64_t inDIM, int64_t outDIM) {
  std::vector<float> ws((size_t)(inDIM * outDIM));
  envo_bf16_to_f32(inDIM * outDIM, W, ws.data());
  envo_linear_f32(path, dst, x, ws.data(), bias, seqLen, inDIM, outDIM);
}

// Scalar fast_exp (quicknncpu.pas:305-330).
float envo_fast_exp(float x) { return fast_exp(x); }

// QNNSiluMul scalar build (quicknncpu.pas:2414-2416): gate[i] = gate/(1+fast_exp(-gate)) * up
void envo_silu_mul(float* gate, const float* up, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float v = gate[i];
    float s = v / (1.0f + fast_exp(-v));
    gate[i] = s * up[i];
  }
}

// QNNSiluInplace scalar build (quicknncpu.pas:2395-2399 form): x = x / (1 + fast_exp(-x))
void envo_silu(float* x, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    float v = x[i];
    x[i] = v / (1.0f + fast_exp(-v));
  }
}

// QNNGatedAdd (quicknncpu.pas:853-859 via QNNAccMul :1752-1758): dst += gate (.) proj per row
void envo_gated_add(float* dst, const float* gate, const float* proj, int64_t seq, int64_t hidden) {
  for (int64_t s = 0; s < seq; ++s) {
    float* d = dst + s * hidden;
    const float* p = proj + s * hidden;
    for (int64_t i = 0; i < hidden; ++i) {
      float t = gate[i] * p[i];
      d[i] = d[i] + t;
    }
  }
}

// QNNAdaLN (quicknncpu.pas:3042-3060), scalar build: per row, mean = sequential fp32 sum / n,
// population variance = sequential sum of squared differences / n, stdInv = 1/sqrt(var +
// EPSILON) with EPSILON = 1e-6 (quicknn_common.pas:51; the eps argument of QNNAdaLN is not used
// by its body), out = (1 + scale[j]) * ((x - mean) * stdInv) + bias[j].
void envo_adaln(float* dst, const float* src, const float* bias, const float* scale, int64_t seq, int64_t hidden) {
  const float EPS = 1e-6f;
  for (int64_t i = 0; i < seq; ++i) {
    const float* in = src + i * hidden;
    float* out = dst + i * hidden;
    float sum = 0.0f;
    for (int64_t j = 0; j < hidden; ++j) sum = sum + in[j];
    const float mean = hidden ? sum / (float)hidden : 0.0f;
    float ssd = 0.0f;
    for (int64_t j = 0; j < hidden; ++j) {
      const float d = in[j] - mean;
      ssd = ssd + d * d;
    }
    const float var = hidden ? ssd / (float)hidden : 0.0f;
    const float stdInv = 1.0f / sqrtf(var + EPS);
    for (int64_t j = 0; j < hidden; ++j) {
      const float norm = (in[j] - mean) * stdInv;
      out[j] = (1.0f + scale[j]) * norm + bias[j];
    }
  }
}

// QNNRMSNorm applied per row (QNNRMSNormRows, quicknncpu.pas:2187-2198 -> 2159-2185):
// inv = 1 / sqrt(sum(x^2) / N + 1e-6), then x * weight * inv (QNNFusedMulScale), or x * inv when
// no weight is given.  Scalar sums in index order.
void envo_rms_norm(float* dst, const float* src, const float* weight, int64_t seq, int64_t hidden) {
  const float EPS = 1e-6f;
  for (int64_t i = 0; i < seq; ++i) {
    const float* in = src + i * hidden;
    float* out = dst + i * hidden;
    float ss = 0.0f;
    for (int64_t j = 0; j < hidden; ++j) ss = ss + in[j] * in[j];
    const float inv = 1.0f / sqrtf((hidden ? ss / (float)hidden : 0.0f) + EPS);
    for (int64_t j = 0; j < hidden; ++j) out[j] = weight ? (in[j] * weight[j]) * inv : in[j] * inv;
  }
}

// QNNGroupNorm (quicknncpu.pas:2259-2313), scalar build: per (batch, group) over the contiguous
// run of channels_per_group * H * W floats, mean = QNNMean (sequential fp32 sum / n, :536-547 and
// :679-685), variance = QNNVariance population form (sequential sum of squared differences / n,
// :566-581 and :687-695), std_inv = 1 / sqrt(variance + EPSILON) (EPSILON = 1e-6,
// quicknn_common.pas:51), then per channel QNNFusedScaleBias with scale = gamma*std_inv and
// bias = beta - mean*gamma*std_inv (:769-780).  act != 0 applies QNNSiluInplace (:2372-2386,
// scalar form) afterwards.  dst may equal src.
void envo_group_norm(float* dst, const float* src, const float* gamma, const float* beta, int batch, int channels,
                     int H, int W, int num_groups, int act) {
  const float EPS = 1e-6f;
  const int cpg = channels / num_groups;
  const int64_t spatial = (int64_t)H * W;
  const int64_t n = (int64_t)cpg * spatial;
  for (int b = 0; b < batch; ++b)
    for (int g = 0; g < num_groups; ++g) {
      const int c_start = g * cpg;
      const float* s1 = src + ((int64_t)b * channels + c_start) * spatial;
      float* d1 = dst + ((int64_t)b * channels + c_start) * spatial;
      float sum = 0.0f;
      for (int64_t i = 0; i < n; ++i) sum = sum + s1[i];
      const float mean = sum / (float)n;
      float ssd = 0.0f;
      for (int64_t i = 0; i < n; ++i) {
        const float dl = s1[i] - mean;
        ssd = ssd + dl * dl;
      }
      const float variance = ssd / (float)n;
      const float std_inv = 1.0f / sqrtf(variance + EPS);
      for (int c = 0; c < cpg; ++c) {
        const float ga = gamma ? gamma[c + c_start] : 1.0f;
        const float be = beta ? beta[c + c_start] : 0.0f;
        const float scale = ga * std_inv;
        const float bias = be - mean * ga * std_inv;
        for (int64_t i = 0; i < spatial; ++i) d1[c * spatial + i] = s1[c * spatial + i] * scale + bias;
      }
    }
  if (act) envo_silu(dst, (int64_t)batch * channels * spatial);
}

// Multi-head attention as the reference's BLAS path runs it, per head h (kv head h / (heads /
// kv_heads)): scores = scale * Q_h K_h^T with cblas_gemm (NoTrans, Trans; restated qgemm),
// masked entries set to -inf (QNNMatTriangularFill, quicknncpu.pas:3017-3029: column c > row r,
// or key_mask[c] == 0), QNNSoftmaxRows (QNNSoftmax scalar build :2421-2444: max, fast_exp(x -
// max), sum, scale by 1/sum), then O_h = P V_h with cblas_gemm (NoTrans, NoTrans).  Sources:
// TTransformerFlux.multiHeadForward (quicknn_transformers.pas:1150-1200) and the Qwen3 attention
// (quicknn_qwen3.pas:726-768).  Q/K/V/dst rows are strided (ldq, ldk, ldv, ldo); head h sits at
// column h * head_dim.  causal keeps column c <= r + (seq_k - seq_q) (the square case of the
// reference when seq_q == seq_k).
int envo_attention(int path, float* dst, const float* Q, const float* K, const float* V, int seq_q, int seq_k,
                   int heads, int kv_heads, int head_dim, int64_t ldq, int64_t ldk, int64_t ldv, int64_t ldo,
                   float scale, int causal, const int32_t* key_mask) {
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads) return -1;
  std::vector<float> sc((size_t)seq_q * seq_k);
  const int per_kv = heads / kv_heads;
  const int64_t off = (int64_t)seq_k - seq_q;
  for (int h = 0; h < heads; ++h) {
    const int kvh = h / per_kv;
    gemm_nt(path, seq_q, seq_k, head_dim, scale, Q + (int64_t)h * head_dim, ldq, K + (int64_t)kvh * head_dim, ldk,
            0.0f, sc.data(), seq_k);
    for (int r = 0; r < seq_q; ++r) {
      float* row = sc.data() + (int64_t)r * seq_k;
      for (int c = 0; c < seq_k; ++c)
        if ((causal && c > r + off) || (key_mask && key_mask[c] == 0)) row[c] = -INFINITY;
      float mx = row[0];
      for (int c = 1; c < seq_k; ++c)
        if (row[c] > mx) mx = row[c];
      float sum = 0.0f;
      for (int c = 0; c < seq_k; ++c) {
        row[c] = fast_exp(row[c] - mx);
        sum = sum + row[c];
      }
      const float inv = 1.0f / sum;
      for (int c = 0; c < seq_k; ++c) row[c] = row[c] * inv;
    }
    gemm_nn(path, seq_q, head_dim, seq_k, 1.0f, sc.data(), seq_k, V + (int64_t)kvh * head_dim, ldv, 0.0f,
            dst + (int64_t)h * head_dim, ldo);
  }
  return 0;
}

// QNNConv2d, im2col build (quicknncpu.pas:1958-2132).  fp32 weights [out_ch, in_ch, kH, kW].
// Restated including its stride-1 copy, which is exact only for "same" padding
// (outW == W); batches processed one after another, the col buffer row-tiled at
// MAX_COL_SIZE floats.
int envo_conv2d(int path, float* dst, const float* src, const float* weights, const float* bias,
                int in_ch, int out_ch, int H, int W, int kH, int kW, int stride, int padding,
                int batch) {
  const int64_t MAX_COL_SIZE = 256LL * 1024 * 1024;
  int64_t outH = (H + 2 * padding - kH) / stride + 1;
  int64_t outW = (W + 2 * padding - kW) / stride + 1;
  if (outH <= 0 || outW <= 0) return -1;
  int64_t outSpatial = outH * outW;
  int64_t col_size = (int64_t)in_ch * kH * kW * outH * outW;
  int64_t tile_rows = outH;
  if (col_size > MAX_COL_SIZE) {
    int64_t row_size = (int64_t)in_ch * kH * kW * outW;
    tile_rows = MAX_COL_SIZE / row_size;
    if (tile_rows < 1) tile_rows = 1;
  }
  std::vector<float> colbuf;
  if (kH * kW != 1) colbuf.resize((size_t)((int64_t)in_ch * kH * kW * tile_rows * outW));
  int64_t K = (int64_t)in_ch * kH * kW;
  for (int b = 0; b < batch; ++b) {
    const float* in_b = src + (int64_t)b * in_ch * H * W;
    float* out_b = dst + (int64_t)b * out_ch * outSpatial;
    for (int64_t tile_start = 0; tile_start < outH; tile_start += tile_rows) {
      int64_t tile_end = std::min(tile_start + tile_rows, outH);
      int64_t tile_pixels = (tile_end - tile_start) * outW;
      const float* col;
      if (kH * kW == 1) {
        col = in_b;  // pointwise conv: col aliases the input (quicknncpu.pas:2074-2075)
      } else {
        float* cp = colbuf.data();
        int64_t col_row = 0;
        for (int ic = 0; ic < in_ch; ++ic)
          for (int kr = 0; kr < kH; ++kr)
            for (int kc = 0; kc < kW; ++kc) {
              for (int64_t oh = tile_start; oh < tile_end; ++oh) {
                int64_t ih = oh * stride + kr - padding;
                float* col_ptr = cp + (col_row * tile_pixels + (oh - tile_start) * outW);
                int64_t input_col = kc - padding;
                if ((uint64_t)ih < (uint64_t)H) {
                  if (stride == 1) {
                    memset(col_ptr, 0, sizeof(float) * outW);
                    int64_t cnt = outW - std::llabs(input_col);
                    if (cnt > 0)
                      memcpy(col_ptr + (input_col < 0 ? -input_col : 0),
                             in_b + (int64_t)ic * H * W + ih * W + (input_col >= 0 ? input_col : 0),
                             sizeof(float) * cnt);
                  } else {
                    for (int64_t ow = 0; ow < outW; ++ow) {
                      int64_t iw = ow * stride - padding + kc;
                      col_ptr[ow] = ((uint64_t)iw < (uint64_t)W) ? in_b[(int64_t)ic * H * W + ih * W + iw] : 0.0f;
                    }
                  }
                } else {
                  memset(col_ptr, 0, sizeof(float) * outW);
                }
              }
              ++col_row;
            }
        col = cp;
      }
      float* out_tile = out_b + tile_start * outW;
      gemm_nn(path, out_ch, tile_pixels, K, 1.0f, weights, K, col, tile_pixels, 0.0f, out_tile, outSpatial);
    }
    if (bias)
      for (int oc = 0; oc < out_ch; ++oc) {
        float bv = bias[oc];
        float* p = out_b + (int64_t)oc * outSpatial;
        for (int64_t i = 0; i < outSpatial; ++i) p[i] = p[i] + bv;  // QNNBiasInplace
      }
  }
  return 0;
}

}  // extern "C"
