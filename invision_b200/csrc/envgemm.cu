// envgemm.cu -- host side of libenvgemm.so: the C ABI declared in include/envgemm.h, the
// device-resident weight registry, TMA descriptor construction and kernel dispatch.
//
// Call path of one Envision Linear (quicknn_kernels.pas:2093 QNNLINEAR_BF16_OR_F32 ->
// quicknncpu.pas:1822 QNNLinearNoBias -> cblas_gemm NT) through this library:
//   envg_linear(dst, x, W, bias, M, K, N, ...)
//     [host pointers] x, bias (and the residual) -> device workspace
//     k_cast_rows     X fp32 -> Xb bf16 (RNE), K padded to a multiple of 8
//     k1_gemm         M > 64: persistent tcgen05 GEMM, fused epilogue writes Y fp32
//     k2_skinny       M <= 64: swap-AB split-K GEMM, fused epilogue
//     [host pointers] Y -> dst, stream synchronised, device status checked
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/envgemm.h"
#include "attention.cuh"
#include "kernels.cuh"
#include "safetensors.hpp"

using namespace envg;

namespace {

constexpr uint32_t WEIGHT_MAGIC = 0xE17A9E11u;
constexpr int K1_BN = 256;
constexpr int K1_STAGES = 4;
constexpr int KPAIR_STAGES = 6;
constexpr int SKINNY_MAX = 64;
constexpr unsigned SCHED_SLOTS = 64;  // k1_gemm_pair schedules in flight
constexpr int PAIR_DYN_UNITS = 12;    // units per CTA pair from which k1_gemm_pair may order them dynamically
constexpr int64_t PAIR_L2_SHARE = 64ll << 20;  // L2 bytes k1_gemm_pair's raster group of A panels may hold
constexpr uint64_t DEFAULT_WAIT_CAP_NS = 2000000000ull;  // 2 s

thread_local std::string t_err;
thread_local char t_buf[1024];

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_buf, sizeof(t_buf), fmt, ap);
  va_end(ap);
  t_err = t_buf;
  return code;
}

#define ENVG_CUDA(call)                                                                                \
  do {                                                                                                 \
    cudaError_t e_ = (call);                                                                           \
    if (e_ != cudaSuccess)                                                                             \
      return fail(ENVG_ERR_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
  } while (0)

#define ENVG_TRY(...)       \
  do {                      \
    int rc_ = (__VA_ARGS__); \
    if (rc_ != ENVG_OK) return rc_; \
  } while (0)

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

struct Buf {
  void* p = nullptr;
  size_t bytes = 0;
};

struct Dev {
  bool ready = false;
  int id = -1;
  int sms = 0;
  cudaStream_t own = nullptr;
  cudaStream_t user = nullptr;
  Buf x, y, xb, wb, part, cnt, bias, gate, act, col, b32, xbatch, ada, xn;
  Buf gn, c1, vec;  // GroupNorm statistics + affine, ResBlock conv1 output, small parameter vectors
  Buf fa, fain;     // attention operands (bf16 Q / K / V^T + key bits), host-call staging
  cudaStream_t aux = nullptr;              // second stream of envg_linear_batch
  cudaStream_t h2d = nullptr, d2h = nullptr;  // copy streams of pipelined host-pointer calls
  std::vector<cudaEvent_t> pipe_events;    // reused event pool of the pipelined host calls
  std::vector<cudaEvent_t> batch_events;   // reused event pool of envg_linear_batch
  int* h_status = nullptr;  // mapped pinned: [0] status code, [1] wait site
  int* d_status = nullptr;
  uint64_t wait_cap_ns = DEFAULT_WAIT_CAP_NS;
  int skinny_max = SKINNY_MAX;
  int gemv_max = 8;      // M <= gemv_max runs k_gemv (fp32 X on CUDA cores); ENVG_GEMV_M_MAX overrides
  bool use_pair = true;  // 256x256 CTA-pair tiles for M > 128 (ENVG_K1=single selects k1_gemm)
  int max_pairs = 0;     // co-resident CTA pairs of k1_gemm_pair
  bool store_tma = true;  // TMA bulk-store epilogue; ENVG_STORE=coalesced selects warp-coalesced stores
  bool pipe_host = true;  // pipeline large host-pointer linears in row chunks (ENVG_PIPE=0 disables)
  int attn_tiles = 0;     // query tiles per attention CTA: 0 = by grid size, ENVG_ATTN_TILES=1|2 forces
  int pair_split = -1;    // k1_gemm_pair split-K: -1 by cost model, 0 off, n forces n (ENVG_PAIR_SPLIT)
  int pair_group_m = 0;   // k1_gemm_pair M-tiles per raster group: 0 by L2 budget (ENVG_PAIR_GROUP_M)
  bool l2_hints = true;   // k1_gemm_pair L2 eviction priorities (ENVG_L2_HINTS=0 disables)
  int pair_dyn = 1;       // k1_gemm_pair unit order: 1 dynamic on long launches with A beyond the L2
                          // share, else fixed; ENVG_PAIR_SCHED=static (0) or =dynamic (2) forces one
  bool gemv_chain = true; // k_gemv runs a linear chained to another's output in one launch (ENVG_GEMV_CHAIN=0)
  Buf sched;              // k1_gemm_pair schedules: SCHED_SLOTS x {next unit, pairs done}, zeroed
  Buf hb;                 // host-pointer batches: the device copies of every linear's x, Y and vectors
  unsigned sched_seq = 0; // slot of the next launch
  bool pdl = true;        // programmatic dependent launch of the GEMM-chain kernels (ENVG_PDL=0 disables)
  bool no_split = false;  // set while a pipelined host call launches its row chunks
  envg_stats st{};
  size_t ws_bytes() const {
    return x.bytes + y.bytes + xb.bytes + wb.bytes + part.bytes + cnt.bytes + sched.bytes + bias.bytes + gate.bytes + act.bytes +
           col.bytes + b32.bytes + xbatch.bytes + ada.bytes + xn.bytes + gn.bytes + c1.bytes + vec.bytes +
           fa.bytes + fain.bytes + hb.bytes;
  }
};

std::recursive_mutex g_mu;
Dev g_dev[64];
int g_cur = -1;

// ---- optional per-launch timing (envg_profile) ---------------------------------------------
enum KernelId {
  KID_K1 = 0, KID_K1_SILU_GATE, KID_K1_CONV, KID_K2, KID_GEMV, KID_CAST, KID_ADALN, KID_TRANSPOSE, KID_IM2COL,
  KID_SELFTEST, KID_GN_STATS, KID_GN_AFFINE, KID_GN_APPLY, KID_ATTN, KID_CAST_HEADS, KID_KEY_BITS, KID_ABSMAX,
  KID_SPLIT_REDUCE, KID_SKINNY_REDUCE, KID_RMSNORM, KID_CAST_X3, KID_COUNT
};
// Profile names are per family: "k1_gemm*" counts k1_gemm and k1_gemm_pair launches (plain,
// SiLU-gate, conv), "k2_set" counts k2_set and the no-alloc path's k2_skinny.
const char* const kKernelNames[KID_COUNT] = {"k1_gemm",     "k1_gemm_silu_gate", "k1_gemm_conv",
                                             "k2_set",      "k_gemv",            "k_cast_rows",
                                             "k_adaln",     "k_transpose_cast",  "k_im2col_nhwc",
                                             "k_wait_selftest", "k_group_stats",     "k_group_affine",
                                             "k_group_apply",   "k_attention",       "k_cast_heads",
                                             "k_key_bits",      "k_absmax_heads",    "k_split_reduce",
                                             "k_skinny_reduce", "k_rmsnorm",      "k_cast_x3"};
struct KAcc {
  uint64_t launches = 0;
  double ms = 0, flops = 0, bytes = 0;
};
struct Pending {
  int kid;
  cudaEvent_t a, b;
  double flops, bytes;
};
bool g_prof_on = false;
KAcc g_prof[KID_COUNT];
std::vector<Pending> g_pending;
std::vector<cudaEvent_t> g_event_pool;

cudaEvent_t take_event() {
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Brackets one launch with events on `s` when profiling is on.
struct ProfScope {
  bool on;
  Pending p;
  cudaStream_t s;
  ProfScope(cudaStream_t s_, int kid, double flops, double bytes) : on(g_prof_on), s(s_) {
    if (!on) return;
    p.kid = kid;
    p.flops = flops;
    p.bytes = bytes;
    p.a = take_event();
    p.b = take_event();
    cudaEventRecord(p.a, s);
  }
  ~ProfScope() {
    if (!on) return;
    cudaEventRecord(p.b, s);
    g_pending.push_back(p);
  }
};

void resolve_pending() {
  for (auto& p : g_pending) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, p.a, p.b) == cudaSuccess) {
      KAcc& k = g_prof[p.kid];
      k.launches++;
      k.ms += ms;
      k.flops += p.flops;
      k.bytes += p.bytes;
    }
    g_event_pool.push_back(p.a);
    g_event_pool.push_back(p.b);
  }
  g_pending.clear();
}

Dev* cur() { return (g_cur >= 0 && g_dev[g_cur].ready) ? &g_dev[g_cur] : nullptr; }
cudaStream_t stream_of(Dev* d) { return d->user ? d->user : d->own; }

int ensure(Dev* d, Buf& b, size_t bytes, bool zero = false) {
  if (bytes == 0) bytes = 256;
  if (b.bytes >= bytes) return ENVG_OK;
  size_t want = (bytes + (2u << 20) - 1) & ~size_t((2u << 20) - 1);
  if (b.p) {
    ENVG_CUDA(cudaStreamSynchronize(stream_of(d)));
    cudaFree(b.p);
    b.p = nullptr;
    b.bytes = 0;
  }
  if (cudaMalloc(&b.p, want) != cudaSuccess) {
    cudaGetLastError();
    return fail(ENVG_ERR_OOM, "device workspace allocation of %zu bytes failed", want);
  }
  if (zero) {  // zero before any stream, blocking or not, can use the buffer
    ENVG_CUDA(cudaMemset(b.p, 0, want));
    ENVG_CUDA(cudaDeviceSynchronize());
  }
  b.bytes = want;
  d->st.workspace_bytes = d->ws_bytes();
  return ENVG_OK;
}

int get_encode() {
  if (g_encode) return ENVG_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  ENVG_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  if (!fn || q != cudaDriverEntryPointSuccess) return fail(ENVG_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return ENVG_OK;
}

// Loads a kernel's code on the current device now (cuFuncLoad, CUDA 12.4+) rather than at its
// first launch, which is when the runtime loads it under lazy module loading.
int load_kernel(const void* sym) {
  using PfnFuncLoad = CUresult (*)(CUfunction);
  static PfnFuncLoad func_load = nullptr;
  static bool looked_up = false;
  if (!looked_up) {
    looked_up = true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuFuncLoad", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      func_load = reinterpret_cast<PfnFuncLoad>(fn);
    else
      cudaGetLastError();
  }
  if (!func_load) return fail(ENVG_ERR_CUDA, "cuFuncLoad unavailable (driver older than CUDA 12.4)");
  cudaFunction_t f = nullptr;
  ENVG_CUDA(cudaGetFuncBySymbol(&f, sym));
  const CUresult r = func_load(reinterpret_cast<CUfunction>(f));
  if (r != CUDA_SUCCESS) return fail(ENVG_ERR_CUDA, "cuFuncLoad failed: %d", (int)r);
  return ENVG_OK;
}

// 2D bf16 K-major map: dims {inner, rows}, 64 x box_rows boxes, 128-byte swizzle, zero fill.
int tmap_2d(CUtensorMap* tm, const void* base, uint64_t inner, uint64_t rows, uint32_t box_rows) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (inner * 2) % 16)
    return fail(ENVG_ERR_ARG, "TMA operand misaligned (base %p, inner %llu)", base, (unsigned long long)inner);
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ENVG_ERR_CUDA, "cuTensorMapEncodeTiled(2D) failed: %d", (int)r);
  return ENVG_OK;
}

// 4D map over an NHWC bf16 activation [B][H][W][Cp]: dims {Cp, W, H, B}, box {64, tw, th, 1}.
int tmap_nhwc(CUtensorMap* tm, const void* base, int Cp, int W, int H, int B, int tw, int th) {
  cuuint64_t dims[4] = {(cuuint64_t)Cp, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)Cp * 2, (cuuint64_t)W * Cp * 2, (cuuint64_t)H * W * Cp * 2};
  cuuint32_t box[4] = {(cuuint32_t)BK, (cuuint32_t)tw, (cuuint32_t)th, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ENVG_ERR_CUDA, "cuTensorMapEncodeTiled(4D) failed: %d", (int)r);
  return ENVG_OK;
}

// fp32 output maps for the TMA-store epilogue: boxes of 32 columns x box_rows rows (one warp's
// 32 rows, or a CTA's 128), 128-byte swizzle.
int tmap_out_2d(CUtensorMap* tm, const float* base, uint64_t cols, uint64_t rows, uint64_t ld,
                uint32_t box_rows = 32) {
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 4};
  cuuint32_t box[2] = {32, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ENVG_ERR_CUDA, "cuTensorMapEncodeTiled(out 2D) failed: %d", (int)r);
  return ENVG_OK;
}
int tmap_out_3d(CUtensorMap* tm, const float* base, uint64_t plane, uint64_t ch, uint64_t nb,
                uint32_t box_rows = 32) {
  cuuint64_t dims[3] = {plane, ch, nb};
  cuuint64_t strides[2] = {plane * 4, ch * plane * 4};
  cuuint32_t box[3] = {32, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ENVG_ERR_CUDA, "cuTensorMapEncodeTiled(out 3D) failed: %d", (int)r);
  return ENVG_OK;
}

// Picks the k1_gemm store path for a row-major Y (and builds its map for the TMA paths).  With
// peer copies of Y (N-split) and `pm` given, the chunks go out as TMA bulk stores, one per copy.
int choose_store(bool use_tma, EpiArgs& e, CUtensorMap* tmY, PeerMaps* pm = nullptr, CUtensorMap* ybig = nullptr,
                 int* ybig_ok = nullptr) {
  if (use_tma && pm && e.nremote > 0 && e.mode != EPI_ALPHA_BETA) {
    bool ok = e.ldy % 4 == 0 && e.col_off % 4 == 0;
    for (int r = 0; r < e.nremote; ++r) ok = ok && (reinterpret_cast<uintptr_t>(e.remote[r] + e.col_off) & 15) == 0;
    if (ok) {
      for (int r = 0; r < e.nremote; ++r)
        ENVG_TRY(tmap_out_2d(&pm->m[r], e.remote[r] + e.col_off, (uint64_t)e.n_out, (uint64_t)e.m_valid,
                             (uint64_t)e.ldy));
      e.store_mode = e.mode == EPI_GATED_RES ? STORE_TMA_ADD_PEERS : STORE_TMA_PEERS;
      return ENVG_OK;
    }
  }
  if (!use_tma || e.nremote != 0) {  // N-split outputs leave through peer / multicast stores
    e.store_mode = STORE_COALESCED;
    return ENVG_OK;
  }
  e.store_mode = STORE_DIRECT;
  // the maps start at the output's first column (col_off > 0: a kept N-split shard inside a wider Y)
  const float* ybase = e.Y + e.col_off;
  const bool aligned = (reinterpret_cast<uintptr_t>(ybase) & 15) == 0 && e.ldy % 4 == 0;
  if (!aligned) {
    if (e.yb) e.store_mode = STORE_COALESCED;  // the bf16 side output is written on the staged paths
    return ENVG_OK;
  }
  int mode = STORE_TMA;
  if (e.mode == EPI_GATED_RES) mode = STORE_TMA_ADD;
  else if (e.mode == EPI_ALPHA_BETA) mode = e.beta == 0.0f ? STORE_TMA : (e.beta == 1.0f ? STORE_TMA_ADD : STORE_DIRECT);
  if (mode == STORE_DIRECT) return ENVG_OK;
  int rc = tmap_out_2d(tmY, ybase, (uint64_t)e.n_out, (uint64_t)e.m_valid, (uint64_t)e.ldy);
  if (rc != ENVG_OK) return rc;
  if (ybig) {  // k1_gemm_pair's last-unit stores (CTA-high boxes)
    rc = tmap_out_2d(ybig, ybase, (uint64_t)e.n_out, (uint64_t)e.m_valid, (uint64_t)e.ldy, 128);
    if (rc != ENVG_OK) return rc;
    *ybig_ok = 1;
  }
  e.store_mode = mode;
  return ENVG_OK;
}

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t rup(int64_t a, int64_t b) { return cdiv(a, b) * b; }

uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float bf16_to_f32(uint16_t b) {
  const uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// IEEE binary16 -> binary32 (exact; subnormals normalised, Inf/NaN kept).
float f16_to_f32(uint16_t h) {
  const uint32_t s = (uint32_t)(h & 0x8000u) << 16;
  int e = (h >> 10) & 0x1f;
  uint32_t m = h & 0x3ffu, u;
  if (e == 31) {
    u = s | 0x7f800000u | (m << 13);
  } else if (e != 0) {
    u = s | ((uint32_t)(e + 112) << 23) | (m << 13);
  } else if (m == 0) {
    u = s;
  } else {
    e = 1;
    while (!(m & 0x400u)) {
      m <<= 1;
      --e;
    }
    u = s | ((uint32_t)(e + 112) << 23) | ((m & 0x3ffu) << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// Reads element (r, k) of the caller's weight as bf16 bits: b = bf16 bits, f = fp32,
// h = IEEE half bits (exactly one is set).
struct WSrc {
  const uint16_t* b;
  const float* f;
  int64_t ld;
  const uint16_t* h = nullptr;
  uint16_t at(int64_t r, int64_t k) const {
    if (b) return b[r * ld + k];
    if (h) return f32_to_bf16_rne(f16_to_f32(h[r * ld + k]));
    return f32_to_bf16_rne(f[r * ld + k]);
  }
  float value(int64_t r, int64_t k) const {
    if (b) return bf16_to_f32(b[r * ld + k]);
    if (h) return f16_to_f32(h[r * ld + k]);
    return f[r * ld + k];
  }
  // The low bf16 part of the bf16x3 form (k_cast_x3): bf16_rn(v - hi), 0 for an infinite hi.
  uint16_t lo_at(int64_t r, int64_t k) const {
    const float v = value(r, k);
    const float hv = bf16_to_f32(f32_to_bf16_rne(v));
    return std::isinf(hv) ? 0 : f32_to_bf16_rne(v - hv);
  }
  // true when every value of rows [r0, r1) is exactly a bf16 (then all lo parts are zero)
  bool bf16_exact(int64_t r0, int64_t r1, int64_t K) const {
    if (b) return true;
    for (int64_t r = r0; r < r1; ++r)
      for (int64_t k = 0; k < K; ++k) {
        const float v = value(r, k);
        if (!(bf16_to_f32(f32_to_bf16_rne(v)) == v) && !std::isnan(v)) return false;
      }
    return true;
  }
};

}  // namespace

struct envg_weight_s {
  uint32_t magic;
  int dev;
  uint16_t* d;
  size_t bytes;
  int64_t rows;   // rows stored on the device (padding included)
  int64_t N;      // rows seen by envg_linear (N argument)
  int64_t K, Kp;  // logical reduction length; device row length (3 * Ks for a bf16x3 weight)
  int64_t Ks;     // K rounded up to 8: the padded length of one K-segment
  bool x3;        // bf16x3: rows hold hi | lo | hi segments of the fp32 weight (k_cast_x3)
  int layout;
  int64_t half;   // GATE_UP: gate rows (N/2)
  bool conv;
  int out_ch, in_ch, kH, kW, Cp;
  CUtensorMap tm256;  // box 64 x 256 rows: B operand of k1_gemm
  CUtensorMap tm128;  // box 64 x 128 rows: A operand of k2_skinny and of convolutions
};

namespace {

int check_weight(Dev* d, envg_weight w) {
  if (!w || w->magic != WEIGHT_MAGIC) return fail(ENVG_ERR_STATE, "invalid or freed weight handle");
  if (w->dev != d->id) return fail(ENVG_ERR_STATE, "weight lives on device %d, current device is %d", w->dev, d->id);
  return ENVG_OK;
}

int finish_weight(Dev* d, envg_weight w, const std::vector<uint16_t>& host) {
  w->bytes = host.size() * 2;
  if (cudaMalloc(reinterpret_cast<void**>(&w->d), std::max<size_t>(w->bytes, 256)) != cudaSuccess) {
    cudaGetLastError();
    return fail(ENVG_ERR_OOM, "weight allocation of %zu bytes failed", w->bytes);
  }
  ENVG_CUDA(cudaMemcpy(w->d, host.data(), w->bytes, cudaMemcpyHostToDevice));
  ENVG_TRY(tmap_2d(&w->tm256, w->d, w->Kp, w->rows, 256));
  ENVG_TRY(tmap_2d(&w->tm128, w->d, w->Kp, w->rows, 128));
  d->st.weight_bytes += w->bytes;
  return ENVG_OK;
}

// Status word written by bounded device waits; reset after reading.
int check_status(Dev* d) {
  volatile int* hs = d->h_status;
  int st = hs[0];
  if (st != 0) {
    int site = hs[1];
    hs[0] = 0;
    hs[1] = 0;
    if (d->cnt.p) cudaMemsetAsync(d->cnt.p, 0, d->cnt.bytes, stream_of(d));  // re-arm split-K counters
    if (d->sched.p) cudaMemsetAsync(d->sched.p, 0, d->sched.bytes, stream_of(d));  // and the schedules
    d->st.last_status = st;
    return fail(st, "device-side wait exceeded its bound (site %d); pipeline abandoned", site);
  }
  return ENVG_OK;
}

int sync_and_check(Dev* d) {
  ENVG_CUDA(cudaStreamSynchronize(stream_of(d)));
  return check_status(d);
}

// ---- kernel launchers ----------------------------------------------------------------------

// Launch on the library stream.  With programmatic stream serialization (Dev::pdl) the kernel may
// start while the previous kernel of the stream finishes: every kernel launched this way calls
// griddep_wait before its first global memory access, so only its prologue overlaps.  While
// per-launch timing (envg_profile) is on, launches are plainly serialized, so that each kernel's
// events bracket that kernel alone and not its wait for the previous one.
template <typename... KArgs, typename... Args>
int launch_pdl(Dev* d, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream_of(d);
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = (d->pdl && !g_prof_on) ? 1 : 0;
  ENVG_CUDA(cudaLaunchKernelEx(&cfg, kern, args...));
  return ENVG_OK;
}

template <bool CONV_B, bool SILU_GATE>
int launch_k1(Dev* d, const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tY, GemmArgs& a, double flops,
              double bytes) {
  using L = K1Smem<K1_BN, K1_STAGES>;
  auto kern = k1_gemm<K1_BN, K1_STAGES, CONV_B, SILU_GATE>;
  static bool attr = false;
  if (!attr) {
    ENVG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    attr = true;
  }
  a.status = d->d_status;
  a.wait_cap_ns = d->wait_cap_ns;
  const int grid = (int)std::min<int64_t>(a.num_tiles, d->sms);
  if (grid <= 0) return ENVG_OK;
  ProfScope ps(stream_of(d), CONV_B ? KID_K1_CONV : (SILU_GATE ? KID_K1_SILU_GATE : KID_K1), flops, bytes);
  kern<<<grid, K1_THREADS, L::TOTAL, stream_of(d)>>>(tA, tB, tY, a);
  ENVG_CUDA(cudaGetLastError());
  d->st.kernel_launches++;
  return ENVG_OK;
}

// Dynamic shared memory attribute and the number of co-resident CTA pairs of one
// k1_gemm_pair instance (queried once).
template <bool CONV_B, bool SILU_GATE>
int k1_pair_capacity(Dev* d, int* pairs) {
  using L = KPairSmem<KPAIR_STAGES>;
  auto kern = k1_gemm_pair<KPAIR_STAGES, CONV_B, SILU_GATE>;
  static bool attr = false;
  static int max_pairs = 0;
  if (!attr) {
    ENVG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * d->sms, 1, 1);
    cfg.blockDim = dim3(K1_THREADS, 1, 1);
    cfg.dynamicSmemBytes = L::TOTAL;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = d->sms / 2;
    }
    max_pairs = n;
    attr = true;
  }
  *pairs = max_pairs;
  return ENVG_OK;
}

template <bool CONV_B, bool SILU_GATE>
int launch_k1_pair(Dev* d, const CUtensorMap& tA, PairSet& set, double flops, double bytes) {
  using L = KPairSmem<KPAIR_STAGES>;
  auto kern = k1_gemm_pair<KPAIR_STAGES, CONV_B, SILU_GATE>;
  int max_pairs = 0;
  ENVG_TRY((k1_pair_capacity<CONV_B, SILU_GATE>(d, &max_pairs)));
  set.status = d->d_status;
  set.wait_cap_ns = d->wait_cap_ns;
  set.l2_hints = d->l2_hints ? 1 : 0;
  set.sched = nullptr;
  // The dynamic order keeps the pairs at work on a contiguous run of the raster, so the A panels
  // of the current raster group are still in L2 when the next pair needs them.  That pays on long
  // launches whose A operand is larger than the L2 share the groups are sized by (config 4: 16
  // and 140 units per pair, A of 151 and 604 MB; fused_in reads 1.9 instead of 6.2 GB).  On
  // shorter launches, or with A resident in L2, the fixed order measured 0-4% faster.
  const int64_t a_bytes = (int64_t)set.lin[0].tiles_m * set.lin[0].num_kb * (2 * BM * BK * 2);
  if (d->pair_dyn == 2 ||
      (d->pair_dyn == 1 && !CONV_B && a_bytes > PAIR_L2_SHARE && set.total >= (int64_t)PAIR_DYN_UNITS * max_pairs)) {
    // each launch takes the next of SCHED_SLOTS zeroed schedules (launches on different streams
    // may run at once); the launch's last pair zeroes its slot again
    ENVG_TRY(ensure(d, d->sched, SCHED_SLOTS * 2 * sizeof(int), true));
    set.sched = reinterpret_cast<int*>(d->sched.p) + 2 * (d->sched_seq++ % SCHED_SLOTS);
  }
  const int pairs = (int)std::min<int64_t>(set.total, max_pairs);
  if (pairs <= 0) return ENVG_OK;
  ProfScope ps(stream_of(d), CONV_B ? KID_K1_CONV : (SILU_GATE ? KID_K1_SILU_GATE : KID_K1), flops, bytes);
  ENVG_TRY(launch_pdl(d, kern, dim3(2 * pairs), dim3(K1_THREADS), L::TOTAL, tA, set));
  d->st.kernel_launches++;
  return ENVG_OK;
}

// A pair launch of one linear (or convolution) described by GemmArgs-style fields.
PairSet set_of_one(const GemmArgs& g, const CUtensorMap& tB, const CUtensorMap& tY) {
  PairSet set;
  memset(&set, 0, sizeof(set));
  PairLin& P = set.lin[0];
  P.num_kb = g.num_kb;
  P.tiles_m = g.tiles_m;
  P.tiles_n = g.tiles_n;
  P.group_m = g.group_m;
  P.splits = g.splits;
  P.kb_per_split = g.kb_per_split;
  P.tiles_per_split = g.tiles_per_split;
  P.split_rows = g.split_rows;
  P.ybig_ok = g.ybig_ok;
  P.epi = g.epi;
  set.tmB[0] = tB;
  set.tmY[0] = tY;
  set.ybig[0] = g.ybig;
  set.n = 1;
  set.total = g.num_tiles;
  set.base[0] = 0;
  set.base[1] = g.num_tiles;
  set.conv = g.conv;
  set.pm = g.pm;
  return set;
}

template <int MPAD, int R>
struct K2Skinny {
  static constexpr int STAGE_BYTES = K2Smem<MPAD, R, 1>::STAGE_BYTES;
  static constexpr int ST = (110 * 1024) / STAGE_BYTES < 2 ? 2 : (110 * 1024) / STAGE_BYTES;  // two CTAs per SM
  using L = K2Smem<MPAD, R, ST>;
  static constexpr auto kern = k2_skinny<MPAD, R, ST>;
};

// Sets k2_skinny<MPAD, R>'s shared-memory attribute once.  With local set, also loads the
// kernel's code on the device now and returns its local memory per thread.
template <int MPAD, int R>
int k2_prepare(size_t* local) {
  using K = K2Skinny<MPAD, R>;
  static bool attr = false;
  if (!attr) {
    ENVG_CUDA(cudaFuncSetAttribute(K::kern, cudaFuncAttributeMaxDynamicSharedMemorySize, K::L::TOTAL));
    attr = true;
  }
  if (local) {
    ENVG_TRY(load_kernel(reinterpret_cast<const void*>(K::kern)));
    cudaFuncAttributes fa;
    ENVG_CUDA(cudaFuncGetAttributes(&fa, K::kern));
    *local = fa.localSizeBytes;
  }
  return ENVG_OK;
}

template <int MPAD, int R>
int launch_k2_t(Dev* d, const CUtensorMap& tW, const CUtensorMap& tX, SkinnyArgs& a, double flops, double bytes) {
  using L = typename K2Skinny<MPAD, R>::L;
  const auto kern = K2Skinny<MPAD, R>::kern;
  ENVG_TRY((k2_prepare<MPAD, R>(nullptr)));
  a.status = d->d_status;
  a.wait_cap_ns = d->wait_cap_ns;
  ProfScope ps(stream_of(d), KID_K2, flops, bytes);
  kern<<<a.n_tiles * a.splits, K1_THREADS, L::TOTAL, stream_of(d)>>>(tW, tX, a);
  ENVG_CUDA(cudaGetLastError());
  d->st.kernel_launches++;
  return ENVG_OK;
}

int launch_k2(Dev* d, int mpad, int R, const CUtensorMap& tW, const CUtensorMap& tX, SkinnyArgs& a, double flops,
              double bytes) {
  if (R == 1) {
    switch (mpad) {
      case 16: return launch_k2_t<16, 1>(d, tW, tX, a, flops, bytes);
      case 32: return launch_k2_t<32, 1>(d, tW, tX, a, flops, bytes);
      case 48: return launch_k2_t<48, 1>(d, tW, tX, a, flops, bytes);
      case 64: return launch_k2_t<64, 1>(d, tW, tX, a, flops, bytes);
    }
  } else {
    switch (mpad) {
      case 16: return launch_k2_t<16, 2>(d, tW, tX, a, flops, bytes);
      case 32: return launch_k2_t<32, 2>(d, tW, tX, a, flops, bytes);
      case 48: return launch_k2_t<48, 2>(d, tW, tX, a, flops, bytes);
      case 64: return launch_k2_t<64, 2>(d, tW, tX, a, flops, bytes);
    }
  }
  return fail(ENVG_ERR_ARG, "skinny path: unsupported padded M %d", mpad);
}

// One 8 < M <= 64 linear for k2_set: A = its bf16 activation copy [M, Kp].
struct K2Job {
  const void* A;
  int64_t M, Kp;
  const CUtensorMap* w128;  // W, box 64 x 128 rows
  int64_t rows_b;
  bool gu;
  EpiArgs e;
  double flops, bytes;
};

// Splits of a skinny linear: about one unit per SM, at least 8 k-blocks (128 KB of W per 128
// rows) per split; more, shorter splits cost more in partials and reductions than they gain.
// Depends only on the linear's shape.
void k2_plan(const Dev* d, int64_t rows_b, int64_t Kp, bool gu, SkinnyArgs& s) {
  const int R = gu ? 2 : 1;
  const int64_t num_kb = cdiv(Kp, BK);
  s.n_tiles = (int)cdiv(rows_b, (int64_t)R * BM);
  s.num_kb = (int)num_kb;
  int splits = std::max(1, d->sms / s.n_tiles);
  if (splits == 1 && s.n_tiles < d->sms) splits = 2;  // fewer tiles than SMs: do not leave half idle
  splits = (int)std::min<int64_t>(splits, std::max<int64_t>(1, num_kb / 8));
  s.kb_per_split = (int)cdiv(num_kb, splits);
  s.splits = (int)cdiv(num_kb, s.kb_per_split);
}

// k2_set over the set, then (when a linear splits K) k_skinny_reduce over its split linears.
template <int MPAD, int R>
int launch_k2_set_t(Dev* d, K2Set& S, const SkinnyReduceSet& rs, double flops, double bytes) {
  constexpr int STAGE = K2SetSmem<MPAD, R, 1>::STAGE_BYTES;
  constexpr int ST = (110 * 1024) / STAGE < 2 ? 2 : (110 * 1024) / STAGE;  // two CTAs per SM
  using L = K2SetSmem<MPAD, R, ST>;
  auto kern = k2_set<MPAD, R, ST>;
  static bool attr[64] = {};
  if (!attr[d->id]) {
    ENVG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    attr[d->id] = true;
  }
  S.status = d->d_status;
  S.wait_cap_ns = d->wait_cap_ns;
  const int grid = std::min(S.total, 2 * d->sms);
  {
    ProfScope ps(stream_of(d), KID_K2, flops, bytes);
    ENVG_TRY(launch_pdl(d, kern, dim3(grid), dim3(K1_THREADS), L::TOTAL, S));
    d->st.kernel_launches++;
  }
  if (rs.n) {
    double rb = 0.0;
    for (int i = 0; i < rs.n; ++i)
      rb += 16.0 * R * (double)(rs.base[i + 1] - rs.base[i]) * rs.splits[i] +
            4.0 * (double)rs.e[i].m_valid * rs.e[i].n_out;
    ProfScope ps(stream_of(d), KID_SKINNY_REDUCE, 0.0, rb);
    ENVG_TRY(launch_pdl(d, k_skinny_reduce<MPAD, R>, dim3((unsigned)cdiv(rs.base[rs.n], 256)), dim3(256), 0, rs));
    d->st.kernel_launches++;
  }
  return ENVG_OK;
}

// Up to K2S_MAX_LIN skinny linears with the same padded M and the same layout kind (plain, or
// GATE_UP with the SiLU-gate) in one persistent k2_set launch.
int launch_k2_set(Dev* d, const K2Job* jobs, int n) {
  if (n <= 0) return ENVG_OK;
  if (n > K2S_MAX_LIN) return fail(ENVG_ERR_STATE, "launch_k2_set: %d linears", n);
  const int mpad = (int)rup(std::max<int64_t>(jobs[0].M, 1), 16);
  K2Set S{};
  S.n = n;
  size_t part_off = 0;
  std::vector<size_t> po(n);
  double flops = 0.0, bytes = 0.0;
  for (int i = 0; i < n; ++i) {
    const K2Job& q = jobs[i];
    if ((int)rup(std::max<int64_t>(q.M, 1), 16) != mpad || q.gu != jobs[0].gu)
      return fail(ENVG_ERR_STATE, "launch_k2_set: mixed padded M or layout");
    ENVG_TRY(tmap_2d(&S.tmX[i], q.A, q.Kp, q.M, mpad));
    S.tmW[i] = *q.w128;
    K2Lin& L = S.lin[i];
    L.R = q.gu ? 2 : 1;
    k2_plan(d, q.rows_b, q.Kp, q.gu, L.s);
    L.s.epi = q.e;
    S.base[i] = S.total;
    S.total += L.s.n_tiles * L.s.splits;
    po[i] = part_off;
    if (L.s.splits > 1) part_off += (size_t)L.s.n_tiles * L.s.splits * L.R * BM * mpad * sizeof(float);
    flops += q.flops;
    bytes += q.bytes;
  }
  S.base[n] = S.total;
  SkinnyReduceSet rs;
  memset(&rs, 0, sizeof(rs));
  if (part_off) {
    ENVG_TRY(ensure(d, d->part, part_off));
    for (int i = 0; i < n; ++i)
      if (S.lin[i].s.splits > 1) {
        S.lin[i].s.partial = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(d->part.p) + po[i]);
        const int j = rs.n++;
        rs.partial[j] = S.lin[i].s.partial;
        rs.splits[j] = S.lin[i].s.splits;
        rs.e[j] = S.lin[i].s.epi;
        rs.base[j + 1] = rs.base[j] + S.lin[i].s.n_tiles * BM * (mpad / 4);
      }
  }
  const bool gu = jobs[0].gu;
  switch (mpad * 2 + (gu ? 1 : 0)) {
    case 32: ENVG_TRY((launch_k2_set_t<16, 1>(d, S, rs, flops, bytes))); break;
    case 64: ENVG_TRY((launch_k2_set_t<32, 1>(d, S, rs, flops, bytes))); break;
    case 96: ENVG_TRY((launch_k2_set_t<48, 1>(d, S, rs, flops, bytes))); break;
    case 128: ENVG_TRY((launch_k2_set_t<64, 1>(d, S, rs, flops, bytes))); break;
    case 33: ENVG_TRY((launch_k2_set_t<16, 2>(d, S, rs, flops, bytes))); break;
    case 65: ENVG_TRY((launch_k2_set_t<32, 2>(d, S, rs, flops, bytes))); break;
    case 97: ENVG_TRY((launch_k2_set_t<48, 2>(d, S, rs, flops, bytes))); break;
    case 129: ENVG_TRY((launch_k2_set_t<64, 2>(d, S, rs, flops, bytes))); break;
    default: return fail(ENVG_ERR_ARG, "skinny path: unsupported padded M %d", mpad);
  }
  return ENVG_OK;
}

// M <= 8 linear on CUDA cores straight from fp32 X (no cast).
// One M <= 8 linear for k_gemv.
struct GemvJob {
  const float* X;
  int64_t M, K;
  envg_weight W;
  bool gu;
  EpiArgs e;
  double flops, bytes;
  int dep = -1;  // index in the set of the linear whose output is X (chained in the launch), or -1
};

// Resident k_gemv<MT> blocks on the whole GPU.
template <int MT>
int gemv_capacity(Dev* d, int* cap) {
  static int per_sm[64] = {};
  if (!per_sm[d->id]) {
    int nb = 0;
    ENVG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k_gemv<MT>, 256, 0));
    per_sm[d->id] = std::max(1, nb);
  }
  *cap = per_sm[d->id] * d->sms;
  return ENVG_OK;
}

// Up to GEMV_MAX_LIN independent skinny linears in one persistent k_gemv launch.
int launch_gemv_set(Dev* d, const GemvJob* jobs, int n) {
  if (n <= 0) return ENVG_OK;
  if (n > GEMV_MAX_LIN) return fail(ENVG_ERR_STATE, "launch_gemv_set: %d linears", n);
  int64_t mt = 1;
  double flops = 0.0, bytes = 0.0;
  for (int i = 0; i < n; ++i) {
    mt = std::max(mt, jobs[i].M);
    flops += jobs[i].flops;
    bytes += jobs[i].bytes;
  }
  auto capacity = [&](int64_t m, int* c) -> int {
    if (m <= 1) return gemv_capacity<1>(d, c);
    if (m <= 2) return gemv_capacity<2>(d, c);
    if (m <= 4) return gemv_capacity<4>(d, c);
    return gemv_capacity<8>(d, c);
  };
  int cap = 0;
  ENVG_TRY(capacity(mt, &cap));
  GemvSet set{};
  set.n = n;
  set.status = d->d_status;
  set.wait_cap_ns = d->wait_cap_ns;
  size_t part_off = 0, cnt_off = 0;
  std::vector<size_t> po(n), co(n), doff(n, 0);
  std::vector<bool> produces(n, false);
  for (int i = 0; i < n; ++i) {
    if (jobs[i].dep >= i) return fail(ENVG_ERR_STATE, "launch_gemv_set: linear %d depends on %d", i, jobs[i].dep);
    if (jobs[i].dep >= 0) produces[jobs[i].dep] = true;
  }
  for (int i = 0; i < n; ++i) {
    const GemvJob& q = jobs[i];
    GemvArgs& a = set.lin[i];
    a.X = q.X;
    a.ldx = q.K;
    a.M = (int)q.M;
    a.K = (int)q.K;
    a.W = q.W->d;
    a.Kp = q.W->Kp;
    a.rows = (int)q.W->rows;
    a.gate_up = q.gu ? 1 : 0;
    a.groups = (int)(q.gu ? cdiv(q.W->half, 32) : cdiv(q.W->rows, 64));
    // About one unit per resident block for the linear on its own: one with many row groups runs
    // without split-K (partials and their reduction cost more than a short tail); one with few
    // groups and a long K splits it, keeping at least 1024 K elements per split.  The choice
    // depends only on the linear (not on the rest of the set), so a batch sums in the same order
    // as a separate call.
    const int64_t kchunks = cdiv(q.K, 256);
    int own_cap = 0;
    ENVG_TRY(capacity(q.M, &own_cap));
    const int64_t splits = std::max<int64_t>(1, std::min<int64_t>(std::max<int64_t>(1, kchunks / 4),
                                                                    (int64_t)own_cap / a.groups));
    a.kchunk = (int)(cdiv(kchunks, splits) * 256);
    a.splits = (int)cdiv(q.K, a.kchunk);
    a.xvec = (q.K % 8 == 0 && (reinterpret_cast<uintptr_t>(q.X) & 15) == 0) ? 1 : 0;
    a.epi = q.e;
    set.base[i] = set.total;
    set.total += a.groups * a.splits;
    po[i] = part_off;
    co[i] = cnt_off;
    if (a.splits > 1) {
      part_off += (size_t)a.groups * a.splits * GEMV_PART * sizeof(float);
      cnt_off += (size_t)rup(a.groups, 64) * sizeof(int);
    }
    if (produces[i]) {  // completion counters read by the chained linear
      doff[i] = cnt_off;
      cnt_off += 64 * sizeof(int);
    }
  }
  set.base[n] = set.total;
  if (part_off) ENVG_TRY(ensure(d, d->part, part_off));
  if (cnt_off) ENVG_TRY(ensure(d, d->cnt, cnt_off, true));
  uint8_t* cnt_base = reinterpret_cast<uint8_t*>(d->cnt.p);
  for (int i = 0; i < n; ++i) {
    if (set.lin[i].splits > 1) {
      set.lin[i].partial = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(d->part.p) + po[i]);
      set.lin[i].counters = reinterpret_cast<int*>(cnt_base + co[i]);
    }
    if (produces[i]) set.lin[i].done = reinterpret_cast<int*>(cnt_base + doff[i]);
  }
  for (int i = 0; i < n; ++i)
    if (jobs[i].dep >= 0) {
      set.lin[i].wait_on = set.lin[jobs[i].dep].done;
      set.lin[i].wait_groups = set.lin[jobs[i].dep].groups;
    }
  const int grid = std::min(set.total, cap);
  ProfScope ps(stream_of(d), KID_GEMV, flops, bytes);
  auto kern = mt <= 1 ? k_gemv<1> : mt <= 2 ? k_gemv<2> : mt <= 4 ? k_gemv<4> : k_gemv<8>;
  ENVG_TRY(launch_pdl(d, kern, dim3(grid), dim3(256), 0, set));
  d->st.kernel_launches++;
  return ENVG_OK;
}

int launch_gemv(Dev* d, const float* X, int64_t M, int64_t K, envg_weight W, bool gu, const EpiArgs& e, double flops,
                double bytes) {
  const GemvJob j{X, M, K, W, gu, e, flops, bytes};
  return launch_gemv_set(d, &j, 1);
}

// QNNAdaLN (EPSILON = 1e-6, quicknn_common.pas:51) fused with the bf16 cast, or into fp32.
int launch_adaln(Dev* d, const float* x, int64_t rows, int64_t K, int64_t Kp, const float* shift, const float* scale,
                 void* out, bool bf16) {
  if (rows == 0) return ENVG_OK;
  ProfScope ps(stream_of(d), KID_ADALN, 0.0, (double)rows * K * 4 + (double)rows * Kp * (bf16 ? 2 : 4) + 8.0 * K);
  ENVG_TRY(launch_pdl(d, k_adaln, dim3((unsigned)rows), dim3(256), 0, x, K, (int)K, (int)Kp, shift, scale, 1e-6f,
                      out, bf16 ? 1 : 0));
  d->st.kernel_launches++;
  return ENVG_OK;
}

// QNNRMSNorm (EPSILON = 1e-6, quicknn_common.pas:51) fused with the bf16 cast, or into fp32.
int launch_rmsnorm(Dev* d, const float* x, int64_t rows, int64_t K, int64_t Kp, const float* weight, void* out,
                   bool bf16) {
  if (rows == 0) return ENVG_OK;
  ProfScope ps(stream_of(d), KID_RMSNORM, 0.0,
               (double)rows * K * 4 + (double)rows * Kp * (bf16 ? 2 : 4) + (weight ? 4.0 * K : 0.0));
  ENVG_TRY(launch_pdl(d, k_rmsnorm, dim3((unsigned)rows), dim3(256), 0, x, K, (int)K, (int)Kp, weight, 1e-6f, out,
                      bf16 ? 1 : 0));
  d->st.kernel_launches++;
  return ENVG_OK;
}

int launch_cast_rows(Dev* d, const float* x, int64_t ldx, int64_t rows, int64_t K, int64_t Kp, void* xb) {
  if (rows == 0) return ENVG_OK;
  int vec8 = (K == Kp && K % 8 == 0 && ldx % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) ? 1 : 0;
  if (vec8 && ldx == K && (reinterpret_cast<uintptr_t>(xb) & 15) == 0) vec8 = 2;
  const int64_t work = vec8 ? rows * K / 8 : rows * Kp;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(work, 256), (int64_t)d->sms * 8));
  ProfScope ps(stream_of(d), KID_CAST, 0.0, (double)rows * K * 4 + (double)rows * Kp * 2);
  ENVG_TRY(launch_pdl(d, k_cast_rows, dim3(blocks), dim3(256), 0, x, ldx, (int)rows, (int)K, (int)Kp,
                      reinterpret_cast<__nv_bfloat16*>(xb), vec8));
  d->st.kernel_launches++;
  return ENVG_OK;
}

// bf16x3 operand layouts (k_cast_x3): activations hi|hi|lo, weights hi|lo|hi.
constexpr int X3_ACT = 4;
constexpr int X3_WEIGHT = 2;

// x fp32 [rows][K] (row stride ldx) -> bf16 [rows][3 * Ks] in the bf16x3 layout lo_mask.
int launch_cast_x3(Dev* d, const float* x, int64_t ldx, int64_t rows, int64_t K, int64_t Ks, void* out,
                      int lo_mask) {
  if (rows == 0) return ENVG_OK;
  const int64_t work = rows * (Ks / 2);
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(work, 256), (int64_t)d->sms * 8));
  ProfScope ps(stream_of(d), KID_CAST_X3, 0.0, (double)rows * K * 4 + (double)rows * 3 * Ks * 2);
  ENVG_TRY(launch_pdl(d, k_cast_x3, dim3(blocks), dim3(256), 0, x, ldx, (int)rows, (int)K, (int)Ks,
                      reinterpret_cast<__nv_bfloat16*>(out), lo_mask));
  d->st.kernel_launches++;
  return ENVG_OK;
}

// src fp32 [R][C] (row stride lds) -> bf16 [C][3 * Rs], the transpose in the bf16x3 layout lo_mask.
int launch_transpose_x3(Dev* d, const float* src, int64_t lds, int R, int C, void* dst, int Rs, int lo_mask) {
  ProfScope ps(stream_of(d), KID_CAST_X3, 0.0, (double)R * C * 4 + (double)C * 3 * Rs * 2);
  dim3 grid((unsigned)cdiv(C, 32), (unsigned)cdiv(Rs, 64), 1);
  ENVG_TRY(launch_pdl(d, k_transpose_cast_x3, grid, dim3(256), 0, src, lds, R, C,
                      reinterpret_cast<__nv_bfloat16*>(dst), Rs, lo_mask));
  d->st.kernel_launches++;
  return ENVG_OK;
}

// fp32 [batch][R][C] -> bf16 [batch][C][Rp]
int launch_transpose_cast(Dev* d, const float* src, int64_t lds, int64_t sbs, int R, int C, void* dst, int64_t ldd,
                          int64_t dbs, int Rp, int batch, const float2* aff = nullptr, int act = 0) {
  ProfScope ps(stream_of(d), KID_TRANSPOSE, 0.0, (double)batch * ((double)R * C * 4 + (double)C * Rp * 2));
  const bool vec = C % 4 == 0 && lds % 4 == 0 && sbs % 4 == 0 && Rp % 8 == 0 && ldd % 8 == 0 && dbs % 8 == 0 &&
                   (reinterpret_cast<uintptr_t>(src) & 15) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
  if (vec) {
    dim3 grid((unsigned)cdiv(C, 64), (unsigned)cdiv(Rp, 64), (unsigned)batch);
    ENVG_TRY(launch_pdl(d, k_transpose_cast_v, grid, dim3(256), 0, src, lds, sbs, R, C,
                        reinterpret_cast<__nv_bfloat16*>(dst), ldd, dbs, Rp, aff, act));
  } else {
    dim3 grid((unsigned)cdiv(C, 32), (unsigned)cdiv(Rp, 64), (unsigned)batch);
    ENVG_TRY(launch_pdl(d, k_transpose_cast, grid, dim3(256), 0, src, lds, sbs, R, C,
                        reinterpret_cast<__nv_bfloat16*>(dst), ldd, dbs, Rp, aff, act));
  }
  d->st.kernel_launches++;
  return ENVG_OK;
}

// ---- split-K for mid-size M ----------------------------------------------------------------
// Below SPLIT_MAX_M rows a linear has at most four 256-row pair tiles in M, and a narrow N leaves
// most CTA pairs idle (Qwen3's k / v at 512 tokens: 8 tiles for 74 pairs).  Such a launch cuts
// K into `splits` contiguous ranges; every (split, tile) unit stores its raw fp32 tile, and
// k_split_reduce adds the splits in split order and applies the epilogue.  The split count
// depends only on (M, N, K) and the device, so repeated calls give identical results.  N-split
// shards (outputs on several ranks) never split K.
// A call of M >= SPLIT_MAX_M rows never splits; the row chunks of a pipelined host call (such a
// call, cut into chunks of PIPE_CHUNK rows) are launched with splitting off (Dev::no_split), so
// they sum in the same order as one launch over all rows.
constexpr int64_t SPLIT_MAX_M = 1024;
constexpr int SPLIT_MIN_KB = 4;        // K blocks per split at least
constexpr int SPLIT_MAX = 16;
constexpr double SPLIT_US_PER_KB = 0.42;  // one 64-deep K block of a 256 x 256 pair tile, measured
constexpr double SPLIT_REDUCE_US = 3.0;   // launch and tail of k_split_reduce

int pair_splits(Dev* d, int64_t M, int tiles, int num_kb, int64_t Mp, int64_t ldp, int* splits, int* kb_per) {
  *splits = 1;
  *kb_per = num_kb;
  if (d->pair_split == 0 || d->no_split || M >= SPLIT_MAX_M || num_kb < 2) return ENVG_OK;
  auto eff = [&](int sp, int* kbp) {
    *kbp = (int)cdiv(num_kb, sp);
    return (int)cdiv(num_kb, *kbp);
  };
  if (d->pair_split > 0) {  // forced count (tests and sweeps)
    *splits = eff(std::min(d->pair_split, num_kb), kb_per);
    return ENVG_OK;
  }
  if (num_kb < 2 * SPLIT_MIN_KB) return ENVG_OK;
  int P = 0;
  ENVG_TRY((k1_pair_capacity<false, false>(d, &P)));
  int best = 1;
  double best_us = (double)cdiv(tiles, P) * num_kb * SPLIT_US_PER_KB;
  for (int sp = 2; sp <= SPLIT_MAX && sp * SPLIT_MIN_KB <= num_kb; ++sp) {
    int kbp = 0;
    const int se = eff(sp, &kbp);
    const double part_bytes = 4.0 * (double)se * (double)Mp * (double)ldp;
    const double us = (double)cdiv((int64_t)tiles * se, P) * kbp * SPLIT_US_PER_KB + SPLIT_REDUCE_US +
                      2.0 * part_bytes / 6.5e6;  // partials written and read back at HBM speed
    if (us < best_us) {
      best_us = us;
      best = se;
    }
  }
  if (best > 1) *splits = eff(best, kb_per);
  return ENVG_OK;
}

int launch_split_reduce(Dev* d, SplitReduceSet& rs) {
  const int64_t work = rs.base[rs.n];
  if (work == 0) return ENVG_OK;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(work, 256), (int64_t)d->sms * 8));
  double bytes = 0.0;
  for (int i = 0; i < rs.n; ++i) {
    const EpiArgs& e = rs.e[i];
    const bool rmw = e.mode == EPI_GATED_RES || (e.mode == EPI_ALPHA_BETA && e.beta != 0.0f);
    bytes += 4.0 * (double)rs.splits[i] * e.m_valid * (rs.silu_gate[i] ? 2.0 * e.n_out : e.n_out) +
             (rmw ? 8.0 : 4.0) * (double)e.m_valid * e.n_out;
  }
  ProfScope ps(stream_of(d), KID_SPLIT_REDUCE, 0.0, bytes);
  ENVG_TRY(launch_pdl(d, k_split_reduce, dim3(blocks), dim3(256), 0, rs));
  d->st.kernel_launches++;
  return ENVG_OK;
}

// One linear of a k1_gemm_pair launch, host side.
struct PairJob {
  const CUtensorMap* tB;  // its weight, 128-row boxes
  int64_t rows_b;         // weight rows on the device
  bool gu;                // SiLU-gate (GATE_UP weight)
  EpiArgs e;              // its epilogue
  double flops, bytes;
};

// M-tiles (256-row A panels) per raster group of k1_gemm_pair.  A group's units sweep all of W's
// column panels while its A panels stay in L2, so each W panel is read from HBM tiles_m / group_m
// times: as many panels as fit a 64 MB share of the 126 MB L2, from 4 to 16.  Measured on config
// 4 (ncu DRAM bytes per launch): the 18432x4096x36864 linear reads 11.1 GB at 4 panels and 2.9 GB
// at 16 (4.33 -> 3.78 ms); the K = 16384 one reads 4.6 GB at 4 and 3.6 GB at 8.
int pair_group_m(const Dev* d, int64_t Kp) {
  if (d->pair_group_m > 0) return d->pair_group_m;
  const int64_t panel = 2 * (int64_t)BM * Kp * 2;
  return (int)std::max<int64_t>(4, std::min<int64_t>(16, PAIR_L2_SHARE / panel));
}

// Linears that share the activation operand A[M, Kp] (M > 128) as k1_gemm_pair launches: one
// launch per kernel variant present (the SiLU-gate variant for unsplit GATE_UP linears, the
// plain one for the rest), each walking all its linears' units; then one k_split_reduce per
// linear that splits K.  Each linear's split count is its own (pair_splits), so a linear gives
// the same bits whether it runs alone or in a set.
int launch_pair_set(Dev* d, const void* A, int64_t M, int64_t Kp, PairJob* jobs, int n) {
  CUtensorMap tA;
  ENVG_TRY(tmap_2d(&tA, A, Kp, M, BM));
  const int num_kb = (int)cdiv(Kp, BK);
  const int tiles_m = (int)cdiv(M, 2 * BM);
  const int64_t Mp = (int64_t)tiles_m * 2 * BM;
  int sp[PSET_MAX], kbp[PSET_MAX];
  size_t off[PSET_MAX], part = 0;
  for (int i = 0; i < n; ++i) {
    const int tiles = tiles_m * (int)cdiv(jobs[i].rows_b, K1_BN);
    sp[i] = 1;
    kbp[i] = num_kb;
    if (jobs[i].e.nremote == 0)
      ENVG_TRY(pair_splits(d, M, tiles, num_kb, Mp, rup(jobs[i].rows_b, 4), &sp[i], &kbp[i]));
    off[i] = part;
    if (sp[i] > 1) part += ((size_t)(sp[i] * Mp * rup(jobs[i].rows_b, 4)) * 4 + 255) & ~size_t(255);
  }
  if (part) ENVG_TRY(ensure(d, d->part, part));
  // Units are handed to CTA pairs in order (pair p takes units p, p + pairs, ...), so the
  // linears with the longest units (most K blocks each) go first and the short ones fill in.
  int order[PSET_MAX];
  for (int i = 0; i < n; ++i) order[i] = i;
  std::stable_sort(order, order + n, [&](int a, int b) { return kbp[a] > kbp[b]; });
  for (int pass = 0; pass < 2; ++pass) {  // pass 0: plain kernel; pass 1: SiLU-gate kernel
    PairSet set;
    memset(&set, 0, sizeof(set));
    double flops = 0.0, bytes = 0.0;
    for (int oi = 0; oi < n; ++oi) {
      const int i = order[oi];
      const bool silu_kernel = jobs[i].gu && sp[i] == 1;
      if (silu_kernel != (pass == 1)) continue;
      const int j = set.n++;
      PairLin& P = set.lin[j];
      P.num_kb = num_kb;
      P.tiles_m = tiles_m;
      P.tiles_n = (int)cdiv(jobs[i].rows_b, K1_BN);
      P.group_m = pair_group_m(d, Kp);
      P.tiles_per_split = P.tiles_m * P.tiles_n;
      set.tmB[j] = *jobs[i].tB;
      if (sp[i] > 1) {
        // the units store raw partials [sp][Mp][ldp]; k_split_reduce finishes Y
        const int64_t ldp = rup(jobs[i].rows_b, 4);
        float* p = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(d->part.p) + off[i]);
        ENVG_TRY(tmap_out_2d(&set.tmY[j], p, (uint64_t)ldp, (uint64_t)(sp[i] * Mp), (uint64_t)ldp));
        ENVG_TRY(tmap_out_2d(&set.ybig[j], p, (uint64_t)ldp, (uint64_t)(sp[i] * Mp), (uint64_t)ldp, 128));
        P.ybig_ok = 1;
        P.splits = sp[i];
        P.kb_per_split = kbp[i];
        P.split_rows = (int)Mp;
        EpiArgs& ep = P.epi;
        ep.Y = p;
        ep.ldy = ldp;
        ep.mode = EPI_PLAIN;
        ep.n_out = (int)ldp;
        ep.m_valid = (int)(sp[i] * Mp);
        ep.vec_ok = 1;
        ep.store_mode = STORE_TMA;
      } else {
        P.epi = jobs[i].e;
        ENVG_TRY(choose_store(d->store_tma, P.epi, &set.tmY[j], n == 1 ? &set.pm : nullptr, &set.ybig[j],
                              &P.ybig_ok));
        if (P.epi.nremote > 0 && P.epi.store_mode >= STORE_TMA_PEERS && n != 1)
          return fail(ENVG_ERR_STATE, "internal: peer-store maps in a pair set");
      }
      set.base[j + 1] = set.base[j] + P.tiles_per_split * std::max(1, P.splits);
      flops += jobs[i].flops;
      bytes += jobs[i].bytes;
    }
    if (set.n == 0) continue;
    set.total = set.base[set.n];
    if (pass == 1) ENVG_TRY((launch_k1_pair<false, true>(d, tA, set, flops, bytes)));
    else ENVG_TRY((launch_k1_pair<false, false>(d, tA, set, flops, bytes)));
  }
  SplitReduceSet rs;
  memset(&rs, 0, sizeof(rs));
  for (int i = 0; i < n; ++i)
    if (sp[i] > 1) {
      const int j = rs.n++;
      rs.ldp[j] = rup(jobs[i].rows_b, 4);
      rs.part[j] = reinterpret_cast<const float*>(reinterpret_cast<uint8_t*>(d->part.p) + off[i]);
      rs.split_elems[j] = Mp * rs.ldp[j];
      rs.splits[j] = sp[i];
      rs.silu_gate[j] = jobs[i].gu ? 1 : 0;
      rs.e[j] = jobs[i].e;
      rs.base[j + 1] = rs.base[j] + (int64_t)rs.e[j].m_valid * cdiv(rs.e[j].n_out, 4);
    }
  if (rs.n) ENVG_TRY(launch_split_reduce(d, rs));
  return ENVG_OK;
}

// Core GEMM on device operands: Y = epilogue(A[M, Kp] . B[rows, Kp]^T).
//   A: bf16 activations (M rows);  B: bf16 weights (rows_b rows), with maps for both boxes.
int gemm_device(Dev* d, const void* A, int64_t M, int64_t Kp, const CUtensorMap& b256, const CUtensorMap& b128,
                int64_t rows_b, bool silu_gate, EpiArgs e, double flops, double bytes) {
  const int64_t num_kb = cdiv(Kp, BK);
  if (M <= d->skinny_max) {
    const K2Job j{A, M, Kp, &b128, rows_b, silu_gate, e, flops, bytes};
    return launch_k2_set(d, &j, 1);
  }
  if (d->use_pair && M > BM) {
    PairJob j{&b128, rows_b, silu_gate, e, flops, bytes};
    return launch_pair_set(d, A, M, Kp, &j, 1);
  }
  CUtensorMap tA;
  ENVG_TRY(tmap_2d(&tA, A, Kp, M, BM));
  GemmArgs g{};
  g.num_kb = (int)num_kb;
  g.tiles_n = (int)cdiv(rows_b, K1_BN);
  g.group_m = 8;
  CUtensorMap tY;
  memset(&tY, 0, sizeof(tY));
  ENVG_TRY(choose_store(d->store_tma, e, &tY, &g.pm));
  g.epi = e;
  g.tiles_m = (int)cdiv(M, BM);
  g.num_tiles = g.tiles_m * g.tiles_n;
  if (silu_gate) return launch_k1<false, true>(d, tA, b256, tY, g, flops, bytes);
  return launch_k1<false, false>(d, tA, b256, tY, g, flops, bytes);
}

int upload_common(Dev* d, WSrc src, int64_t N, int64_t K, int64_t n0, int64_t n1, int layout, envg_weight* out) {
  if (!out) return fail(ENVG_ERR_ARG, "out handle pointer is NULL");
  *out = nullptr;
  if (N <= 0 || K <= 0) return fail(ENVG_ERR_ARG, "weight shape [%lld, %lld] invalid", (long long)N, (long long)K);
  const bool round_bf16 = (layout & ENVG_LAYOUT_ROUND_BF16) != 0;
  layout &= ~ENVG_LAYOUT_ROUND_BF16;
  if (layout != ENVG_LAYOUT_PLAIN && layout != ENVG_LAYOUT_GATE_UP)
    return fail(ENVG_ERR_ARG, "unknown layout flag %d", layout);
  const bool gu = layout == ENVG_LAYOUT_GATE_UP;
  if (gu && (N % 2)) return fail(ENVG_ERR_ARG, "GATE_UP weight needs an even row count, got %lld", (long long)N);
  const int64_t lim = gu ? N / 2 : N;
  if (n0 < 0 || n1 > lim || n0 >= n1)
    return fail(ENVG_ERR_ARG, "shard [%lld, %lld) outside [0, %lld)", (long long)n0, (long long)n1, (long long)lim);
  // An fp32 / fp16 weight whose values are not all bf16 numbers keeps its low parts: the bf16x3
  // form (k_cast_x3), unless the caller asked for plain RNE rounding.
  bool x3 = !round_bf16 && !src.b;
  if (x3) x3 = !(src.bf16_exact(n0, n1, K) && (!gu || src.bf16_exact(N / 2 + n0, N / 2 + n1, K)));
  auto* w = new envg_weight_s();
  w->magic = WEIGHT_MAGIC;
  w->dev = d->id;
  w->K = K;
  w->Ks = rup(K, 8);
  w->x3 = x3;
  w->Kp = x3 ? 3 * w->Ks : w->Ks;
  w->layout = layout;
  w->conv = false;
  std::vector<uint16_t> host;
  // device row rd <- source row rs: hi parts, or hi | lo | hi for a bf16x3 weight
  auto put = [&](int64_t rd, int64_t rs) {
    uint16_t* row = &host[(size_t)(rd * w->Kp)];
    for (int64_t k = 0; k < K; ++k) {
      const uint16_t hb = src.at(rs, k);
      row[k] = hb;
      if (x3) {
        row[w->Ks + k] = src.lo_at(rs, k);
        row[2 * w->Ks + k] = hb;
      }
    }
  };
  const int64_t cnt = n1 - n0;
  if (!gu) {
    w->N = cnt;
    w->rows = cnt;
    host.assign((size_t)(w->rows * w->Kp), 0);
    for (int64_t r = 0; r < cnt; ++r) put(r, n0 + r);
  } else {
    // Interleave per 128-row block: device rows [256t, 256t+128) = gate rows [128t, 128t+128),
    // rows [256t+128, 256t+256) = the matching up rows; missing rows are zero.
    const int64_t half = N / 2;
    w->half = cnt;
    w->N = 2 * cnt;
    const int64_t hp = rup(cnt, BM);
    w->rows = 2 * hp;
    host.assign((size_t)(w->rows * w->Kp), 0);
    for (int64_t j = 0; j < cnt; ++j) {
      const int64_t t = j / BM, i = j % BM;
      const int64_t rg = 2 * BM * t + i, ru = rg + BM;
      put(rg, n0 + j);
      put(ru, half + n0 + j);
    }
  }
  int rc = finish_weight(d, w, host);
  if (rc != ENVG_OK) {
    if (w->d) cudaFree(w->d);
    w->magic = 0;
    delete w;
    return rc;
  }
  *out = w;
  return ENVG_OK;
}

int conv_upload_common(Dev* d, WSrc src, int out_ch, int in_ch, int kH, int kW, envg_weight* out) {
  if (!out) return fail(ENVG_ERR_ARG, "out handle pointer is NULL");
  *out = nullptr;
  if (out_ch <= 0 || in_ch <= 0 || kH <= 0 || kW <= 0)
    return fail(ENVG_ERR_ARG, "conv weight shape [%d, %d, %d, %d] invalid", out_ch, in_ch, kH, kW);
  // Device layout W'[out_ch][kH][kW][Cp] (Cp = in_ch rounded up to 64, zero filled): the
  // reduction index becomes (kh, kw, c), matching the NHWC activation tiles.
  auto* w = new envg_weight_s();
  w->magic = WEIGHT_MAGIC;
  w->dev = d->id;
  w->conv = true;
  w->out_ch = out_ch;
  w->in_ch = in_ch;
  w->kH = kH;
  w->kW = kW;
  w->Cp = (int)rup(in_ch, BK);
  w->K = (int64_t)in_ch * kH * kW;
  w->Kp = (int64_t)kH * kW * w->Cp;
  w->Ks = w->Kp;
  w->N = out_ch;
  w->rows = out_ch;
  w->layout = ENVG_LAYOUT_PLAIN;
  std::vector<uint16_t> host((size_t)(w->rows * w->Kp), 0);
  for (int o = 0; o < out_ch; ++o)
    for (int c = 0; c < in_ch; ++c)
      for (int kh = 0; kh < kH; ++kh)
        for (int kw = 0; kw < kW; ++kw)
          host[(size_t)(o * w->Kp + ((int64_t)kh * kW + kw) * w->Cp + c)] = src.at(o, ((int64_t)c * kH + kh) * kW + kw);
  int rc = finish_weight(d, w, host);
  if (rc != ENVG_OK) {
    if (w->d) cudaFree(w->d);
    w->magic = 0;
    delete w;
    return rc;
  }
  *out = w;
  return ENVG_OK;
}


// A read-only mapping of a whole file (the reference maps its safetensors files the same way,
// safetensor.pas:275-326).
struct MappedFile {
  void* p = MAP_FAILED;
  size_t size = 0;
  ~MappedFile() {
    if (p != MAP_FAILED) munmap(p, size);
  }
  int open(const char* path) {
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) return fail(ENVG_ERR_ARG, "cannot open %s", path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
      ::close(fd);
      return fail(ENVG_ERR_ARG, "cannot stat %s", path);
    }
    size = (size_t)st.st_size;
    p = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (p == MAP_FAILED) return fail(ENVG_ERR_OOM, "mmap of %s (%zu bytes) failed", path, size);
    return ENVG_OK;
  }
};

int st_dtype(const std::string& dt) {
  if (dt == "BF16") return ENVG_DTYPE_BF16;
  if (dt == "F16") return ENVG_DTYPE_F16;
  if (dt == "F32") return ENVG_DTYPE_F32;
  return ENVG_DTYPE_OTHER;
}

// Finds `name` and checks that its byte count matches dtype x shape.  *count = element count.
int st_lookup(const char* path, const char* name, envg_st::TensorInfo* ti, int64_t* count) {
  if (!path || !name) return fail(ENVG_ERR_ARG, "path and tensor name must be set");
  const std::string why = envg_st::find_tensor(path, name, ti);
  if (!why.empty()) return fail(ENVG_ERR_ARG, "safetensors %s: %s", path, why.c_str());
  if (ti->shape.size() > 8) return fail(ENVG_ERR_UNSUPPORTED, "tensor %s has %zu dims (> 8)", name, ti->shape.size());
  int64_t n = 1;
  for (int64_t v : ti->shape) {
    if (v < 0) return fail(ENVG_ERR_ARG, "tensor %s has a negative dimension", name);
    n *= v;
  }
  *count = n;
  const int64_t eb = envg_st::dtype_bytes(ti->dtype);
  if (eb && n * eb != ti->end - ti->begin)
    return fail(ENVG_ERR_ARG, "tensor %s: %lld bytes of data for %lld elements of %s", name,
                (long long)(ti->end - ti->begin), (long long)n, ti->dtype.c_str());
  return ENVG_OK;
}

// Maps the file and points `src` at the tensor's data.  Data that is not aligned to its element
// size (the format does not promise it) is copied into `copy` first.
int st_source(const char* path, const envg_st::TensorInfo& ti, int64_t ld, MappedFile* mf,
              std::vector<uint32_t>* copy, WSrc* src) {
  ENVG_TRY(mf->open(path));
  const int dt = st_dtype(ti.dtype);
  if (dt == ENVG_DTYPE_OTHER)
    return fail(ENVG_ERR_UNSUPPORTED, "tensor dtype %s cannot be uploaded (BF16, F16 or F32 only)", ti.dtype.c_str());
  const size_t nbytes = (size_t)(ti.end - ti.begin);
  const unsigned char* base = static_cast<const unsigned char*>(mf->p) + ti.data_start + ti.begin;
  const void* data = base;
  const size_t align = dt == ENVG_DTYPE_F32 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(base) % align) {
    copy->assign((nbytes + 3) / 4, 0);
    memcpy(copy->data(), base, nbytes);
    data = copy->data();
  }
  *src = WSrc{nullptr, nullptr, ld};
  if (dt == ENVG_DTYPE_BF16) src->b = static_cast<const uint16_t*>(data);
  if (dt == ENVG_DTYPE_F16) src->h = static_cast<const uint16_t*>(data);
  if (dt == ENVG_DTYPE_F32) src->f = static_cast<const float*>(data);
  return ENVG_OK;
}

const char* epi_name(int e) {
  switch (e) {
    case ENVG_EPI_NONE: return "NONE";
    case ENVG_EPI_BIAS: return "BIAS";
    case ENVG_EPI_SILU_GATE: return "SILU_GATE";
    case ENVG_EPI_GATED_RESIDUAL: return "GATED_RESIDUAL";
    case ENVG_EPI_SILU: return "SILU";
  }
  return "?";
}

}  // namespace

// ---- scratch of envg_linear_noalloc ----------------------------------------------------------
// Layout: [0, 2 MiB) bf16 activations [M, Kp]; then split-K partial sums; the last 64 KiB hold
// the per-tile split-K counters.  Host code must not take this symbol's address directly (it
// names a host-side stand-in); noalloc_scratch() asks the runtime for the device address.
constexpr size_t NOALLOC_XB_BYTES = 2u << 20;
constexpr size_t NOALLOC_CNT_BYTES = 64u << 10;
constexpr size_t NOALLOC_PART_BYTES = ENVG_NOALLOC_SCRATCH_BYTES - NOALLOC_XB_BYTES - NOALLOC_CNT_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[ENVG_NOALLOC_SCRATCH_BYTES];
void* g_noalloc_ptr[64] = {};

// Device address of the scratch array on the current device (looked up once per device).
int noalloc_scratch(Dev* d, uint8_t** out) {
  if (!g_noalloc_ptr[d->id]) {
    void* p = nullptr;
    ENVG_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    if (!p) return fail(ENVG_ERR_CUDA, "cudaGetSymbolAddress returned NULL for the no-alloc scratch");
    g_noalloc_ptr[d->id] = p;
  }
  *out = reinterpret_cast<uint8_t*>(g_noalloc_ptr[d->id]);
  return ENVG_OK;
}

// Run by envg_init: everything envg_linear_noalloc would otherwise set up on first use, some of
// which takes device memory.  With lazy module loading the runtime loads a kernel's code on its
// first use and may map a new block of device memory for it, and a kernel that needs more local
// memory per thread than the context holds grows that reservation at its first launch.  So this
// loads every kernel the entry point launches (the eight k2_skinny shapes, k_cast_rows and, for
// bf16x3 weights, k_cast_x3),
// raises the context's stack limit to their largest local-memory need, looks up the scratch
// array and issues one memset into it.
int noalloc_preload(Dev* d) {
  size_t need = 0, l = 0;
  ENVG_TRY((k2_prepare<16, 1>(&l))); need = std::max(need, l);
  ENVG_TRY((k2_prepare<32, 1>(&l))); need = std::max(need, l);
  ENVG_TRY((k2_prepare<48, 1>(&l))); need = std::max(need, l);
  ENVG_TRY((k2_prepare<64, 1>(&l))); need = std::max(need, l);
  ENVG_TRY((k2_prepare<16, 2>(&l))); need = std::max(need, l);
  ENVG_TRY((k2_prepare<32, 2>(&l))); need = std::max(need, l);
  ENVG_TRY((k2_prepare<48, 2>(&l))); need = std::max(need, l);
  ENVG_TRY((k2_prepare<64, 2>(&l))); need = std::max(need, l);
  ENVG_TRY(load_kernel(reinterpret_cast<const void*>(k_cast_rows)));
  ENVG_TRY(load_kernel(reinterpret_cast<const void*>(k_cast_x3)));
  cudaFuncAttributes fa;
  ENVG_CUDA(cudaFuncGetAttributes(&fa, k_cast_rows));
  need = std::max(need, fa.localSizeBytes);
  ENVG_CUDA(cudaFuncGetAttributes(&fa, k_cast_x3));
  need = std::max(need, fa.localSizeBytes);
  size_t have = 0;
  ENVG_CUDA(cudaDeviceGetLimit(&have, cudaLimitStackSize));
  if (need > have) ENVG_CUDA(cudaDeviceSetLimit(cudaLimitStackSize, need));
  uint8_t* scratch = nullptr;
  ENVG_TRY(noalloc_scratch(d, &scratch));
  ENVG_CUDA(cudaMemsetAsync(scratch + NOALLOC_XB_BYTES + NOALLOC_PART_BYTES, 0, sizeof(int), d->own));
  ENVG_CUDA(cudaStreamSynchronize(d->own));
  return ENVG_OK;
}

// =============================================================================================
// C ABI
// =============================================================================================
extern "C" {

const char* envg_version(void) { return "envgemm 0.1 sm_100a (tcgen05/TMA)"; }

const char* envg_last_error(void) { return t_err.c_str(); }

int envg_init(int ndev, const int* dev_ids) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (ndev != 1)
    return fail(ENVG_ERR_UNSUPPORTED, "envg_init: ndev=%d; this build drives one device per process", ndev);
  const int id = dev_ids ? dev_ids[0] : 0;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    return fail(ENVG_ERR_CUDA, "no CUDA device visible");
  }
  if (id < 0 || id >= count || id >= 64) return fail(ENVG_ERR_ARG, "device id %d out of range (%d devices)", id, count);
  ENVG_CUDA(cudaSetDevice(id));
  Dev* d = &g_dev[id];
  g_cur = id;
  if (d->ready) return ENVG_OK;
  cudaDeviceProp prop;
  ENVG_CUDA(cudaGetDeviceProperties(&prop, id));
  if (prop.major != 10)
    return fail(ENVG_ERR_UNSUPPORTED, "device %d is sm_%d%d; libenvgemm is built for sm_100a", id, prop.major, prop.minor);
  ENVG_TRY(get_encode());
  d->id = id;
  d->sms = prop.multiProcessorCount;
  ENVG_CUDA(cudaStreamCreateWithFlags(&d->own, cudaStreamNonBlocking));
  ENVG_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&d->h_status), 2 * sizeof(int), cudaHostAllocMapped));
  d->h_status[0] = d->h_status[1] = 0;
  ENVG_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&d->d_status), d->h_status, 0));
  if (const char* s = getenv("ENVG_WAIT_CAP")) {
    long long ms = atoll(s);
    if (ms > 0) d->wait_cap_ns = (uint64_t)ms * 1000000ull;
  }
  if (const char* s = getenv("ENVG_K1")) d->use_pair = strcmp(s, "single") != 0;
  if (const char* s = getenv("ENVG_STORE")) d->store_tma = strcmp(s, "coalesced") != 0;
  if (const char* s = getenv("ENVG_PIPE")) d->pipe_host = strcmp(s, "0") != 0;
  if (const char* s = getenv("ENVG_PDL")) d->pdl = strcmp(s, "0") != 0;
  if (const char* s = getenv("ENVG_L2_HINTS")) d->l2_hints = strcmp(s, "0") != 0;
  if (const char* s = getenv("ENVG_PAIR_SCHED")) d->pair_dyn = !strcmp(s, "static") ? 0 : !strcmp(s, "dynamic") ? 2 : 1;
  if (const char* s = getenv("ENVG_GEMV_CHAIN")) d->gemv_chain = strcmp(s, "0") != 0;
  if (const char* s = getenv("ENVG_PAIR_GROUP_M")) {
    const int v = atoi(s);
    if (v >= 1 && v <= 64) d->pair_group_m = v;
  }
  if (const char* s = getenv("ENVG_PAIR_SPLIT")) {
    const int v = atoi(s);
    if (v >= 0 && v <= 64) d->pair_split = v;
  }
  if (const char* s = getenv("ENVG_ATTN_TILES")) {
    const int v = atoi(s);
    if (v == 1 || v == 2) d->attn_tiles = v;
  }
  if (const char* s = getenv("ENVG_GEMV_M_MAX")) {
    int v = atoi(s);
    if (v >= 0 && v <= 8) d->gemv_max = v;
  }
  if (const char* s = getenv("ENVG_SKINNY_M_MAX")) {
    int v = atoi(s);
    if (v >= 0 && v <= SKINNY_MAX) d->skinny_max = v;
  }
  d->st = envg_stats{};
  d->st.device = id;
  ENVG_TRY(noalloc_preload(d));
  d->ready = true;
  return ENVG_OK;
}

int envg_shutdown(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return ENVG_OK;
  cudaStreamSynchronize(stream_of(d));
  Buf* bufs[] = {&d->x,    &d->y,   &d->xb,  &d->wb,  &d->part,  &d->cnt,
                 &d->bias, &d->gate, &d->act, &d->col, &d->b32, &d->xbatch, &d->ada, &d->xn,
                 &d->gn,   &d->c1,   &d->vec,  &d->fa,  &d->fain, &d->sched, &d->hb};
  for (Buf* b : bufs) {
    if (b->p) cudaFree(b->p);
    *b = Buf{};
  }
  if (d->own) cudaStreamDestroy(d->own);
  if (d->aux) cudaStreamDestroy(d->aux);
  if (d->h2d) cudaStreamDestroy(d->h2d);
  if (d->d2h) cudaStreamDestroy(d->d2h);
  d->h2d = d->d2h = nullptr;
  for (cudaEvent_t e : d->pipe_events) cudaEventDestroy(e);
  d->pipe_events.clear();
  for (cudaEvent_t e : d->batch_events) cudaEventDestroy(e);
  d->batch_events.clear();
  d->aux = nullptr;
  if (d->h_status) cudaFreeHost(d->h_status);
  d->own = nullptr;
  d->user = nullptr;
  d->h_status = d->d_status = nullptr;
  d->ready = false;
  g_cur = -1;
  return ENVG_OK;
}

int envg_set_stream(void* stream) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  d->user = reinterpret_cast<cudaStream_t>(stream);
  return ENVG_OK;
}

int envg_sync(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  return sync_and_check(d);
}

int envg_set_wait_cap_ns(uint64_t ns) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  d->wait_cap_ns = ns ? ns : DEFAULT_WAIT_CAP_NS;
  return ENVG_OK;
}

int envg_get_stats(envg_stats* out) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!out) return fail(ENVG_ERR_ARG, "stats pointer is NULL");
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  d->st.workspace_bytes = d->ws_bytes();
  *out = d->st;
  return ENVG_OK;
}

int envg_weight_upload(const uint16_t* w_bf16, const float* w_f32, int64_t N, int64_t K, int layout_flags,
                       envg_weight* out) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  if ((w_bf16 == nullptr) == (w_f32 == nullptr)) return fail(ENVG_ERR_ARG, "exactly one of w_bf16 / w_f32 must be set");
  const int64_t lim = (layout_flags == ENVG_LAYOUT_GATE_UP) ? N / 2 : N;
  return upload_common(d, WSrc{w_bf16, w_f32, K}, N, K, 0, lim, layout_flags, out);
}

int envg_weight_upload_shard(const uint16_t* w_bf16, const float* w_f32, int64_t N, int64_t K, int64_t n0, int64_t n1,
                             int layout_flags, envg_weight* out) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  if ((w_bf16 == nullptr) == (w_f32 == nullptr)) return fail(ENVG_ERR_ARG, "exactly one of w_bf16 / w_f32 must be set");
  return upload_common(d, WSrc{w_bf16, w_f32, K}, N, K, n0, n1, layout_flags, out);
}

int envg_conv_weight_upload(const uint16_t* w_bf16, const float* w_f32, int out_ch, int in_ch, int kH, int kW,
                            envg_weight* out) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  if (!out) return fail(ENVG_ERR_ARG, "out handle pointer is NULL");
  *out = nullptr;
  if ((w_bf16 == nullptr) == (w_f32 == nullptr)) return fail(ENVG_ERR_ARG, "exactly one of w_bf16 / w_f32 must be set");
  return conv_upload_common(d, WSrc{w_bf16, w_f32, (int64_t)in_ch * kH * kW}, out_ch, in_ch, kH, kW, out);
}

int envg_weight_free(envg_weight w) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!w || w->magic != WEIGHT_MAGIC) return fail(ENVG_ERR_STATE, "invalid or already freed weight handle");
  Dev* d = (w->dev >= 0 && w->dev < 64 && g_dev[w->dev].ready) ? &g_dev[w->dev] : nullptr;
  if (d) cudaStreamSynchronize(stream_of(d));
  cudaFree(w->d);
  if (d) d->st.weight_bytes -= std::min<uint64_t>(d->st.weight_bytes, w->bytes);
  w->magic = 0;
  delete w;
  return ENVG_OK;
}

int envg_safetensors_tensor_info(const char* path, const char* name, envg_tensor_info* out) {
  if (!out) return fail(ENVG_ERR_ARG, "info pointer is NULL");
  memset(out, 0, sizeof(*out));
  envg_st::TensorInfo ti;
  int64_t count = 0;
  ENVG_TRY(st_lookup(path, name, &ti, &count));
  out->dtype = st_dtype(ti.dtype);
  out->ndim = (int)ti.shape.size();
  for (size_t i = 0; i < ti.shape.size(); ++i) out->shape[i] = ti.shape[i];
  out->offset = ti.data_start + ti.begin;
  out->nbytes = ti.end - ti.begin;
  snprintf(out->dtype_name, sizeof(out->dtype_name), "%s", ti.dtype.c_str());
  return ENVG_OK;
}

int envg_safetensors_read_f32(const char* path, const char* name, float* dst, int64_t count) {
  if (!dst && count) return fail(ENVG_ERR_ARG, "dst is NULL");
  envg_st::TensorInfo ti;
  int64_t n = 0;
  ENVG_TRY(st_lookup(path, name, &ti, &n));
  if (n != count)
    return fail(ENVG_ERR_ARG, "tensor %s has %lld elements, dst holds %lld", name, (long long)n, (long long)count);
  MappedFile mf;
  std::vector<uint32_t> copy;
  WSrc src{};
  ENVG_TRY(st_source(path, ti, 0, &mf, &copy, &src));
  for (int64_t i = 0; i < n; ++i) {
    if (src.b) {
      const uint32_t u = (uint32_t)src.b[i] << 16;
      memcpy(&dst[i], &u, 4);
    } else if (src.h) {
      dst[i] = f16_to_f32(src.h[i]);
    } else {
      dst[i] = src.f[i];
    }
  }
  return ENVG_OK;
}

int envg_weight_upload_safetensors(const char* path, const char* name, int layout_flags, int64_t n0, int64_t n1,
                                   envg_weight* out) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!out) return fail(ENVG_ERR_ARG, "out handle pointer is NULL");
  *out = nullptr;
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  envg_st::TensorInfo ti;
  int64_t n = 0;
  ENVG_TRY(st_lookup(path, name, &ti, &n));
  const size_t nd = ti.shape.size();
  if (nd != 2 && nd != 4)
    return fail(ENVG_ERR_ARG, "tensor %s has %zu dims; a weight is 2-D [N, K] or 4-D [O, C, kH, kW]", name, nd);
  const int64_t N = ti.shape[0], K = n / std::max<int64_t>(1, N);
  MappedFile mf;
  std::vector<uint32_t> copy;
  WSrc src{};
  ENVG_TRY(st_source(path, ti, K, &mf, &copy, &src));
  if (nd == 4) {
    if (n0 != 0 || n1 != 0) return fail(ENVG_ERR_ARG, "convolution weights are uploaded whole (n0 = n1 = 0)");
    if ((layout_flags & ~ENVG_LAYOUT_ROUND_BF16) != ENVG_LAYOUT_PLAIN)
      return fail(ENVG_ERR_ARG, "convolution weights take ENVG_LAYOUT_PLAIN");
    for (int i = 0; i < 4; ++i)
      if (ti.shape[i] <= 0 || ti.shape[i] > INT32_MAX) return fail(ENVG_ERR_ARG, "conv weight %s: bad shape", name);
    return conv_upload_common(d, src, (int)ti.shape[0], (int)ti.shape[1], (int)ti.shape[2], (int)ti.shape[3], out);
  }
  if (n0 == 0 && n1 == 0) n1 = (layout_flags & ~ENVG_LAYOUT_ROUND_BF16) == ENVG_LAYOUT_GATE_UP ? N / 2 : N;
  return upload_common(d, src, N, K, n0, n1, layout_flags, out);
}

}  // extern "C"

namespace {
constexpr int64_t PIPE_MIN_M = 1024;   // host calls from this many rows are pipelined
constexpr int64_t PIPE_CHUNK = 512;    // rows per chunk (a multiple of the 256-row pair tile)

cudaEvent_t pipe_event(Dev* d, size_t i) {
  while (d->pipe_events.size() <= i) {
    cudaEvent_t e = nullptr;
    cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    d->pipe_events.push_back(e);
  }
  return d->pipe_events[i];
}

// Row normalisation fused into the activation cast of a linear: none, QNNAdaLN (shift, scale) or
// QNNRMSNorm (weight, which may be NULL).
struct Prologue {
  enum Kind { NONE = 0, ADALN, RMS } kind = NONE;
  const float* shift = nullptr;
  const float* scale = nullptr;
  const float* rms_w = nullptr;
};

// Copies a host prologue's K-long vectors into d->ada on stream s; out is the device-side prologue.
int stage_prologue(Dev* d, const Prologue& p, int64_t K, cudaStream_t s, Prologue& out) {
  out = p;
  if (p.kind == Prologue::ADALN) {
    ENVG_TRY(ensure(d, d->ada, (size_t)(2 * K) * 4));
    float* a = reinterpret_cast<float*>(d->ada.p);
    ENVG_CUDA(cudaMemcpyAsync(a, p.shift, (size_t)K * 4, cudaMemcpyHostToDevice, s));
    ENVG_CUDA(cudaMemcpyAsync(a + K, p.scale, (size_t)K * 4, cudaMemcpyHostToDevice, s));
    d->st.h2d_bytes += (double)(2 * K) * 4;
    out.shift = a;
    out.scale = a + K;
  } else if (p.kind == Prologue::RMS && p.rms_w) {
    ENVG_TRY(ensure(d, d->ada, (size_t)K * 4));
    float* a = reinterpret_cast<float*>(d->ada.p);
    ENVG_CUDA(cudaMemcpyAsync(a, p.rms_w, (size_t)K * 4, cudaMemcpyHostToDevice, s));
    d->st.h2d_bytes += (double)K * 4;
    out.rms_w = a;
  }
  return ENVG_OK;
}

// Normalises (or only casts) rows of x into out: bf16 padded to Kp, or fp32 with K columns
// (bf16 = false, only for a prologue other than NONE).  For a bf16x3 weight (x3), Kp is its
// device row length 3 * Ks and out receives the activation layout hi|hi|lo; a prologue first
// writes its fp32 rows into the workspace d->xn.
int launch_prologue(Dev* d, const Prologue& p, const float* x, int64_t rows, int64_t K, int64_t Kp, void* out,
                    bool bf16, bool x3 = false) {
  if (x3) {
    const float* src = x;
    if (p.kind != Prologue::NONE) {
      ENVG_TRY(ensure(d, d->xn, (size_t)(rows * K) * 4));
      ENVG_TRY(launch_prologue(d, p, x, rows, K, K, d->xn.p, false));
      src = reinterpret_cast<const float*>(d->xn.p);
    }
    return launch_cast_x3(d, src, K, rows, K, Kp / 3, out, X3_ACT);
  }
  switch (p.kind) {
    case Prologue::ADALN: return launch_adaln(d, x, rows, K, Kp, p.shift, p.scale, out, bf16);
    case Prologue::RMS: return launch_rmsnorm(d, x, rows, K, Kp, p.rms_w, out, bf16);
    default: return launch_cast_rows(d, x, K, rows, K, Kp, out);
  }
}

// Host-pointer linear with M >= PIPE_MIN_M, cut into row chunks: the copy-in of chunk c + 1 (on
// d->h2d), the cast + GEMM of chunk c (on the compute stream) and the copy-out of chunk c - 1
// (on d->d2h) overlap, so PCIe moves X and Y in both directions at once while the GPU computes.
// Rows are independent, so every output is computed exactly as in one launch.  Synchronous.
int linear_host_pipelined(Dev* d, float* dst, const float* x, envg_weight W, const float* bias, int64_t M, int64_t K,
                          int64_t N, int epilogue, const float* gate, const Prologue& pro) {
  const bool gu = W->layout == ENVG_LAYOUT_GATE_UP;
  const int64_t n_out = gu ? N / 2 : N;
  cudaStream_t s = stream_of(d);
  if (!d->h2d) ENVG_CUDA(cudaStreamCreateWithFlags(&d->h2d, cudaStreamNonBlocking));
  if (!d->d2h) ENVG_CUDA(cudaStreamCreateWithFlags(&d->d2h, cudaStreamNonBlocking));
  ENVG_TRY(ensure(d, d->x, (size_t)(M * K) * 4));
  ENVG_TRY(ensure(d, d->y, (size_t)(M * n_out) * 4));
  ENVG_TRY(ensure(d, d->xb, (size_t)(M * W->Kp) * 2));
  float* dx = reinterpret_cast<float*>(d->x.p);
  float* dy = reinterpret_cast<float*>(d->y.p);
  // small vectors first, on the compute stream
  const float *dbias = nullptr, *dgate = nullptr;
  if (bias) {
    ENVG_TRY(ensure(d, d->bias, (size_t)N * 4));
    ENVG_CUDA(cudaMemcpyAsync(d->bias.p, bias, (size_t)N * 4, cudaMemcpyHostToDevice, s));
    d->st.h2d_bytes += (double)N * 4;
    dbias = reinterpret_cast<float*>(d->bias.p);
  }
  if (epilogue == ENVG_EPI_GATED_RESIDUAL) {
    ENVG_TRY(ensure(d, d->gate, (size_t)N * 4));
    ENVG_CUDA(cudaMemcpyAsync(d->gate.p, gate, (size_t)N * 4, cudaMemcpyHostToDevice, s));
    d->st.h2d_bytes += (double)N * 4;
    dgate = reinterpret_cast<float*>(d->gate.p);
  }
  Prologue dpro;
  ENVG_TRY(stage_prologue(d, pro, K, s, dpro));
  // chunks of PIPE_CHUNK rows, the remainder joining the last one.  Small chunks shorten the
  // pipeline's fill (the first copy-in) and drain (the last copy-out).  Every chunk has more
  // than 128 rows and runs without split-K, so it takes the CTA-pair kernel with the same
  // per-tile summation order as one launch over all M >= PIPE_MIN_M rows (which never splits).
  const int64_t nch = std::max<int64_t>(1, M / PIPE_CHUNK);
  struct NoSplit {
    Dev* d;
    ~NoSplit() { d->no_split = false; }
  } no_split_guard{d};
  d->no_split = true;
  auto chunk = [&](int64_t c, int64_t& r0, int64_t& rows) {
    r0 = c * PIPE_CHUNK;
    rows = (c == nch - 1) ? M - r0 : PIPE_CHUNK;
  };
  // event 0: the small vectors are queued on s (the copy streams start after them)
  ENVG_CUDA(cudaEventRecord(pipe_event(d, 0), s));
  ENVG_CUDA(cudaStreamWaitEvent(d->h2d, pipe_event(d, 0), 0));
  for (int64_t c = 0; c < nch; ++c) {
    int64_t r0, rows;
    chunk(c, r0, rows);
    ENVG_CUDA(cudaMemcpyAsync(dx + r0 * K, x + r0 * K, (size_t)(rows * K) * 4, cudaMemcpyHostToDevice, d->h2d));
    d->st.h2d_bytes += (double)(rows * K) * 4;
    if (epilogue == ENVG_EPI_GATED_RESIDUAL) {
      ENVG_CUDA(cudaMemcpyAsync(dy + r0 * n_out, dst + r0 * n_out, (size_t)(rows * n_out) * 4,
                                cudaMemcpyHostToDevice, d->h2d));
      d->st.h2d_bytes += (double)(rows * n_out) * 4;
    }
    ENVG_CUDA(cudaEventRecord(pipe_event(d, 1 + 2 * c), d->h2d));  // chunk c is on the device
  }
  for (int64_t c = 0; c < nch; ++c) {
    int64_t r0, rows;
    chunk(c, r0, rows);
    ENVG_CUDA(cudaStreamWaitEvent(s, pipe_event(d, 1 + 2 * c), 0));
    void* xb = reinterpret_cast<uint8_t*>(d->xb.p) + (size_t)(r0 * W->Kp) * 2;
    ENVG_TRY(launch_prologue(d, dpro, dx + r0 * K, rows, K, W->Kp, xb, true, W->x3));
    EpiArgs e{};
    e.Y = dy + r0 * n_out;
    e.ldy = n_out;
    e.bias = dbias;
    e.bias_mode = dbias ? 1 : 0;
    e.mode = (epilogue == ENVG_EPI_GATED_RESIDUAL) ? EPI_GATED_RES : EPI_PLAIN;
    e.gate = dgate;
    e.alpha = 1.0f;
    e.n_out = (int)n_out;
    e.m_valid = (int)rows;
    e.half_n = (int)(gu ? W->half : 0);
    e.vec_ok = ((reinterpret_cast<uintptr_t>(e.Y) & 15) == 0 && n_out % 4 == 0) ? 1 : 0;
    const double fl = 2.0 * (double)rows * (double)N * (double)K;
    ENVG_TRY(gemm_device(d, xb, rows, W->Kp, W->tm256, W->tm128, W->rows, gu, e, fl,
                         2.0 * (double)N * K + 2.0 * (double)rows * W->Kp + 4.0 * (double)rows * n_out));
    ENVG_CUDA(cudaEventRecord(pipe_event(d, 2 + 2 * c), s));  // chunk c of Y is done
    ENVG_CUDA(cudaStreamWaitEvent(d->d2h, pipe_event(d, 2 + 2 * c), 0));
    ENVG_CUDA(cudaMemcpyAsync(dst + r0 * n_out, dy + r0 * n_out, (size_t)(rows * n_out) * 4, cudaMemcpyDeviceToHost,
                              d->d2h));
    d->st.d2h_bytes += (double)(rows * n_out) * 4;
  }
  d->st.calls++;
  d->st.flops += 2.0 * (double)M * (double)N * (double)K;
  ENVG_CUDA(cudaStreamSynchronize(d->d2h));
  return sync_and_check(d);
}

// envg_linear, envg_linear_adaln and envg_linear_rmsnorm.  With a prologue, X is first normalised
// per row (QNNAdaLN or QNNRMSNorm) inside the activation-cast kernel.
int linear_core(Dev* d, float* dst, const float* x, envg_weight W, const float* bias, int64_t M, int64_t K, int64_t N,
                int epilogue, const float* gate, int flags, const Prologue& pro) {
  ENVG_TRY(check_weight(d, W));
  if (W->conv) return fail(ENVG_ERR_ARG, "envg_linear: handle holds a convolution weight");
  if (M < 0) return fail(ENVG_ERR_ARG, "envg_linear: M=%lld < 0", (long long)M);
  if (K != W->K || N != W->N)
    return fail(ENVG_ERR_ARG, "envg_linear: [K=%lld, N=%lld] does not match the weight [N=%lld, K=%lld]", (long long)K,
                (long long)N, (long long)W->N, (long long)W->K);
  if (M > INT32_MAX / 2) return fail(ENVG_ERR_ARG, "envg_linear: M=%lld too large", (long long)M);
  const bool gu = W->layout == ENVG_LAYOUT_GATE_UP;
  if (epilogue == ENVG_EPI_SILU_GATE && !gu)
    return fail(ENVG_ERR_ARG, "envg_linear: SILU_GATE needs a weight uploaded with ENVG_LAYOUT_GATE_UP");
  if (gu && epilogue != ENVG_EPI_SILU_GATE)
    return fail(ENVG_ERR_ARG, "envg_linear: a GATE_UP weight only supports the SILU_GATE epilogue");
  if (epilogue != ENVG_EPI_NONE && epilogue != ENVG_EPI_BIAS && epilogue != ENVG_EPI_SILU_GATE &&
      epilogue != ENVG_EPI_GATED_RESIDUAL)
    return fail(ENVG_ERR_ARG, "envg_linear: epilogue %s (%d) not valid for a linear", epi_name(epilogue), epilogue);
  if (epilogue == ENVG_EPI_BIAS && !bias) return fail(ENVG_ERR_ARG, "envg_linear: BIAS epilogue without bias");
  if (epilogue == ENVG_EPI_GATED_RESIDUAL && !gate)
    return fail(ENVG_ERR_ARG, "envg_linear: GATED_RESIDUAL epilogue without gate");
  if (M == 0) return ENVG_OK;
  if (!dst || !x) return fail(ENVG_ERR_ARG, "envg_linear: dst or x is NULL");
  if ((const void*)dst == (const void*)x) return fail(ENVG_ERR_ARG, "envg_linear: dst aliases x");
  const bool devp = (flags & ENVG_DEVICE_PTRS) != 0;
  const int64_t n_out = gu ? N / 2 : N;
  cudaStream_t s = stream_of(d);
  if (!devp && M >= PIPE_MIN_M && d->pipe_host)
    return linear_host_pipelined(d, dst, x, W, bias, M, K, N, epilogue, gate, pro);

  const float *dx = x, *dbias = bias, *dgate = gate;
  float* dy = dst;
  Prologue dpro = pro;
  if (!devp) {
    ENVG_TRY(stage_prologue(d, pro, K, s, dpro));
    ENVG_TRY(ensure(d, d->x, (size_t)(M * K) * 4));
    ENVG_TRY(ensure(d, d->y, (size_t)(M * n_out) * 4));
    ENVG_CUDA(cudaMemcpyAsync(d->x.p, x, (size_t)(M * K) * 4, cudaMemcpyHostToDevice, s));
    d->st.h2d_bytes += (double)(M * K) * 4;
    dx = reinterpret_cast<float*>(d->x.p);
    dy = reinterpret_cast<float*>(d->y.p);
    if (bias) {
      ENVG_TRY(ensure(d, d->bias, (size_t)N * 4));
      ENVG_CUDA(cudaMemcpyAsync(d->bias.p, bias, (size_t)N * 4, cudaMemcpyHostToDevice, s));
      d->st.h2d_bytes += (double)N * 4;
      dbias = reinterpret_cast<float*>(d->bias.p);
    }
    if (epilogue == ENVG_EPI_GATED_RESIDUAL) {
      ENVG_TRY(ensure(d, d->gate, (size_t)N * 4));
      ENVG_CUDA(cudaMemcpyAsync(d->gate.p, gate, (size_t)N * 4, cudaMemcpyHostToDevice, s));
      ENVG_CUDA(cudaMemcpyAsync(dy, dst, (size_t)(M * n_out) * 4, cudaMemcpyHostToDevice, s));
      d->st.h2d_bytes += (double)N * 4 + (double)(M * n_out) * 4;
      dgate = reinterpret_cast<float*>(d->gate.p);
    }
  }
  EpiArgs e{};
  e.Y = dy;
  e.ldy = n_out;
  e.bias = dbias;
  e.bias_mode = dbias ? 1 : 0;
  e.act = 0;
  e.mode = (epilogue == ENVG_EPI_GATED_RESIDUAL) ? EPI_GATED_RES : EPI_PLAIN;
  e.gate = dgate;
  e.alpha = 1.0f;
  e.beta = 0.0f;
  e.n_out = (int)n_out;
  e.m_valid = (int)M;
  e.half_n = (int)(gu ? W->half : 0);
  e.vec_ok = ((reinterpret_cast<uintptr_t>(dy) & 15) == 0 && n_out % 4 == 0) ? 1 : 0;
  const double lin_flops = 2.0 * (double)M * (double)N * (double)K;
  const double out_bytes = 4.0 * (double)M * n_out + (dbias ? 4.0 * N : 0.0) +
                           (epilogue == ENVG_EPI_GATED_RESIDUAL ? 4.0 * (double)M * n_out + 4.0 * N : 0.0);
  if (M <= d->gemv_max && !W->x3) {
    if (dpro.kind != Prologue::NONE) {  // normalised X kept in fp32 for the CUDA-core path
      ENVG_TRY(ensure(d, d->xn, (size_t)(M * K) * 4));
      ENVG_TRY(launch_prologue(d, dpro, dx, M, K, K, d->xn.p, false));
      dx = reinterpret_cast<const float*>(d->xn.p);
    }
    // fp32 X read directly: W once, X once per 64-row group (from L2)
    ENVG_TRY(launch_gemv(d, dx, M, K, W, gu, e, lin_flops, 2.0 * (double)N * K + 4.0 * (double)M * K + out_bytes));
  } else {
    ENVG_TRY(ensure(d, d->xb, (size_t)(M * W->Kp) * 2));
    ENVG_TRY(launch_prologue(d, dpro, dx, M, K, W->Kp, d->xb.p, true, W->x3));
    ENVG_TRY(gemm_device(d, d->xb.p, M, W->Kp, W->tm256, W->tm128, W->rows, gu, e, lin_flops,
                         2.0 * (double)N * K + 2.0 * (double)M * W->Kp + out_bytes));
  }

  d->st.calls++;
  d->st.flops += 2.0 * (double)M * (double)N * (double)K;
  if (!devp) {
    ENVG_CUDA(cudaMemcpyAsync(dst, dy, (size_t)(M * n_out) * 4, cudaMemcpyDeviceToHost, s));
    d->st.d2h_bytes += (double)(M * n_out) * 4;
    return sync_and_check(d);
  }
  if (!(flags & ENVG_ASYNC)) return sync_and_check(d);
  return ENVG_OK;
}
}  // namespace

extern "C" {

int envg_linear(float* dst, const float* x, envg_weight W, const float* bias, int64_t M, int64_t K, int64_t N,
                int epilogue, const float* gate, int flags) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  return linear_core(d, dst, x, W, bias, M, K, N, epilogue, gate, flags, Prologue{});
}

int envg_linear_adaln(float* dst, const float* x, const float* shift, const float* scale, envg_weight W,
                      const float* bias, int64_t M, int64_t K, int64_t N, int epilogue, const float* gate, int flags) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  if (!shift || !scale) return fail(ENVG_ERR_ARG, "envg_linear_adaln: shift and scale are required");
  Prologue p;
  p.kind = Prologue::ADALN;
  p.shift = shift;
  p.scale = scale;
  return linear_core(d, dst, x, W, bias, M, K, N, epilogue, gate, flags, p);
}

int envg_linear_rmsnorm(float* dst, const float* x, const float* weight, envg_weight W, const float* bias, int64_t M,
                        int64_t K, int64_t N, int epilogue, const float* gate, int flags) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  Prologue p;
  p.kind = Prologue::RMS;
  p.rms_w = weight;
  return linear_core(d, dst, x, W, bias, M, K, N, epilogue, gate, flags, p);
}

namespace {
EpiArgs linear_epi(const envg_linear_desc& q);  // the epilogue arguments of one linear (below)
}  // namespace

int envg_linear_noalloc(float* dst, const float* x, envg_weight W, const float* bias, int64_t M, int64_t K, int64_t N,
                        int epilogue, const float* gate, int flags) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  ENVG_TRY(check_weight(d, W));
  if (W->conv) return fail(ENVG_ERR_ARG, "envg_linear_noalloc: handle holds a convolution weight");
  if (!(flags & ENVG_DEVICE_PTRS))
    return fail(ENVG_ERR_ARG, "envg_linear_noalloc: needs device pointers (ENVG_DEVICE_PTRS); it stages nothing");
  if (K != W->K || N != W->N)
    return fail(ENVG_ERR_ARG, "envg_linear_noalloc: [K=%lld, N=%lld] does not match the weight [N=%lld, K=%lld]",
                (long long)K, (long long)N, (long long)W->N, (long long)W->K);
  const bool gu = W->layout == ENVG_LAYOUT_GATE_UP;
  if ((epilogue == ENVG_EPI_SILU_GATE) != gu)
    return fail(ENVG_ERR_ARG, "envg_linear_noalloc: SILU_GATE goes with (and only with) a GATE_UP weight");
  if (epilogue != ENVG_EPI_NONE && epilogue != ENVG_EPI_BIAS && epilogue != ENVG_EPI_SILU_GATE &&
      epilogue != ENVG_EPI_GATED_RESIDUAL)
    return fail(ENVG_ERR_ARG, "envg_linear_noalloc: epilogue %d not valid for a linear", epilogue);
  if (epilogue == ENVG_EPI_BIAS && !bias) return fail(ENVG_ERR_ARG, "envg_linear_noalloc: BIAS epilogue without bias");
  if (epilogue == ENVG_EPI_GATED_RESIDUAL && !gate)
    return fail(ENVG_ERR_ARG, "envg_linear_noalloc: GATED_RESIDUAL epilogue without gate");
  if (M < 0 || M > SKINNY_MAX)
    return fail(ENVG_ERR_ARG, "envg_linear_noalloc: M=%lld outside [0, %d] (the allocation-free path is skinny-M only)",
                (long long)M, SKINNY_MAX);
  if ((size_t)M * (size_t)W->Kp * 2 > NOALLOC_XB_BYTES)
    return fail(ENVG_ERR_ARG, "envg_linear_noalloc: M*Kp*2 = %lld bytes exceeds the %zu-byte activation scratch",
                (long long)(M * W->Kp * 2), NOALLOC_XB_BYTES);
  const int R = gu ? 2 : 1;
  const int64_t n_tiles = cdiv(W->rows, (int64_t)R * BM);
  if ((size_t)n_tiles * sizeof(int) > NOALLOC_CNT_BYTES)
    return fail(ENVG_ERR_ARG, "envg_linear_noalloc: %lld row tiles exceed the %zu-entry counter scratch",
                (long long)n_tiles, NOALLOC_CNT_BYTES / sizeof(int));
  if (M == 0) return ENVG_OK;
  if (!dst || !x) return fail(ENVG_ERR_ARG, "envg_linear_noalloc: dst or x is NULL");
  if ((const void*)dst == (const void*)x) return fail(ENVG_ERR_ARG, "envg_linear_noalloc: dst aliases x");
  uint8_t* scratch = nullptr;
  ENVG_TRY(noalloc_scratch(d, &scratch));
  uint8_t* xb = scratch;
  float* part = reinterpret_cast<float*>(scratch + NOALLOC_XB_BYTES);
  int* cnt = reinterpret_cast<int*>(scratch + NOALLOC_XB_BYTES + NOALLOC_PART_BYTES);
  cudaStream_t s = stream_of(d);
  const int64_t n_out = gu ? N / 2 : N;

  if (W->x3) ENVG_TRY(launch_cast_x3(d, x, K, M, K, W->Ks, xb, X3_ACT));
  else ENVG_TRY(launch_cast_rows(d, x, K, M, K, W->Kp, xb));
  const int mpad = (int)rup(M, 16);
  const int64_t num_kb = cdiv(W->Kp, BK);
  SkinnyArgs a{};
  a.n_tiles = (int)n_tiles;
  a.num_kb = (int)num_kb;
  int splits = std::max<int64_t>(1, (2 * d->sms) / n_tiles);
  splits = (int)std::min<int64_t>(splits, std::max<int64_t>(1, num_kb / 2));
  const size_t part_per_split = (size_t)n_tiles * R * BM * mpad * sizeof(float);
  splits = (int)std::max<size_t>(1, std::min<size_t>((size_t)splits, NOALLOC_PART_BYTES / part_per_split));
  a.kb_per_split = (int)cdiv(num_kb, splits);
  a.splits = (int)cdiv(num_kb, a.kb_per_split);
  if (a.splits > 1) {
    ENVG_CUDA(cudaMemsetAsync(cnt, 0, (size_t)n_tiles * sizeof(int), s));  // counters start at zero
    a.partial = part;
    a.counters = cnt;
  }
  a.epi = linear_epi(envg_linear_desc{dst, x, W, bias, M, K, N, epilogue, gate});
  CUtensorMap tX;
  ENVG_TRY(tmap_2d(&tX, xb, W->Kp, M, mpad));
  ENVG_TRY(launch_k2(d, mpad, R, W->tm128, tX, a, 2.0 * (double)M * N * K,
                     2.0 * (double)N * K + 2.0 * (double)M * W->Kp + 4.0 * (double)M * n_out));
  d->st.calls++;
  d->st.flops += 2.0 * (double)M * (double)N * (double)K;
  if (!(flags & ENVG_ASYNC)) return sync_and_check(d);
  return ENVG_OK;
}

namespace {
// Validation shared by envg_linear and envg_linear_batch (device pointers).
int check_linear_args(Dev* d, const envg_linear_desc& q) {
  ENVG_TRY(check_weight(d, q.W));
  if (q.W->conv) return fail(ENVG_ERR_ARG, "linear: handle holds a convolution weight");
  if (q.M < 0 || q.M > INT32_MAX / 2) return fail(ENVG_ERR_ARG, "linear: M=%lld out of range", (long long)q.M);
  if (q.K != q.W->K || q.N != q.W->N)
    return fail(ENVG_ERR_ARG, "linear: [K=%lld, N=%lld] does not match the weight [N=%lld, K=%lld]", (long long)q.K,
                (long long)q.N, (long long)q.W->N, (long long)q.W->K);
  const bool gu = q.W->layout == ENVG_LAYOUT_GATE_UP;
  if ((q.epilogue == ENVG_EPI_SILU_GATE) != gu)
    return fail(ENVG_ERR_ARG, "linear: SILU_GATE goes with (and only with) a GATE_UP weight");
  if (q.epilogue != ENVG_EPI_NONE && q.epilogue != ENVG_EPI_BIAS && q.epilogue != ENVG_EPI_SILU_GATE &&
      q.epilogue != ENVG_EPI_GATED_RESIDUAL)
    return fail(ENVG_ERR_ARG, "linear: epilogue %d not valid for a linear", q.epilogue);
  if (q.epilogue == ENVG_EPI_BIAS && !q.bias) return fail(ENVG_ERR_ARG, "linear: BIAS epilogue without bias");
  if (q.epilogue == ENVG_EPI_GATED_RESIDUAL && !q.gate) return fail(ENVG_ERR_ARG, "linear: GATED_RESIDUAL without gate");
  if (q.M > 0 && (!q.dst || !q.x)) return fail(ENVG_ERR_ARG, "linear: dst or x is NULL");
  if (q.M > 0 && (const void*)q.dst == (const void*)q.x) return fail(ENVG_ERR_ARG, "linear: dst aliases x");
  return ENVG_OK;
}

EpiArgs linear_epi(const envg_linear_desc& q) {
  const bool gu = q.W->layout == ENVG_LAYOUT_GATE_UP;
  const int64_t n_out = gu ? q.N / 2 : q.N;
  EpiArgs e{};
  e.Y = q.dst;
  e.ldy = n_out;
  e.bias = q.bias;
  e.bias_mode = q.bias ? 1 : 0;
  e.mode = (q.epilogue == ENVG_EPI_GATED_RESIDUAL) ? EPI_GATED_RES : EPI_PLAIN;
  e.gate = q.gate;
  e.alpha = 1.0f;
  e.n_out = (int)n_out;
  e.m_valid = (int)q.M;
  e.half_n = (int)(gu ? q.W->half : 0);
  e.vec_ok = ((reinterpret_cast<uintptr_t>(q.dst) & 15) == 0 && n_out % 4 == 0) ? 1 : 0;
  return e;
}

// Convolution of an NHWC bf16 activation `act` ([batch][H][W][Cp], Cp = W->Cp) into NCHW fp32 dy.
// residual: dy += conv + bias (stride 1 only; the residual add of QNNAddInplace,
// src/quicknncpu.pas:704-709, fused into the store).
int conv_core(Dev* d, envg_weight W, const void* act, float* dy, const float* dbias, int H, int W_, int stride, int pad,
              int batch, int act_silu, bool residual) {
  cudaStream_t s = stream_of(d);
  const int out_ch = W->out_ch, kH = W->kH, kW = W->kW, Cp = W->Cp;
  const int outH = (H + 2 * pad - kH) / stride + 1;
  const int outW = (W_ + 2 * pad - kW) / stride + 1;
  if (residual && stride != 1) return fail(ENVG_ERR_UNSUPPORTED, "conv residual add needs stride 1");
  const int64_t plane = (int64_t)outH * outW;
  const int64_t out_elems = (int64_t)batch * out_ch * plane;
  EpiArgs e{};
  e.Y = dy;
  e.bias = dbias;
  e.bias_mode = dbias ? 2 : 0;
  e.act = act_silu;
  e.mode = residual ? EPI_GATED_RES : EPI_PLAIN;
  e.alpha = 1.0f;
  e.m_valid = out_ch;
  if (stride == 1) {
    // Implicit im2col: each B tile is one 4D TMA box of the NHWC activation.
    int tw = 1;
    while (tw < outW && tw < 256) tw <<= 1;
    const int th = 256 / tw;
    const bool pair = d->use_pair && out_ch > BM;
    CUtensorMap tB;
    if (pair)  // each CTA of the pair fetches half of the 256-pixel tile
      ENVG_TRY(tmap_nhwc(&tB, act, Cp, W_, H, batch, th >= 2 ? tw : tw / 2, th >= 2 ? th / 2 : 1));
    else
      ENVG_TRY(tmap_nhwc(&tB, act, Cp, W_, H, batch, tw, th));
    GemmArgs g{};
    g.num_kb = (int)(W->Kp / BK);
    g.tiles_m = (int)cdiv(out_ch, pair ? 2 * BM : BM);
    g.conv.tileW = tw;
    g.conv.tileH = th;
    g.conv.outH = outH;
    g.conv.outW = outW;
    g.conv.tiles_w = (int)cdiv(outW, tw);
    g.conv.tiles_h = (int)cdiv(outH, th);
    g.conv.KW = kW;
    g.conv.pad = pad;
    g.conv.cblocks = Cp / BK;
    g.conv.img_stride = (int64_t)out_ch * plane;
    g.conv.plane = plane;
    g.tiles_n = batch * g.conv.tiles_w * g.conv.tiles_h;
    g.num_tiles = g.tiles_m * g.tiles_n;
    g.group_m = 1;
    e.ldy = plane;
    e.n_out = (int)plane;
    e.vec_ok = ((reinterpret_cast<uintptr_t>(dy) & 15) == 0 && outW % 4 == 0) ? 1 : 0;
    CUtensorMap tY;
    memset(&tY, 0, sizeof(tY));
    e.store_mode = (tw >= 32) ? STORE_COALESCED : STORE_DIRECT;  // a 32-pixel chunk stays in one row
    if (d->store_tma && (reinterpret_cast<uintptr_t>(dy) & 15) == 0 && outW % 32 == 0) {
      ENVG_TRY(tmap_out_3d(&tY, dy, (uint64_t)plane, (uint64_t)out_ch, (uint64_t)batch));
      if (pair) {
        ENVG_TRY(tmap_out_3d(&g.ybig, dy, (uint64_t)plane, (uint64_t)out_ch, (uint64_t)batch, 128));
        g.ybig_ok = 1;
      }
      e.store_mode = residual ? STORE_TMA_ADD : STORE_TMA;
    }
    g.epi = e;
    const double cflops = 2.0 * out_ch * (double)plane * batch * (double)W->K;
    const double cbytes = 2.0 * (double)batch * H * W_ * Cp + 2.0 * out_ch * (double)W->Kp + 4.0 * (double)out_elems +
                          (dbias ? 4.0 * out_ch : 0.0);
    if (pair) {
      PairSet set = set_of_one(g, tB, tY);
      ENVG_TRY((launch_k1_pair<true, false>(d, W->tm128, set, cflops, cbytes)));
    }
    else ENVG_TRY(launch_k1<true, false>(d, W->tm128, tB, tY, g, cflops, cbytes));
  } else {
    // Strided convolution: explicit bf16 im2col, then one GEMM per image.
    const int64_t colK = W->Kp;
    ENVG_TRY(ensure(d, d->col, (size_t)batch * plane * colK * 2));
    const int64_t total = (int64_t)batch * plane * kH * kW * (Cp / 8);
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(total, 256), (int64_t)d->sms * 16));
    ProfScope ps_im(s, KID_IM2COL, 0.0, 2.0 * (double)batch * H * W_ * Cp + 2.0 * (double)batch * plane * colK);
    k_im2col_nhwc<<<blocks, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(act), batch, H, W_, Cp, kH, kW,
                                         stride, pad, outH, outW, reinterpret_cast<__nv_bfloat16*>(d->col.p));
    ENVG_CUDA(cudaGetLastError());
    d->st.kernel_launches++;
    for (int b = 0; b < batch; ++b) {
      const void* colb = reinterpret_cast<const uint8_t*>(d->col.p) + (size_t)b * plane * colK * 2;
      CUtensorMap tB;
      ENVG_TRY(tmap_2d(&tB, colb, colK, plane, 256));
      CUtensorMap tA = W->tm128;
      GemmArgs g{};
      g.num_kb = (int)(colK / BK);
      g.tiles_m = (int)cdiv(out_ch, BM);
      g.tiles_n = (int)cdiv(plane, K1_BN);
      g.num_tiles = g.tiles_m * g.tiles_n;
      g.group_m = 8;
      EpiArgs eb = e;
      eb.Y = dy + (int64_t)b * out_ch * plane;
      eb.ldy = plane;
      eb.n_out = (int)plane;
      eb.vec_ok = ((reinterpret_cast<uintptr_t>(eb.Y) & 15) == 0 && plane % 4 == 0) ? 1 : 0;
      CUtensorMap tY;
      memset(&tY, 0, sizeof(tY));
      ENVG_TRY(choose_store(d->store_tma, eb, &tY));
      g.epi = eb;
      ENVG_TRY(launch_k1<false, false>(d, tA, tB, tY, g, 2.0 * out_ch * (double)plane * (double)W->K,
                                       2.0 * (double)plane * colK + 2.0 * out_ch * (double)colK + 4.0 * out_ch * (double)plane));
    }
  }
  return ENVG_OK;
}

constexpr float GN_EPS = 1e-6f;  // EPSILON of QNNGroupNorm (src/quicknn_common.pas:51)

int gn_chunks(int C, int64_t HW, int groups) { return (int)cdiv((int64_t)(C / groups) * HW, GN_CHUNK); }

// Bytes of GroupNorm scratch for one tensor: chunk partials (3 doubles each) + float2 affine.
size_t gn_bytes(int batch, int C, int64_t HW, int groups) {
  return (size_t)rup((int64_t)batch * groups * gn_chunks(C, HW, groups) * 24, 256) + (size_t)batch * C * 8;
}

// Per-(b, c) GroupNorm affine {gamma*std_inv, beta - mean*gamma*std_inv} of a device NCHW tensor,
// written after the partials in d->gn (which must hold gn_bytes()).
int launch_group_affine(Dev* d, const float* src, int batch, int C, int64_t HW, int groups, const float* gamma,
                        const float* beta, float2** aff_out) {
  cudaStream_t s = stream_of(d);
  const int cpg = C / groups, chunks = gn_chunks(C, HW, groups);
  // d->gn: [0, 256) the finished-CTA counter (always at offset 0: zeroed when the buffer is
  // allocated, re-armed by every launch), then the chunk partials, then the affine
  double* part = reinterpret_cast<double*>(d->gn.p);
  float2* aff = reinterpret_cast<float2*>(reinterpret_cast<uint8_t*>(d->gn.p) +
                                          rup((int64_t)batch * groups * chunks * 24, 256));
  {
    ProfScope ps(s, KID_GN_STATS, 0.0, 4.0 * batch * (double)C * HW + 24.0 * batch * groups * chunks);
    k_group_stats<<<dim3((unsigned)chunks, (unsigned)(batch * groups)), GN_THREADS, 0, s>>>(src, C, HW, cpg, groups,
                                                                                           part, chunks);
    ENVG_CUDA(cudaGetLastError());
    d->st.kernel_launches++;
  }
  {
    // one warp per group, all groups in parallel (a single finishing CTA doing them all is slower)
    ProfScope ps(s, KID_GN_AFFINE, 0.0, 24.0 * batch * groups * chunks + 8.0 * C + 8.0 * batch * C);
    k_group_affine<<<(unsigned)cdiv((int64_t)batch * groups * 32, 256), 256, 0, s>>>(part, chunks, batch, C, cpg,
                                                                                     groups, gamma, beta, GN_EPS, aff);
    ENVG_CUDA(cudaGetLastError());
    d->st.kernel_launches++;
  }
  *aff_out = aff;
  return ENVG_OK;
}

int check_gn_geometry(int batch, int C, int H, int W, int groups) {
  if (batch < 0 || C <= 0 || H <= 0 || W <= 0 || groups <= 0 || C % groups)
    return fail(ENVG_ERR_ARG, "group norm: batch %d, channels %d, %dx%d, %d groups invalid", batch, C, H, W, groups);
  if ((int64_t)batch * groups > 65535)
    return fail(ENVG_ERR_UNSUPPORTED, "group norm: batch x groups = %lld > 65535", (long long)batch * groups);
  return ENVG_OK;
}

// Copies host vectors into d->vec (sized beforehand by the caller) and returns device pointers.
struct VecStage {
  Dev* d;
  bool devp;
  size_t off = 0;
  int put(const float* v, int64_t n, const float** out) {
    if (!v || devp) {
      *out = v;
      return ENVG_OK;
    }
    float* dv = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(d->vec.p) + off);
    ENVG_CUDA(cudaMemcpyAsync(dv, v, (size_t)n * 4, cudaMemcpyHostToDevice, stream_of(d)));
    d->st.h2d_bytes += (double)n * 4;
    off += (size_t)rup(n * 4, 256);
    *out = dv;
    return ENVG_OK;
  }
};

cudaEvent_t batch_event(Dev* d, size_t i) {
  while (d->batch_events.size() <= i) {
    cudaEvent_t e = nullptr;
    cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    d->batch_events.push_back(e);
  }
  return d->batch_events[i];
}
}  // namespace

}  // extern "C"

namespace {
// envg_linear_batch and envg_linear_nsplit_batch.  ns[i] (optional) makes linear i an N-split
// shard whose epilogue writes into every rank's copy of Y.
int batch_core(Dev* d, const envg_linear_desc* descs, const envg_nsplit_desc* ns, int n, int flags) {
  if (n < 0 || (n > 0 && !descs)) return fail(ENVG_ERR_ARG, "envg_linear_batch: bad descriptor array");
  if (!(flags & ENVG_DEVICE_PTRS)) return fail(ENVG_ERR_ARG, "envg_linear_batch: needs device pointers");
  for (int i = 0; i < n; ++i) ENVG_TRY(check_linear_args(d, descs[i]));
  // An N-split shard keeps its output on this rank (columns [col0, col0 + width) of y_local only)
  // with ENVG_KEEP_SHARDED, or when the descriptor names no peer copies and no multicast address.
  auto keeps_shard = [&](int i) {
    return ns && ((flags & ENVG_KEEP_SHARDED) || (ns[i].npeers == 0 && !ns[i].y_multicast));
  };
  auto nsplit_epi = [&](int i, EpiArgs& e) -> int {
    if (!ns) return ENVG_OK;
    const envg_nsplit_desc& x = ns[i];
    const int64_t n_out = e.n_out;
    if (x.col0 < 0 || x.col0 + n_out > x.ldy)
      return fail(ENVG_ERR_ARG, "nsplit: columns [%lld, %lld) outside ldy %lld", (long long)x.col0,
                  (long long)(x.col0 + n_out), (long long)x.ldy);
    const bool keep = keeps_shard(i);
    if (!keep && !x.y_multicast && (x.npeers < 1 || x.npeers > 8 || !x.y_peers))
      return fail(ENVG_ERR_ARG, "nsplit: give a multicast address or 1..8 peer copies of Y");
    e.ldy = x.ldy;
    e.col_off = (int)x.col0;
    bool aligned = (reinterpret_cast<uintptr_t>(e.Y) & 15) == 0 && x.ldy % 4 == 0 && x.col0 % 4 == 0;
    if (keep) {
      e.nremote = 0;  // the epilogue stores into this rank's y_local only
    } else if (x.y_multicast) {
      e.nremote = -1;
      e.remote[0] = x.y_multicast;
      aligned = aligned && (reinterpret_cast<uintptr_t>(x.y_multicast) & 15) == 0;
    } else {
      e.nremote = x.npeers;
      for (int r = 0; r < x.npeers; ++r) {
        if (!x.y_peers[r]) return fail(ENVG_ERR_ARG, "nsplit: peer copy %d is NULL", r);
        e.remote[r] = x.y_peers[r];
        aligned = aligned && (reinterpret_cast<uintptr_t>(x.y_peers[r]) & 15) == 0;
      }
    }
    e.vec_ok = (aligned && n_out % 4 == 0) ? 1 : 0;
    return ENVG_OK;
  };
  if (!d->aux) ENVG_CUDA(cudaStreamCreateWithFlags(&d->aux, cudaStreamNonBlocking));
  cudaStream_t s = stream_of(d);

  // Distinct inputs that take the tcgen05 path (M > gemv_max) get one bf16 copy each, packed in
  // one workspace; `src_of[i]` maps linear i to its copy.
  std::vector<int> src_of(n, -1);
  std::vector<int> first_use;  // linear index of each copy's first use
  std::vector<size_t> offset;
  size_t total = 0;
  // true when linear t writes into the fp32 input of linear c
  auto writes_input_of = [&](int t, const envg_linear_desc& c) {
    const envg_linear_desc& pr = descs[t];
    const bool gu = pr.W->layout == ENVG_LAYOUT_GATE_UP;
    const char* y0 = reinterpret_cast<const char*>(pr.dst);
    const char* y1 = y0 + (size_t)(pr.M * (gu ? pr.N / 2 : pr.N)) * 4;
    const char* x0 = reinterpret_cast<const char*>(c.x);
    const char* x1 = x0 + (size_t)(c.M * c.K) * 4;
    return pr.M > 0 && x0 < y1 && y0 < x1;
  };
  for (int i = 0; i < n; ++i) {
    const envg_linear_desc& q = descs[i];
    if (q.M == 0 || q.M <= d->gemv_max || q.W->x3) continue;  // k_gemv reads fp32 x; bf16x3: below
    for (size_t j = 0; j < first_use.size(); ++j) {
      const envg_linear_desc& p = descs[first_use[j]];
      if (p.x == q.x && p.M == q.M && p.W->Kp == q.W->Kp && p.K == q.K) {
        // the copy holds x as it was before first_use[j]; reuse it only if nothing since wrote x
        bool stale = false;
        for (int t = first_use[j]; t < i && !stale; ++t) stale = writes_input_of(t, q);
        if (stale) continue;
        src_of[i] = (int)j;
        break;
      }
    }
    if (src_of[i] < 0) {
      src_of[i] = (int)first_use.size();
      first_use.push_back(i);
      offset.push_back(total);
      total += ((size_t)(q.M * q.W->Kp) * 2 + 255) & ~size_t(255);
    }
  }
  ENVG_TRY(ensure(d, d->xbatch, total));
  uint8_t* base = reinterpret_cast<uint8_t*>(d->xbatch.p);

  // Event plan: ev[0] = start of the batch on s; ev[1 + j] = copy j done on aux;
  // ev[1 + ncopies + i] = linear i done on s.
  const size_t ncopies = first_use.size();
  ENVG_CUDA(cudaEventRecord(batch_event(d, 0), s));
  ENVG_CUDA(cudaStreamWaitEvent(d->aux, batch_event(d, 0), 0));
  cudaStream_t saved = d->user;
  size_t next_copy = 0;
  // Producers of copy j: earlier linears whose output overlaps copy j's input.
  auto produces = [&](int p, size_t j) {
    const envg_linear_desc& q = descs[first_use[j]];
    const envg_linear_desc& pr = descs[p];
    const bool gu = pr.W->layout == ENVG_LAYOUT_GATE_UP;
    const char* y0 = reinterpret_cast<const char*>(pr.dst);
    const char* y1 = y0 + (size_t)(pr.M * (gu ? pr.N / 2 : pr.N)) * 4;
    const char* x0 = reinterpret_cast<const char*>(q.x);
    const char* x1 = x0 + (size_t)(q.M * q.K) * 4;
    return pr.M > 0 && x0 < y1 && y0 < x1;
  };
  // A copy whose input is exactly the output of one earlier linear on the tcgen05 path (k1 or k2; same
  // [M, K] shape, K % 8 == 0, overwrite epilogue) is written by that linear's epilogue as a bf16
  // side output instead of by a cast: fused_from[j] = the producer, yb_copy[p] = the copy.
  std::vector<int> fused_from(ncopies, -1), yb_copy(n, -1);
  for (size_t j = 0; j < ncopies; ++j) {
    const envg_linear_desc& q = descs[first_use[j]];
    if (q.W->Kp != q.K) continue;
    int prod = -1, count = 0;
    for (int p = 0; p < first_use[j]; ++p)
      if (produces(p, j)) {
        ++count;
        prod = p;
      }
    if (count != 1) continue;
    const envg_linear_desc& pr = descs[prod];
    const int64_t pn = pr.W->layout == ENVG_LAYOUT_GATE_UP ? pr.N / 2 : pr.N;
    if ((const void*)pr.dst != (const void*)q.x || pr.M != q.M || pn != q.K) continue;
    if (pr.epilogue == ENVG_EPI_GATED_RESIDUAL || src_of[prod] < 0) continue;
    if (ns) continue;  // an N-split producer computes only its own columns of the consumer's input
    if (yb_copy[prod] >= 0) continue;
    fused_from[j] = prod;
    yb_copy[prod] = (int)j;
  }
  // Cast j may be issued once every producer (index < issued) has been issued on s.
  auto ready = [&](size_t j, int issued) {
    for (int p = issued; p < first_use[j]; ++p)
      if (produces(p, j)) return false;
    return true;
  };
  auto issue_cast = [&](size_t j) -> int {
    const envg_linear_desc& q = descs[first_use[j]];
    for (int p = 0; p < first_use[j]; ++p)
      if (produces(p, j)) ENVG_CUDA(cudaStreamWaitEvent(d->aux, batch_event(d, 1 + ncopies + p), 0));
    d->user = d->aux;
    int rc = launch_cast_rows(d, q.x, q.K, q.M, q.K, q.W->Kp, base + offset[j]);
    d->user = saved;
    if (rc != ENVG_OK) return rc;
    ENVG_CUDA(cudaEventRecord(batch_event(d, 1 + j), d->aux));
    return ENVG_OK;
  };
  // Consecutive independent M <= gemv_max linears go out as one persistent k_gemv launch; until
  // that launch, their events do not exist, so casts that read their outputs wait.
  std::vector<GemvJob> gq;
  std::vector<int> gidx;
  auto flush_gemv = [&]() -> int {
    if (gq.empty()) return ENVG_OK;
    ENVG_TRY(launch_gemv_set(d, gq.data(), (int)gq.size()));
    for (size_t k = 0; k < gidx.size(); ++k) {
      ENVG_CUDA(cudaEventRecord(batch_event(d, 1 + ncopies + gidx[k]), s));
      d->st.calls++;
      d->st.flops += gq[k].flops;
    }
    gq.clear();
    gidx.clear();
    return ENVG_OK;
  };
  // Consecutive independent skinny (gemv_max < M <= skinny_max) linears with the same padded M
  // and layout kind go out as one persistent k2_set launch, in the same way.  (Keeping a plain
  // and a GATE_UP queue open side by side, so that a Qwen3 layer runs as {gate_up} then
  // {q, k, v, o, down}, measured slower: the merged set's static unit assignment is unbalanced.)
  std::vector<K2Job> kq;
  std::vector<int> kidx;
  auto flush_k2 = [&]() -> int {
    if (kq.empty()) return ENVG_OK;
    ENVG_TRY(launch_k2_set(d, kq.data(), (int)kq.size()));
    for (size_t k = 0; k < kidx.size(); ++k) {
      ENVG_CUDA(cudaEventRecord(batch_event(d, 1 + ncopies + kidx[k]), s));
      d->st.calls++;
      d->st.flops += kq[k].flops;
    }
    kq.clear();
    kidx.clear();
    return ENVG_OK;
  };
  // Consecutive independent linears on the CTA-pair path (M > 128) that read the same bf16
  // input copy go out as one pair-set launch (launch_pair_set), in the same way.
  std::vector<PairJob> pq;
  std::vector<int> pidx;
  int pair_src = -1;
  auto flush_pair = [&]() -> int {
    if (pq.empty()) return ENVG_OK;
    const envg_linear_desc& f = descs[pidx.front()];
    ENVG_TRY(launch_pair_set(d, base + offset[pair_src], f.M, f.W->Kp, pq.data(), (int)pq.size()));
    for (size_t k = 0; k < pidx.size(); ++k) {
      ENVG_CUDA(cudaEventRecord(batch_event(d, 1 + ncopies + pidx[k]), s));
      d->st.calls++;
      d->st.flops += pq[k].flops;
    }
    pq.clear();
    pidx.clear();
    pair_src = -1;
    return ENVG_OK;
  };
  auto out_range = [&](const envg_linear_desc& c, const char** y0, const char** y1) {
    const bool gu = c.W->layout == ENVG_LAYOUT_GATE_UP;
    *y0 = reinterpret_cast<const char*>(c.dst);
    *y1 = *y0 + (size_t)(c.M * (gu ? c.N / 2 : c.N)) * 4;
  };
  auto reads_output_of = [&](const envg_linear_desc& c, const envg_linear_desc& pr) {
    const bool gu = pr.W->layout == ENVG_LAYOUT_GATE_UP;
    const char* y0 = reinterpret_cast<const char*>(pr.dst);
    const char* y1 = y0 + (size_t)(pr.M * (gu ? pr.N / 2 : pr.N)) * 4;
    const char* x0 = reinterpret_cast<const char*>(c.x);
    const char* x1 = x0 + (size_t)(c.M * c.K) * 4;
    return pr.M > 0 && x0 < y1 && y0 < x1;
  };
  // Every epilogue reads its linear's bias (N floats) and, for the gated residual, its gate
  // (N floats).  Inside one launch a member must neither read a vector that another member
  // writes nor write over one that another member reads.
  auto vectors_meet_output = [&](const envg_linear_desc& c, const envg_linear_desc& pr) {
    if (pr.M <= 0 || c.M <= 0) return false;
    const char *y0, *y1;
    out_range(pr, &y0, &y1);
    auto hits = [&](const float* v) {
      const char* v0 = reinterpret_cast<const char*>(v);
      return v && v0 < y1 && y0 < v0 + (size_t)c.N * 4;
    };
    return hits(c.bias) || (c.epilogue == ENVG_EPI_GATED_RESIDUAL && hits(c.gate));
  };
  auto vector_hazard = [&](const envg_linear_desc& a, const envg_linear_desc& b) {
    return vectors_meet_output(a, b) || vectors_meet_output(b, a);
  };
  for (int i = 0; i < n; ++i) {
    const envg_linear_desc& q = descs[i];
    const bool is_k2 = src_of[i] >= 0 && q.M <= d->skinny_max;
    const bool is_pair = src_of[i] >= 0 && !is_k2 && d->use_pair && q.M > BM && (!ns || keeps_shard(i));
    const bool is_x3 = q.M > 0 && q.W->x3;
    if (src_of[i] >= 0 || is_x3) ENVG_TRY(flush_gemv());  // a tcgen05 linear follows the pending gemv ones
    if (!is_k2) ENVG_TRY(flush_k2());
    if (!is_pair) ENVG_TRY(flush_pair());
    // casts run one linear ahead of the GEMMs, in order, as soon as their inputs exist; a cast
    // that reads the output of a linear still waiting in a group waits for that group's launch
    int first_pending = i;
    if (!gidx.empty()) first_pending = std::min(first_pending, gidx.front());
    if (!kidx.empty()) first_pending = std::min(first_pending, kidx.front());
    if (!pidx.empty()) first_pending = std::min(first_pending, pidx.front());
    while (next_copy < ncopies && first_use[next_copy] <= i + 1 && ready(next_copy, first_pending)) {
      if (fused_from[next_copy] < 0) ENVG_TRY(issue_cast(next_copy));  // else written by its producer on s
      ++next_copy;
    }
    if (q.M == 0) continue;
    const bool gu = q.W->layout == ENVG_LAYOUT_GATE_UP;
    EpiArgs e = linear_epi(q);
    ENVG_TRY(nsplit_epi(i, e));
    if (yb_copy[i] >= 0) {
      e.yb = reinterpret_cast<__nv_bfloat16*>(base + offset[yb_copy[i]]);
      e.ldyb = descs[first_use[yb_copy[i]]].W->Kp;
    }
    const int64_t n_out = gu ? q.N / 2 : q.N;
    const double fl = 2.0 * (double)q.M * (double)q.N * (double)q.K;
    const double ob = 4.0 * (double)q.M * n_out + (q.bias ? 4.0 * q.N : 0.0) +
                      (q.epilogue == ENVG_EPI_GATED_RESIDUAL ? 4.0 * (double)q.M * n_out + 4.0 * q.N : 0.0);
    if (is_x3) {
      // A bf16x3 weight (fp32 values kept as hi / lo parts) takes its own activation layout
      // hi|hi|lo, made here on s after every earlier linear, then runs alone.
      ENVG_TRY(ensure(d, d->xb, (size_t)(q.M * q.W->Kp) * 2));
      ENVG_TRY(launch_cast_x3(d, q.x, q.K, q.M, q.K, q.W->Ks, d->xb.p, X3_ACT));
      ENVG_TRY(gemm_device(d, d->xb.p, q.M, q.W->Kp, q.W->tm256, q.W->tm128, q.W->rows, gu, e, fl,
                           2.0 * (double)q.N * q.K + 2.0 * (double)q.M * q.W->Kp + ob));
    } else if (src_of[i] < 0) {
      const char *qy0, *qy1;
      out_range(q, &qy0, &qy1);
      // a set runs its linears at once: none may read or write over another's output, and since
      // k_gemv reads fp32 X directly (no cast copy), none may write over another's input either.
      // One exception: a linear whose X is exactly the whole output of one pending linear (Qwen3's
      // down after gate_up at M = 1) joins the set chained to it; its units wait in the kernel
      // until that linear's outputs are all stored.
      int dep = -1;
      for (size_t j = 0; j < gidx.size(); ++j) {
        const envg_linear_desc& pk = descs[gidx[j]];
        const char *ky0, *ky1;
        out_range(pk, &ky0, &ky1);
        const int64_t pn = pk.W->layout == ENVG_LAYOUT_GATE_UP ? pk.N / 2 : pk.N;
        bool chain = dep < 0 && !ns && (const void*)q.x == (const void*)pk.dst && q.M == pk.M && q.K == pn;
        for (const GemvJob& g : gq) chain = chain && g.dep != (int)j;  // one reader per producer
        if (reads_output_of(q, pk) && chain) {
          dep = (int)j;
          if ((qy0 < ky1 && ky0 < qy1) || writes_input_of(i, pk) || vector_hazard(q, pk)) {
            ENVG_TRY(flush_gemv());
            dep = -1;
            break;
          }
          continue;
        }
        if (reads_output_of(q, pk) || (qy0 < ky1 && ky0 < qy1) || writes_input_of(i, pk) || vector_hazard(q, pk)) {
          ENVG_TRY(flush_gemv());
          dep = -1;
          break;
        }
      }
      if (!d->gemv_chain) dep = -1;
      if (dep < 0) {  // a pending linear it reads (not chainable) was flushed above; recheck
        for (int k : gidx)
          if (reads_output_of(q, descs[k])) {
            ENVG_TRY(flush_gemv());
            break;
          }
      }
      GemvJob gj{q.x, q.M, q.K, q.W, gu, e, fl, 2.0 * (double)q.N * q.K + 4.0 * (double)q.M * q.K + ob};
      gj.dep = dep;
      gq.push_back(gj);
      gidx.push_back(i);
      if ((int)gq.size() == GEMV_MAX_LIN) ENVG_TRY(flush_gemv());
      continue;
    } else if (is_k2) {
      const int mpad = (int)rup(q.M, 16);
      bool flush = !kq.empty() && ((int)rup(kq.front().M, 16) != mpad || kq.front().gu != gu ||
                                   (int)kq.size() == K2S_MAX_LIN);
      const char *qy0, *qy1;
      out_range(q, &qy0, &qy1);
      for (int k : kidx) {  // a set runs its linears at once: no reads of, or writes over, its outputs
        const char *ky0, *ky1;
        out_range(descs[k], &ky0, &ky1);
        flush = flush || reads_output_of(q, descs[k]) || (qy0 < ky1 && ky0 < qy1) || vector_hazard(q, descs[k]);
      }
      if (flush) ENVG_TRY(flush_k2());
      if ((size_t)src_of[i] >= next_copy) {
        // its cast waits for a linear of the pending group: launch the group, then cast
        ENVG_TRY(flush_k2());
        while (next_copy < ncopies && first_use[next_copy] <= i + 1 && ready(next_copy, i)) {
          if (fused_from[next_copy] < 0) ENVG_TRY(issue_cast(next_copy));
          ++next_copy;
        }
        if ((size_t)src_of[i] >= next_copy) return fail(ENVG_ERR_STATE, "envg_linear_batch: internal schedule error");
      }
      if (fused_from[src_of[i]] < 0) ENVG_CUDA(cudaStreamWaitEvent(s, batch_event(d, 1 + src_of[i]), 0));
      kq.push_back(K2Job{base + offset[src_of[i]], q.M, q.W->Kp, &q.W->tm128, q.W->rows, gu, e, fl,
                         2.0 * (double)q.N * q.K + 2.0 * (double)q.M * q.W->Kp + ob});
      kidx.push_back(i);
      continue;
    } else if (is_pair) {
      bool flush = !pq.empty() && (src_of[i] != pair_src || (int)pq.size() == PSET_MAX);
      const char *qy0, *qy1;
      out_range(q, &qy0, &qy1);
      for (int k : pidx) {
        const char *py0, *py1;
        out_range(descs[k], &py0, &py1);
        flush = flush || reads_output_of(q, descs[k]) || (qy0 < py1 && py0 < qy1) || vector_hazard(q, descs[k]);
      }
      if (flush) ENVG_TRY(flush_pair());
      if ((size_t)src_of[i] >= next_copy) {
        // its cast waits for a linear of the pending group: launch the group, then cast
        ENVG_TRY(flush_pair());
        while (next_copy < ncopies && first_use[next_copy] <= i + 1 && ready(next_copy, i)) {
          if (fused_from[next_copy] < 0) ENVG_TRY(issue_cast(next_copy));
          ++next_copy;
        }
        if ((size_t)src_of[i] >= next_copy) return fail(ENVG_ERR_STATE, "envg_linear_batch: internal schedule error");
      }
      if (fused_from[src_of[i]] < 0) ENVG_CUDA(cudaStreamWaitEvent(s, batch_event(d, 1 + src_of[i]), 0));
      pq.push_back(PairJob{&q.W->tm128, q.W->rows, gu, e, fl, 2.0 * (double)q.N * q.K + 2.0 * (double)q.M * q.W->Kp + ob});
      pidx.push_back(i);
      pair_src = src_of[i];
      continue;
    } else {
      ENVG_TRY(flush_gemv());
      if ((size_t)src_of[i] >= next_copy) return fail(ENVG_ERR_STATE, "envg_linear_batch: internal schedule error");
      if (fused_from[src_of[i]] < 0) ENVG_CUDA(cudaStreamWaitEvent(s, batch_event(d, 1 + src_of[i]), 0));
      ENVG_TRY(gemm_device(d, base + offset[src_of[i]], q.M, q.W->Kp, q.W->tm256, q.W->tm128, q.W->rows, gu, e, fl,
                           2.0 * (double)q.N * q.K + 2.0 * (double)q.M * q.W->Kp + ob));
    }
    ENVG_CUDA(cudaEventRecord(batch_event(d, 1 + ncopies + i), s));
    d->st.calls++;
    d->st.flops += fl;
  }
  ENVG_TRY(flush_gemv());
  ENVG_TRY(flush_k2());
  ENVG_TRY(flush_pair());
  if (!(flags & ENVG_ASYNC)) return sync_and_check(d);
  return ENVG_OK;
}
// envg_linear_batch on host pointers.  The linears' copies and GEMMs are queued back to back and
// the call synchronises once, so the copy-in of one linear, the GEMMs and the copy-out of an
// earlier one overlap (PCIe carries both directions at once): the call costs about the larger of
// its total copy-in and copy-out instead of the sum over the linears of each one's larger
// direction.  Copy-ins queue on d->h2d, GEMMs on the compute stream, copy-outs on d->d2h.  Each
// linear is computed exactly as envg_linear computes it from host pointers: from PIPE_MIN_M rows
// on in row chunks of PIPE_CHUNK rows without split-K, else in one launch.  An input shared by
// several linears (the same x, M and K) is copied once.  When one linear's output overlaps
// another's output, or an input of a later linear (x, bias, gate), the linears run one call
// after another instead.
int batch_host(Dev* d, const envg_linear_desc* descs, int n, int flags) {
  if (n < 0 || (n > 0 && !descs)) return fail(ENVG_ERR_ARG, "envg_linear_batch: bad descriptor array");
  for (int i = 0; i < n; ++i) ENVG_TRY(check_linear_args(d, descs[i]));
  auto n_out_of = [](const envg_linear_desc& q) { return q.W->layout == ENVG_LAYOUT_GATE_UP ? q.N / 2 : q.N; };
  auto overlap = [](const void* a, size_t na, const void* b, size_t nb) {
    const char* pa = static_cast<const char*>(a);
    const char* pb = static_cast<const char*>(b);
    return a && b && na && nb && pa < pb + nb && pb < pa + na;
  };
  bool sequential = !d->pipe_host;
  for (int j = 0; j < n && !sequential; ++j) {
    const envg_linear_desc& b = descs[j];
    if (b.M == 0) continue;
    const size_t yb = (size_t)(b.M * n_out_of(b)) * 4;
    for (int i = 0; i < j && !sequential; ++i) {
      const envg_linear_desc& a = descs[i];
      if (a.M == 0) continue;
      const size_t ya = (size_t)(a.M * n_out_of(a)) * 4;
      sequential = overlap(a.dst, ya, b.dst, yb) || overlap(a.dst, ya, b.x, (size_t)(b.M * b.K) * 4) ||
                   overlap(a.dst, ya, b.bias, b.bias ? (size_t)b.N * 4 : 0) ||
                   overlap(a.dst, ya, b.gate, b.gate ? (size_t)b.N * 4 : 0);
    }
  }
  if (sequential) {
    for (int i = 0; i < n; ++i) {
      const envg_linear_desc& q = descs[i];
      ENVG_TRY(linear_core(d, q.dst, q.x, q.W, q.bias, q.M, q.K, q.N, q.epilogue, q.gate, ENVG_HOST_PTRS, Prologue{}));
    }
    return ENVG_OK;
  }
  // device copies: one per distinct input, an output, bias and gate per linear
  auto a256 = [](size_t b) { return (b + 255) & ~size_t(255); };
  std::vector<int> xsrc(n, -1);  // the descriptor whose copy of x this one reads
  std::vector<size_t> xoff(n, 0), yoff(n, 0), boff(n, 0), goff(n, 0);
  size_t total = 0;
  for (int i = 0; i < n; ++i) {
    const envg_linear_desc& q = descs[i];
    if (q.M == 0) continue;
    for (int k = 0; k < i && xsrc[i] < 0; ++k)
      if (descs[k].M == q.M && descs[k].K == q.K && descs[k].x == q.x) xsrc[i] = xsrc[k];
    if (xsrc[i] < 0) {
      xsrc[i] = i;
      xoff[i] = total;
      total += a256((size_t)(q.M * q.K) * 4);
    }
    yoff[i] = total;
    total += a256((size_t)(q.M * n_out_of(q)) * 4);
    if (q.bias) {
      boff[i] = total;
      total += a256((size_t)q.N * 4);
    }
    if (q.epilogue == ENVG_EPI_GATED_RESIDUAL) {
      goff[i] = total;
      total += a256((size_t)q.N * 4);
    }
  }
  if (total == 0) return ENVG_OK;
  ENVG_TRY(ensure(d, d->hb, total));
  uint8_t* base = reinterpret_cast<uint8_t*>(d->hb.p);
  cudaStream_t s = stream_of(d);
  if (!d->h2d) ENVG_CUDA(cudaStreamCreateWithFlags(&d->h2d, cudaStreamNonBlocking));
  if (!d->d2h) ENVG_CUDA(cudaStreamCreateWithFlags(&d->d2h, cudaStreamNonBlocking));
  // the copy streams start after the work already queued on s
  size_t ev = 0;
  ENVG_CUDA(cudaEventRecord(pipe_event(d, ev), s));
  ENVG_CUDA(cudaStreamWaitEvent(d->h2d, pipe_event(d, ev), 0));
  ENVG_CUDA(cudaStreamWaitEvent(d->d2h, pipe_event(d, ev), 0));
  ++ev;
  uint64_t calls = d->st.calls;  // one per linear, as envg_linear counts them (not one per chunk)
  for (int i = 0; i < n; ++i) {
    const envg_linear_desc& q = descs[i];
    if (q.M == 0) continue;
    const int64_t n_out = n_out_of(q);
    float* dx = reinterpret_cast<float*>(base + xoff[xsrc[i]]);
    float* dy = reinterpret_cast<float*>(base + yoff[i]);
    const float *dbias = nullptr, *dgate = nullptr;
    if (q.bias) {
      dbias = reinterpret_cast<float*>(base + boff[i]);
      ENVG_CUDA(cudaMemcpyAsync(const_cast<float*>(dbias), q.bias, (size_t)q.N * 4, cudaMemcpyHostToDevice, d->h2d));
      d->st.h2d_bytes += (double)q.N * 4;
    }
    if (q.epilogue == ENVG_EPI_GATED_RESIDUAL) {
      dgate = reinterpret_cast<float*>(base + goff[i]);
      ENVG_CUDA(cudaMemcpyAsync(const_cast<float*>(dgate), q.gate, (size_t)q.N * 4, cudaMemcpyHostToDevice, d->h2d));
      d->st.h2d_bytes += (double)q.N * 4;
    }
    const bool chunked = q.M >= PIPE_MIN_M;
    const int64_t nch = chunked ? std::max<int64_t>(1, q.M / PIPE_CHUNK) : 1;
    for (int64_t c = 0; c < nch; ++c) {
      const int64_t r0 = chunked ? c * PIPE_CHUNK : 0;
      const int64_t rows = (c == nch - 1) ? q.M - r0 : PIPE_CHUNK;
      if (xsrc[i] == i) {
        ENVG_CUDA(cudaMemcpyAsync(dx + r0 * q.K, q.x + r0 * q.K, (size_t)(rows * q.K) * 4, cudaMemcpyHostToDevice,
                                  d->h2d));
        d->st.h2d_bytes += (double)(rows * q.K) * 4;
      }
      if (q.epilogue == ENVG_EPI_GATED_RESIDUAL) {
        ENVG_CUDA(cudaMemcpyAsync(dy + r0 * n_out, q.dst + r0 * n_out, (size_t)(rows * n_out) * 4,
                                  cudaMemcpyHostToDevice, d->h2d));
        d->st.h2d_bytes += (double)(rows * n_out) * 4;
      }
      // every copy queued on h2d so far (this chunk's included) has landed
      ENVG_CUDA(cudaEventRecord(pipe_event(d, ev), d->h2d));
      ENVG_CUDA(cudaStreamWaitEvent(s, pipe_event(d, ev), 0));
      ++ev;
      {
        struct NoSplit {
          Dev* d;
          bool prev;
          ~NoSplit() { d->no_split = prev; }
        } guard{d, d->no_split};
        d->no_split = chunked;
        ENVG_TRY(linear_core(d, dy + r0 * n_out, dx + r0 * q.K, q.W, dbias, rows, q.K, q.N, q.epilogue, dgate,
                             ENVG_DEVICE_PTRS | ENVG_ASYNC, Prologue{}));
      }
      ENVG_CUDA(cudaEventRecord(pipe_event(d, ev), s));
      ENVG_CUDA(cudaStreamWaitEvent(d->d2h, pipe_event(d, ev), 0));
      ++ev;
      ENVG_CUDA(cudaMemcpyAsync(q.dst + r0 * n_out, dy + r0 * n_out, (size_t)(rows * n_out) * 4,
                                cudaMemcpyDeviceToHost, d->d2h));
      d->st.d2h_bytes += (double)(rows * n_out) * 4;
    }
    d->st.calls = ++calls;
  }
  ENVG_CUDA(cudaStreamSynchronize(d->d2h));
  ENVG_CUDA(cudaStreamSynchronize(d->h2d));
  return sync_and_check(d);
}

}  // namespace

extern "C" {

int envg_linear_batch(const envg_linear_desc* descs, int n, int flags) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  if (!(flags & ENVG_DEVICE_PTRS)) return batch_host(d, descs, n, flags);
  return batch_core(d, descs, nullptr, n, flags);
}

int envg_linear_nsplit_batch(const envg_nsplit_desc* descs, int n, int flags) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  if (n < 0 || (n > 0 && !descs)) return fail(ENVG_ERR_ARG, "envg_linear_nsplit_batch: bad descriptor array");
  std::vector<envg_linear_desc> lin((size_t)n);
  for (int i = 0; i < n; ++i) lin[i] = descs[i].lin;
  return batch_core(d, lin.data(), descs, n, flags);
}

int envg_linear_nsplit(float* y_local, float* const* y_peers, int npeers, float* y_multicast, int64_t ldy,
                       int64_t col0, const float* x, envg_weight W, const float* bias, int64_t M, int64_t K,
                       int64_t N, int epilogue, const float* gate, int flags) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  if (!(flags & ENVG_DEVICE_PTRS)) return fail(ENVG_ERR_ARG, "envg_linear_nsplit: needs device pointers");
  envg_linear_desc q{y_local, x, W, bias, M, K, N, epilogue, gate};
  ENVG_TRY(check_linear_args(d, q));
  const bool gu = W->layout == ENVG_LAYOUT_GATE_UP;
  const int64_t n_out = gu ? N / 2 : N;
  if (col0 < 0 || col0 + n_out > ldy) return fail(ENVG_ERR_ARG, "envg_linear_nsplit: columns [%lld, %lld) outside ldy %lld",
                                                  (long long)col0, (long long)(col0 + n_out), (long long)ldy);
  const bool keep = (flags & ENVG_KEEP_SHARDED) || (npeers == 0 && !y_multicast);
  if (!keep && !y_multicast && (npeers < 1 || npeers > 8 || !y_peers))
    return fail(ENVG_ERR_ARG, "envg_linear_nsplit: give a multicast address or 1..8 peer copies of Y");
  if (M == 0) return ENVG_OK;
  EpiArgs e = linear_epi(q);
  e.ldy = ldy;
  e.col_off = (int)col0;
  bool aligned = (reinterpret_cast<uintptr_t>(y_local) & 15) == 0 && ldy % 4 == 0 && col0 % 4 == 0;
  if (keep) {
    e.nremote = 0;  // the epilogue stores into this rank's y_local only
  } else if (y_multicast) {
    e.nremote = -1;
    e.remote[0] = y_multicast;
    aligned = aligned && (reinterpret_cast<uintptr_t>(y_multicast) & 15) == 0;
  } else {
    e.nremote = npeers;
    for (int r = 0; r < npeers; ++r) {
      if (!y_peers[r]) return fail(ENVG_ERR_ARG, "envg_linear_nsplit: peer copy %d is NULL", r);
      e.remote[r] = y_peers[r];
      aligned = aligned && (reinterpret_cast<uintptr_t>(y_peers[r]) & 15) == 0;
    }
  }
  e.vec_ok = (aligned && n_out % 4 == 0) ? 1 : 0;
  const double fl = 2.0 * (double)M * (double)N * (double)K;
  const double ob = 4.0 * (double)M * n_out + (bias ? 4.0 * N : 0.0);
  if (M <= d->gemv_max && !W->x3) {
    ENVG_TRY(launch_gemv(d, x, M, K, W, gu, e, fl, 2.0 * (double)N * K + 4.0 * (double)M * K + ob));
  } else {
    ENVG_TRY(ensure(d, d->xb, (size_t)(M * W->Kp) * 2));
    if (W->x3) ENVG_TRY(launch_cast_x3(d, x, K, M, K, W->Ks, d->xb.p, X3_ACT));
    else ENVG_TRY(launch_cast_rows(d, x, K, M, K, W->Kp, d->xb.p));
    ENVG_TRY(gemm_device(d, d->xb.p, M, W->Kp, W->tm256, W->tm128, W->rows, gu, e, fl,
                         2.0 * (double)N * K + 2.0 * (double)M * W->Kp + ob));
  }
  d->st.calls++;
  d->st.flops += fl;
  if (!(flags & ENVG_ASYNC)) return sync_and_check(d);
  return ENVG_OK;
}

int envg_conv2d(float* dst, const float* src, envg_weight W, const float* bias, int in_ch, int out_ch, int H, int W_,
                int kH, int kW, int stride, int pad, int batch, int epilogue, int flags) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  ENVG_TRY(check_weight(d, W));
  if (!W->conv) return fail(ENVG_ERR_ARG, "envg_conv2d: handle holds a linear weight");
  if (in_ch != W->in_ch || out_ch != W->out_ch || kH != W->kH || kW != W->kW)
    return fail(ENVG_ERR_ARG, "envg_conv2d: geometry [%d,%d,%d,%d] does not match the weight [%d,%d,%d,%d]", out_ch,
                in_ch, kH, kW, W->out_ch, W->in_ch, W->kH, W->kW);
  if (stride <= 0 || pad < 0 || H <= 0 || W_ <= 0 || batch < 0)
    return fail(ENVG_ERR_ARG, "envg_conv2d: invalid stride/pad/size");
  if (epilogue != ENVG_EPI_NONE && epilogue != ENVG_EPI_BIAS && epilogue != ENVG_EPI_SILU)
    return fail(ENVG_ERR_ARG, "envg_conv2d: epilogue %s (%d) not valid for a convolution", epi_name(epilogue), epilogue);
  if (epilogue == ENVG_EPI_BIAS && !bias) return fail(ENVG_ERR_ARG, "envg_conv2d: BIAS epilogue without bias");
  const int outH = (H + 2 * pad - kH) / stride + 1;
  const int outW = (W_ + 2 * pad - kW) / stride + 1;
  if (outH <= 0 || outW <= 0) return fail(ENVG_ERR_ARG, "envg_conv2d: empty output");
  if (batch == 0) return ENVG_OK;
  if (!dst || !src) return fail(ENVG_ERR_ARG, "envg_conv2d: dst or src is NULL");
  const bool devp = (flags & ENVG_DEVICE_PTRS) != 0;
  cudaStream_t s = stream_of(d);
  const int64_t in_elems = (int64_t)batch * in_ch * H * W_;
  const int64_t plane = (int64_t)outH * outW;
  const int64_t out_elems = (int64_t)batch * out_ch * plane;
  const float* dsrc = src;
  const float* dbias = bias;
  float* dy = dst;
  if (!devp) {
    ENVG_TRY(ensure(d, d->x, (size_t)in_elems * 4));
    ENVG_TRY(ensure(d, d->y, (size_t)out_elems * 4));
    ENVG_CUDA(cudaMemcpyAsync(d->x.p, src, (size_t)in_elems * 4, cudaMemcpyHostToDevice, s));
    d->st.h2d_bytes += (double)in_elems * 4;
    dsrc = reinterpret_cast<float*>(d->x.p);
    dy = reinterpret_cast<float*>(d->y.p);
    if (bias) {
      ENVG_TRY(ensure(d, d->bias, (size_t)out_ch * 4));
      ENVG_CUDA(cudaMemcpyAsync(d->bias.p, bias, (size_t)out_ch * 4, cudaMemcpyHostToDevice, s));
      d->st.h2d_bytes += (double)out_ch * 4;
      dbias = reinterpret_cast<float*>(d->bias.p);
    }
  }
  // NCHW fp32 -> NHWC bf16 with channels padded to Cp.
  const int Cp = W->Cp;
  ENVG_TRY(ensure(d, d->act, (size_t)batch * H * W_ * Cp * 2));
  ENVG_TRY(launch_transpose_cast(d, dsrc, (int64_t)H * W_, (int64_t)in_ch * H * W_, in_ch, H * W_, d->act.p, Cp,
                                 (int64_t)H * W_ * Cp, Cp, batch));
  ENVG_TRY(conv_core(d, W, d->act.p, dy, dbias, H, W_, stride, pad, batch, epilogue == ENVG_EPI_SILU ? 1 : 0, false));
  d->st.calls++;
  d->st.flops += 2.0 * (double)out_ch * (double)plane * (double)batch * (double)W->K;
  if (!devp) {
    ENVG_CUDA(cudaMemcpyAsync(dst, dy, (size_t)out_elems * 4, cudaMemcpyDeviceToHost, s));
    d->st.d2h_bytes += (double)out_elems * 4;
    return sync_and_check(d);
  }
  if (!(flags & ENVG_ASYNC)) return sync_and_check(d);
  return ENVG_OK;
}

int envg_group_norm(float* dst, const float* src, const float* gamma, const float* beta, int batch, int channels, int H,
                    int W_, int num_groups, int act_silu, int flags) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  ENVG_TRY(check_gn_geometry(batch, channels, H, W_, num_groups));
  if (batch == 0) return ENVG_OK;
  if (!dst || !src) return fail(ENVG_ERR_ARG, "group norm: dst or src is NULL");
  const bool devp = (flags & ENVG_DEVICE_PTRS) != 0;
  cudaStream_t s = stream_of(d);
  const int64_t HW = (int64_t)H * W_, elems = (int64_t)batch * channels * HW;
  const float* dsrc = src;
  float* dy = dst;
  ENVG_TRY(ensure(d, d->gn, gn_bytes(batch, channels, HW, num_groups), true));
  if (!devp) {
    ENVG_TRY(ensure(d, d->x, (size_t)elems * 4));
    ENVG_TRY(ensure(d, d->vec, (size_t)2 * rup((int64_t)channels * 4, 256)));
    ENVG_CUDA(cudaMemcpyAsync(d->x.p, src, (size_t)elems * 4, cudaMemcpyHostToDevice, s));
    d->st.h2d_bytes += (double)elems * 4;
    dsrc = reinterpret_cast<float*>(d->x.p);
    dy = reinterpret_cast<float*>(d->x.p);  // applied in place on the device copy
  }
  VecStage vs{d, devp};
  const float *g = nullptr, *b = nullptr;
  ENVG_TRY(vs.put(gamma, channels, &g));
  ENVG_TRY(vs.put(beta, channels, &b));
  float2* aff = nullptr;
  ENVG_TRY(launch_group_affine(d, dsrc, batch, channels, HW, num_groups, g, b, &aff));
  {
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(elems, 256), (int64_t)d->sms * 8));
    ProfScope ps(s, KID_GN_APPLY, 0.0, 8.0 * (double)elems);
    k_group_apply<<<blocks, 256, 0, s>>>(dsrc, dy, HW, batch * channels, aff, act_silu);
    ENVG_CUDA(cudaGetLastError());
    d->st.kernel_launches++;
  }
  d->st.calls++;
  if (!devp) {
    ENVG_CUDA(cudaMemcpyAsync(dst, dy, (size_t)elems * 4, cudaMemcpyDeviceToHost, s));
    d->st.d2h_bytes += (double)elems * 4;
    return sync_and_check(d);
  }
  if (!(flags & ENVG_ASYNC)) return sync_and_check(d);
  return ENVG_OK;
}

int envg_vae_resblock(float* dst, const float* src, const envg_resblock* rb, int batch, int H, int W_, int num_groups,
                      int flags) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  if (!rb) return fail(ENVG_ERR_ARG, "resblock: descriptor is NULL");
  const int Ci = rb->in_ch, Co = rb->out_ch;
  ENVG_TRY(check_weight(d, rb->conv1));
  ENVG_TRY(check_weight(d, rb->conv2));
  auto conv_is = [](envg_weight w, int o, int c, int k) {
    return w->conv && w->out_ch == o && w->in_ch == c && w->kH == k && w->kW == k;
  };
  if (!conv_is(rb->conv1, Co, Ci, 3)) return fail(ENVG_ERR_ARG, "resblock: conv1 is not a 3x3 %d -> %d conv", Ci, Co);
  if (!conv_is(rb->conv2, Co, Co, 3)) return fail(ENVG_ERR_ARG, "resblock: conv2 is not a 3x3 %d -> %d conv", Co, Co);
  if (rb->skip) {
    ENVG_TRY(check_weight(d, rb->skip));
    if (!conv_is(rb->skip, Co, Ci, 1)) return fail(ENVG_ERR_ARG, "resblock: skip is not a 1x1 %d -> %d conv", Ci, Co);
  } else if (Ci != Co) {
    return fail(ENVG_ERR_ARG, "resblock: in_ch %d != out_ch %d needs a skip conv", Ci, Co);
  }
  ENVG_TRY(check_gn_geometry(batch, Ci, H, W_, num_groups));
  ENVG_TRY(check_gn_geometry(batch, Co, H, W_, num_groups));
  if (batch == 0) return ENVG_OK;
  if (!dst || !src) return fail(ENVG_ERR_ARG, "resblock: dst or src is NULL");
  if ((const void*)dst == (const void*)src) return fail(ENVG_ERR_ARG, "resblock: dst aliases src");
  const bool devp = (flags & ENVG_DEVICE_PTRS) != 0;
  cudaStream_t s = stream_of(d);
  const int64_t HW = (int64_t)H * W_;
  const int64_t in_elems = (int64_t)batch * Ci * HW, out_elems = (int64_t)batch * Co * HW;
  const int Cp = (int)std::max(rb->conv1->Cp, rb->conv2->Cp);
  ENVG_TRY(ensure(d, d->gn, std::max(gn_bytes(batch, Ci, HW, num_groups), gn_bytes(batch, Co, HW, num_groups)), true));
  ENVG_TRY(ensure(d, d->act, (size_t)batch * HW * Cp * 2));
  ENVG_TRY(ensure(d, d->c1, (size_t)out_elems * 4));
  const float* dsrc = src;
  float* dy = dst;
  if (!devp) {
    ENVG_TRY(ensure(d, d->x, (size_t)in_elems * 4));
    ENVG_TRY(ensure(d, d->y, (size_t)out_elems * 4));
    ENVG_TRY(ensure(d, d->vec, (size_t)2 * rup((int64_t)Ci * 4, 256) + 5 * rup((int64_t)Co * 4, 256)));
    ENVG_CUDA(cudaMemcpyAsync(d->x.p, src, (size_t)in_elems * 4, cudaMemcpyHostToDevice, s));
    d->st.h2d_bytes += (double)in_elems * 4;
    dsrc = reinterpret_cast<float*>(d->x.p);
    dy = reinterpret_cast<float*>(d->y.p);
  }
  VecStage vs{d, devp};
  const float *g1, *b1, *cb1, *g2, *b2, *cb2, *sb;
  ENVG_TRY(vs.put(rb->norm1_gamma, Ci, &g1));
  ENVG_TRY(vs.put(rb->norm1_beta, Ci, &b1));
  ENVG_TRY(vs.put(rb->conv1_bias, Co, &cb1));
  ENVG_TRY(vs.put(rb->norm2_gamma, Co, &g2));
  ENVG_TRY(vs.put(rb->norm2_beta, Co, &b2));
  ENVG_TRY(vs.put(rb->conv2_bias, Co, &cb2));
  ENVG_TRY(vs.put(rb->skip_bias, Co, &sb));
  float* c1 = reinterpret_cast<float*>(d->c1.p);
  // skip path into dst
  if (rb->skip) {
    const int Cs = rb->skip->Cp;
    ENVG_TRY(launch_transpose_cast(d, dsrc, HW, (int64_t)Ci * HW, Ci, (int)HW, d->act.p, Cs, HW * Cs, Cs, batch));
    ENVG_TRY(conv_core(d, rb->skip, d->act.p, dy, sb, H, W_, 1, 0, batch, 0, false));
  } else {
    ENVG_CUDA(cudaMemcpyAsync(dy, dsrc, (size_t)in_elems * 4, cudaMemcpyDeviceToDevice, s));
  }
  // conv1(SiLU(GN1(src)))
  float2* aff = nullptr;
  ENVG_TRY(launch_group_affine(d, dsrc, batch, Ci, HW, num_groups, g1, b1, &aff));
  const int C1p = rb->conv1->Cp, C2p = rb->conv2->Cp;
  ENVG_TRY(launch_transpose_cast(d, dsrc, HW, (int64_t)Ci * HW, Ci, (int)HW, d->act.p, C1p, HW * C1p, C1p, batch, aff, 1));
  ENVG_TRY(conv_core(d, rb->conv1, d->act.p, c1, cb1, H, W_, 1, 1, batch, 0, false));
  // dst += conv2(SiLU(GN2(c1)))
  ENVG_TRY(launch_group_affine(d, c1, batch, Co, HW, num_groups, g2, b2, &aff));
  ENVG_TRY(launch_transpose_cast(d, c1, HW, (int64_t)Co * HW, Co, (int)HW, d->act.p, C2p, HW * C2p, C2p, batch, aff, 1));
  ENVG_TRY(conv_core(d, rb->conv2, d->act.p, dy, cb2, H, W_, 1, 1, batch, 0, true));
  d->st.calls++;
  d->st.flops += 2.0 * (double)batch * HW * ((double)Co * rb->conv1->K + (double)Co * rb->conv2->K +
                                             (rb->skip ? (double)Co * Ci : 0.0));
  if (!devp) {
    ENVG_CUDA(cudaMemcpyAsync(dst, dy, (size_t)out_elems * 4, cudaMemcpyDeviceToHost, s));
    d->st.d2h_bytes += (double)out_elems * 4;
    return sync_and_check(d);
  }
  if (!(flags & ENVG_ASYNC)) return sync_and_check(d);
  return ENVG_OK;
}

int envg_attention(float* dst, const float* Q, const float* K, const float* V, int seq_q, int seq_k, int heads,
                   int kv_heads, int head_dim, int64_t ldq, int64_t ldk, int64_t ldv, int64_t ldo, float scale,
                   int causal, const int32_t* key_mask, int flags) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  if (head_dim != FA_D) return fail(ENVG_ERR_UNSUPPORTED, "attention: head_dim %d (this build: 128)", head_dim);
  if (seq_q < 0 || seq_k <= 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads)
    return fail(ENVG_ERR_ARG, "attention: seq_q %d, seq_k %d, heads %d, kv_heads %d invalid", seq_q, seq_k, heads,
                kv_heads);
  if (heads > 65535) return fail(ENVG_ERR_UNSUPPORTED, "attention: more than 65535 heads");
  if (causal && seq_k < seq_q) return fail(ENVG_ERR_ARG, "attention: causal needs seq_k >= seq_q");
  if (ldq < (int64_t)heads * FA_D || ldk < (int64_t)kv_heads * FA_D || ldv < (int64_t)kv_heads * FA_D ||
      ldo < (int64_t)heads * FA_D)
    return fail(ENVG_ERR_ARG, "attention: a row stride is shorter than its heads x head_dim");
  if (!(scale > 0.0f)) return fail(ENVG_ERR_ARG, "attention: scale must be positive");
  if (seq_q == 0) return ENVG_OK;
  if (!dst || !Q || !K || !V) return fail(ENVG_ERR_ARG, "attention: NULL operand");
  const bool devp = (flags & ENVG_DEVICE_PTRS) != 0;
  cudaStream_t s = stream_of(d);
  // two query tiles per CTA when that still fills the GPU (one wave or more)
  const bool two = d->attn_tiles == 2 || (d->attn_tiles == 0 && cdiv(seq_q, 2 * FA_BQ) * heads >= d->sms);
  const int sq_pad = (int)rup(seq_q, two ? 2 * FA_BQ : FA_BQ), sk_pad = (int)rup(seq_k, FA_BKV);
  const int64_t wq = (int64_t)heads * FA_D, wk = (int64_t)kv_heads * FA_D;
  // device operands: Qh | Kh | Vt (fp16) | key bits | per-head max |x|
  const size_t qb = (size_t)heads * sq_pad * FA_D * 2, kb = (size_t)kv_heads * sk_pad * FA_D * 2;
  const size_t words = (size_t)sk_pad / 32;
  const size_t nmax = (size_t)heads + 2 * (size_t)kv_heads;
  ENVG_TRY(ensure(d, d->fa, qb + 2 * kb + words * 4 + nmax * 4));
  uint8_t* fa = reinterpret_cast<uint8_t*>(d->fa.p);
  __half* Qh = reinterpret_cast<__half*>(fa);
  __half* Kh = reinterpret_cast<__half*>(fa + qb);
  __half* Vt = reinterpret_cast<__half*>(fa + qb + kb);
  uint32_t* bits = reinterpret_cast<uint32_t*>(fa + qb + 2 * kb);
  float* amax = reinterpret_cast<float*>(fa + qb + 2 * kb + words * 4);
  const float *dq = Q, *dk = K, *dv = V;
  const int32_t* dm = key_mask;
  float* dout = dst;
  int64_t lq = ldq, lkk = ldk, lv = ldv, lo = ldo;
  if (!devp) {
    // host rows are packed to the heads' width on the device
    const size_t bq = (size_t)seq_q * wq * 4, bk = (size_t)seq_k * wk * 4, bo = bq;
    const size_t bm = key_mask ? (size_t)rup(seq_k * 4, 256) : 0;
    ENVG_TRY(ensure(d, d->fain, bq + 2 * bk + bm + bo));
    uint8_t* st = reinterpret_cast<uint8_t*>(d->fain.p);
    float* q_d = reinterpret_cast<float*>(st);
    float* k_d = reinterpret_cast<float*>(st + bq);
    float* v_d = reinterpret_cast<float*>(st + bq + bk);
    int32_t* m_d = reinterpret_cast<int32_t*>(st + bq + 2 * bk);
    float* o_d = reinterpret_cast<float*>(st + bq + 2 * bk + bm);
    ENVG_CUDA(cudaMemcpy2DAsync(q_d, wq * 4, Q, ldq * 4, wq * 4, seq_q, cudaMemcpyHostToDevice, s));
    ENVG_CUDA(cudaMemcpy2DAsync(k_d, wk * 4, K, ldk * 4, wk * 4, seq_k, cudaMemcpyHostToDevice, s));
    ENVG_CUDA(cudaMemcpy2DAsync(v_d, wk * 4, V, ldv * 4, wk * 4, seq_k, cudaMemcpyHostToDevice, s));
    if (key_mask) ENVG_CUDA(cudaMemcpyAsync(m_d, key_mask, (size_t)seq_k * 4, cudaMemcpyHostToDevice, s));
    d->st.h2d_bytes += (double)(bq + 2 * bk) + (key_mask ? seq_k * 4.0 : 0.0);
    dq = q_d, dk = k_d, dv = v_d, dm = key_mask ? m_d : nullptr, dout = o_d;
    lq = wq, lkk = wk, lv = wk, lo = wq;
  }
  // operand preparation: per-head max |x|, then scaled fp16 copies (V transposed) and key bits
  {
    ENVG_CUDA(cudaMemsetAsync(amax, 0, nmax * 4, s));
    ProfScope ps(s, KID_ABSMAX, 0.0, 4.0 * ((double)seq_q * wq + 2.0 * seq_k * wk));
    AbsmaxArgs am{};
    const float* xs[3] = {dq, dk, dv};
    const int64_t lds[3] = {lq, lkk, lv};
    const int seqs[3] = {seq_q, seq_k, seq_k};
    const int hs[3] = {heads, kv_heads, kv_heads};
    const int bases[3] = {0, heads, heads + kv_heads};
    for (int z = 0; z < 3; ++z) {
      am.X[z] = xs[z];
      am.ld[z] = lds[z];
      am.seq[z] = seqs[z];
      am.heads[z] = hs[z];
      am.base[z] = bases[z];
      am.vec[z] = (lds[z] % 4 == 0 && (reinterpret_cast<uintptr_t>(xs[z]) & 15) == 0) ? 1 : 0;
    }
    k_absmax_heads<<<dim3((unsigned)cdiv(std::max(seq_q, seq_k), 64), (unsigned)std::max(heads, kv_heads), 3), 256, 0,
                     s>>>(am, amax);
    ENVG_CUDA(cudaGetLastError());
    d->st.kernel_launches += 1;
  }
  {
    const bool vq = (lq % 4 == 0) && ((reinterpret_cast<uintptr_t>(dq) & 15) == 0);
    const bool vk = (lkk % 4 == 0) && ((reinterpret_cast<uintptr_t>(dk) & 15) == 0);
    ProfScope ps(s, KID_CAST_HEADS, 0.0, 4.0 * ((double)seq_q * wq + 2.0 * seq_k * wk) + (double)qb + 2.0 * kb);
    k_cast_heads<<<dim3((unsigned)cdiv((int64_t)sq_pad * 16, 256), (unsigned)heads), 256, 0, s>>>(
        dq, lq, seq_q, sq_pad, amax, Qh, vq);
    ENVG_CUDA(cudaGetLastError());
    k_cast_heads<<<dim3((unsigned)cdiv((int64_t)sk_pad * 16, 256), (unsigned)kv_heads), 256, 0, s>>>(
        dk, lkk, seq_k, sk_pad, amax + heads, Kh, vk);
    ENVG_CUDA(cudaGetLastError());
    k_v_transpose<<<dim3((unsigned)(sk_pad / 64), FA_D / 32, (unsigned)kv_heads), 256, 0, s>>>(
        dv, lv, seq_k, sk_pad, amax + heads + kv_heads, Vt);
    ENVG_CUDA(cudaGetLastError());
    d->st.kernel_launches += 3;
  }
  {
    ProfScope ps(s, KID_KEY_BITS, 0.0, (dm ? 4.0 * seq_k : 0.0) + 4.0 * words);
    k_key_bits<<<(unsigned)cdiv((int64_t)words, 128), 128, 0, s>>>(dm, seq_k, (int)words, bits);
    ENVG_CUDA(cudaGetLastError());
    d->st.kernel_launches++;
  }
  CUtensorMap tQ, tK, tV;
  // 16-bit element maps (TMA copies the fp16 bits unchanged)
  ENVG_TRY(tmap_2d(&tQ, Qh, FA_D, (uint64_t)heads * sq_pad, FA_BQ));
  ENVG_TRY(tmap_2d(&tK, Kh, FA_D, (uint64_t)kv_heads * sk_pad, FA_BKV));
  ENVG_TRY(tmap_2d(&tV, Vt, (uint64_t)sk_pad, (uint64_t)kv_heads * FA_D, FA_D));
  FaArgs a{};
  a.seq_q = seq_q;
  a.seq_k = seq_k;
  a.heads = heads;
  a.kv_heads = kv_heads;
  a.sq_pad = sq_pad;
  a.sk_pad = sk_pad;
  a.causal = causal ? 1 : 0;
  a.sl2 = scale * 1.4426950408889634f;
  a.kbits = bits;
  a.full_blocks = dm ? 0 : seq_k / FA_BKV;  // without a key mask every whole block inside seq_k is valid
  a.amax = amax;
  a.out = dout;
  a.ldo = lo;
  a.status = d->d_status;
  a.wait_cap_ns = d->wait_cap_ns;
  static bool attr_set[64] = {};
  if (!attr_set[d->id]) {
    ENVG_CUDA(cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, FaSmem::TOTAL));
    ENVG_CUDA(cudaFuncSetAttribute(k_attention2, cudaFuncAttributeMaxDynamicSharedMemorySize, Fa2Smem::TOTAL));
    attr_set[d->id] = true;
  }
  {
    // visible (q, k) pairs: all of them, or the causal triangle
    double pairs = (double)seq_q * seq_k;
    if (causal) pairs = (double)seq_q * seq_k - 0.5 * (double)seq_q * (seq_q - 1);
    const double fl = 4.0 * FA_D * pairs * heads;
    ProfScope ps(s, KID_ATTN, fl, (double)qb + 2.0 * kb * (double)(sq_pad / FA_BQ) + 4.0 * seq_q * wq);
    if (two)
      k_attention2<<<dim3((unsigned)(sq_pad / (2 * FA_BQ)), (unsigned)heads), FA2_THREADS, Fa2Smem::TOTAL, s>>>(tQ, tK,
                                                                                                        tV, a);
    else
      k_attention<<<dim3((unsigned)(sq_pad / FA_BQ), (unsigned)heads), FA_THREADS, FaSmem::TOTAL, s>>>(tQ, tK, tV, a);
    const cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) {
      cudaFuncAttributes fa{};
      cudaFuncGetAttributes(&fa, two ? (const void*)k_attention2 : (const void*)k_attention);
      return fail(ENVG_ERR_CUDA, "attention launch (%s, %d threads, %d B smem) failed: %s; kernel: %d regs, max %d "
                  "threads, %zu B local", two ? "k_attention2" : "k_attention", two ? FA2_THREADS : FA_THREADS,
                  two ? Fa2Smem::TOTAL : FaSmem::TOTAL, cudaGetErrorString(le), fa.numRegs, fa.maxThreadsPerBlock,
                  fa.localSizeBytes);
    }
    d->st.kernel_launches++;
    d->st.flops += fl;
  }
  d->st.calls++;
  if (!devp) {
    ENVG_CUDA(cudaMemcpy2DAsync(dst, ldo * 4, dout, wq * 4, wq * 4, seq_q, cudaMemcpyDeviceToHost, s));
    d->st.d2h_bytes += (double)seq_q * wq * 4;
    return sync_and_check(d);
  }
  if (!(flags & ENVG_ASYNC)) return sync_and_check(d);
  return ENVG_OK;
}

int envg_sgemm(int order, int transA, int transB, int64_t M, int64_t N, int64_t K, float alpha, const float* A,
               int64_t lda, const float* B, int64_t ldb, float beta, float* C, int64_t ldc) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  const int RowMajor = 101, NoTrans = 111, Trans = 112;
  if (order != RowMajor) return fail(ENVG_ERR_ARG, "ERROR : Operation is not supported using the provided arguments!");
  if ((transA != NoTrans && transA != Trans) || (transB != NoTrans && transB != Trans) ||
      (transA == Trans && transB == Trans))
    return fail(ENVG_ERR_ARG, "ERROR : Operation is not supported using the provided arguments!");
  if (M < 0 || N < 0 || K < 0) return fail(ENVG_ERR_ARG, "envg_sgemm: negative size");
  if (M == 0 || N == 0) return ENVG_OK;
  if (!A || !B || !C) return fail(ENVG_ERR_ARG, "envg_sgemm: NULL operand");
  const bool ta = transA == Trans, tb = transB == Trans;
  const int64_t arows = ta ? K : M, acols = ta ? M : K;
  const int64_t brows = tb ? N : K, bcols = tb ? K : N;
  if (lda < std::max<int64_t>(1, acols) || ldb < std::max<int64_t>(1, bcols) || ldc < std::max<int64_t>(1, N))
    return fail(ENVG_ERR_ARG, "envg_sgemm: leading dimension too small");
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2) return fail(ENVG_ERR_ARG, "envg_sgemm: size too large");
  cudaStream_t s = stream_of(d);
  // Both operands in the bf16x3 layout (k_cast_x3): A as hi|hi|lo, B as hi|lo|hi, so the
  // tensor-core GEMM over Kp = 3 * Ks sums a_hi b_hi + a_hi b_lo + a_lo b_hi.
  const int64_t Ks = rup(std::max<int64_t>(K, 1), 8);
  const int64_t Kp = 3 * Ks;
  ENVG_TRY(ensure(d, d->x, (size_t)(arows * acols) * 4));
  ENVG_TRY(ensure(d, d->b32, (size_t)(brows * bcols) * 4));
  ENVG_TRY(ensure(d, d->y, (size_t)(M * N) * 4));
  ENVG_TRY(ensure(d, d->xb, (size_t)(M * Kp) * 2));
  ENVG_TRY(ensure(d, d->wb, (size_t)(N * Kp) * 2));
  if (K > 0) {
    ENVG_CUDA(cudaMemcpy2DAsync(d->x.p, acols * 4, A, lda * 4, acols * 4, arows, cudaMemcpyHostToDevice, s));
    ENVG_CUDA(cudaMemcpy2DAsync(d->b32.p, bcols * 4, B, ldb * 4, bcols * 4, brows, cudaMemcpyHostToDevice, s));
    d->st.h2d_bytes += (double)(arows * acols + brows * bcols) * 4;
  }
  if (beta != 0.0f) {
    ENVG_CUDA(cudaMemcpy2DAsync(d->y.p, N * 4, C, ldc * 4, N * 4, M, cudaMemcpyHostToDevice, s));
    d->st.h2d_bytes += (double)(M * N) * 4;
  }
  const float* a32 = reinterpret_cast<const float*>(d->x.p);
  const float* b32 = reinterpret_cast<const float*>(d->b32.p);
  if (K == 0) {
    ENVG_CUDA(cudaMemsetAsync(d->xb.p, 0, (size_t)(M * Kp) * 2, s));
    ENVG_CUDA(cudaMemsetAsync(d->wb.p, 0, (size_t)(N * Kp) * 2, s));
  } else {
    if (!ta) ENVG_TRY(launch_cast_x3(d, a32, K, M, K, Ks, d->xb.p, X3_ACT));
    else ENVG_TRY(launch_transpose_x3(d, a32, M, (int)K, (int)M, d->xb.p, (int)Ks, X3_ACT));
    if (tb) ENVG_TRY(launch_cast_x3(d, b32, K, N, K, Ks, d->wb.p, X3_WEIGHT));
    else ENVG_TRY(launch_transpose_x3(d, b32, N, (int)K, (int)N, d->wb.p, (int)Ks, X3_WEIGHT));
  }
  CUtensorMap b256, b128;
  ENVG_TRY(tmap_2d(&b256, d->wb.p, Kp, N, 256));
  ENVG_TRY(tmap_2d(&b128, d->wb.p, Kp, N, 128));
  EpiArgs e{};
  e.Y = reinterpret_cast<float*>(d->y.p);
  e.ldy = N;
  e.mode = EPI_ALPHA_BETA;
  e.alpha = alpha;
  e.beta = beta;
  e.n_out = (int)N;
  e.m_valid = (int)M;
  e.vec_ok = (N % 4 == 0) ? 1 : 0;
  ENVG_TRY(gemm_device(d, d->xb.p, M, Kp, b256, b128, N, false, e, 2.0 * (double)M * N * K,
                       2.0 * (double)(M + N) * Kp + (beta != 0.0f ? 8.0 : 4.0) * (double)M * N));
  ENVG_CUDA(cudaMemcpy2DAsync(C, ldc * 4, d->y.p, N * 4, N * 4, M, cudaMemcpyDeviceToHost, s));
  d->st.d2h_bytes += (double)(M * N) * 4;
  d->st.calls++;
  d->st.flops += 2.0 * (double)M * (double)N * (double)K;
  return sync_and_check(d);
}

int envg_profile(int enable) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  if (enable) {
    ENVG_CUDA(cudaStreamSynchronize(stream_of(d)));
    resolve_pending();
    for (auto& k : g_prof) k = KAcc{};
  }
  g_prof_on = enable != 0;
  return ENVG_OK;
}

int envg_profile_read(envg_kernel_stat* out, int max, int* count) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  if (!out || !count || max < 0) return fail(ENVG_ERR_ARG, "envg_profile_read: bad arguments");
  ENVG_CUDA(cudaStreamSynchronize(stream_of(d)));
  resolve_pending();
  int n = 0;
  for (int k = 0; k < KID_COUNT && n < max; ++k) {
    if (!g_prof[k].launches) continue;
    envg_kernel_stat& o = out[n++];
    memset(&o, 0, sizeof(o));
    strncpy(o.name, kKernelNames[k], sizeof(o.name) - 1);
    o.launches = g_prof[k].launches;
    o.ms = g_prof[k].ms;
    o.flops = g_prof[k].flops;
    o.bytes = g_prof[k].bytes;
  }
  *count = n;
  return ENVG_OK;
}

int envg_selftest_wait_timeout(uint64_t cap_ns) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  Dev* d = cur();
  if (!d) return fail(ENVG_ERR_STATE, "envg_init has not been called");
  k_wait_selftest<<<1, 32, 0, stream_of(d)>>>(d->d_status, cap_ns);
  ENVG_CUDA(cudaGetLastError());
  d->st.kernel_launches++;
  return sync_and_check(d);
}

}  // extern "C"
