// C++ harness of the library boundary, driven by tests/test_abi.py and tests/test_gpu_abi.py.
// It links libenvgemm.so like any C/C++ host and calls it through include/quicknn_cuda.hpp with
// the reference's argument order (QNNLinear(dst, x, W, B, seqLen, inDIM, outDIM), ...).
//   abi_harness nogpu  -> expects envg_init to fail cleanly (no sm_100 device), exit 0
//   abi_harness gpu    -> runs QNNLinear / QNNLinearSiluMul / QNNConv2d on a B200 and checks them
//                         against double-precision loops on the same bf16-rounded operands
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

#include "quicknn_cuda.hpp"

using namespace quicknn_cuda;

static uint16_t bf16_rne(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static float bf16_to_f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// sum|d| / sum|ref| of y against ref
static double mean_rel(const std::vector<float>& y, const std::vector<double>& ref) {
  double num = 0, den = 0;
  for (size_t i = 0; i < y.size(); ++i) {
    num += std::fabs((double)y[i] - ref[i]);
    den += std::fabs(ref[i]);
  }
  return den > 0 ? num / den : num;
}

static int run_gpu() {
  check(envg_init(1, nullptr), "envg_init");
  std::mt19937 rng(1234);
  std::normal_distribution<float> nd(0.f, 1.f);
  const int M = 200, K = 320, N = 264;
  std::vector<float> x(M * K), b(N);
  std::vector<uint16_t> w(N * K);
  for (auto& v : x) v = nd(rng);
  for (auto& v : w) v = bf16_rne(0.02f * nd(rng));
  for (auto& v : b) v = 0.01f * nd(rng);
  QNNWeight W(w.data(), nullptr, N, K);
  std::vector<float> y(M * N, NAN);
  QNNLinear(y.data(), x.data(), W, b.data(), M, K, N);
  std::vector<double> ref(M * N);
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) {
      double s = b[n];
      for (int k = 0; k < K; ++k) s += (double)x[m * K + k] * bf16_to_f(w[n * K + k]);
      ref[m * N + n] = s;
    }
  double e1 = mean_rel(y, ref);
  // skinny path through the same entry
  std::vector<float> y1(3 * N, NAN);
  QNNLinearNoBias(y1.data(), x.data(), W, 3, K, N);
  std::vector<double> ref1(3 * N);
  for (int m = 0; m < 3; ++m)
    for (int n = 0; n < N; ++n) ref1[m * N + n] = ref[m * N + n] - b[n];
  double e2 = mean_rel(y1, ref1);
  // fused gate/up + SiLU-gate
  const int H = 136;
  std::vector<uint16_t> wg(2 * H * K);
  for (auto& v : wg) v = bf16_rne(0.02f * nd(rng));
  QNNWeight WG(wg.data(), nullptr, 2 * H, K, ENVG_LAYOUT_GATE_UP);
  std::vector<float> ys(M * H, NAN);
  QNNLinearSiluMul(ys.data(), x.data(), WG, M, K, H);
  std::vector<double> refs(M * H);
  for (int m = 0; m < M; ++m)
    for (int j = 0; j < H; ++j) {
      double g = 0, u = 0;
      for (int k = 0; k < K; ++k) {
        g += (double)x[m * K + k] * bf16_to_f(wg[j * K + k]);
        u += (double)x[m * K + k] * bf16_to_f(wg[(H + j) * K + k]);
      }
      refs[m * H + j] = g / (1.0 + std::exp(-g)) * u;
    }
  double e3 = mean_rel(ys, refs);
  // argument errors come back as exceptions (the reference asserts)
  bool threw = false;
  try {
    QNNLinear(y.data(), x.data(), W, nullptr, M, K + 8, N);
  } catch (const std::runtime_error&) {
    threw = true;
  }
  std::printf("linear %.3e skinny %.3e silu-gate %.3e threw %d\n", e1, e2, e3, (int)threw);
  W.reset();
  WG.reset();
  const bool ok = e1 < 2e-3 && e2 < 2e-3 && e3 < 4e-3 && threw;
  return ok ? 0 : 1;
}

int main(int argc, char** argv) {
  const char* mode = argc > 1 ? argv[1] : "nogpu";
  if (std::strcmp(mode, "gpu") == 0) {
    try {
      return run_gpu();
    } catch (const std::exception& e) {
      std::printf("exception: %s\n", e.what());
      return 2;
    }
  }
  // no GPU: init must fail with a status, not crash, and leave an error message
  int rc = envg_init(1, nullptr);
  std::printf("init rc %d: %s\n", rc, envg_last_error());
  if (rc == ENVG_OK) return 3;
  bool threw = false;
  try {
    QNNWeight W(nullptr, nullptr, 4, 4);
  } catch (const std::runtime_error& e) {
    threw = true;
    std::printf("upload without init: %s\n", e.what());
  }
  return threw ? 0 : 4;
}
