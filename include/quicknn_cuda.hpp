// quicknn_cuda.hpp -- C++ host-side mirror of Envision's QNN operator surface for the dense-linear
// path, on top of the C ABI in envgemm.h.
//
// The reference's model code calls these procedures (src/quicknn_kernels.pas); this header keeps
// their names, argument order and meaning so that a C++ host (or a test written like the
// reference's call sites) reads the same:
//   QNNLinear(dst, x, W, B, seqLen, inDIM, outDIM)          quicknn_kernels.pas:897-911
//   QNNLinearNoBias(dst, x, W, seqLen, inDIM, outDIM)       quicknn_kernels.pas:913-927
//   QNNLINEAR_BF16_OR_F32(dst, src, weight, weight_bf16, seq, srcDim, dstDim)
//                                                           quicknn_kernels.pas:2093-2103
//   QNNMatMulNT(C, A, B, M, K, N)                           quicknn_kernels.pas:847-861
//   QNNConv2d(dst, src, weights, bias, in_ch, out_ch, H, W, kH, kW, stride, padding, batch)
//                                                           quicknn_kernels.pas:990-1010
// plus the fused forms of the element-wise ops around a linear in the model, and the other
// compute-heavy neighbours of the path:
//   QNNLinearSiluMul   = linear into [gate | up] then QNNSiluMul (quicknncpu.pas:2404-2419)
//   QNNLinearGatedAdd  = linear then QNNGatedAdd (quicknncpu.pas:853-859)
//   QNNAdaLNLinear     = QNNAdaLN then a linear (quicknncpu.pas:3042-3060)
//   QNNGroupNorm(dst, src, gamma, beta, batch, channels, H, W, num_groups)
//                                                           quicknncpu.pas:2259-2313
//   QNNFlashAttention(dst, Q, K, V, heads, seq_q, seq_k, head_dim, scale)
//                                                           quicknncpu.pas:2763-2860
//   QNNResBlock::forward(dst, src, batch, H, W, num_groups) quicknn_vae.pas:164-187
// The weight argument is a device-resident QNNWeight in place of the reference's fp32/bf16
// TMemoryBlock.  Where the reference asserts (e.g. quicknn_kernels.pas:484-486), these functions
// throw std::runtime_error carrying the library's message; host pointers are used throughout,
// as in the reference (the call is synchronous).
#ifndef QUICKNN_CUDA_HPP
#define QUICKNN_CUDA_HPP

#include <cstdint>
#include <stdexcept>
#include <string>

#include "envgemm.h"

namespace quicknn_cuda {

inline void check(int rc, const char* what) {
  if (rc != ENVG_OK) throw std::runtime_error(std::string("ERROR ") + what + " : " + envg_last_error());
}

// A weight uploaded once into HBM (bf16).  Owns its envg_weight handle.
class QNNWeight {
 public:
  QNNWeight() = default;
  // W[N, K] row-major as raw bf16 bits (w_bf16) or fp32 (rounded to bf16 at upload).
  QNNWeight(const uint16_t* w_bf16, const float* w_f32, int64_t N, int64_t K, int layout = ENVG_LAYOUT_PLAIN)
      : N_(N), K_(K), layout_(layout) {
    check(envg_weight_upload(w_bf16, w_f32, N, K, layout, &h_), "QNNWeight upload");
  }
  // Convolution weight [out_ch, in_ch, kH, kW].
  static QNNWeight conv(const uint16_t* w_bf16, const float* w_f32, int out_ch, int in_ch, int kH, int kW) {
    QNNWeight w;
    check(envg_conv_weight_upload(w_bf16, w_f32, out_ch, in_ch, kH, kW, &w.h_), "QNNWeight conv upload");
    w.N_ = out_ch;
    w.K_ = (int64_t)in_ch * kH * kW;
    w.conv_ = true;
    w.out_ch_ = out_ch;
    w.in_ch_ = in_ch;
    w.kH_ = kH;
    w.kW_ = kW;
    return w;
  }
  // Tensor `name` of a .safetensors file (TSafeTensorFiles.getTensorDataMemBlockBF16,
  // safetensor.pas:650-683, then upload): 2-D [N, K] -> linear weight, 4-D -> conv weight.
  static QNNWeight from_safetensors(const char* path, const char* name, int layout = ENVG_LAYOUT_PLAIN) {
    envg_tensor_info info;
    check(envg_safetensors_tensor_info(path, name, &info), "QNNWeight safetensors");
    QNNWeight w;
    check(envg_weight_upload_safetensors(path, name, layout, 0, 0, &w.h_), "QNNWeight safetensors upload");
    w.N_ = info.shape[0];
    w.layout_ = layout;
    if (info.ndim == 4) {
      w.conv_ = true;
      w.out_ch_ = (int)info.shape[0];
      w.in_ch_ = (int)info.shape[1];
      w.kH_ = (int)info.shape[2];
      w.kW_ = (int)info.shape[3];
      w.K_ = info.shape[1] * info.shape[2] * info.shape[3];
    } else {
      w.K_ = info.shape[1];
    }
    return w;
  }
  QNNWeight(const QNNWeight&) = delete;
  QNNWeight& operator=(const QNNWeight&) = delete;
  QNNWeight(QNNWeight&& o) noexcept { *this = static_cast<QNNWeight&&>(o); }
  QNNWeight& operator=(QNNWeight&& o) noexcept {
    if (this != &o) {
      reset();
      h_ = o.h_;
      N_ = o.N_;
      K_ = o.K_;
      layout_ = o.layout_;
      conv_ = o.conv_;
      out_ch_ = o.out_ch_;
      in_ch_ = o.in_ch_;
      kH_ = o.kH_;
      kW_ = o.kW_;
      o.h_ = nullptr;
    }
    return *this;
  }
  ~QNNWeight() { reset(); }
  void reset() {
    if (h_) envg_weight_free(h_);
    h_ = nullptr;
  }
  bool assigned() const { return h_ != nullptr; }
  envg_weight handle() const { return h_; }
  int64_t N() const { return N_; }
  int64_t K() const { return K_; }
  int layout() const { return layout_; }
  bool is_conv() const { return conv_; }
  int out_ch() const { return out_ch_; }
  int in_ch() const { return in_ch_; }
  int kH() const { return kH_; }
  int kW() const { return kW_; }

 private:
  envg_weight h_ = nullptr;
  int64_t N_ = 0, K_ = 0;
  int layout_ = ENVG_LAYOUT_PLAIN;
  bool conv_ = false;
  int out_ch_ = 0, in_ch_ = 0, kH_ = 0, kW_ = 0;
};

inline void QNNLinear(float* dst, const float* x, const QNNWeight& W, const float* B, int seqLen, int inDIM,
                      int outDIM) {
  if (!W.assigned()) throw std::runtime_error("ERROR QNNLinear : weight not assigned!");
  check(envg_linear(dst, x, W.handle(), B, seqLen, inDIM, outDIM, B ? ENVG_EPI_BIAS : ENVG_EPI_NONE, nullptr,
                    ENVG_HOST_PTRS),
        "QNNLinear");
}

inline void QNNLinearNoBias(float* dst, const float* x, const QNNWeight& W, int seqLen, int inDIM, int outDIM) {
  QNNLinear(dst, x, W, nullptr, seqLen, inDIM, outDIM);
}

inline void QNNLINEAR_BF16_OR_F32(float* dst, const float* src, const QNNWeight* weight,
                                  const QNNWeight* weight_bf16, int seq, int srcDim, int dstDim) {
  const QNNWeight* w = (weight_bf16 && weight_bf16->assigned()) ? weight_bf16 : weight;
  if (!w || !w->assigned())
    throw std::runtime_error("ERROR QNNLINEAR_BF16_OR_F32 : no weight or weight_16 assigned!");
  QNNLinearNoBias(dst, src, *w, seq, srcDim, dstDim);
}

inline void QNNMatMulNT(float* C, const float* A, const QNNWeight& B, int M, int K, int N) {
  QNNLinearNoBias(C, A, B, M, K, N);
}

// dst[seqLen, mlpDIM] = silu(x.Wg^T) * (x.Wu^T) with W_gate_up = [gate | up] uploaded as GATE_UP.
inline void QNNLinearSiluMul(float* dst, const float* x, const QNNWeight& W_gate_up, int seqLen, int inDIM,
                             int mlpDIM) {
  if (W_gate_up.layout() != ENVG_LAYOUT_GATE_UP) throw std::runtime_error("ERROR QNNLinearSiluMul : not a gate/up weight");
  check(envg_linear(dst, x, W_gate_up.handle(), nullptr, seqLen, inDIM, 2LL * mlpDIM, ENVG_EPI_SILU_GATE, nullptr,
                    ENVG_HOST_PTRS),
        "QNNLinearSiluMul");
}

// h[seqLen, outDIM] += gate (.) (x.W^T + B)
inline void QNNLinearGatedAdd(float* h, const float* x, const QNNWeight& W, const float* gate, int seqLen, int inDIM,
                              int outDIM, const float* B = nullptr) {
  check(envg_linear(h, x, W.handle(), B, seqLen, inDIM, outDIM, ENVG_EPI_GATED_RESIDUAL, gate, ENVG_HOST_PTRS),
        "QNNLinearGatedAdd");
}

inline void QNNConv2d(float* dst, const float* src, const QNNWeight& weights, const float* bias, int in_ch,
                      int out_ch, int H, int W, int kH, int kW, int stride, int padding, int batch) {
  if (!weights.is_conv()) throw std::runtime_error("ERROR [Conv2D] : not a convolution weight");
  check(envg_conv2d(dst, src, weights.handle(), bias, in_ch, out_ch, H, W, kH, kW, stride, padding, batch,
                    bias ? ENVG_EPI_BIAS : ENVG_EPI_NONE, ENVG_HOST_PTRS),
        "[Conv2D]");
}

// QNNAdaLN(xn, x, shift, scale, seqLen, inDIM) followed by QNNLinear(dst, xn, W, B, ...)
// (quicknncpu.pas:3042-3060; quicknn_transformers.pas:1400-1456): the normalisation runs inside
// the activation cast.
inline void QNNAdaLNLinear(float* dst, const float* x, const float* shift, const float* scale, const QNNWeight& W,
                           const float* B, int seqLen, int inDIM, int outDIM) {
  check(envg_linear_adaln(dst, x, shift, scale, W.handle(), B, seqLen, inDIM, outDIM,
                          W.layout() == ENVG_LAYOUT_GATE_UP ? ENVG_EPI_SILU_GATE : (B ? ENVG_EPI_BIAS : ENVG_EPI_NONE),
                          nullptr, ENVG_HOST_PTRS),
        "QNNAdaLNLinear");
}

// QNNGroupNorm(dst, src, gamma, beta, batch, channels, H, W, num_groups) (quicknncpu.pas:2259-2313).
inline void QNNGroupNorm(float* dst, const float* src, const float* gamma, const float* beta, int batch,
                         int channels, int H, int W, int num_groups) {
  if (num_groups <= 0 || channels % num_groups)
    throw std::runtime_error("ERROR [GroupNorm] : channels not divisible by groups");
  check(envg_group_norm(dst, src, gamma, beta, batch, channels, H, W, num_groups, 0, ENVG_HOST_PTRS), "[GroupNorm]");
}

// QNNFlashAttention(dst, Q, K, V, heads, seq_q, seq_k, head_dim, scale) (quicknncpu.pas:2763-2860):
// Q/K/V/dst [seq, heads * head_dim], head h at column h * head_dim.  head_dim 128.
inline void QNNFlashAttention(float* dst, const float* Q, const float* K, const float* V, int heads, int seq_q,
                              int seq_k, int head_dim, float scale) {
  const int64_t hid = (int64_t)heads * head_dim;
  check(envg_attention(dst, Q, K, V, seq_q, seq_k, heads, heads, head_dim, hid, hid, hid, hid, scale, 0, nullptr,
                       ENVG_HOST_PTRS),
        "[FlashAttention]");
}

// One VAE ResBlock (TVAEResBlock.forward, quicknn_vae.pas:164-187) with its conv weights on the
// device; the vectors stay host pointers.
struct QNNResBlock {
  int in_ch = 0, out_ch = 0;
  const float *norm1_gamma = nullptr, *norm1_beta = nullptr, *conv1_bias = nullptr;
  const float *norm2_gamma = nullptr, *norm2_beta = nullptr, *conv2_bias = nullptr, *skip_bias = nullptr;
  const QNNWeight* conv1 = nullptr;
  const QNNWeight* conv2 = nullptr;
  const QNNWeight* skip = nullptr;  // nullptr when in_ch == out_ch

  void forward(float* dst, const float* src, int batch, int H, int W, int num_groups) const {
    envg_resblock rb{};
    rb.in_ch = in_ch;
    rb.out_ch = out_ch;
    rb.norm1_gamma = norm1_gamma;
    rb.norm1_beta = norm1_beta;
    rb.conv1 = conv1 ? conv1->handle() : nullptr;
    rb.conv1_bias = conv1_bias;
    rb.norm2_gamma = norm2_gamma;
    rb.norm2_beta = norm2_beta;
    rb.conv2 = conv2 ? conv2->handle() : nullptr;
    rb.conv2_bias = conv2_bias;
    rb.skip = skip ? skip->handle() : nullptr;
    rb.skip_bias = skip_bias;
    check(envg_vae_resblock(dst, src, &rb, batch, H, W, num_groups, ENVG_HOST_PTRS), "[VAE ResBlock]");
  }
};

}  // namespace quicknn_cuda

#endif  // QUICKNN_CUDA_HPP
