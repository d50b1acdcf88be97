"""ctypes front end of the CPU checkers -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import this module.
It wraps two shared libraries built by ``oracle/Makefile``:

* ``liboracle.so`` -- the C++ restatement of the reference CPU path (``envg_oracle.cpp``;
  each function there cites the Envision source line it restates);
* ``_ref/libsgemm2.so`` -- the reference's own ``src/sgemm2.cpp`` compiled unmodified
  (``cpp_sgemm``, sgemm2.cpp:530-547).  Optional: present only when it was built here.

Arrays are numpy; every call checks dtype and contiguity before handing pointers to C.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PATH_AVX2 = 0
PATH_SCALAR = 1
ROW_MAJOR, NO_TRANS, TRANS = 101, 111, 112

_lib = None
_ref = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i64 = ctypes.c_int64


def _p(a, ct=_f32p):
    return None if a is None else a.ctypes.data_as(ct)


def _chk(a, dtype):
    assert isinstance(a, np.ndarray) and a.dtype == dtype and a.flags.c_contiguous, (a.dtype, dtype)
    return a


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            raise RuntimeError("oracle/liboracle.so missing: run `make -C oracle`")
        L = ctypes.CDLL(path)
        L.envo_set_threads.argtypes = [ctypes.c_int]
        L.envo_set_threads.restype = ctypes.c_int
        L.envo_get_threads.restype = ctypes.c_int
        L.envo_bf16_to_f32.argtypes = [_i64, _u16p, _f32p]
        L.envo_f32_to_bf16_trunc.argtypes = [_i64, _f32p, _u16p]
        L.envo_sdot.argtypes = [ctypes.c_int, _i64, _f32p, _f32p]
        L.envo_sdot.restype = ctypes.c_float
        L.envo_qgemm.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _i64, _i64, _i64,
                                 ctypes.c_float, _f32p, _i64, _f32p, _i64, ctypes.c_float, _f32p, _i64]
        L.envo_qgemm.restype = ctypes.c_int
        L.envo_linear_f32.argtypes = [ctypes.c_int, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64]
        L.envo_linear_bf16.argtypes = [ctypes.c_int, _f32p, _f32p, _u16p, _f32p, _i64, _i64, _i64]
        L.envo_fast_exp.argtypes = [ctypes.c_float]
        L.envo_fast_exp.restype = ctypes.c_float
        L.envo_silu_mul.argtypes = [_f32p, _f32p, _i64]
        L.envo_silu.argtypes = [_f32p, _i64]
        L.envo_gated_add.argtypes = [_f32p, _f32p, _f32p, _i64, _i64]
        L.envo_conv2d.argtypes = [ctypes.c_int, _f32p, _f32p, _f32p, _f32p] + [ctypes.c_int] * 9
        L.envo_adaln.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64]
        L.envo_rms_norm.argtypes = [_f32p, _f32p, ctypes.c_void_p, _i64, _i64]
        L.envo_group_norm.argtypes = [_f32p, _f32p, _f32p, _f32p] + [ctypes.c_int] * 6
        L.envo_attention.argtypes = [ctypes.c_int, _f32p, _f32p, _f32p, _f32p] + [ctypes.c_int] * 5 + \
            [_i64] * 4 + [ctypes.c_float, ctypes.c_int, ctypes.POINTER(ctypes.c_int32)]
        L.envo_attention.restype = ctypes.c_int
        L.envo_conv2d.restype = ctypes.c_int
        _lib = L
    return _lib


def ref_lib():
    """The reference's own sgemm2.cpp, or None when it was not built."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libsgemm2.so")
        if not os.path.exists(path):
            return None
        L = ctypes.CDLL(path)
        ci = ctypes.c_int
        L.cpp_sgemm.argtypes = [ci, ci, ci, ci, ci, ctypes.c_float, _f32p, ci, _f32p, ci,
                                ctypes.c_float, _f32p, ci, ci, ci]
        L.cpp_sgemm.restype = None
        _ref = L
    return _ref


def set_threads(n):
    return lib().envo_set_threads(int(n))


def bf16_to_f32(w_bits):
    w_bits = _chk(np.ascontiguousarray(w_bits), np.uint16)
    out = np.empty(w_bits.shape, np.float32)
    lib().envo_bf16_to_f32(w_bits.size, _p(w_bits, _u16p), _p(out))
    return out


def f32_to_bf16_trunc(x):
    x = _chk(np.ascontiguousarray(x), np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().envo_f32_to_bf16_trunc(x.size, _p(x), _p(out, _u16p))
    return out


def f32_to_bf16_rne(x):
    """Round-to-nearest-even fp32 -> bf16 bits (the rounding the CUDA path applies to X)."""
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u >> 16) & 1) + 0x7FFF
    out = ((u + r) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def qgemm(transA, transB, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, path=PATH_AVX2):
    for a in (A, B, C):
        _chk(a, np.float32)
    rc = lib().envo_qgemm(path, ROW_MAJOR, transA, transB, M, N, K, alpha, _p(A), lda, _p(B), ldb,
                          beta, _p(C), ldc)
    assert rc == 0
    return C


def linear_bf16(x, w_bits, bias=None, path=PATH_AVX2):
    """QNNLinearNoBias_BF16 (+ QNNLinear bias): Y[M,N] = X[M,K] . widen(W[N,K])^T (+ b)."""
    x = _chk(np.ascontiguousarray(x), np.float32)
    w_bits = _chk(np.ascontiguousarray(w_bits), np.uint16)
    M, K = x.shape
    N = w_bits.shape[0]
    assert w_bits.shape == (N, K)
    if bias is not None:
        bias = _chk(np.ascontiguousarray(bias), np.float32)
        assert bias.shape == (N,)
    y = np.zeros((M, N), np.float32)
    lib().envo_linear_bf16(path, _p(y), _p(x), _p(w_bits, _u16p), _p(bias), M, K, N)
    return y


def linear_f32(x, w, bias=None, path=PATH_AVX2):
    x = _chk(np.ascontiguousarray(x), np.float32)
    w = _chk(np.ascontiguousarray(w), np.float32)
    M, K = x.shape
    N = w.shape[0]
    if bias is not None:
        bias = _chk(np.ascontiguousarray(bias), np.float32)
    y = np.zeros((M, N), np.float32)
    lib().envo_linear_f32(path, _p(y), _p(x), _p(w), _p(bias), M, K, N)
    return y


def fast_exp(x):
    return lib().envo_fast_exp(float(x))


def silu_mul(gate, up):
    """QNNSiluMul (scalar build): returns silu(gate) * up (inputs unchanged)."""
    g = np.array(gate, np.float32, copy=True, order="C")
    u = _chk(np.ascontiguousarray(up), np.float32)
    lib().envo_silu_mul(_p(g), _p(u), g.size)
    return g


def silu(x):
    g = np.array(x, np.float32, copy=True, order="C")
    lib().envo_silu(_p(g), g.size)
    return g


def gated_add(dst, gate, proj):
    """QNNGatedAdd: returns dst + gate (.) proj, row by row (inputs unchanged)."""
    d = np.array(dst, np.float32, copy=True, order="C")
    g = _chk(np.ascontiguousarray(gate), np.float32)
    p = _chk(np.ascontiguousarray(proj), np.float32)
    seq, hidden = d.shape
    lib().envo_gated_add(_p(d), _p(g), _p(p), seq, hidden)
    return d


def rms_norm(src, weight=None):
    """QNNRMSNormRows: per row x * weight / sqrt(mean(x^2) + 1e-6) (returns a new array)."""
    src = _chk(np.ascontiguousarray(src), np.float32)
    seq, hidden = src.shape
    out = np.empty_like(src)
    wp = None
    if weight is not None:
        weight = _chk(np.ascontiguousarray(weight), np.float32)
        wp = weight.ctypes.data
    lib().envo_rms_norm(_p(out), _p(src), wp, seq, hidden)
    return out


def adaln(src, shift, scale):
    """QNNAdaLN: per row (1 + scale) * (x - mean) / sqrt(var + 1e-6) + shift (returns a new array)."""
    src = _chk(np.ascontiguousarray(src), np.float32)
    shift = _chk(np.ascontiguousarray(shift), np.float32)
    scale = _chk(np.ascontiguousarray(scale), np.float32)
    seq, hidden = src.shape
    out = np.empty_like(src)
    lib().envo_adaln(_p(out), _p(src), _p(shift), _p(scale), seq, hidden)
    return out


def group_norm(src, gamma, beta, num_groups, act=False):
    """QNNGroupNorm (+ QNNSiluInplace when act): src fp32 [B, C, H, W] -> new array."""
    src = _chk(np.ascontiguousarray(src), np.float32)
    B, C, H, W = src.shape
    g = None if gamma is None else _chk(np.ascontiguousarray(gamma), np.float32)
    b = None if beta is None else _chk(np.ascontiguousarray(beta), np.float32)
    out = np.empty_like(src)
    lib().envo_group_norm(_p(out), _p(src), _p(g) if g is not None else None, _p(b) if b is not None else None,
                          B, C, H, W, num_groups, 1 if act else 0)
    return out


def vae_resblock(src, p, num_groups, path=PATH_AVX2):
    """TVAEResBlock.forward (quicknn_vae.pas:164-187) on fp32 weights.

    p: dict with norm1_gamma, norm1_beta, conv1_w [O, C, 3, 3], conv1_b, norm2_gamma, norm2_beta,
    conv2_w [O, O, 3, 3], conv2_b and, when in_ch != out_ch, skip_w [O, C, 1, 1], skip_b.
    dst := skip(src); work := SiLU(GN1(src)); c1 := conv1(work); work := SiLU(GN2(c1));
    c1 := conv2(work); dst += c1 (QNNAddInplace, quicknncpu.pas:704-709)."""
    src = _chk(np.ascontiguousarray(src), np.float32)
    if p.get("skip_w") is not None:
        dst = conv2d(src, p["skip_w"], p.get("skip_b"), 1, 0, path=path)
    else:
        dst = src.copy()
    work = group_norm(src, p["norm1_gamma"], p["norm1_beta"], num_groups, act=True)
    c1 = conv2d(work, p["conv1_w"], p["conv1_b"], 1, 1, path=path)
    work = group_norm(c1, p["norm2_gamma"], p["norm2_beta"], num_groups, act=True)
    c2 = conv2d(work, p["conv2_w"], p["conv2_b"], 1, 1, path=path)
    return (dst + c2).astype(np.float32)


def attention(q, k, v, heads, kv_heads, head_dim, scale=None, causal=False, key_mask=None, path=PATH_AVX2):
    """Per-head cblas_gemm + QNNSoftmaxRows + cblas_gemm (the reference's BLAS attention).

    q [seq_q, >= heads*head_dim], k/v [seq_k, >= kv_heads*head_dim] fp32 (row strides = their
    widths); returns [seq_q, heads*head_dim]."""
    q = _chk(np.ascontiguousarray(q), np.float32)
    k = _chk(np.ascontiguousarray(k), np.float32)
    v = _chk(np.ascontiguousarray(v), np.float32)
    seq_q, seq_k = q.shape[0], k.shape[0]
    if scale is None:
        scale = 1.0 / np.sqrt(head_dim)
    out = np.zeros((seq_q, heads * head_dim), np.float32)
    m = None
    if key_mask is not None:
        m = np.ascontiguousarray(key_mask, dtype=np.int32)
    rc = lib().envo_attention(path, _p(out), _p(q), _p(k), _p(v), seq_q, seq_k, heads, kv_heads, head_dim,
                              q.shape[1], k.shape[1], v.shape[1], out.shape[1], float(scale), 1 if causal else 0,
                              m.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)) if m is not None else None)
    assert rc == 0
    return out


def conv2d(src, w, bias, stride, padding, path=PATH_AVX2):
    """QNNConv2d: src fp32 [B,C,H,W], w fp32 [O,C,kH,kW] -> fp32 [B,O,outH,outW] (NCHW)."""
    src = _chk(np.ascontiguousarray(src), np.float32)
    w = _chk(np.ascontiguousarray(w), np.float32)
    B, C, H, W = src.shape
    O, C2, kH, kW = w.shape
    assert C2 == C
    if bias is not None:
        bias = _chk(np.ascontiguousarray(bias), np.float32)
    outH = (H + 2 * padding - kH) // stride + 1
    outW = (W + 2 * padding - kW) // stride + 1
    y = np.zeros((B, O, outH, outW), np.float32)
    rc = lib().envo_conv2d(path, _p(y), _p(src), _p(w), _p(bias), C, O, H, W, kH, kW, stride, padding, B)
    assert rc == 0
    return y


def sgemm2_nt(A, B, M, N, K, threads=0):
    """The reference's cpp_sgemm(NoTrans, Trans) on pre-zeroed C (it ignores beta, sgemm2.cpp:312-324)."""
    L = ref_lib()
    if L is None:
        raise RuntimeError("oracle/_ref/libsgemm2.so not built")
    A = _chk(np.ascontiguousarray(A), np.float32)
    B = _chk(np.ascontiguousarray(B), np.float32)
    C = np.zeros((M, N), np.float32)
    L.cpp_sgemm(NO_TRANS, TRANS, M, N, K, 1.0, _p(A), K, _p(B), K, 0.0, _p(C), N, 0, 0)
    return C


def sgemm2_nn(A, B, M, N, K):
    L = ref_lib()
    if L is None:
        raise RuntimeError("oracle/_ref/libsgemm2.so not built")
    A = _chk(np.ascontiguousarray(A), np.float32)
    B = _chk(np.ascontiguousarray(B), np.float32)
    C = np.zeros((M, N), np.float32)
    L.cpp_sgemm(NO_TRANS, NO_TRANS, M, N, K, 1.0, _p(A), K, _p(B), N, 0.0, _p(C), N, 0, 0)
    return C


def parity_stats(y, ref):
    """(max|d| / max|ref|, sum|d| / sum|ref|): the acceptance metrics of the hot path."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    d = np.abs(y - ref)
    mref = np.abs(ref).max()
    sref = np.abs(ref).sum()
    return (float(d.max() / mref) if mref > 0 else float(d.max()),
            float(d.sum() / sref) if sref > 0 else float(d.sum()))
