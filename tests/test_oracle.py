"""CPU: the restated reference path (oracle/envg_oracle.cpp) against fp64 and against the
reference's own compiled sgemm2.cpp (oracle/_ref), including the reference's edge behaviour."""
import math

import numpy as np
import pytest

from oracle import oracle as O


def f64_linear(x, w, b=None):
    y = x.astype(np.float64) @ w.astype(np.float64).T
    return y if b is None else y + b


@pytest.mark.parametrize("M", [1, 3, 8, 17, 63, 64, 65, 129])
@pytest.mark.parametrize("K", [8, 128, 2560])
@pytest.mark.parametrize("N", [1, 4, 7, 9, 257])
def test_gemm_nt_avx2_vs_fp64(M, K, N):
    """8x8 tiling, 4-column sDot_x4 groups and the qdot column tail against fp64."""
    rng = np.random.default_rng(M * 1000 + K + N)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.standard_normal((N, K), dtype=np.float32)
    y = O.linear_f32(x, w, path=O.PATH_AVX2)
    mx, mean = O.parity_stats(y, f64_linear(x, w))
    assert mx < 1e-5 and mean < 1e-5


@pytest.mark.parametrize("M,K,N", [(17, 127, 9), (64, 131, 257), (3, 8, 7), (65, 2561, 4)])
def test_gemm_nt_scalar_build_vs_fp64(M, K, N):
    rng = np.random.default_rng(K)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.standard_normal((N, K), dtype=np.float32)
    mx, mean = O.parity_stats(O.linear_f32(x, w, path=O.PATH_SCALAR), f64_linear(x, w))
    assert mx < 1e-4 and mean < 1e-5


def test_avx2_k_tail_quirk_is_restated():
    """ops_avx2.inc:1442-1460: for K % 8 != 0 the 4-column kernel reloads its accumulators from B
    and returns sum(A_tail*B_tail + B_tail); qdot columns (N % 4 tail) stay correct."""
    rng = np.random.default_rng(5)
    M, K, N = 2, 11, 5
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.standard_normal((N, K), dtype=np.float32)
    y = O.linear_f32(x, w, path=O.PATH_AVX2)
    tail = slice(8, 11)
    expect4 = (x[:, None, tail] * w[None, :4, tail] + w[None, :4, tail]).sum(-1)
    np.testing.assert_allclose(y[:, :4], expect4, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(y[:, 4], f64_linear(x, w)[:, 4], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("ta,tb", [(111, 111), (112, 111), (111, 112)])
def test_qgemm_all_transposes_and_beta(ta, tb):
    rng = np.random.default_rng(ta + tb)
    M, N, K = 19, 23, 37
    A = rng.standard_normal((K, M) if ta == 112 else (M, K), dtype=np.float32)
    B = rng.standard_normal((N, K) if tb == 112 else (K, N), dtype=np.float32)
    C = rng.standard_normal((M, N), dtype=np.float32)
    Am = A.T if ta == 112 else A
    Bm = B.T if tb == 112 else B
    ref = 0.5 * Am.astype(np.float64) @ Bm.astype(np.float64) + 2.0 * C
    out = O.qgemm(ta, tb, M, N, K, 0.5, A, A.shape[1], B, B.shape[1], 2.0, C.copy(), N, path=O.PATH_SCALAR)
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-4)


def test_restated_gemm_equals_reference_sgemm2():
    """O1 (restated Pascal qgemm) against the reference's own C++ sgemm2 (K % 128 == 0, where
    sgemm2 is complete): equal within fp32 round-off."""
    if O.ref_lib() is None:
        pytest.skip("oracle/_ref/libsgemm2.so not built (reference tree absent)")
    rng = np.random.default_rng(3)
    for M, N, K in [(64, 96, 256), (17, 9, 128), (128, 300, 2560)]:
        x = rng.standard_normal((M, K), dtype=np.float32)
        w = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
        y_ref = O.sgemm2_nt(x, w, M, N, K)
        y_o1 = O.linear_f32(x, w)
        mx, mean = O.parity_stats(y_o1, y_ref)
        assert mx < 2e-6 and mean < 1e-6, (M, N, K, mx, mean)
        y_nn = O.sgemm2_nn(x, np.ascontiguousarray(w.T), M, N, K)
        out = np.zeros((M, N), np.float32)
        O.qgemm(111, 111, M, N, K, 1.0, x, K, np.ascontiguousarray(w.T), N, 0.0, out, N)
        assert O.parity_stats(out, y_nn)[0] < 2e-6


def test_bf16_conversions():
    x = np.array([1.0, -2.5, 1.00390625, 1.01171875, 3.4e38, 1e-40, 0.0, -0.0], np.float32)
    assert np.array_equal(O.bf16_to_f32(O.f32_to_bf16_trunc(x))[:4], np.array([1.0, -2.5, 1.0, 1.0078125], np.float32))
    rne = O.bf16_to_f32(O.f32_to_bf16_rne(x))
    assert rne[2] == 1.0 and rne[3] == 1.015625  # ties to even, round up
    w = np.arange(0, 65536, 7, dtype=np.uint16)
    f = O.bf16_to_f32(w)
    assert np.array_equal(f.view(np.uint32) >> 16, w.astype(np.uint32))


def test_fast_exp_and_silu_mul():
    for v in [-87.0, -10.0, -1.0, -0.1, 0.0, 0.3, 1.0, 5.0, 20.0, 88.0]:
        assert abs(O.fast_exp(v) - math.exp(v)) <= 2e-6 * math.exp(v)
    assert O.fast_exp(-90.0) == 0.0 and O.fast_exp(90.0) == pytest.approx(1e38)
    rng = np.random.default_rng(1)
    g = rng.standard_normal(1000, dtype=np.float32) * 3
    u = rng.standard_normal(1000, dtype=np.float32)
    ref = g.astype(np.float64) / (1 + np.exp(-g.astype(np.float64))) * u
    np.testing.assert_allclose(O.silu_mul(g, u), ref, rtol=1e-5, atol=1e-6)


def test_gated_add():
    rng = np.random.default_rng(2)
    d = rng.standard_normal((5, 7), dtype=np.float32)
    gate = rng.standard_normal(7, dtype=np.float32)
    p = rng.standard_normal((5, 7), dtype=np.float32)
    np.testing.assert_array_equal(O.gated_add(d, gate, p), d + (gate * p))


def conv_f64(src, w, b, stride, pad):
    B, C, H, W = src.shape
    Oc, _, kH, kW = w.shape
    oH = (H + 2 * pad - kH) // stride + 1
    oW = (W + 2 * pad - kW) // stride + 1
    xp = np.zeros((B, C, H + 2 * pad, W + 2 * pad))
    xp[:, :, pad:pad + H, pad:pad + W] = src
    out = np.zeros((B, Oc, oH, oW))
    for kh in range(kH):
        for kw in range(kW):
            patch = xp[:, :, kh:kh + stride * oH:stride, kw:kw + stride * oW:stride]
            out += np.einsum("bchw,oc->bohw", patch, w[:, :, kh, kw])
    return out + (0 if b is None else b[None, :, None, None])


@pytest.mark.parametrize("B,C,H,W,Oc,k,stride,pad", [(1, 8, 9, 11, 5, 3, 1, 1), (2, 3, 6, 6, 4, 1, 1, 0),
                                                    (1, 4, 9, 7, 6, 3, 2, 1), (1, 5, 8, 8, 3, 3, 2, 0)])
def test_conv2d_vs_fp64(B, C, H, W, Oc, k, stride, pad):
    rng = np.random.default_rng(C * H)
    src = rng.standard_normal((B, C, H, W), dtype=np.float32)
    w = rng.standard_normal((Oc, C, k, k), dtype=np.float32)
    b = rng.standard_normal(Oc, dtype=np.float32)
    y = O.conv2d(src, w, b, stride, pad)
    np.testing.assert_allclose(y, conv_f64(src, w, b, stride, pad), rtol=1e-4, atol=1e-4)


def test_conv2d_stride1_valid_padding_quirk():
    """quicknncpu.pas:2091-2093: the stride-1 im2col copies outW - |kernel_col - pad| values, which
    drops the last kernel_col columns when outW < W (padding 0, kW > 1).  Restated as is."""
    rng = np.random.default_rng(0)
    src = rng.standard_normal((1, 2, 6, 6), dtype=np.float32)
    w = rng.standard_normal((3, 2, 3, 3), dtype=np.float32)
    y = O.conv2d(src, w, None, 1, 0)
    exact = conv_f64(src, w, None, 1, 0)
    assert not np.allclose(y, exact, atol=1e-3)
    # same padding is exact
    y1 = O.conv2d(src, w, None, 1, 1)
    np.testing.assert_allclose(y1, conv_f64(src, w, None, 1, 1), rtol=1e-4, atol=1e-4)


def test_rms_norm_vs_fp64():
    rng = np.random.default_rng(10)
    x = (0.5 + 2 * rng.standard_normal((5, 2560))).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(2560)).astype(np.float32)
    xd = x.astype(np.float64)
    inv = 1 / np.sqrt((xd * xd).mean(1, keepdims=True) + 1e-6)
    np.testing.assert_allclose(O.rms_norm(x, w), xd * w * inv, rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(O.rms_norm(x), xd * inv, rtol=2e-5, atol=2e-5)


def test_adaln_vs_fp64():
    rng = np.random.default_rng(9)
    x = (3 + 2 * rng.standard_normal((7, 3072))).astype(np.float32)
    shift = (0.1 * rng.standard_normal(3072)).astype(np.float32)
    scale = (0.1 * rng.standard_normal(3072)).astype(np.float32)
    y = O.adaln(x, shift, scale)
    xd = x.astype(np.float64)
    mu = xd.mean(1, keepdims=True)
    var = ((xd - mu) ** 2).mean(1, keepdims=True)
    ref = (1 + scale) * (xd - mu) / np.sqrt(var + 1e-6) + shift
    np.testing.assert_allclose(y, ref, rtol=2e-4, atol=2e-4)


def _gn_fp64(x, gamma, beta, G, eps=1e-6):
    B, C, H, W = x.shape
    xd = x.astype(np.float64).reshape(B, G, -1)
    mu = xd.mean(2, keepdims=True)
    var = ((xd - mu) ** 2).mean(2, keepdims=True)
    y = ((xd - mu) / np.sqrt(var + eps)).reshape(B, C, H, W)
    return y * gamma.reshape(1, C, 1, 1) + beta.reshape(1, C, 1, 1)


def test_group_norm_vs_fp64():
    rng = np.random.default_rng(21)
    x = (1.5 + 2 * rng.standard_normal((2, 64, 12, 10))).astype(np.float32)
    gamma = (1 + 0.1 * rng.standard_normal(64)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(64)).astype(np.float32)
    y = O.group_norm(x, gamma, beta, 32)
    np.testing.assert_allclose(y, _gn_fp64(x, gamma, beta, 32), rtol=2e-4, atol=2e-4)
    ys = O.group_norm(x, gamma, beta, 8, act=True)
    r = _gn_fp64(x, gamma, beta, 8)
    np.testing.assert_allclose(ys, r / (1 + np.exp(-r)), rtol=2e-3, atol=2e-3)   # fast_exp SiLU


def test_vae_resblock_composition():
    """The ResBlock oracle is skip + conv2(SiLU(GN2(conv1(SiLU(GN1(x)))))), checked against fp64."""
    rng = np.random.default_rng(22)
    B, Ci, Co, H, W, G = 1, 32, 64, 8, 8, 8
    x = rng.standard_normal((B, Ci, H, W)).astype(np.float32)
    p = {"norm1_gamma": (1 + 0.1 * rng.standard_normal(Ci)).astype(np.float32),
         "norm1_beta": (0.1 * rng.standard_normal(Ci)).astype(np.float32),
         "conv1_w": (0.05 * rng.standard_normal((Co, Ci, 3, 3))).astype(np.float32),
         "conv1_b": (0.01 * rng.standard_normal(Co)).astype(np.float32),
         "norm2_gamma": (1 + 0.1 * rng.standard_normal(Co)).astype(np.float32),
         "norm2_beta": (0.1 * rng.standard_normal(Co)).astype(np.float32),
         "conv2_w": (0.05 * rng.standard_normal((Co, Co, 3, 3))).astype(np.float32),
         "conv2_b": (0.01 * rng.standard_normal(Co)).astype(np.float32),
         "skip_w": (0.1 * rng.standard_normal((Co, Ci, 1, 1))).astype(np.float32),
         "skip_b": (0.01 * rng.standard_normal(Co)).astype(np.float32)}
    y = O.vae_resblock(x, p, G, path=O.PATH_SCALAR)

    def conv(a, w, b, pad):
        a = a.astype(np.float64)
        O_, C, kh, kw = w.shape
        ap = np.pad(a, ((0, 0), (0, 0), (pad, pad), (pad, pad)))
        out = np.zeros((a.shape[0], O_, H, W))
        for i in range(kh):
            for j in range(kw):
                out += np.einsum("oc,bchw->bohw", w[:, :, i, j], ap[:, :, i:i + H, j:j + W])
        return out + b.reshape(1, -1, 1, 1)

    def silu(v):
        return v / (1 + np.exp(-v))

    h = conv(silu(_gn_fp64(x, p["norm1_gamma"], p["norm1_beta"], G)), p["conv1_w"], p["conv1_b"], 1)
    h = conv(silu(_gn_fp64(h, p["norm2_gamma"], p["norm2_beta"], G)), p["conv2_w"], p["conv2_b"], 1)
    ref = conv(x, p["skip_w"], p["skip_b"], 0) + h
    np.testing.assert_allclose(y, ref, rtol=5e-3, atol=5e-3)


def _attn_fp64(q, k, v, H, KVH, D, causal=False, mask=None):
    Sq, Sk = q.shape[0], k.shape[0]
    out = np.zeros((Sq, H * D))
    for h in range(H):
        g = h // (H // KVH)
        s = q[:, h * D:(h + 1) * D].astype(np.float64) @ k[:, g * D:(g + 1) * D].astype(np.float64).T / np.sqrt(D)
        if causal:
            s = np.where(np.arange(Sk)[None, :] > np.arange(Sq)[:, None] + (Sk - Sq), -np.inf, s)
        if mask is not None:
            s = np.where(np.asarray(mask)[None, :] == 0, -np.inf, s)
        s = np.exp(s - s.max(1, keepdims=True))
        s /= s.sum(1, keepdims=True)
        out[:, h * D:(h + 1) * D] = s @ v[:, g * D:(g + 1) * D].astype(np.float64)
    return out


@pytest.mark.parametrize("Sq,Sk,H,KVH,causal", [(37, 37, 2, 2, False), (64, 80, 4, 2, False), (50, 50, 4, 1, True),
                                               (20, 45, 2, 2, True)])
def test_attention_vs_fp64(Sq, Sk, H, KVH, causal):
    rng = np.random.default_rng(Sq + Sk + H)
    D = 32
    q = rng.standard_normal((Sq, H * D)).astype(np.float32)
    k = rng.standard_normal((Sk, KVH * D)).astype(np.float32)
    v = rng.standard_normal((Sk, KVH * D)).astype(np.float32)
    mask = (rng.random(Sk) > 0.2).astype(np.int32)
    mask[0] = 1
    for m in (None, mask):
        y = O.attention(q, k, v, H, KVH, D, causal=causal, key_mask=m, path=O.PATH_SCALAR)
        np.testing.assert_allclose(y, _attn_fp64(q, k, v, H, KVH, D, causal, m), rtol=1e-4, atol=1e-4)
