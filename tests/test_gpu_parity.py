"""GPU parity: libenvgemm (through its C ABI) against the CPU restatement of the reference.

Every case runs the same seeded inputs through the CUDA path and through the oracle
(oracle/envg_oracle.cpp, which restates src/quicknncpu.pas qgemm/gemm_nt/gemm_nn and the
epilogue ops) and applies the acceptance bounds of tests/common.py.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.common import TOL_MAX_PRODUCT, TOL_MEAN_PRODUCT, TOL_X3_MAX, TOL_X3_MEAN, assert_parity, inputs

pytestmark = pytest.mark.gpu

# (M, K, N): model shapes scaled to oracle-friendly sizes, tile edges and ragged tails.
LINEAR_SHAPES = [
    (1024, 3072, 9216),   # FLUX2-Klein QKV
    (256, 512, 768),
    (200, 136, 300),      # ragged M and N, K not a multiple of 64
    (129, 64, 257),       # one row / one column past a tile
    (384, 1024, 512),
    (65, 256, 128),       # smallest M on the large-M path
]
SKINNY_SHAPES = [
    (1, 3072, 18432),     # adaLN modulation (config 2, M = 1)
    (1, 2560, 1024),      # Qwen3 k/v at M = 1
    (16, 2560, 4096),     # Qwen3 q at M = 16
    (17, 512, 200),
    (33, 256, 136),
    (64, 1024, 512),
    (48, 4096, 256),
]


@pytest.mark.parametrize("M,K,N", LINEAR_SHAPES + SKINNY_SHAPES)
@pytest.mark.parametrize("with_bias", [True, False])
def test_linear_vs_oracle(gpu, M, K, N, with_bias):
    x, w, b = inputs(M, K, N, seed=M * 7 + K + N, bias=with_bias)
    W = gpu.Weight(w)
    y = np.full((M, N), np.nan, np.float32)
    gpu.linear(y, x, W, bias=b)
    ref = O.linear_bf16(x, w, b, path=O.PATH_AVX2)
    assert_parity(y, ref, what=f"linear {M}x{K}x{N} bias={with_bias}")


# BASELINE config 3 (Qwen3-4B layer) at M = 512, whole outputs: q, o, the fused gate+up
# tensor as one plain linear, and down (quicknn_qwen3.pas:712-714,772,782-789).
CONFIG3_M512 = [(512, 2560, 4096), (512, 4096, 2560), (512, 2560, 2 * 9728), (512, 9728, 2560)]


@pytest.mark.parametrize("M,K,N", CONFIG3_M512)
def test_config3_m512_vs_oracle(gpu, M, K, N):
    x, w, _ = inputs(M, K, N, seed=M + K + 3 * N, bias=False)
    W = gpu.Weight(w)
    y = np.full((M, N), np.nan, np.float32)
    gpu.linear(y, x, W)
    assert_parity(y, O.linear_bf16(x, w, path=O.PATH_AVX2), what=f"config 3 {M}x{K}x{N}")
    W.free()


@pytest.mark.parametrize("M,K,N", [(70, 131, 96), (5, 45, 33), (130, 1001, 260)])
def test_linear_k_not_multiple_of_8(gpu, M, K, N):
    """K % 8 != 0: the AVX2 build of the reference discards its main-loop sum here
    (ops_avx2.inc:1442-1460), so parity is against the scalar build of the same GEMM."""
    x, w, b = inputs(M, K, N, seed=3 + K)
    W = gpu.Weight(w)
    y = np.zeros((M, N), np.float32)
    gpu.linear(y, x, W, bias=b)
    ref = O.linear_bf16(x, w, b, path=O.PATH_SCALAR)
    assert_parity(y, ref, what=f"K%8 {M}x{K}x{N}")


F32_WEIGHT_CASES = [
    # (M, K, N, gate_up): every GEMM path (k2_set for M <= 64 (M <= 8 included), CTA-pair above)
    (96, 256, 192, False),
    (1, 2560, 1024, False),     # Qwen3 k at M = 1 (fp32 weights, quicknn_qwen3.pas:712-714)
    (16, 1000, 300, False),     # ragged K (padded segments)
    (300, 512, 640, False),
    (512, 2560, 1024, False),   # Qwen3 k at M = 512
    (40, 512, 2 * 200, True),   # gate/up pair with the SiLU-gate epilogue
    (260, 384, 2 * 136, True),
]


@pytest.mark.parametrize("M,K,N,gate_up", F32_WEIGHT_CASES)
def test_linear_f32_weight_vs_oracle(gpu, M, K, N, gate_up):
    """An fp32 weight that is not made of bf16 numbers (QNNLinearNoBias on fp32 W,
    quicknncpu.pas:1822-1828): the oracle multiplies the same unrounded W and X the reference
    does.  The upload keeps W as bf16x3 hi/lo parts, so the result holds the acceptance bounds and
    the much tighter bf16x3 bounds."""
    rng = np.random.default_rng(11 + M + K + N)
    x = rng.standard_normal((M, K), dtype=np.float32)
    wf = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    b = (0.01 * rng.standard_normal(N)).astype(np.float32)
    W = gpu.Weight(wf, layout=gpu.LAYOUT_GATE_UP if gate_up else gpu.LAYOUT_PLAIN)
    if gate_up:
        y = np.full((M, N // 2), np.nan, np.float32)
        gpu.linear(y, x, W, bias=b, epilogue=gpu.EPI_SILU_GATE)
        g = O.linear_f32(x, wf, b)
        ref = O.silu_mul(np.ascontiguousarray(g[:, :N // 2]), np.ascontiguousarray(g[:, N // 2:]))
    else:
        y = np.full((M, N), np.nan, np.float32)
        gpu.linear(y, x, W, bias=b)
        ref = O.linear_f32(x, wf, b, path=O.PATH_AVX2 if K % 8 == 0 else O.PATH_SCALAR)
    what = f"f32 weight {M}x{K}x{N} gate_up={gate_up}"
    assert_parity(y, ref, what=what)
    assert_parity(y, ref, TOL_X3_MAX, TOL_X3_MEAN, what=what + " (bf16x3 bounds)")
    W.free()


def test_linear_f32_weight_upload_forms(gpu):
    """fp32 weights made of bf16 numbers (the reference's widened bf16 checkpoints,
    safetensor.pas:584-647) are stored as plain bf16 and give exactly the bf16 upload's bits;
    LAYOUT_ROUND_BF16 rounds any fp32 weight to bf16 (RNE), again bit for bit the bf16 upload of
    the rounded bits."""
    M, K, N = 96, 256, 192
    rng = np.random.default_rng(12)
    x = rng.standard_normal((M, K), dtype=np.float32)
    wf = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    wb = O.f32_to_bf16_rne(wf)
    ys = {}
    for name, w, layout in (("bits", wb, gpu.LAYOUT_PLAIN), ("widened", O.bf16_to_f32(wb), gpu.LAYOUT_PLAIN),
                            ("rounded", wf, gpu.LAYOUT_PLAIN | gpu.LAYOUT_ROUND_BF16)):
        W = gpu.Weight(w, layout=layout)
        ys[name] = np.zeros((M, N), np.float32)
        gpu.linear(ys[name], x, W)
        W.free()
    np.testing.assert_array_equal(ys["widened"], ys["bits"])
    np.testing.assert_array_equal(ys["rounded"], ys["bits"])
    assert_parity(ys["bits"], O.linear_bf16(x, wb))


def test_f32_weight_in_batch_and_noalloc(gpu):
    """A bf16x3 weight inside envg_linear_batch (between linears that share and chain inputs) and
    through envg_linear_noalloc gives the bits of its own envg_linear call."""
    import torch

    rng = np.random.default_rng(13)
    K, N = 512, 384
    wf = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    wb = O.f32_to_bf16_rne((0.02 * rng.standard_normal((K, N))).astype(np.float32))
    Wf, Wb = gpu.Weight(wf), gpu.Weight(wb)
    for M in (4, 16, 300):
        x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()
        y1, y2, y3 = (torch.empty(M, N, device="cuda"), torch.empty(M, K, device="cuda"),
                      torch.empty(M, N, device="cuda"))
        gpu.linear_batch([dict(dst=y1, x=x, W=Wf), dict(dst=y2, x=y1, W=Wb), dict(dst=y3, x=y2, W=Wf)])
        torch.cuda.synchronize()
        got = [t.cpu().numpy() for t in (y1, y2, y3)]
        r1, r2, r3 = torch.empty_like(y1), torch.empty_like(y2), torch.empty_like(y3)
        gpu.linear(r1, x, Wf)
        gpu.linear(r2, r1, Wb)
        gpu.linear(r3, r2, Wf)
        torch.cuda.synchronize()
        for g, r in zip(got, (r1, r2, r3)):
            np.testing.assert_array_equal(g, r.cpu().numpy())
        assert_parity(got[0], O.linear_f32(x.cpu().numpy(), wf), TOL_X3_MAX, TOL_X3_MEAN, what=f"batch x3 M={M}")
        if M <= 64:
            yn = torch.empty(M, N, device="cuda")
            gpu.linear_noalloc(yn, x, Wf)
            torch.cuda.synchronize()
            assert_parity(yn.cpu().numpy(), O.linear_f32(x.cpu().numpy(), wf), TOL_X3_MAX, TOL_X3_MEAN,
                          what=f"noalloc x3 M={M}")
    Wf.free()
    Wb.free()


@pytest.mark.parametrize("M,K,H", [(256, 512, 384), (4608 // 8, 3072, 1152), (1, 3072, 640), (16, 512, 200), (130, 256, 130)])
def test_silu_gate_vs_oracle(gpu, M, K, H):
    """Fused gate/up linear + QNNSiluMul: W = [gate (H rows) | up (H rows)], Y [M, H]."""
    x, w, _ = inputs(M, K, 2 * H, seed=H + M)
    W = gpu.Weight(w, layout=gpu.LAYOUT_GATE_UP)
    y = np.zeros((M, H), np.float32)
    gpu.linear(y, x, W)
    gu = O.linear_bf16(x, w)
    ref = O.silu_mul(np.ascontiguousarray(gu[:, :H]), np.ascontiguousarray(gu[:, H:]))
    # the two GEMM halves through the plain path, at the GEMM bounds
    Wp = gpu.Weight(w)
    yg = np.zeros((M, 2 * H), np.float32)
    gpu.linear(yg, x, Wp)
    assert_parity(yg, gu, what=f"silu-gate halves {M}x{K}x{2 * H}")
    # the fused epilogue applies exactly silu(g) * u to those GEMM values
    np.testing.assert_allclose(y, O.silu_mul(np.ascontiguousarray(yg[:, :H]), np.ascontiguousarray(yg[:, H:])),
                               rtol=2e-5, atol=2e-6)
    assert_parity(y, ref, TOL_MAX_PRODUCT, TOL_MEAN_PRODUCT, what=f"silu-gate {M}x{K}x{H}")


@pytest.mark.parametrize("M,K,N", [(512, 1024, 768), (8, 3072, 3072), (200, 256, 100), (150, 128, 101)])
def test_gated_residual_vs_oracle(gpu, M, K, N):
    x, w, b = inputs(M, K, N, seed=N + 5)
    rng = np.random.default_rng(N)
    h0 = rng.standard_normal((M, N), dtype=np.float32)
    gate = rng.standard_normal(N).astype(np.float32)
    W = gpu.Weight(w)
    h = h0.copy()
    gpu.linear(h, x, W, bias=b, epilogue=gpu.EPI_GATED_RESIDUAL, gate=gate)
    proj = O.linear_bf16(x, w, b)
    ref = O.gated_add(h0, gate, proj)
    # compare the update (h - h0) so the residual does not hide GEMM error
    assert_parity(h - h0, ref - h0, what=f"gated residual {M}x{K}x{N}")


CONV_CASES = [
    # (B, C, H, W, O, k, stride, pad)
    (1, 64, 32, 32, 128, 3, 1, 1),
    (1, 128, 16, 48, 64, 3, 1, 1),
    (2, 16, 20, 24, 32, 3, 1, 1),     # channels padded to 64, odd width
    (1, 64, 8, 300, 64, 3, 1, 1),     # width above one 256-pixel tile
    (1, 96, 16, 16, 200, 1, 1, 0),    # 1x1 (conv_shortcut shape)
    (1, 32, 17, 19, 48, 3, 2, 1),     # strided: explicit im2col path
    (1, 64, 12, 96, 128, 3, 1, 1),    # TMA-store epilogue with a skipped overhang chunk
    (2, 64, 6, 64, 64, 3, 1, 1),      # two images, 4 rows per pixel tile
    (1, 64, 3, 256, 160, 3, 1, 1),    # one row per pixel tile, out_ch past one 128 block
]


@pytest.mark.parametrize("B,C,H,Wd,O_,k,stride,pad", CONV_CASES)
@pytest.mark.parametrize("silu", [False, True])
def test_conv2d_vs_oracle(gpu, B, C, H, Wd, O_, k, stride, pad, silu):
    rng = np.random.default_rng(B * 1000 + C + H + O_)
    src = rng.standard_normal((B, C, H, Wd), dtype=np.float32)
    wb = O.f32_to_bf16_rne((0.02 * rng.standard_normal((O_, C, k, k))).astype(np.float32))
    bias = (0.01 * rng.standard_normal(O_)).astype(np.float32)
    W = gpu.Weight(wb.reshape(O_, -1), conv=(O_, C, k, k))
    outH = (H + 2 * pad - k) // stride + 1
    outW = (Wd + 2 * pad - k) // stride + 1
    y = np.full((B, O_, outH, outW), np.nan, np.float32)
    gpu.conv2d(y, src, W, bias, stride, pad, epilogue=gpu.EPI_SILU if silu else gpu.EPI_BIAS)
    ref = O.conv2d(src, O.bf16_to_f32(wb), bias, stride, pad)
    if silu:
        ref = O.silu(ref)
    assert_parity(y, ref, what=f"conv {B}x{C}x{H}x{Wd}->{O_} k{k} s{stride} silu={silu}")


@pytest.mark.parametrize("ta,tb", [(111, 112), (111, 111), (112, 111)])
@pytest.mark.parametrize("M,N,K", [(96, 80, 72), (8, 300, 128), (257, 129, 64), (512, 512, 128), (200, 96, 45)])
def test_sgemm_vs_oracle(gpu, ta, tb, M, N, K):
    """The cblas_sgemm slot on the reference's own fp32 operands (cblas_gemm -> qgemm,
    quicknncpu.pas:335-365,1398-1496): the oracle multiplies the unrounded A and B.  512x512x128
    is a head of the FLUX attention score product Q.K^T (quicknn_transformers.pas:1174-1183)."""
    rng = np.random.default_rng(M + N + K + ta + tb)
    A = rng.standard_normal((K, M) if ta == 112 else (M, K), dtype=np.float32)
    B = rng.standard_normal((N, K) if tb == 112 else (K, N), dtype=np.float32)
    C0 = rng.standard_normal((M, N), dtype=np.float32)
    lda, ldb = A.shape[1], B.shape[1]
    path = O.PATH_AVX2 if K % 8 == 0 else O.PATH_SCALAR
    for alpha, beta in ((1.0, 0.0), (0.5, 2.0), (1.5, 1.0)):
        C = C0.copy()
        gpu.sgemm(101, ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, N)
        ref = C0.copy()
        O.qgemm(ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, ref, N, path=path)
        what = f"sgemm {ta},{tb} {M}x{N}x{K} a={alpha} b={beta}"
        assert_parity(C, ref, what=what)
        assert_parity(C, ref, TOL_X3_MAX, TOL_X3_MEAN, what=what + " (bf16x3 bounds)")


def test_qnn_matmul_mirror_vs_oracle(gpu):
    """The QNNMatMulNT / NN / TN mirror (quicknncpu.pas:1760-1797) with the reference's own
    arguments: NT with a device weight (bf16 W, fp32 X) and NT / NN / TN on fp32 host operands
    through the cblas_gemm slot, each against the oracle's qgemm on the same unrounded inputs."""
    rng = np.random.default_rng(41)
    M, K, N = 200, 256, 320
    x, w, _ = inputs(M, K, N, seed=41, bias=False)
    W = gpu.Weight(w)
    C = np.full((M, N), np.nan, np.float32)
    gpu.QNNMatMulNT(C, x, W, M, K, N)
    assert_parity(C, O.linear_bf16(x, w), what="QNNMatMulNT device weight")
    W.free()
    A = rng.standard_normal((M, K), dtype=np.float32)
    Bnt = rng.standard_normal((N, K), dtype=np.float32)
    Bnn = rng.standard_normal((K, N), dtype=np.float32)
    for name, fn, B, ta, tb, ldb in (("NT", gpu.QNNMatMulNT, Bnt, 111, 112, K),
                                     ("NN", gpu.QNNMatMulNN, Bnn, 111, 111, N)):
        C = np.full((M, N), np.nan, np.float32)
        fn(C, A, B, M, K, N)
        ref = np.zeros((M, N), np.float32)
        O.qgemm(ta, tb, M, N, K, 1.0, A, K, B, ldb, 0.0, ref, N)
        assert_parity(C, ref, TOL_X3_MAX, TOL_X3_MEAN, what=f"QNNMatMul{name} fp32 operands")
    S = 192  # TN with the reference's lda = ldb = K: square products
    At = rng.standard_normal((S, S), dtype=np.float32)
    Bs = rng.standard_normal((S, S), dtype=np.float32)
    C = np.full((S, S), np.nan, np.float32)
    gpu.QNNMatMulTN(C, At, Bs, S, S, S)
    ref = np.zeros((S, S), np.float32)
    O.qgemm(112, 111, S, S, S, 1.0, At, S, Bs, S, 0.0, ref, S)
    assert_parity(C, ref, TOL_X3_MAX, TOL_X3_MEAN, what="QNNMatMulTN fp32 operands")


def test_m_zero_is_noop(gpu):
    x, w, _ = inputs(4, 64, 64, seed=1, bias=False)
    W = gpu.Weight(w)
    y = np.full((0, 64), 7.0, np.float32)
    gpu.linear(y, np.zeros((0, 64), np.float32), W)


def test_bounded_wait_times_out_cleanly(gpu):
    """A wait nothing satisfies returns ENVG_ERR_TIMEOUT and the context stays usable."""
    rc = gpu.selftest_wait_timeout(20_000_000)  # 20 ms bound
    assert rc == gpu.ERR_TIMEOUT
    assert "bound" in gpu.last_error()
    x, w, b = inputs(128, 256, 256, seed=9)
    W = gpu.Weight(w)
    y = np.zeros((128, 256), np.float32)
    gpu.linear(y, x, W, bias=b)
    assert_parity(y, O.linear_bf16(x, w, b))


def test_device_pointer_mode_and_canaries(gpu):
    """torch CUDA tensors go through ENVG_DEVICE_PTRS; guard zones around Y stay untouched."""
    import torch

    M, K, N = 300, 512, 520
    x, w, b = inputs(M, K, N, seed=21)
    W = gpu.Weight(w)
    guard = 4096
    ybuf = torch.full((M * N + 2 * guard,), 12345.0, device="cuda")
    y = ybuf[guard:guard + M * N].view(M, N)
    gpu.linear(y, torch.from_numpy(x).cuda(), W, bias=torch.from_numpy(b).cuda())
    torch.cuda.synchronize()
    assert torch.all(ybuf[:guard] == 12345.0) and torch.all(ybuf[guard + M * N:] == 12345.0)
    assert_parity(y.cpu().numpy(), O.linear_bf16(x, w, b))


def test_errors_are_codes_not_crashes(gpu):
    x, w, _ = inputs(8, 64, 32, seed=2, bias=False)
    W = gpu.Weight(w)
    y = np.zeros((8, 32), np.float32)
    with pytest.raises(gpu.EnvgError) as e:
        gpu.linear(y, np.zeros((8, 48), np.float32), W)  # K mismatch
    assert e.value.code == gpu.ERR_ARG
    with pytest.raises(gpu.EnvgError):
        gpu.linear(y, x, W, epilogue=gpu.EPI_SILU_GATE)  # needs a GATE_UP weight
    W.free()
    with pytest.raises(gpu.EnvgError) as e:
        gpu.linear(y, x, W)  # freed handle -> NULL
    assert e.value.code == gpu.ERR_STATE


@pytest.mark.parametrize("env", [{"ENVG_STORE": "coalesced"}, {"ENVG_STORE": "coalesced", "ENVG_K1": "single"},
                                 {"ENVG_K1": "single"}, {"ENVG_PAIR_SPLIT": "3"}, {"ENVG_PAIR_SPLIT": "0"},
                                 {"ENVG_PAIR_SCHED": "static"}, {"ENVG_PAIR_GROUP_M": "4", "ENVG_L2_HINTS": "0"}])
def test_alternate_kernel_paths_in_subprocess(env):
    """The warp-coalesced store epilogue, the single-CTA k1_gemm and a forced (or disabled) split-K of
    k1_gemm_pair (selected by environment at init) on a few linear / SiLU-gate / gated-residual /
    conv cases, in a fresh process."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "import numpy as np\n"
        "from invision_b200 import envg\n"
        "from oracle import oracle as O\n"
        "from tests.common import inputs, assert_parity, TOL_MAX_PRODUCT, TOL_MEAN_PRODUCT\n"
        "envg.init(0)\n"
        "for (M, K, N) in [(300, 512, 520), (129, 64, 257), (1024, 3072, 9216)]:\n"
        "    x, w, b = inputs(M, K, N, seed=M + N)\n"
        "    W = envg.Weight(w); y = np.zeros((M, N), np.float32); envg.linear(y, x, W, bias=b)\n"
        "    assert_parity(y, O.linear_bf16(x, w, b))\n"
        "x, w, _ = inputs(256, 512, 768, seed=4)\n"
        "W = envg.Weight(w, layout=envg.LAYOUT_GATE_UP); y = np.zeros((256, 384), np.float32); envg.linear(y, x, W)\n"
        "g = O.linear_bf16(x, w)\n"
        "assert_parity(y, O.silu_mul(np.ascontiguousarray(g[:, :384]), np.ascontiguousarray(g[:, 384:])), "
        "TOL_MAX_PRODUCT, TOL_MEAN_PRODUCT)\n"
        "x, w, b = inputs(200, 256, 100, seed=8); rng = np.random.default_rng(1)\n"
        "h0 = rng.standard_normal((200, 100), dtype=np.float32); gate = rng.standard_normal(100).astype(np.float32)\n"
        "W = envg.Weight(w); h = h0.copy(); envg.linear(h, x, W, bias=b, epilogue=envg.EPI_GATED_RESIDUAL, gate=gate)\n"
        "ref = O.gated_add(h0, gate, O.linear_bf16(x, w, b)); assert_parity(h - h0, ref - h0)\n"
        "rng = np.random.default_rng(3); src = rng.standard_normal((1, 64, 12, 96), dtype=np.float32)\n"
        "wb = O.f32_to_bf16_rne((0.02 * rng.standard_normal((256, 64, 3, 3))).astype(np.float32))\n"
        "bias = (0.01 * rng.standard_normal(256)).astype(np.float32)\n"
        "W = envg.Weight(wb.reshape(256, -1), conv=(256, 64, 3, 3)); y = np.zeros((1, 256, 12, 96), np.float32)\n"
        "envg.conv2d(y, src, W, bias, 1, 1, epilogue=envg.EPI_SILU)\n"
        "assert_parity(y, O.silu(O.conv2d(src, O.bf16_to_f32(wb), bias, 1, 1)))\n"
        "print('ok')\n" % root)
    r = subprocess.run([sys.executable, "-c", code], env={**os.environ, **env}, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-3000:]


_SCHED_CASE = r"""
import sys
import numpy as np
from invision_b200 import envg
from tests.common import inputs
envg.init(0)
out = {}
for (M, K, N) in [(2048, 1024, 4096), (600, 512, 1040), (4608, 3072, 768)]:
    x, w, b = inputs(M, K, N, seed=M + K)
    W = envg.Weight(w)
    y = np.zeros((M, N), np.float32)
    envg.linear(y, x, W, bias=b)
    out["%d_%d_%d" % (M, K, N)] = y
np.savez(sys.argv[1], **out)
"""


def test_pair_unit_order_does_not_change_results(tmp_path):
    """The CTA-pair GEMM hands out its units dynamically (the next free pair takes the next unit;
    ENVG_PAIR_SCHED=dynamic forces it on launches of any length) or statically
    (ENVG_PAIR_SCHED=static): every tile is computed the same way, so the outputs are bit-identical,
    with and without split-K, for one tile wave and for many."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    res = {}
    for mode in ("dynamic", "static"):
        env = dict(os.environ)
        env["ENVG_PAIR_SCHED"] = mode
        f = str(tmp_path / f"{mode}.npz")
        r = subprocess.run([sys.executable, "-c", _SCHED_CASE, f], cwd=root, env=env, capture_output=True,
                           text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-3000:]
        res[mode] = np.load(f)
    for k in res["static"].files:
        np.testing.assert_array_equal(res["dynamic"][k], res["static"][k], err_msg=k)


@pytest.mark.parametrize("M,K,N", [(1, 3072, 18432), (8, 2560, 1024), (3, 131, 257), (5, 4096, 2560), (2, 64, 70)])
def test_gemv_path_is_fp32_exact(gpu, M, K, N):
    """M <= 8 runs k_gemv: fp32 X times bf16 W in fp32 (no bf16 rounding of X), so it matches the
    reference's fp32 GEMM (scalar build) to fp32 round-off, far inside the GEMM bound."""
    x, w, b = inputs(M, K, N, seed=600 + M + K)
    W = gpu.Weight(w)
    y = np.zeros((M, N), np.float32)
    gpu.linear(y, x, W, bias=b)
    assert_parity(y, O.linear_bf16(x, w, b, path=O.PATH_SCALAR), 1e-5, 5e-6, what=f"gemv {M}x{K}x{N}")


@pytest.mark.parametrize("M", [1, 4, 8])
def test_gemv_silu_gate_and_gated_residual(gpu, M):
    K, H = 768, 300
    x, w, _ = inputs(M, K, 2 * H, seed=M + 31)
    W = gpu.Weight(w, layout=gpu.LAYOUT_GATE_UP)
    y = np.zeros((M, H), np.float32)
    gpu.linear(y, x, W)
    g = O.linear_bf16(x, w, path=O.PATH_SCALAR)
    assert_parity(y, O.silu_mul(np.ascontiguousarray(g[:, :H]), np.ascontiguousarray(g[:, H:])), 1e-5, 5e-6,
                  what=f"gemv silu-gate M={M}")
    x2, w2, b2 = inputs(M, K, H, seed=M + 77)
    rng = np.random.default_rng(M)
    h0 = rng.standard_normal((M, H), dtype=np.float32)
    gate = rng.standard_normal(H).astype(np.float32)
    W2 = gpu.Weight(w2)
    h = h0.copy()
    gpu.linear(h, x2, W2, bias=b2, epilogue=gpu.EPI_GATED_RESIDUAL, gate=gate)
    ref = O.gated_add(h0, gate, O.linear_bf16(x2, w2, b2, path=O.PATH_SCALAR))
    assert_parity(h - h0, ref - h0, 1e-5, 1e-5, what=f"gemv gated residual M={M}")


@pytest.mark.parametrize("M", [300, 40])
def test_linear_batch_equals_separate_calls(gpu, M):
    """envg_linear_batch (one cast per distinct input, casts overlapped on a second stream, a
    chained input waiting for its producer) gives bit-identical results to envg_linear calls, on
    the CTA-pair path (M = 300) and the skinny k2_set path (M = 40)."""
    import torch

    dev = "cuda"
    H, F = 256, 384
    rng = np.random.default_rng(5)
    x = torch.from_numpy(rng.standard_normal((M, H), dtype=np.float32)).to(dev)
    x2 = torch.from_numpy(rng.standard_normal((M, H), dtype=np.float32)).to(dev)
    xs = torch.from_numpy(rng.standard_normal((4, H), dtype=np.float32)).to(dev)

    def wt(n, k, seed):
        return O.f32_to_bf16_rne((0.02 * np.random.default_rng(seed).standard_normal((n, k))).astype(np.float32))

    Wq, Wk, Wv = gpu.Weight(wt(H, H, 1)), gpu.Weight(wt(H, H, 2)), gpu.Weight(wt(H, H, 3))
    Wgu = gpu.Weight(wt(2 * F, H, 4), layout=gpu.LAYOUT_GATE_UP)
    Wd = gpu.Weight(wt(H, F, 5))
    Ws = gpu.Weight(wt(520, H, 6))
    Wr, Wr2 = gpu.Weight(wt(201, H, 7)), gpu.Weight(wt(96, 201, 8))
    b = torch.from_numpy((0.01 * rng.standard_normal(H)).astype(np.float32)).to(dev)
    outs = {k: torch.empty(M, H, device=dev) for k in ("q", "k", "v", "d", "q2")}
    outs["gu"] = torch.empty(M, F, device=dev)
    outs["s"] = torch.empty(4, 520, device=dev)
    outs["r"] = torch.empty(M, 201, device=dev)
    outs["r2"] = torch.empty(M, 96, device=dev)
    # chains: gu -> d (SiLU-gate producer) and q -> q2 (bias producer) hand their bf16 copy over in
    # the producer's epilogue; r -> r2 (K = 201, not a multiple of 8) goes through a cast.
    calls = [dict(dst=outs["q"], x=x, W=Wq, bias=b), dict(dst=outs["k"], x=x, W=Wk),
             dict(dst=outs["v"], x=x, W=Wv, bias=b), dict(dst=outs["gu"], x=x2, W=Wgu),
             dict(dst=outs["d"], x=outs["gu"], W=Wd, bias=b), dict(dst=outs["s"], x=xs, W=Ws),
             dict(dst=outs["q2"], x=outs["q"], W=Wk), dict(dst=outs["r"], x=x2, W=Wr),
             dict(dst=outs["r2"], x=outs["r"], W=Wr2)]
    gpu.linear_batch(calls)
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy() for k, v in outs.items()}
    for c in calls:  # the same linears one by one
        gpu.linear(c["dst"], c["x"], c["W"], bias=c.get("bias"))
    torch.cuda.synchronize()
    for k, v in outs.items():
        np.testing.assert_array_equal(got[k], v.cpu().numpy(), err_msg=k)


@pytest.mark.parametrize("M", [16, 64])
def test_skinny_chain_batch_split_producer(gpu, M):
    """A skinny gate_up whose K splits (its k_skinny_reduce writes down's bf16 input) chained into
    down, in one batch: bit-identical to separate calls, and within the bound of the oracle."""
    import torch

    K, F, H = 2048, 1024, 256
    rng = np.random.default_rng(M + 3)
    x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()
    wgu = O.f32_to_bf16_rne((0.02 * rng.standard_normal((2 * F, K))).astype(np.float32))
    wd = O.f32_to_bf16_rne((0.02 * rng.standard_normal((H, F))).astype(np.float32))
    Wgu, Wd = gpu.Weight(wgu, layout=gpu.LAYOUT_GATE_UP), gpu.Weight(wd)
    g, y = torch.empty(M, F, device="cuda"), torch.empty(M, H, device="cuda")
    gpu.linear_batch([dict(dst=g, x=x, W=Wgu), dict(dst=y, x=g, W=Wd)])
    torch.cuda.synchronize()
    gb, yb = g.cpu().numpy(), y.cpu().numpy()
    gpu.linear(g, x, Wgu)
    gpu.linear(y, g, Wd)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(gb, g.cpu().numpy())
    np.testing.assert_array_equal(yb, y.cpu().numpy())
    gu = O.linear_bf16(x.cpu().numpy(), wgu)
    gref = O.silu_mul(np.ascontiguousarray(gu[:, :F]), np.ascontiguousarray(gu[:, F:]))
    assert_parity(gb, gref, TOL_MAX_PRODUCT, TOL_MEAN_PRODUCT, what=f"skinny chain gate_up M={M}")
    assert_parity(yb, O.linear_bf16(gb, wd), what=f"skinny chain down M={M}")


@pytest.mark.parametrize("M", [1, 3, 8])
def test_gemv_chained_in_one_launch(gpu, M):
    """M <= 8: a linear whose input is exactly the output of an earlier linear of the batch runs in
    the same persistent k_gemv launch, its units waiting in the kernel for the producer's outputs
    (Qwen3 gate_up -> down, quicknn_qwen3.pas:782-789), and chains of chains (a -> b -> c, one with
    split-K); a producer read by two later linears chains only the first.  Bit-identical to
    separate calls, and within the bounds of the oracle."""
    import torch

    rng = np.random.default_rng(50 + M)

    def wt(n, k):
        return O.f32_to_bf16_rne((0.02 * rng.standard_normal((n, k))).astype(np.float32))

    K, F, H = 2560, 1536, 2048
    wgu, wd, wc, we = wt(2 * F, K), wt(H, F), wt(640, H), wt(384, H)
    Wgu, Wd, Wc, We = (gpu.Weight(wgu, layout=gpu.LAYOUT_GATE_UP), gpu.Weight(wd), gpu.Weight(wc),
                       gpu.Weight(we))
    x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()
    g, y, c, e = (torch.empty(M, n, device="cuda") for n in (F, H, 640, 384))
    calls = [dict(dst=g, x=x, W=Wgu), dict(dst=y, x=g, W=Wd), dict(dst=c, x=y, W=Wc), dict(dst=e, x=y, W=We)]
    launches0 = gpu.stats()["kernel_launches"]
    gpu.linear_batch(calls)
    torch.cuda.synchronize()
    launches = gpu.stats()["kernel_launches"] - launches0
    got = [t.cpu().numpy() for t in (g, y, c, e)]
    for t in (g, y, c, e):
        t.fill_(float("nan"))
    for cl in calls:
        gpu.linear(cl["dst"], cl["x"], cl["W"])
    torch.cuda.synchronize()
    for a_, t, name in zip(got, (g, y, c, e), "gyce"):
        np.testing.assert_array_equal(a_, t.cpu().numpy(), err_msg=name)
    # gate_up, down and the first reader of down in one launch; the second reader in another
    assert launches == 2, launches
    gu = O.linear_f32(x.cpu().numpy(), O.bf16_to_f32(wgu))
    gref = O.silu_mul(np.ascontiguousarray(gu[:, :F]), np.ascontiguousarray(gu[:, F:]))
    assert_parity(got[0], gref, TOL_MAX_PRODUCT, TOL_MEAN_PRODUCT, what=f"chain gate_up M={M}")
    assert_parity(got[1], O.linear_bf16(got[0], wd), what=f"chain down M={M}")
    assert_parity(got[2], O.linear_bf16(got[1], wc), what=f"chain c M={M}")
    assert_parity(got[3], O.linear_bf16(got[1], we), what=f"chain e M={M}")
    for W in (Wgu, Wd, Wc, We):
        W.free()


@pytest.mark.parametrize("M", [16, 1])
def test_skinny_batch_queue_hazards(gpu, M):
    """A batch of skinny plain and gate/up linears that overwrite each other's inputs (write after
    read) and outputs (write after write, within one kind and across kinds) gives the same
    results as the calls one by one: a k2_set or k_gemv launch never holds two linears that write
    the same output, nor runs a linear before an earlier one has read what it overwrites."""
    import torch

    H, F = 256, 384
    rng = np.random.default_rng(21)

    def wt(n, k):
        return O.f32_to_bf16_rne((0.02 * rng.standard_normal((n, k))).astype(np.float32))

    Wa, Wc = gpu.Weight(wt(H, F)), gpu.Weight(wt(F, H))
    Wgu = gpu.Weight(wt(2 * F, H), layout=gpu.LAYOUT_GATE_UP)
    x0 = torch.from_numpy(rng.standard_normal((M, F), dtype=np.float32)).cuda()
    x2 = torch.from_numpy(rng.standard_normal((M, H), dtype=np.float32)).cuda()
    x = x0.clone()
    ya, yc, yd = torch.empty(M, H, device="cuda"), torch.empty(M, F, device="cuda"), torch.empty(M, F, device="cuda")
    calls = [dict(dst=ya, x=x, W=Wa),     # plain, reads x
             dict(dst=x, x=x2, W=Wgu),    # gate/up, then overwrites x (write after read)
             dict(dst=yc, x=x2, W=Wc),    # plain, writes yc
             dict(dst=yc, x=ya, W=Wc),    # plain, writes yc again (write after write, same kind)
             dict(dst=yd, x=x2, W=Wgu),   # gate/up, writes yd
             dict(dst=yd, x=x2, W=Wc)]    # plain over yd (write after write, other kind)
    gpu.linear_batch(calls)
    torch.cuda.synchronize()
    outs = (ya, x, yc, yd)
    got = [t.cpu().numpy() for t in outs]
    x.copy_(x0)
    for c in calls:
        gpu.linear(c["dst"], c["x"], c["W"])
    torch.cuda.synchronize()
    for g, t, name in zip(got, outs, ("ya", "x", "yc", "yd")):
        np.testing.assert_array_equal(g, t.cpu().numpy(), err_msg=name)


@pytest.mark.parametrize("M", [1, 16, 300])
def test_batch_vector_hazards(gpu, M):
    """Linears of one k_gemv (M = 1), k2_set (M = 16) or CTA-pair (M = 300) launch run at once, so a
    batch must not put into one launch a linear whose bias or gate is another member's output (read
    after write: the adaLN modulation feeding a gated residual), nor one that overwrites a vector
    another member reads (write after read).  The batch equals the calls one by one."""
    import torch

    K, N = 256, 384
    rng = np.random.default_rng(31 + M)

    def wt(n, k):
        return gpu.Weight(O.f32_to_bf16_rne((0.02 * rng.standard_normal((n, k))).astype(np.float32)))

    Wb, Wg, Wr, Wo = wt(N, K), wt(N, K), wt(N, K), wt(N, K)
    x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()  # one input: one pair set
    h0 = torch.from_numpy(rng.standard_normal((M, N), dtype=np.float32)).cuda()
    yb, yg, yo = (torch.empty(M, N, device="cuda") for _ in range(3))
    h = h0.clone()
    bias_v, gate_v = yb.view(-1)[:N], yg.view(-1)[:N]  # first N floats of two outputs
    calls = [dict(dst=yb, x=x, W=Wb),                                  # writes the bias vector
             dict(dst=yg, x=x, W=Wg),                                  # writes the gate vector
             dict(dst=h, x=x, W=Wr, bias=bias_v, gate=gate_v,          # reads both (read after write)
                  epilogue=gpu.EPI_GATED_RESIDUAL),
             dict(dst=yb, x=x, W=Wo)]                                  # overwrites the bias (write after read)
    gpu.linear_batch(calls)
    torch.cuda.synchronize()
    got = [t.cpu().numpy() for t in (yb, yg, h)]
    h.copy_(h0)
    for c in calls:
        gpu.linear(c["dst"], c["x"], c["W"], bias=c.get("bias"), epilogue=c.get("epilogue"), gate=c.get("gate"))
    torch.cuda.synchronize()
    for g, t, name in zip(got, (yb, yg, h), ("yb", "yg", "h")):
        np.testing.assert_array_equal(g, t.cpu().numpy(), err_msg=name)
    for W in (Wb, Wg, Wr, Wo):
        W.free()


@pytest.mark.parametrize("M,K,N", [(512, 3072, 1024), (4, 3072, 768), (130, 200, 264)])
def test_adaln_linear_vs_oracle(gpu, M, K, N):
    """QNNAdaLN + QNNLinear fused (envg_linear_adaln) against the oracle's QNNAdaLN then linear."""
    rng = np.random.default_rng(M + K)
    x = (1.5 + 2 * rng.standard_normal((M, K))).astype(np.float32)
    shift = (0.1 * rng.standard_normal(K)).astype(np.float32)
    scale = (0.1 * rng.standard_normal(K)).astype(np.float32)
    _, w, b = inputs(M, K, N, seed=K + N)
    W = gpu.Weight(w)
    y = np.zeros((M, N), np.float32)
    gpu.QNNAdaLNLinear(y, x, shift, scale, W, b, M, K, N)
    xn = O.adaln(x, shift, scale)
    ref = O.linear_bf16(xn, w, b, path=O.PATH_SCALAR if K % 8 else O.PATH_AVX2)
    if M <= 8:  # fp32 path: far inside the GEMM bound
        assert_parity(y, ref, 1e-4, 2e-5, what=f"adaln gemv {M}x{K}x{N}")
    else:
        assert_parity(y, ref, what=f"adaln {M}x{K}x{N}")


@pytest.mark.parametrize("M,K,N,wt", [(512, 2560, 1024, True), (4, 2560, 640, True), (16, 2560, 512, True),
                                      (130, 200, 264, False), (1, 200, 96, False)])
def test_rmsnorm_linear_vs_oracle(gpu, M, K, N, wt):
    """QNNRMSNormRows + QNNLinear fused (envg_linear_rmsnorm) against the oracle's QNNRMSNormRows then
    linear: the gemv path (M <= 8, fp32 normalised input), k2 (M = 16) and the pair kernel."""
    rng = np.random.default_rng(M + K + 7)
    x = (0.3 + 3 * rng.standard_normal((M, K))).astype(np.float32)
    nw = (1 + 0.2 * rng.standard_normal(K)).astype(np.float32) if wt else None
    _, w, b = inputs(M, K, N, seed=K + N + 1)
    W = gpu.Weight(w)
    y = np.zeros((M, N), np.float32)
    gpu.QNNRMSNormLinear(y, x, nw, W, b, M, K, N)
    ref = O.linear_bf16(O.rms_norm(x, nw), w, b, path=O.PATH_SCALAR if K % 8 else O.PATH_AVX2)
    if M <= 8:
        assert_parity(y, ref, 1e-4, 2e-5, what=f"rmsnorm gemv {M}x{K}x{N}")
    else:
        assert_parity(y, ref, what=f"rmsnorm {M}x{K}x{N}")


@pytest.mark.parametrize("M", [3, 200])
def test_rmsnorm_gate_up_vs_oracle(gpu, M):
    """The Qwen3 MLP input: post_attention_layernorm fused into the gate/up linear with SiLU-gate."""
    K, H = 512, 384
    rng = np.random.default_rng(M + 5)
    x = (2 * rng.standard_normal((M, K))).astype(np.float32)
    nw = (1 + 0.2 * rng.standard_normal(K)).astype(np.float32)
    _, w, _ = inputs(M, K, 2 * H, seed=M + 9, bias=False)
    W = gpu.Weight(w, layout=gpu.LAYOUT_GATE_UP)
    y = np.zeros((M, H), np.float32)
    gpu.QNNRMSNormLinear(y, x, nw, W, None, M, K, H)
    gu = O.linear_bf16(O.rms_norm(x, nw), w)
    ref = O.silu_mul(np.ascontiguousarray(gu[:, :H]), np.ascontiguousarray(gu[:, H:]))
    yg = np.zeros((M, 2 * H), np.float32)
    gpu.linear_rmsnorm(yg, x, gpu.Weight(w), weight=nw)
    assert_parity(yg, gu, what=f"rmsnorm gate_up halves M={M}")
    np.testing.assert_allclose(y, O.silu_mul(np.ascontiguousarray(yg[:, :H]), np.ascontiguousarray(yg[:, H:])),
                               rtol=2e-5, atol=2e-6)
    # silu(g) * u compounds the two halves' errors: the product bound of the SiLU-gate tests
    assert_parity(y, ref, TOL_MAX_PRODUCT, TOL_MEAN_PRODUCT, what=f"rmsnorm gate_up M={M}")


def test_safetensors_upload_matches_array_upload(gpu, tmp_path):
    """Weights uploaded straight from a .safetensors file (BF16, F16, F32; plain, GATE_UP, a shard
    and a 4-D conv weight) give the same outputs, bit for bit, as the same values uploaded from
    arrays, and pass parity against the oracle."""
    from tests.common import write_safetensors

    rng = np.random.default_rng(77)
    M, K, N = 96, 320, 272
    x = rng.standard_normal((M, K), dtype=np.float32)
    w_bf = O.f32_to_bf16_rne((0.02 * rng.standard_normal((N, K))).astype(np.float32))
    w_h = (0.02 * rng.standard_normal((N, K))).astype(np.float16)
    w_f = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    conv = O.f32_to_bf16_rne((0.02 * rng.standard_normal((24, 16, 3, 3))).astype(np.float32))
    p = write_safetensors(str(tmp_path / "w.safetensors"), {
        "bf": ("BF16", [N, K], w_bf.tobytes()), "h": ("F16", [N, K], w_h.tobytes()),
        "f": ("F32", [N, K], w_f.tobytes()), "conv": ("BF16", list(conv.shape), conv.tobytes())},
        pad_to=0, extra_header_bytes=1)   # odd data offset: the unaligned path
    for name, arr in (("bf", w_bf), ("h", w_h.astype(np.float32)), ("f", w_f)):
        y_file = np.full((M, N), np.nan, np.float32)
        y_arr = np.full((M, N), np.nan, np.float32)
        gpu.linear(y_file, x, gpu.Weight.from_safetensors(p, name))
        gpu.linear(y_arr, x, gpu.Weight(arr))
        np.testing.assert_array_equal(y_file, y_arr, err_msg=name)
        if arr.dtype == np.uint16:
            assert_parity(y_file, O.linear_bf16(x, arr, None, path=O.PATH_AVX2), what=f"safetensors {name}")
        else:  # F16 / F32 values that are not bf16 numbers keep their precision (bf16x3)
            assert_parity(y_file, O.linear_f32(x, arr, None, path=O.PATH_AVX2), TOL_X3_MAX, TOL_X3_MEAN,
                          what=f"safetensors {name}")
    # GATE_UP from file, and a shard of it
    y_file = np.zeros((M, N // 2), np.float32)
    y_arr = np.zeros((M, N // 2), np.float32)
    gpu.linear(y_file, x, gpu.Weight.from_safetensors(p, "bf", layout=gpu.LAYOUT_GATE_UP))
    gpu.linear(y_arr, x, gpu.Weight(w_bf, layout=gpu.LAYOUT_GATE_UP))
    np.testing.assert_array_equal(y_file, y_arr)
    ys_file = np.zeros((M, 40), np.float32)
    ys_arr = np.zeros((M, 40), np.float32)
    gpu.linear(ys_file, x, gpu.Weight.from_safetensors(p, "bf", layout=gpu.LAYOUT_GATE_UP, shard=(16, 56)))
    gpu.linear(ys_arr, x, gpu.Weight(w_bf, layout=gpu.LAYOUT_GATE_UP, shard=(16, 56)))
    np.testing.assert_array_equal(ys_file, ys_arr)
    # 4-D conv weight
    src = rng.standard_normal((1, 16, 20, 20), dtype=np.float32)
    bias = (0.01 * rng.standard_normal(24)).astype(np.float32)
    yc_file = np.zeros((1, 24, 20, 20), np.float32)
    yc_arr = np.zeros((1, 24, 20, 20), np.float32)
    gpu.conv2d(yc_file, src, gpu.Weight.from_safetensors(p, "conv"), bias, 1, 1)
    gpu.conv2d(yc_arr, src, gpu.Weight(conv.reshape(24, -1), conv=(24, 16, 3, 3)), bias, 1, 1)
    np.testing.assert_array_equal(yc_file, yc_arr)
    with pytest.raises(gpu.EnvgError):
        gpu.Weight.from_safetensors(p, "conv", shard=(0, 8))


def _resblock_params(rng, Ci, Co, skip):
    def bfw(shape, s):
        return O.f32_to_bf16_rne((s * rng.standard_normal(shape)).astype(np.float32))

    p = {"norm1_gamma": (1 + 0.1 * rng.standard_normal(Ci)).astype(np.float32),
         "norm1_beta": (0.1 * rng.standard_normal(Ci)).astype(np.float32),
         "conv1_w": bfw((Co, Ci, 3, 3), 0.03), "conv1_b": (0.01 * rng.standard_normal(Co)).astype(np.float32),
         "norm2_gamma": (1 + 0.1 * rng.standard_normal(Co)).astype(np.float32),
         "norm2_beta": (0.1 * rng.standard_normal(Co)).astype(np.float32),
         "conv2_w": bfw((Co, Co, 3, 3), 0.03), "conv2_b": (0.01 * rng.standard_normal(Co)).astype(np.float32)}
    if skip:
        p["skip_w"] = bfw((Co, Ci, 1, 1), 0.1)
        p["skip_b"] = (0.01 * rng.standard_normal(Co)).astype(np.float32)
    return p


def _oracle_params(p):
    q = dict(p)
    for k in ("conv1_w", "conv2_w", "skip_w"):
        if k in q:
            q[k] = O.bf16_to_f32(q[k])
    return q


@pytest.mark.parametrize("B,C,H,W,G,silu", [(1, 128, 32, 32, 32, True), (2, 64, 24, 40, 8, False),
                                             (1, 96, 7, 9, 32, True), (1, 32, 256, 256, 32, True)])
def test_group_norm_vs_oracle(gpu, B, C, H, W, G, silu):
    rng = np.random.default_rng(B + C + H + W)
    x = (0.5 + 2 * rng.standard_normal((B, C, H, W))).astype(np.float32)
    gamma = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(C)).astype(np.float32)
    y = np.full_like(x, np.nan)
    gpu.group_norm(y, x, gamma, beta, G, silu=silu)
    ref = O.group_norm(x, gamma, beta, G, act=silu)
    # fp32 elementwise op: statistics in fp64 partials vs the reference's sequential fp32 sums
    assert_parity(y, ref, tol_max=1e-4, tol_mean=1e-5, what=f"group_norm {B}x{C}x{H}x{W} G{G} silu={silu}")


@pytest.mark.parametrize("B,Ci,Co,H,W,G", [(1, 128, 256, 32, 32, 32),   # skip conv, TMA reduce-add store
                                           (1, 128, 128, 24, 40, 32),   # identity skip, non-TMA residual store
                                           (2, 64, 64, 16, 16, 16),
                                           (1, 64, 128, 9, 13, 32)])    # ragged image
def test_vae_resblock_vs_oracle(gpu, B, Ci, Co, H, W, G):
    rng = np.random.default_rng(Ci * 7 + Co + H)
    x = rng.standard_normal((B, Ci, H, W)).astype(np.float32)
    p = _resblock_params(rng, Ci, Co, Ci != Co)
    rb = gpu.ResBlock(p)
    y = np.full((B, Co, H, W), np.nan, np.float32)
    rb.forward(y, x, G)
    ref = O.vae_resblock(x, _oracle_params(p), G)
    assert_parity(y, ref, what=f"resblock {B}x{Ci}->{Co} {H}x{W} G{G}")


def test_vae_resblock_device_pointers_match_host(gpu):
    import torch

    rng = np.random.default_rng(5)
    B, Ci, Co, H, W, G = 1, 64, 128, 64, 64, 32
    x = rng.standard_normal((B, Ci, H, W)).astype(np.float32)
    p = _resblock_params(rng, Ci, Co, True)
    rb = gpu.ResBlock(p)
    y_host = np.zeros((B, Co, H, W), np.float32)
    rb.forward(y_host, x, G)
    vecs = {k: torch.from_numpy(v).cuda() for k, v in p.items() if not k.endswith("_w")}
    xd = torch.from_numpy(x).cuda()
    yd = torch.full((B, Co, H, W), float("nan"), device="cuda")
    rb.forward(yd, xd, G, vecs=vecs)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(yd.cpu().numpy(), y_host)


def test_resblock_argument_errors(gpu):
    rng = np.random.default_rng(6)
    p = _resblock_params(rng, 64, 128, False)   # in != out without a skip conv
    rb = gpu.ResBlock(p)
    x = np.zeros((1, 64, 8, 8), np.float32)
    y = np.zeros((1, 128, 8, 8), np.float32)
    with pytest.raises(gpu.EnvgError) as e:
        rb.forward(y, x, 32)
    assert "skip" in str(e.value)
    p2 = _resblock_params(rng, 64, 64, False)
    rb2 = gpu.ResBlock(p2)
    with pytest.raises(gpu.EnvgError):
        rb2.forward(np.zeros((1, 64, 8, 8), np.float32), x, 48)   # 64 % 48 != 0


ATTN_CASES = [
    # seq_q, seq_k, heads, kv_heads, causal, masked
    (256, 256, 2, 2, False, False),
    (200, 333, 3, 3, False, False),     # ragged q and k tiles
    (130, 130, 4, 2, True, False),      # GQA + causal
    (512, 512, 2, 1, True, True),       # causal + key mask
    (64, 300, 2, 2, False, True),
    (1, 200, 2, 2, True, False),        # one query row, causal with offset (sees all keys)
]


@pytest.mark.parametrize("Sq,Sk,H,KVH,causal,masked", ATTN_CASES)
def test_attention_vs_oracle(gpu, Sq, Sk, H, KVH, causal, masked):
    rng = np.random.default_rng(Sq * 3 + Sk + H)
    D = 128
    q = rng.standard_normal((Sq, H * D)).astype(np.float32)
    k = rng.standard_normal((Sk, KVH * D)).astype(np.float32)
    v = rng.standard_normal((Sk, KVH * D)).astype(np.float32)
    mask = None
    if masked:
        mask = (rng.random(Sk) > 0.25).astype(np.int32)
        mask[0] = 1
    y = np.full((Sq, H * D), np.nan, np.float32)
    gpu.attention(y, q, k, v, H, KVH, causal=causal, key_mask=mask)
    ref = O.attention(q, k, v, H, KVH, D, causal=causal, key_mask=mask)
    assert_parity(y, ref, what=f"attention {Sq}x{Sk} H{H}/{KVH} causal={causal} masked={masked}")


def test_attention_large_scores_and_strides(gpu):
    """Scores spread over a wide range (the running max moves several times) and strided rows
    (the reference's [seq, hidden] buffers with the heads at an offset)."""
    import torch

    rng = np.random.default_rng(3)
    Sq, Sk, H, D = 384, 640, 2, 128
    q = (3.0 * rng.standard_normal((Sq, H * D + 64))).astype(np.float32)
    k = (3.0 * rng.standard_normal((Sk, H * D + 32))).astype(np.float32)
    k[:, :H * D] += np.linspace(0, 4, Sk, dtype=np.float32)[:, None]   # later keys score higher
    v = rng.standard_normal((Sk, H * D)).astype(np.float32)
    ref = O.attention(q[:, :H * D].copy(), k[:, :H * D].copy(), v, H, H, D)
    yd = torch.full((Sq, H * D + 16), float("nan"), device="cuda")
    gpu.attention(yd, torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), H, H)
    torch.cuda.synchronize()
    y = yd.cpu().numpy()
    assert np.isnan(y[:, H * D:]).all()          # columns past the heads untouched
    assert_parity(np.ascontiguousarray(y[:, :H * D]), ref, what="attention wide scores, strided")


def test_attention_argument_errors(gpu):
    q = np.zeros((4, 128), np.float32)
    with pytest.raises(gpu.EnvgError) as e:
        gpu.attention(np.zeros((4, 64), np.float32), q[:, :64].copy(), q[:, :64].copy(), q[:, :64].copy(), 1, 1,
                      head_dim=64)
    assert e.value.code == gpu.ERR_UNSUPPORTED
    with pytest.raises(gpu.EnvgError):
        gpu.attention(np.zeros((8, 128), np.float32), np.zeros((8, 128), np.float32), q, q, 1, 1, causal=True)
    with pytest.raises(gpu.EnvgError):
        gpu.attention(np.zeros((4, 384), np.float32), np.zeros((4, 384), np.float32), q, q, 3, 2)


def test_attention_two_tile_kernel_in_subprocess():
    """k_attention2 (two query tiles per CTA, P in tensor memory), forced with ENVG_ATTN_TILES=2 so
    that small, oracle-sized cases reach it: ragged, GQA, causal and masked."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "import numpy as np\n"
        "from invision_b200 import envg\n"
        "from oracle import oracle as O\n"
        "from tests.common import assert_parity\n"
        "envg.init(0)\n"
        "for (Sq, Sk, H, KVH, causal, masked) in [(256, 256, 2, 2, False, False), (300, 333, 3, 3, False, False),\n"
        "        (130, 130, 4, 2, True, False), (512, 512, 2, 1, True, True), (64, 300, 2, 2, False, True),\n"
        "        (700, 900, 2, 2, True, False)]:\n"
        "    rng = np.random.default_rng(Sq + Sk + H)\n"
        "    q = rng.standard_normal((Sq, H * 128)).astype(np.float32)\n"
        "    k = rng.standard_normal((Sk, KVH * 128)).astype(np.float32)\n"
        "    v = rng.standard_normal((Sk, KVH * 128)).astype(np.float32)\n"
        "    k[:, :] += np.linspace(0, 3, Sk, dtype=np.float32)[:, None]\n"
        "    mask = None\n"
        "    if masked:\n"
        "        mask = (rng.random(Sk) > 0.25).astype(np.int32); mask[0] = 1\n"
        "    y = np.full((Sq, H * 128), np.nan, np.float32)\n"
        "    envg.attention(y, q, k, v, H, KVH, causal=causal, key_mask=mask)\n"
        "    assert_parity(y, O.attention(q, k, v, H, KVH, 128, causal=causal, key_mask=mask),\n"
        "                  what=f'attention2 {Sq}x{Sk} H{H}/{KVH} causal={causal} masked={masked}')\n"
        "print('ok')\n" % root)
    r = subprocess.run([sys.executable, "-c", code], env={**os.environ, "ENVG_ATTN_TILES": "2"}, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-3000:]


def test_linear_batch_groups_skinny_linears(gpu):
    """Consecutive M <= 8 linears of a batch run as one persistent k_gemv launch (several weights per
    launch, a chained one after a flush); results are bit-identical to separate envg_linear calls and
    within the fp32-exact bound of the reference."""
    import torch

    dev = "cuda"
    rng = np.random.default_rng(9)
    H, F = 2560, 1536

    def wt(n, k, seed):
        return O.f32_to_bf16_rne((0.02 * np.random.default_rng(seed).standard_normal((n, k))).astype(np.float32))

    ws = {"q": wt(4096, H, 1), "k": wt(1024, H, 2), "gu": wt(2 * F, H, 3), "d": wt(H, F, 4), "o": wt(H, 4096, 5)}
    W = {k: gpu.Weight(v, layout=gpu.LAYOUT_GATE_UP if k == "gu" else gpu.LAYOUT_PLAIN) for k, v in ws.items()}
    x4 = torch.from_numpy(rng.standard_normal((4, H), dtype=np.float32)).to(dev)
    x1 = torch.from_numpy(rng.standard_normal((1, 4096), dtype=np.float32)).to(dev)
    b = torch.from_numpy((0.01 * rng.standard_normal(4096)).astype(np.float32)).to(dev)
    outs = {"q": torch.empty(4, 4096, device=dev), "k": torch.empty(4, 1024, device=dev),
            "gu": torch.empty(4, F, device=dev), "d": torch.empty(4, H, device=dev), "o": torch.empty(1, H, device=dev)}
    calls = [dict(dst=outs["q"], x=x4, W=W["q"], bias=b), dict(dst=outs["k"], x=x4, W=W["k"]),
             dict(dst=outs["gu"], x=x4, W=W["gu"]), dict(dst=outs["d"], x=outs["gu"], W=W["d"]),
             dict(dst=outs["o"], x=x1, W=W["o"])]
    gpu.linear_batch(calls)
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy() for k, v in outs.items()}
    for c in calls:
        gpu.linear(c["dst"], c["x"], c["W"], bias=c.get("bias"))
    torch.cuda.synchronize()
    for k, v in outs.items():
        np.testing.assert_array_equal(got[k], v.cpu().numpy(), err_msg=k)
    ref = O.linear_bf16(x4.cpu().numpy(), ws["q"], b.cpu().numpy(), path=O.PATH_SCALAR)
    assert_parity(got["q"], ref, tol_max=1e-5, tol_mean=5e-6, what="grouped gemv q")


@pytest.mark.parametrize("M", [16, 48])
def test_linear_batch_groups_skinny_tcgen05_linears(gpu, M):
    """8 < M <= 64: consecutive independent linears of a batch share one persistent k2_set launch
    (with a chained one after its producer's group); bit-identical to separate envg_linear calls,
    and within the GEMM bound of the reference."""
    import torch

    dev = "cuda"
    rng = np.random.default_rng(M)
    H, F = 2560, 1536

    def wt(n, k, seed):
        return O.f32_to_bf16_rne((0.02 * np.random.default_rng(seed).standard_normal((n, k))).astype(np.float32))

    ws = {"q": wt(4096, H, 1), "k": wt(1024, H, 2), "gu": wt(2 * F, H, 3), "d": wt(H, F, 4), "o": wt(H, 4096, 5)}
    W = {k: gpu.Weight(v, layout=gpu.LAYOUT_GATE_UP if k == "gu" else gpu.LAYOUT_PLAIN) for k, v in ws.items()}
    x = torch.from_numpy(rng.standard_normal((M, H), dtype=np.float32)).to(dev)
    x2 = torch.from_numpy(rng.standard_normal((M, 4096), dtype=np.float32)).to(dev)
    b = torch.from_numpy((0.01 * rng.standard_normal(4096)).astype(np.float32)).to(dev)
    outs = {"q": torch.empty(M, 4096, device=dev), "k": torch.empty(M, 1024, device=dev),
            "gu": torch.empty(M, F, device=dev), "d": torch.empty(M, H, device=dev), "o": torch.empty(M, H, device=dev)}
    calls = [dict(dst=outs["q"], x=x, W=W["q"], bias=b), dict(dst=outs["k"], x=x, W=W["k"]),
             dict(dst=outs["gu"], x=x, W=W["gu"]), dict(dst=outs["d"], x=outs["gu"], W=W["d"]),
             dict(dst=outs["o"], x=x2, W=W["o"])]
    gpu.linear_batch(calls)
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy() for k, v in outs.items()}
    for c in calls:
        gpu.linear(c["dst"], c["x"], c["W"], bias=c.get("bias"))
    torch.cuda.synchronize()
    for k, v in outs.items():
        np.testing.assert_array_equal(got[k], v.cpu().numpy(), err_msg=k)
    assert_parity(got["q"], O.linear_bf16(x.cpu().numpy(), ws["q"], b.cpu().numpy(), path=O.PATH_AVX2),
                  what=f"grouped k2 q M={M}")
    assert_parity(got["o"], O.linear_bf16(x2.cpu().numpy(), ws["o"], None, path=O.PATH_AVX2), what=f"grouped k2 o M={M}")


@pytest.mark.parametrize("epi", ["bias", "silu_gate", "gated_residual", "adaln", "rmsnorm"])
def test_host_pipelined_linear_equals_device_call(gpu, epi):
    """Host-pointer linears with M >= 1024 run in row chunks with copies overlapped; the result is
    bit-identical to the same linear on device pointers (one launch), and within the GEMM bound."""
    import torch

    M, K, N = 2600, 768, 1024   # chunks of 1024 and 1576 rows
    rng = np.random.default_rng(31)
    x, w, b = inputs(M, K, N, seed=44)
    layout = gpu.LAYOUT_GATE_UP if epi == "silu_gate" else gpu.LAYOUT_PLAIN
    W = gpu.Weight(w, layout=layout)
    n_out = N // 2 if epi == "silu_gate" else N
    h0 = rng.standard_normal((M, n_out)).astype(np.float32)
    gate = rng.standard_normal(N).astype(np.float32)
    shift = (0.1 * rng.standard_normal(K)).astype(np.float32)
    scale = (0.1 * rng.standard_normal(K)).astype(np.float32)
    yh = h0.copy() if epi == "gated_residual" else np.zeros((M, n_out), np.float32)
    yd = torch.from_numpy(yh.copy()).cuda()
    xd, bd = torch.from_numpy(x).cuda(), torch.from_numpy(b).cuda()
    if epi == "adaln":
        gpu.linear_adaln(yh, x, shift, scale, W, bias=b)
        gpu.linear_adaln(yd, xd, torch.from_numpy(shift).cuda(), torch.from_numpy(scale).cuda(), W, bias=bd)
    elif epi == "rmsnorm":
        gpu.linear_rmsnorm(yh, x, W, weight=1 + scale, bias=b)
        gpu.linear_rmsnorm(yd, xd, W, weight=torch.from_numpy(1 + scale).cuda(), bias=bd)
    elif epi == "gated_residual":
        gpu.linear(yh, x, W, bias=b, epilogue=gpu.EPI_GATED_RESIDUAL, gate=gate)
        gpu.linear(yd, xd, W, bias=bd, epilogue=gpu.EPI_GATED_RESIDUAL, gate=torch.from_numpy(gate).cuda())
    else:
        gpu.linear(yh, x, W, bias=b)
        gpu.linear(yd, xd, W, bias=bd)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(yh, yd.cpu().numpy())
    if epi == "bias":
        assert_parity(yh, O.linear_bf16(x, w, b, path=O.PATH_AVX2), what="pipelined host linear")
