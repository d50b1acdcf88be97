"""GPU: split-K of k1_gemm_pair for mid-size M (below 1024 rows), where the 256 x 256 pair tiles
of a narrow N leave CTA pairs idle.  Each split sums one contiguous K range into raw fp32
partials and k_split_reduce adds them in split order before the epilogue, so:

* results match the reference GEMM (oracle) within the acceptance bounds, for every epilogue
  (bias, SiLU gate, gated residual, alpha/beta) and for forced split counts with ragged K ranges;
* repeated calls are bit-identical (the reduction order is fixed);
* Y(2X) = 2 Y(X) and row permutations hold bit for bit (powers of two and row order commute with
  every fp32 sum);
* in envg_linear_batch, a split linear whose output feeds the next one writes the bf16 copy of
  that output itself, bit-identical to separate calls.

The shapes are Qwen3-4B's linears at 512 prompt tokens.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle as O
from tests.common import TOL_MAX_PRODUCT, TOL_MEAN_PRODUCT, TOL_X3_MAX, TOL_X3_MEAN, assert_parity, inputs

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# (name, M, K, N, gate_up)
QWEN3_M512 = [
    ("k", 512, 2560, 1024, False),
    ("q", 512, 2560, 4096, False),
    ("o", 512, 4096, 2560, False),
    ("down", 512, 9728, 2560, False),
    ("gate_up narrow", 512, 2560, 2 * 1536, True),
    ("ragged", 777, 3000, 1000, False),
]


def _weight(N, K, seed):
    rng = np.random.default_rng(seed)
    return O.f32_to_bf16_rne((0.02 * rng.standard_normal((N, K))).astype(np.float32))


@pytest.mark.parametrize("name,M,K,N,gate_up", QWEN3_M512)
def test_split_linear_properties(gpu, name, M, K, N, gate_up):
    import torch

    dev = "cuda"
    w = _weight(N, K, seed=K + N)
    W = gpu.Weight(w, layout=gpu.LAYOUT_GATE_UP if gate_up else gpu.LAYOUT_PLAIN)
    out = N // 2 if gate_up else N
    g = torch.Generator(device=dev)
    g.manual_seed(M + K)
    x = torch.randn(M, K, generator=g, device=dev)
    b = 0.01 * torch.randn(N, generator=g, device=dev)
    y = torch.empty(M, out, device=dev)
    gpu.linear(y, x, W, bias=b)
    y_again = torch.empty_like(y)
    gpu.linear(y_again, x, W, bias=b)
    torch.cuda.synchronize()
    assert torch.equal(y, y_again), f"{name}: repeated call differs"

    perm = torch.randperm(M, generator=torch.Generator().manual_seed(5)).to(dev)
    yp = torch.empty_like(y)
    gpu.linear(yp, x[perm].contiguous(), W, bias=b)
    torch.cuda.synchronize()
    assert torch.equal(yp, y[perm]), f"{name}: row permutation changed results"

    if not gate_up:
        y1 = torch.empty_like(y)
        y2 = torch.empty_like(y)
        gpu.linear(y1, x, W)
        gpu.linear(y2, 2.0 * x, W)
        torch.cuda.synchronize()
        assert torch.equal(y2, 2.0 * y1), f"{name}: Y(2X) != 2 Y(X)"

    rows = np.sort(np.random.default_rng(3).choice(M, 24, replace=False))
    xs = x[torch.from_numpy(rows).to(dev)].cpu().numpy()
    ref = O.linear_bf16(xs, w, b.cpu().numpy(), path=O.PATH_AVX2)
    got = y[torch.from_numpy(rows).to(dev)].cpu().numpy()
    if gate_up:
        ref = O.silu_mul(np.ascontiguousarray(ref[:, :out]), np.ascontiguousarray(ref[:, out:]))
        assert_parity(got, ref, TOL_MAX_PRODUCT, TOL_MEAN_PRODUCT, what=f"{name}: 24 sampled rows")
    else:
        assert_parity(got, ref, what=f"{name}: 24 sampled rows")
    W.free()


def test_split_gated_residual_and_sgemm(gpu):
    """Read-modify-write epilogues through k_split_reduce: the gated residual (Y += gate * (XW + b))
    and the sgemm's alpha / beta."""
    M, K, N = 512, 4096, 768
    x, w, b = inputs(M, K, N, seed=21)
    rng = np.random.default_rng(22)
    h0 = rng.standard_normal((M, N), dtype=np.float32)
    gate = rng.standard_normal(N).astype(np.float32)
    W = gpu.Weight(w)
    h = h0.copy()
    gpu.linear(h, x, W, bias=b, epilogue=gpu.EPI_GATED_RESIDUAL, gate=gate)
    ref = O.gated_add(h0, gate, O.linear_bf16(x, w, b))
    assert_parity(h - h0, ref - h0, what="split gated residual")
    W.free()

    Ms, Ns, Ks = 300, 256, 2048
    A = rng.standard_normal((Ms, Ks), dtype=np.float32)
    B = rng.standard_normal((Ks, Ns), dtype=np.float32)
    C0 = rng.standard_normal((Ms, Ns), dtype=np.float32)
    for alpha, beta in ((0.5, 1.0), (1.5, 2.0), (1.0, 0.0)):
        C = C0.copy()
        gpu.sgemm(101, 111, 111, Ms, Ns, Ks, alpha, A, Ks, B, Ns, beta, C, Ns)
        ref = C0.copy()
        O.qgemm(111, 111, Ms, Ns, Ks, alpha, A, Ks, B, Ns, beta, ref, Ns, path=O.PATH_AVX2)
        assert_parity(C, ref, what=f"split sgemm alpha={alpha} beta={beta}")
        assert_parity(C, ref, TOL_X3_MAX, TOL_X3_MEAN, what=f"split sgemm alpha={alpha} beta={beta} (bf16x3 bounds)")


def test_split_linear_in_batch_writes_bf16_copy(gpu):
    """A split linear whose output is the next linear's input: the batch takes the bf16 copy from
    k_split_reduce instead of a cast, and both outputs equal separate calls bit for bit."""
    import torch

    dev = "cuda"
    M, H, F = 512, 2560, 1024
    w1, w2 = _weight(F, H, 1), _weight(H, F, 2)
    W1, W2 = gpu.Weight(w1), gpu.Weight(w2)
    x = torch.randn(M, H, generator=torch.Generator(device=dev).manual_seed(4), device=dev)
    b1 = 0.01 * torch.randn(F, generator=torch.Generator(device=dev).manual_seed(5), device=dev)
    y1, y2 = torch.empty(M, F, device=dev), torch.empty(M, H, device=dev)
    gpu.linear_batch([dict(dst=y1, x=x, W=W1, bias=b1), dict(dst=y2, x=y1, W=W2)])
    torch.cuda.synchronize()
    r1, r2 = torch.empty_like(y1), torch.empty_like(y2)
    gpu.linear(r1, x, W1, bias=b1)
    gpu.linear(r2, r1, W2)
    torch.cuda.synchronize()
    assert torch.equal(y1, r1) and torch.equal(y2, r2)
    W1.free()
    W2.free()


def test_forced_split_counts_in_subprocess():
    """Forced split counts (ENVG_PAIR_SPLIT) with K ranges that do not divide evenly, against the
    oracle, on plain, bias and SiLU-gate linears; 16 splits of 2 K blocks each included."""
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "import numpy as np\n"
        "from invision_b200 import envg\n"
        "from oracle import oracle as O\n"
        "from tests.common import inputs, assert_parity, TOL_MAX_PRODUCT, TOL_MEAN_PRODUCT\n"
        "envg.init(0)\n"
        "for (M, K, N) in [(257, 1000, 520), (512, 2048, 256), (130, 4096, 130)]:\n"
        "    x, w, b = inputs(M, K, N, seed=M + K)\n"
        "    W = envg.Weight(w); y = np.zeros((M, N), np.float32); envg.linear(y, x, W, bias=b)\n"
        "    assert_parity(y, O.linear_bf16(x, w, b), what=f'{M}x{K}x{N}')\n"
        "x, w, b = inputs(384, 1536, 2 * 320, seed=6)\n"
        "W = envg.Weight(w, layout=envg.LAYOUT_GATE_UP); y = np.zeros((384, 320), np.float32)\n"
        "envg.linear(y, x, W, bias=b)\n"
        "g = O.linear_bf16(x, w, b)\n"
        "assert_parity(y, O.silu_mul(np.ascontiguousarray(g[:, :320]), np.ascontiguousarray(g[:, 320:])), "
        "TOL_MAX_PRODUCT, TOL_MEAN_PRODUCT, what='gate_up')\n"
        "print('ok')\n" % ROOT)
    for n in ("2", "7", "16"):
        r = subprocess.run([sys.executable, "-c", code], env={**os.environ, "ENVG_PAIR_SPLIT": n},
                           capture_output=True, text=True, timeout=300)
        assert r.returncode == 0 and "ok" in r.stdout, f"ENVG_PAIR_SPLIT={n}: " + r.stderr[-3000:]


def test_pair_set_batch_equals_separate_calls(gpu):
    """Qwen3's q, k, v and a gate_up on one input at M = 512 go out as pair-set launches (k and v
    split K, q does not; the SiLU-gate linear needs the other kernel variant), plus a gated
    residual on the same input: every output equals its separate call bit for bit."""
    import torch

    dev = "cuda"
    M, H = 512, 2560
    ws = {"q": _weight(4096, H, 11), "k": _weight(1024, H, 12), "v": _weight(1024, H, 13),
          "gu": _weight(2 * 1536, H, 14), "r": _weight(768, H, 15)}
    W = {k: gpu.Weight(v, layout=gpu.LAYOUT_GATE_UP if k == "gu" else gpu.LAYOUT_PLAIN) for k, v in ws.items()}
    g = torch.Generator(device=dev).manual_seed(21)
    x = torch.randn(M, H, generator=g, device=dev)
    b = 0.01 * torch.randn(4096, generator=g, device=dev)
    gate = torch.randn(768, generator=g, device=dev)
    h0 = torch.randn(M, 768, generator=g, device=dev)
    outs = {"q": torch.empty(M, 4096, device=dev), "k": torch.empty(M, 1024, device=dev),
            "v": torch.empty(M, 1024, device=dev), "gu": torch.empty(M, 1536, device=dev), "r": h0.clone()}
    calls = [dict(dst=outs["q"], x=x, W=W["q"], bias=b), dict(dst=outs["k"], x=x, W=W["k"]),
             dict(dst=outs["v"], x=x, W=W["v"]), dict(dst=outs["gu"], x=x, W=W["gu"]),
             dict(dst=outs["r"], x=x, W=W["r"], epilogue=gpu.EPI_GATED_RESIDUAL, gate=gate)]
    gpu.linear_batch(calls)
    torch.cuda.synchronize()
    got = {k: v.clone() for k, v in outs.items()}
    outs["r"].copy_(h0)
    for c in calls:
        kw = {k: c[k] for k in ("bias", "epilogue", "gate") if k in c}
        gpu.linear(c["dst"], c["x"], c["W"], **kw)
    torch.cuda.synchronize()
    for k in outs:
        assert torch.equal(got[k], outs[k]), k
    ref = O.linear_bf16(x[:16].cpu().numpy(), ws["k"], path=O.PATH_AVX2)
    assert_parity(got["k"][:16].cpu().numpy(), ref, what="pair set k, 16 rows")
    for w in W.values():
        w.free()


def test_batch_rereads_an_input_that_an_earlier_linear_overwrote(gpu):
    """[y1 = x W1; x = h W2; y3 = x W3]: the third linear reads x after the second rewrote it, so
    it must not reuse the bf16 copy made for the first (equal to three separate calls)."""
    import torch

    dev = "cuda"
    M, K = 300, 512
    w1, w2, w3 = _weight(640, K, 31), _weight(K, 384, 32), _weight(256, K, 33)
    W1, W2, W3 = gpu.Weight(w1), gpu.Weight(w2), gpu.Weight(w3)
    g = torch.Generator(device=dev).manual_seed(5)
    x0 = torch.randn(M, K, generator=g, device=dev)
    h = torch.randn(M, 384, generator=g, device=dev)
    x = x0.clone()
    y1, y3 = torch.empty(M, 640, device=dev), torch.empty(M, 256, device=dev)
    gpu.linear_batch([dict(dst=y1, x=x, W=W1), dict(dst=x, x=h, W=W2), dict(dst=y3, x=x, W=W3)])
    torch.cuda.synchronize()
    xr = x0.clone()
    r1, r3 = torch.empty_like(y1), torch.empty_like(y3)
    gpu.linear(r1, xr, W1)
    gpu.linear(xr, h, W2)
    gpu.linear(r3, xr, W3)
    torch.cuda.synchronize()
    assert torch.equal(y1, r1) and torch.equal(x, xr) and torch.equal(y3, r3)
    for w in (W1, W2, W3):
        w.free()
