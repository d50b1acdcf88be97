"""GPU, at the full BASELINE sizes: properties that do not depend on size, plus oracle parity on
sampled rows.  The oracle cannot compute a whole config-4 output in test time (18432 x 36864 x
4096), so these pin the full-size kernels by:

* row permutation: Y(P X) = P Y(X), bit for bit (rows are independent);
* row slices: Y(X[a:b]) = Y(X)[a:b], bit for bit (another M, another grid; same per-row work --
  from 1024 rows up, where no launch splits K);
* scaling by 2: Y(2 X) = 2 Y(X), bit for bit without bias (a power of two commutes with the bf16
  rounding of X and with every fp32 product and sum);
* 256 sampled rows against the reference GEMM (oracle), within the acceptance bounds (config 4
  is checked on at least 256 rows, the sample its CPU baseline plan names).
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.common import assert_parity

pytestmark = pytest.mark.gpu

FULL = [
    ("config 2 qkv", 4608, 3072, 9216, True),
    ("config 2 down", 4608, 9216, 3072, True),
    ("config 4 fused_in", 18432, 4096, 36864, False),
    ("config 4 out", 18432, 16384, 4096, False),
]


SAMPLED_ROWS = 256


def _weight(N, K, seed):
    rng = np.random.default_rng(seed)
    w = (0.02 * rng.standard_normal((N, K), dtype=np.float32))
    return O.f32_to_bf16_rne(w)


@pytest.mark.parametrize("name,M,K,N,bias", FULL)
def test_full_size_properties(gpu, name, M, K, N, bias):
    import torch

    dev = "cuda"
    w = _weight(N, K, seed=K + N)
    W = gpu.Weight(w)
    g = torch.Generator(device=dev)
    g.manual_seed(M + K)
    x = torch.randn(M, K, generator=g, device=dev)
    b = (0.01 * torch.randn(N, generator=g, device=dev)) if bias else None
    y = torch.empty(M, N, device=dev)
    gpu.linear(y, x, W, bias=b)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()

    # row permutation
    perm = torch.randperm(M, generator=torch.Generator().manual_seed(7)).to(dev)
    yp = torch.empty_like(y)
    gpu.linear(yp, x[perm].contiguous(), W, bias=b)
    torch.cuda.synchronize()
    assert torch.equal(yp, y[perm]), f"{name}: row permutation changed results"

    # a row slice (a different M and grid, still >= 1024 rows)
    a0, a1 = 1000, 1000 + 1100
    ys = torch.empty(a1 - a0, N, device=dev)
    gpu.linear(ys, x[a0:a1].contiguous(), W, bias=b)
    torch.cuda.synchronize()
    assert torch.equal(ys, y[a0:a1]), f"{name}: row slice changed results"

    # scaling by 2 (exact without bias)
    if not bias:
        y2 = torch.empty_like(y)
        gpu.linear(y2, 2.0 * x, W)
        torch.cuda.synchronize()
        assert torch.equal(y2, 2.0 * y), f"{name}: Y(2X) != 2 Y(X)"

    # sampled rows against the reference GEMM
    rows = np.sort(np.random.default_rng(3).choice(M, SAMPLED_ROWS, replace=False))
    xs = x[torch.from_numpy(rows).to(dev)].cpu().numpy()
    ref = O.linear_bf16(xs, w, b.cpu().numpy() if bias else None, path=O.PATH_AVX2)
    got = y[torch.from_numpy(rows).to(dev)].cpu().numpy()
    assert_parity(got, ref, what=f"{name}: {SAMPLED_ROWS} sampled rows of {M}")
    W.free()


CONV_FULL = [
    # (C, H, W, out_ch): BASELINE config 5 and its sweep
    (512, 128, 128, 512),
    (256, 256, 256, 256),
]


@pytest.mark.parametrize("C,H,Wd,Oc", CONV_FULL)
def test_full_size_conv_properties(gpu, C, H, Wd, Oc):
    """Config 5 conv (3x3 + bias + SiLU, padding 1): batch consistency (two images in one call
    equal two calls, bit for bit) and oracle parity on 24x24 output windows of image 0: the
    top-left corner (zero padding on two sides) and one interior window."""
    import torch

    dev = "cuda"
    rng = np.random.default_rng(5 + C)
    wb = O.f32_to_bf16_rne((0.02 * rng.standard_normal((Oc, C, 3, 3))).astype(np.float32))
    W = gpu.Weight(wb.reshape(Oc, -1), conv=(Oc, C, 3, 3))
    bias = torch.from_numpy((0.01 * rng.standard_normal(Oc)).astype(np.float32)).to(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    src = torch.randn(2, C, H, Wd, generator=g, device=dev)
    y = torch.empty(2, Oc, H, Wd, device=dev)
    gpu.conv2d(y, src, W, bias, 1, 1, epilogue=gpu.EPI_SILU)
    y0 = torch.empty(1, Oc, H, Wd, device=dev)
    gpu.conv2d(y0, src[1:].contiguous(), W, bias, 1, 1, epilogue=gpu.EPI_SILU)
    torch.cuda.synchronize()
    assert torch.equal(y0[0], y[1])
    wf = O.bf16_to_f32(wb)
    # corner: output [0, 24) needs input [0, 25) (row/column -1 is the zero padding)
    win = src[0:1, :, :25, :25].cpu().numpy()
    ref = O.silu(O.conv2d(np.ascontiguousarray(win), wf, bias.cpu().numpy(), 1, 1))
    got = y[0:1, :, :24, :24].cpu().numpy()
    assert_parity(np.ascontiguousarray(got), np.ascontiguousarray(ref[:, :, :24, :24]),
                  what=f"config 5 conv {C} ch {H}x{Wd}, 24x24 corner")
    # interior: output [r0, r0 + 24) needs input [r0 - 1, r0 + 25); a padded oracle run over that
    # slab gives the window at offset 1
    r0, c0 = H // 2 - 7, Wd // 2 + 3
    slab = src[0:1, :, r0 - 1:r0 + 25, c0 - 1:c0 + 25].cpu().numpy()
    ref = O.silu(O.conv2d(np.ascontiguousarray(slab), wf, bias.cpu().numpy(), 1, 1))
    got = y[0:1, :, r0:r0 + 24, c0:c0 + 24].cpu().numpy()
    assert_parity(np.ascontiguousarray(got), np.ascontiguousarray(ref[:, :, 1:25, 1:25]),
                  what=f"config 5 conv {C} ch {H}x{Wd}, interior 24x24 window")
    W.free()
