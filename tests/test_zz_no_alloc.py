"""GPU: envg_linear_noalloc, the allocation-free skinny-M linear, against envg_linear and against
the CPU restatement of the reference's GEMM.

Some callers cannot let the library allocate device memory: a host whose own allocator has
reserved the GPU's memory and forbids other libraries to allocate, or a caller sharing the GPU
with streams that must not be stalled by the device-wide wait of cudaFree.  envg_linear_noalloc
serves them from one fixed __device__ scratch array.  This file is collected last on purpose, so
a run that stops at its first failure has already run every other test; it also passes alone in
a fresh process.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.common import TOL_MAX, TOL_MAX_PRODUCT, TOL_MEAN, TOL_MEAN_PRODUCT, assert_parity, inputs

pytestmark = pytest.mark.gpu

CASES = [
    # (M, K, N, epilogue)
    (1, 3072, 18432, "bias"),     # adaLN modulation shape
    (16, 2560, 4096, "bias"),     # Qwen3 q at M = 16
    (64, 4096, 1024, "none"),     # largest M, split-K
    (7, 512, 2 * 384, "silu_gate"),
    (16, 2560, 2560, "gated_residual"),  # FLUX-style gated residual update of the hidden state
]


def _call_noalloc(envg, y, x, W, bias, epi, gate=None):
    L = envg.lib()
    return L.envg_linear_noalloc(y.data_ptr(), x.data_ptr(), W.h, bias.data_ptr() if bias is not None else None,
                                 x.shape[0], x.shape[1], W.N, epi, gate.data_ptr() if gate is not None else None,
                                 envg.DEVICE_PTRS)


@pytest.mark.parametrize("M,K,N,kind", CASES)
def test_noalloc_matches_envg_linear_twice(gpu, M, K, N, kind):
    import torch

    envg = gpu
    x, w, b = inputs(M, K, N, seed=77 + M + K)
    silu = kind == "silu_gate"
    gated = kind == "gated_residual"
    W = envg.Weight(w, layout=envg.LAYOUT_GATE_UP if silu else envg.LAYOUT_PLAIN)
    epi = {"silu_gate": envg.EPI_SILU_GATE, "bias": envg.EPI_BIAS, "gated_residual": envg.EPI_GATED_RESIDUAL}.get(
        kind, envg.EPI_NONE)
    bias = torch.from_numpy(b).cuda() if kind in ("bias", "gated_residual") else None
    rng = np.random.default_rng(M + N)
    gate_h = rng.standard_normal(N).astype(np.float32) if gated else None
    gate = torch.from_numpy(gate_h).cuda() if gated else None
    xt = torch.from_numpy(x).cuda()
    n_out = N // 2 if silu else N
    # the gated residual reads dst as the residual: every call starts from the same h0
    h0 = rng.standard_normal((M, n_out), dtype=np.float32) if gated else np.full((M, n_out), np.nan, np.float32)
    y_ref = torch.from_numpy(h0).cuda()
    envg.linear(y_ref, xt, W, bias=bias, epilogue=epi, gate=gate)  # the existing entry point
    torch.cuda.synchronize()
    ref = y_ref.cpu().numpy()

    ys = [torch.from_numpy(h0).cuda() for _ in range(2)]
    torch.cuda.synchronize()
    ws_before = envg.stats()["workspace_bytes"]
    free_before = torch.cuda.mem_get_info()[0]
    outs = []
    for y in ys:  # two calls in a row share (and reuse) the scratch array
        rc = _call_noalloc(envg, y, xt, W, bias, epi, gate)
        assert rc == envg.OK, envg.last_error()
        torch.cuda.synchronize()
        outs.append(y.cpu().numpy())
    assert envg.stats()["workspace_bytes"] == ws_before, "the library workspace grew"
    assert torch.cuda.mem_get_info()[0] == free_before, "device memory was allocated"
    # the oracle: the reference's fp32 GEMM on the same X and widened bf16 W, then its epilogue
    bref = b if bias is not None else None
    lin = O.linear_bf16(x, w, bref)
    if silu:
        oracle = O.silu_mul(np.ascontiguousarray(lin[:, :n_out]), np.ascontiguousarray(lin[:, n_out:]))
    elif gated:
        oracle = O.gated_add(h0, gate_h, lin)
    else:
        oracle = lin
    # silu(g) * u multiplies two GEMM outputs, so it carries the product bound (tests/common.py);
    # for M <= 8 envg_linear multiplies fp32 X exactly while this entry rounds X to bf16.  The
    # gated residual is compared on the update (y - h0), so the residual does not hide GEMM error.
    tmax, tmean = (TOL_MAX_PRODUCT, TOL_MEAN_PRODUCT) if silu else (TOL_MAX, TOL_MEAN)
    base = h0 if gated else 0.0
    for o in outs:
        assert_parity(o - base, ref - base, tmax, tmean, what=f"noalloc {M}x{K}x{N} {kind} vs envg_linear")
        assert_parity(o - base, oracle - base, tmax, tmean, what=f"noalloc {M}x{K}x{N} {kind} vs oracle")
    np.testing.assert_array_equal(outs[0], outs[1])  # the second call reuses the scratch exactly
    W.free()


def test_noalloc_rejects_what_it_cannot_hold(gpu):
    import torch

    envg = gpu
    L = envg.lib()
    x, w, _ = inputs(65, 256, 128, seed=5, bias=False)
    W = envg.Weight(w)
    xt = torch.from_numpy(x).cuda()
    y = torch.empty(65, 128, device="cuda")
    rc = L.envg_linear_noalloc(y.data_ptr(), xt.data_ptr(), W.h, None, 65, 256, 128, envg.EPI_NONE, None,
                               envg.DEVICE_PTRS)
    assert rc == envg.ERR_ARG and "M=65" in envg.last_error()
    # host pointers are refused: the entry point stages nothing
    xn = np.zeros((4, 256), np.float32)
    yn = np.zeros((4, 128), np.float32)
    rc = L.envg_linear_noalloc(yn.ctypes.data, xn.ctypes.data, W.h, None, 4, 256, 128, envg.EPI_NONE, None,
                               envg.HOST_PTRS)
    assert rc == envg.ERR_ARG and "device pointers" in envg.last_error()
    # dst may not alias x
    xa = torch.zeros(4, 256, device="cuda")
    Wsq = envg.Weight(inputs(4, 256, 256, seed=8, bias=False)[1])
    rc = L.envg_linear_noalloc(xa.data_ptr(), xa.data_ptr(), Wsq.h, None, 4, 256, 256, envg.EPI_NONE, None,
                               envg.DEVICE_PTRS)
    assert rc == envg.ERR_ARG and "aliases" in envg.last_error()
    Wsq.free()
    # activation scratch limit: M * Kp * 2 bytes <= 2 MiB
    x2, w2, _ = inputs(64, 16392, 128, seed=6, bias=False)
    W2 = envg.Weight(w2)
    xt2 = torch.from_numpy(x2).cuda()
    y2 = torch.empty(64, 128, device="cuda")
    rc = L.envg_linear_noalloc(y2.data_ptr(), xt2.data_ptr(), W2.h, None, 64, 16392, 128, envg.EPI_NONE, None,
                               envg.DEVICE_PTRS)
    assert rc == envg.ERR_ARG and "scratch" in envg.last_error()
    W.free()
    W2.free()


_FRESH = r"""
import sys
import torch
from invision_b200 import envg
from tests.common import inputs
envg.init(0)
cases = []
for M, K, N, kind in %r:
    x, w, b = inputs(M, K, N, seed=M + K)
    silu = kind == "silu_gate"
    W = envg.Weight(w, layout=envg.LAYOUT_GATE_UP if silu else envg.LAYOUT_PLAIN)
    epi = envg.EPI_SILU_GATE if silu else (envg.EPI_BIAS if kind == "bias" else envg.EPI_NONE)
    bias = torch.from_numpy(b).cuda() if kind == "bias" else None
    y = torch.empty(M, N // 2 if silu else N, device="cuda")
    cases.append((y, torch.from_numpy(x).cuda(), W, bias, epi))
torch.cuda.synchronize()
free_before = torch.cuda.mem_get_info()[0]
L = envg.lib()
for y, x, W, bias, epi in cases:
    rc = L.envg_linear_noalloc(y.data_ptr(), x.data_ptr(), W.h, bias.data_ptr() if bias is not None else None,
                               x.shape[0], x.shape[1], W.N, epi, None, envg.DEVICE_PTRS)
    if rc != envg.OK:
        sys.exit("rc %%d: %%s" %% (rc, envg.last_error()))
torch.cuda.synchronize()
free_after = torch.cuda.mem_get_info()[0]
print("free", free_before, free_after)
sys.exit(0 if free_after == free_before else "device memory dropped by %%d bytes" %% (free_before - free_after))
"""


def test_noalloc_first_calls_in_a_fresh_process(gpu):
    """The first call of each kernel shape in a new process allocates nothing either: envg_init has
    already loaded the code of every kernel the entry point launches."""
    import os
    import subprocess
    import sys

    cases = CASES + [(33, 1024, 256, "none"), (48, 512, 2 * 128, "silu_gate"), (64, 256, 2 * 64, "silu_gate")]
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _FRESH % (cases,)], cwd=root, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
