"""envg_linear_batch on host pointers: the linears' copies and GEMMs overlap, and every output
must be bit-identical to the same linear called alone through envg_linear with host pointers
(which the parity tests pin to the oracle), including the row-chunked path from 1024 rows on,
a shared input, the SiLU-gate, the gated residual and the M <= 8 CUDA-core path.  One case per
fallback: outputs that overlap, and a later linear reading an earlier one's output."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.common import assert_parity

pytestmark = pytest.mark.gpu


def _w(rng, n, k):
    """bf16 weight bits, as a checkpoint holds them."""
    return O.f32_to_bf16_rne((0.02 * rng.standard_normal((n, k))).astype(np.float32))


def _alone(gpu, c):
    y = c["dst0"].copy()
    gpu.linear(y, c["x"], c["W"], bias=c.get("bias"), epilogue=c.get("epilogue"), gate=c.get("gate"))
    return y


def test_host_batch_matches_single_calls(gpu):
    rng = np.random.default_rng(11)
    x1 = rng.standard_normal((1536, 512)).astype(np.float32)   # chunked (>= 1024 rows), shared
    x2 = rng.standard_normal((300, 1024)).astype(np.float32)
    x3 = rng.standard_normal((4, 768)).astype(np.float32)      # M <= 8: k_gemv
    x4 = rng.standard_normal((40, 256)).astype(np.float32)     # skinny k2 path
    wa = _w(rng, 640, 512)
    Wa = gpu.Weight(wa)
    Wb = gpu.Weight((0.02 * rng.standard_normal((384, 512))).astype(np.float32))  # fp32: the bf16x3 path
    Wgu = gpu.Weight(_w(rng, 512, 1024), layout=gpu.LAYOUT_GATE_UP)
    Wc = gpu.Weight(_w(rng, 1000, 768))
    Wd = gpu.Weight(_w(rng, 136, 256))
    ba = rng.standard_normal(640).astype(np.float32)
    gate = rng.standard_normal(136).astype(np.float32)
    calls = [
        dict(x=x1, W=Wa, bias=ba, dst0=np.full((1536, 640), np.nan, np.float32)),
        dict(x=x1, W=Wb, dst0=np.full((1536, 384), np.nan, np.float32)),
        dict(x=x2, W=Wgu, dst0=np.full((300, 256), np.nan, np.float32)),
        dict(x=x3, W=Wc, dst0=np.full((4, 1000), np.nan, np.float32)),
        dict(x=x4, W=Wd, epilogue=gpu.EPI_GATED_RESIDUAL, gate=gate,
             dst0=rng.standard_normal((40, 136)).astype(np.float32)),
    ]
    ref = [_alone(gpu, c) for c in calls]
    for c in calls:
        c["dst"] = c["dst0"].copy()
    before = gpu.stats()
    gpu.linear_batch(calls)
    after = gpu.stats()
    for i, (c, r) in enumerate(zip(calls, ref)):
        assert np.array_equal(c["dst"], r, equal_nan=True), f"linear {i} differs from its single call"
    assert after["calls"] - before["calls"] == len(calls)
    # the shared input crossed PCIe once
    h2d = after["h2d_bytes"] - before["h2d_bytes"]
    expect = (x1.nbytes + x2.nbytes + x3.nbytes + x4.nbytes + ba.nbytes + gate.nbytes + calls[4]["dst0"].nbytes)
    assert h2d == expect
    # and the chunked linear still agrees with the oracle
    assert_parity(calls[0]["dst"], O.linear_bf16(x1, wa, ba, path=O.PATH_AVX2), what="host batch, chunked")
    for W in (Wa, Wb, Wgu, Wc, Wd):
        W.free()


def test_host_batch_falls_back_on_overlap(gpu):
    rng = np.random.default_rng(12)
    x = rng.standard_normal((64, 256)).astype(np.float32)
    W1 = gpu.Weight(_w(rng, 256, 256))
    W2 = gpu.Weight(_w(rng, 128, 256))
    # linear 2 reads linear 1's output: it must see the finished values
    y1 = np.full((64, 256), np.nan, np.float32)
    y2 = np.full((64, 128), np.nan, np.float32)
    gpu.linear_batch([dict(x=x, W=W1, dst=y1), dict(x=y1, W=W2, dst=y2)])
    r1 = np.full_like(y1, np.nan)
    gpu.linear(r1, x, W1)
    r2 = np.full_like(y2, np.nan)
    gpu.linear(r2, r1, W2)
    assert np.array_equal(y1, r1) and np.array_equal(y2, r2)
    # two outputs in one buffer, overlapping: the later linear's values win, as in two calls
    buf = np.full((64, 256), np.nan, np.float32)
    gpu.linear_batch([dict(x=x, W=W1, dst=buf), dict(x=x, W=W1, dst=buf)])
    assert np.array_equal(buf, r1)
    W1.free()
    W2.free()
