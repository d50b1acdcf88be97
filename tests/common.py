"""Seeded synthetic inputs and the acceptance check shared by the parity tests."""
import json
import os
import struct

import numpy as np

from oracle import oracle as O

# Acceptance bounds for the bf16-operand / fp32-accumulate GEMM against the reference's fp32 CPU
# GEMM: max|d| / max|ref| <= 1e-2 and sum|d| / sum|ref| <= 2e-3.
TOL_MAX = 1e-2
TOL_MEAN = 2e-3


def inputs(M, K, N, seed, bias=True):
    """X ~ N(0,1) fp32, W = bf16_rne(0.02 N(0,1)) as bits, b ~ 0.01 N(0,1) fp32."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = O.f32_to_bf16_rne((0.02 * rng.standard_normal((N, K))).astype(np.float32))
    b = (0.01 * rng.standard_normal(N)).astype(np.float32) if bias else None
    return x, w, b


# bf16x3 operands (fp32 weights that are not bf16 numbers, and envg_sgemm): hi/lo parts make the
# tensor-core product match the reference's fp32 GEMM to about 1e-5 relative.  These bounds, 10-20x
# below the acceptance bounds, show that no bf16 rounding of either operand is left (rounding one
# fp32 operand to bf16 alone gives a mean-rel near 1.5e-3).
TOL_X3_MAX = 1e-3
TOL_X3_MEAN = 1e-4

# A fused epilogue that multiplies two GEMM outputs (SiLU-gate: silu(g) * u) carries the relative
# error of both factors, so its output is held to twice the GEMM bounds; the GEMM halves feeding
# it are checked separately at TOL_MAX / TOL_MEAN.
TOL_MAX_PRODUCT = 2 * TOL_MAX
TOL_MEAN_PRODUCT = 2 * TOL_MEAN


def _log(what, mx, mean):
    path = os.environ.get("ENVG_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"case": what, "max_rel": mx, "mean_rel": mean}) + "\n")


def assert_parity(y, ref, tol_max=TOL_MAX, tol_mean=TOL_MEAN, what=""):
    assert y.shape == ref.shape, (y.shape, ref.shape)
    assert np.isfinite(y).all(), f"{what}: non-finite output"
    mx, mean = O.parity_stats(y, ref)
    _log(what, mx, mean)
    assert mx <= tol_max and mean <= tol_mean, f"{what}: max-rel {mx:.3e} (<= {tol_max}), mean-rel {mean:.3e} (<= {tol_mean})"
    return mx, mean


def write_safetensors(path, tensors, pad_to=8, metadata=None, extra_header_bytes=0):
    """tensors: {name: (dtype_str, shape, raw_bytes)} in file order."""
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, (dt, shape, raw) in tensors.items():
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hj = json.dumps(header).encode()
    if pad_to:
        hj += b" " * ((-(8 + len(hj))) % pad_to)
    hj += b" " * extra_header_bytes
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)
    return path
