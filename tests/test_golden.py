"""CPU: pin the restated oracle to outputs of the reference's own sgemm2.cpp (fixtures made by
tests/golden/make_golden.py; the reference ships no golden vectors of its own)."""
import os

import numpy as np
import pytest

from oracle import oracle as O

FIX = os.path.join(os.path.dirname(__file__), "golden", "sgemm2_golden.npz")


def cases():
    z = np.load(FIX)
    n = len([k for k in z.files if k.endswith("_meta")])
    return [(z[f"c{i}_meta"], z[f"c{i}_a"], z[f"c{i}_b"], z[f"c{i}_c"]) for i in range(n)]


@pytest.mark.parametrize("idx", range(6))
def test_oracle_matches_reference_sgemm2_golden(idx):
    meta, a, b, c = cases()[idx]
    op, M, N, K = (int(v) for v in meta)
    out = np.zeros((M, N), np.float32)
    if op == 0:
        O.qgemm(O.NO_TRANS, O.TRANS, M, N, K, 1.0, a, K, b, K, 0.0, out, N, path=O.PATH_AVX2)
    else:
        O.qgemm(O.NO_TRANS, O.NO_TRANS, M, N, K, 1.0, a, K, b, N, 0.0, out, N, path=O.PATH_AVX2)
    mx, mean = O.parity_stats(out, c)
    assert mx < 2e-6 and mean < 1e-6, (mx, mean)


def test_golden_reproduced_by_reference_build():
    """When the reference's sgemm2 is built here, it reproduces the fixtures bit for bit."""
    if O.ref_lib() is None:
        pytest.skip("oracle/_ref/libsgemm2.so not built")
    for meta, a, b, c in cases():
        op, M, N, K = (int(v) for v in meta)
        got = O.sgemm2_nt(a, b, M, N, K) if op == 0 else O.sgemm2_nn(a, b, M, N, K)
        np.testing.assert_array_equal(got, c)
