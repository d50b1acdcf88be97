"""Generates tests/golden/sgemm2_golden.npz from the reference's own C++ GEMM.

The reference ships no golden vectors for its GEMM.  This script runs src/sgemm2.cpp's
cpp_sgemm (compiled unmodified from the reference tree into oracle/_ref/libsgemm2.so by
oracle/Makefile) on seeded inputs and stores inputs and outputs, so that the restated oracle can
be pinned against the reference's own arithmetic on machines without the reference tree.

    make -C oracle && python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import oracle as O  # noqa: E402

# (op, M, N, K): K a multiple of 128, where sgemm2_nt is complete (sgemm2.cpp:348-395)
CASES = [("nt", 32, 48, 256), ("nt", 17, 9, 128), ("nt", 8, 24, 384), ("nt", 1, 16, 2560),
         ("nn", 24, 40, 128), ("nn", 5, 33, 256)]


def main():
    if O.ref_lib() is None:
        raise SystemExit("oracle/_ref/libsgemm2.so missing: run `make -C oracle` with the reference tree present")
    out = {}
    for i, (op, M, N, K) in enumerate(CASES):
        rng = np.random.default_rng(100 + i)
        a = rng.standard_normal((M, K), dtype=np.float32)
        w = O.bf16_to_f32(O.f32_to_bf16_rne((0.02 * rng.standard_normal((N, K))).astype(np.float32)))
        if op == "nt":
            c = O.sgemm2_nt(a, w, M, N, K)
            b = w
        else:
            b = np.ascontiguousarray(w.T)
            c = O.sgemm2_nn(a, b, M, N, K)
        out[f"c{i}_a"] = a
        out[f"c{i}_b"] = b
        out[f"c{i}_c"] = c
        out[f"c{i}_meta"] = np.array([0 if op == "nt" else 1, M, N, K], np.int64)
    np.savez_compressed(os.path.join(HERE, "sgemm2_golden.npz"), **out)
    print(f"wrote {len(CASES)} cases")


if __name__ == "__main__":
    main()
