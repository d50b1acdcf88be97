"""GPU: the C++ harness (tests/abi/abi_harness.cpp) drives the library through the QNN-named C++
mirror (include/quicknn_cuda.hpp) with host pointers, as a compiled host would."""
import subprocess

import pytest

pytestmark = pytest.mark.gpu


def test_cpp_harness_on_gpu(tmp_path):
    from tests.abi.build_harness import build

    exe = build(str(tmp_path))
    r = subprocess.run([exe, "gpu"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
