"""CPU: the product library loads, exports every entry point include/envgemm.h declares, and
fails with status codes (not crashes) when no GPU is present or it is not initialised."""
import ctypes
import subprocess

import numpy as np
import pytest

from invision_b200 import envg


def test_library_exports_every_header_symbol():
    L = envg.lib()
    names = envg.header_symbols()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/envgemm.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", envg.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(names) <= exported


def test_version_string():
    assert "sm_100a" in envg.version()


def _no_gpu():
    try:
        import torch

        return not torch.cuda.is_available()
    except Exception:
        return True


@pytest.mark.skipif(not _no_gpu(), reason="checks the no-GPU behaviour")
def test_init_without_gpu_returns_cuda_error():
    L = envg.lib()
    ids = (ctypes.c_int * 1)(0)
    assert L.envg_init(1, ids) == envg.ERR_CUDA
    assert envg.last_error()


def test_multi_device_init_is_refused():
    L = envg.lib()
    ids = (ctypes.c_int * 2)(0, 1)
    assert L.envg_init(2, ids) == envg.ERR_UNSUPPORTED


@pytest.mark.skipif(not _no_gpu(), reason="checks the uninitialised state")
def test_calls_before_init_return_state_error():
    L = envg.lib()
    y = np.zeros((4, 4), np.float32)
    assert L.envg_linear(y.ctypes.data, y.ctypes.data, None, None, 4, 4, 4, 0, None, 0) == envg.ERR_STATE
    assert "envg_init" in envg.last_error()
    assert L.envg_sync() == envg.ERR_STATE
    assert L.envg_sgemm(101, 111, 112, 4, 4, 4, 1.0, y.ctypes.data, 4, y.ctypes.data, 4, 0.0, y.ctypes.data, 4) \
        == envg.ERR_STATE
    assert L.envg_weight_free(None) == envg.ERR_STATE


def test_mirror_asserts_like_the_reference():
    with pytest.raises(AssertionError, match="no weight"):
        envg.QNNLINEAR_BF16_OR_F32(None, None, None, None, 1, 1, 1)


@pytest.mark.skipif(not _no_gpu(), reason="checks the no-GPU behaviour")
def test_cpp_harness_links_and_fails_cleanly_without_gpu(tmp_path):
    """A C++ host compiled against include/quicknn_cuda.hpp links the .so and gets status codes /
    exceptions (not crashes) when no sm_100 GPU is present."""
    from tests.abi.build_harness import build

    exe = build(str(tmp_path))
    r = subprocess.run([exe, "nogpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
