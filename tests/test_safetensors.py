"""CPU: the safetensors header parser and host-side reader of libenvgemm.so.

The files are written here byte by byte in the format Envision reads (src/safetensor.pas:466-513):
an 8-byte little-endian header length, the JSON header, then the raw data.  Reading back must
reproduce BF16ToSingle (bits << 16, quicknn_common.pas:1991-2008), FP16ToSingle (exact IEEE
widening) and F32 copies."""
import json
import struct

import numpy as np
import pytest

from invision_b200 import envg
from tests.common import write_safetensors


def bf16_bits(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_widen(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


@pytest.fixture
def stfile(tmp_path):
    rng = np.random.default_rng(5)
    w_bf = bf16_bits(rng.standard_normal((24, 40)).astype(np.float32))
    w_h = rng.standard_normal((8, 16)).astype(np.float16)
    # F16 specials: subnormals, zero signs, inf, largest normal
    w_h.ravel()[:6] = np.array([np.float16(6e-8), np.float16(-3e-5), np.float16(0.0), np.float16(-0.0),
                                np.float16(np.inf), np.float16(65504.0)], np.float16)
    w_f = rng.standard_normal((5, 7)).astype(np.float32)
    conv = bf16_bits(rng.standard_normal((4, 3, 3, 3)).astype(np.float32))
    bias = rng.standard_normal(24).astype(np.float32)
    tensors = {
        "blk.w": ("BF16", w_bf.shape, w_bf.tobytes()),
        "blk.h": ("F16", w_h.shape, w_h.tobytes()),
        "blk.f": ("F32", w_f.shape, w_f.tobytes()),
        "vae.conv": ("BF16", conv.shape, conv.tobytes()),
        "blk.bias": ("F32", bias.shape, bias.tobytes()),
        "q.scale": ("F8_E4M3", [4], bytes(4)),
    }
    p = write_safetensors(str(tmp_path / "m.safetensors"), tensors, metadata={"format": "pt"})
    return p, dict(w_bf=w_bf, w_h=w_h, w_f=w_f, conv=conv, bias=bias)


def test_tensor_info(stfile):
    p, t = stfile
    i = envg.safetensors_tensor_info(p, "blk.w")
    assert i["dtype"] == envg.DTYPE_BF16 and i["dtype_name"] == "BF16"
    assert i["shape"] == [24, 40] and i["nbytes"] == 24 * 40 * 2
    with open(p, "rb") as f:
        f.seek(i["offset"])
        assert f.read(i["nbytes"]) == t["w_bf"].tobytes()
    assert envg.safetensors_tensor_info(p, "vae.conv")["shape"] == [4, 3, 3, 3]
    assert envg.safetensors_tensor_info(p, "blk.h")["dtype"] == envg.DTYPE_F16
    q = envg.safetensors_tensor_info(p, "q.scale")
    assert q["dtype"] == envg.DTYPE_OTHER and q["dtype_name"] == "F8_E4M3"


def test_read_f32_matches_reference_widening(stfile):
    p, t = stfile
    np.testing.assert_array_equal(envg.safetensors_read_f32(p, "blk.w"), bf16_widen(t["w_bf"]))
    np.testing.assert_array_equal(envg.safetensors_read_f32(p, "blk.h"), t["w_h"].astype(np.float32))
    np.testing.assert_array_equal(envg.safetensors_read_f32(p, "blk.f"), t["w_f"])
    np.testing.assert_array_equal(envg.safetensors_read_f32(p, "blk.bias"), t["bias"])


def test_f16_widening_exhaustive(tmp_path):
    """All 65536 half bit patterns widen exactly as IEEE says (NaNs stay NaN)."""
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    p = write_safetensors(str(tmp_path / "h.safetensors"), {"h": ("F16", [65536], h.tobytes())})
    got = envg.safetensors_read_f32(p, "h")
    want = h.astype(np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_unaligned_data_section(tmp_path):
    """The format does not promise aligned data; an odd header length must still read right."""
    rng = np.random.default_rng(1)
    f = rng.standard_normal(33).astype(np.float32)
    b = bf16_bits(rng.standard_normal(9).astype(np.float32))
    p = write_safetensors(str(tmp_path / "u.safetensors"), {"b": ("BF16", [9], b.tobytes()),
                                                            "f": ("F32", [33], f.tobytes())},
                          pad_to=0, extra_header_bytes=3)
    assert envg.safetensors_tensor_info(p, "f")["offset"] % 4 != 0
    np.testing.assert_array_equal(envg.safetensors_read_f32(p, "f"), f)
    np.testing.assert_array_equal(envg.safetensors_read_f32(p, "b"), bf16_widen(b))


def test_errors(stfile, tmp_path):
    p, _ = stfile
    with pytest.raises(envg.EnvgError) as e:
        envg.safetensors_tensor_info(p, "nope")
    assert e.value.code == envg.ERR_ARG and "not found" in str(e.value)
    with pytest.raises(envg.EnvgError) as e:
        envg.safetensors_read_f32(p, "q.scale")
    assert e.value.code == envg.ERR_UNSUPPORTED
    with pytest.raises(envg.EnvgError):
        envg.safetensors_tensor_info(str(tmp_path / "missing.safetensors"), "x")
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(struct.pack("<Q", 1 << 40) + b"{}")
    with pytest.raises(envg.EnvgError) as e:
        envg.safetensors_tensor_info(str(bad), "x")
    assert "header length" in str(e.value)
    short = tmp_path / "short.safetensors"
    hj = json.dumps({"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}).encode()
    short.write_bytes(struct.pack("<Q", len(hj)) + hj + bytes(8))
    with pytest.raises(envg.EnvgError) as e:
        envg.safetensors_tensor_info(str(short), "x")
    assert "outside the file" in str(e.value)
    mism = tmp_path / "mism.safetensors"
    hj = json.dumps({"x": {"dtype": "BF16", "shape": [4, 4], "data_offsets": [0, 16]}}).encode()
    mism.write_bytes(struct.pack("<Q", len(hj)) + hj + bytes(16))
    with pytest.raises(envg.EnvgError) as e:
        envg.safetensors_read_f32(str(mism), "x")
    assert "elements" in str(e.value)


def test_upload_needs_init(stfile):
    """The upload entry is a device operation: without envg_init it reports a state error."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("checks the uninitialised state")
    p, _ = stfile
    with pytest.raises(envg.EnvgError) as e:
        envg.Weight.from_safetensors(p, "blk.w")
    assert e.value.code == envg.ERR_STATE
