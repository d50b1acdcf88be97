"""ctypes binding of libenvgemm.so (the C ABI in include/envgemm.h) plus a mirror of Envision's
QNN operator names for this path.

Two calling modes, picked from the argument types:

* numpy arrays  -> host pointers (``ENVG_HOST_PTRS``): the library copies inputs to the GPU,
  runs, copies the result back and synchronises -- what the Pascal host does;
* torch CUDA tensors -> device pointers (``ENVG_DEVICE_PTRS``) on the current torch stream.

There is no CPU fallback: if the shared library is missing or the GPU is absent, calls raise
``EnvgError``.  The QNN-named mirror functions (``QNNLinear`` and friends) keep the reference's
argument order and meaning (``src/quicknn_kernels.pas``) and raise ``AssertionError`` with an
``ERROR ...`` message where the reference asserts.
"""
import ctypes
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libenvgemm.so")
HEADER_PATH = os.path.join(os.path.dirname(HERE), "include", "envgemm.h")

OK = 0
ERR_ARG, ERR_OOM, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT, ERR_STATE, ERR_UNSUPPORTED = -1, -2, -3, -4, -5, -6, -7
LAYOUT_PLAIN, LAYOUT_GATE_UP, LAYOUT_ROUND_BF16 = 0, 1, 4
EPI_NONE, EPI_BIAS, EPI_SILU_GATE, EPI_GATED_RESIDUAL, EPI_SILU = 0, 1, 2, 3, 4
HOST_PTRS, DEVICE_PTRS, ASYNC, KEEP_SHARDED = 0, 1, 2, 4
ROW_MAJOR, NO_TRANS, TRANS = 101, 111, 112
DTYPE_OTHER, DTYPE_BF16, DTYPE_F16, DTYPE_F32 = 0, 1, 2, 3
CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy


class EnvgError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"envgemm error {code}: {msg}")
        self.code = code


class KernelStat(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("launches", ctypes.c_uint64), ("ms", ctypes.c_double),
                ("flops", ctypes.c_double), ("bytes", ctypes.c_double)]


class LinearDesc(ctypes.Structure):
    _fields_ = [("dst", ctypes.c_void_p), ("x", ctypes.c_void_p), ("W", ctypes.c_void_p), ("bias", ctypes.c_void_p),
                ("M", ctypes.c_int64), ("K", ctypes.c_int64), ("N", ctypes.c_int64), ("epilogue", ctypes.c_int),
                ("gate", ctypes.c_void_p)]


class TensorInfo(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int), ("ndim", ctypes.c_int), ("shape", ctypes.c_int64 * 8),
                ("offset", ctypes.c_int64), ("nbytes", ctypes.c_int64), ("dtype_name", ctypes.c_char * 16)]


class ResBlockDesc(ctypes.Structure):
    _fields_ = [("in_ch", ctypes.c_int), ("out_ch", ctypes.c_int),
                ("norm1_gamma", ctypes.c_void_p), ("norm1_beta", ctypes.c_void_p),
                ("conv1", ctypes.c_void_p), ("conv1_bias", ctypes.c_void_p),
                ("norm2_gamma", ctypes.c_void_p), ("norm2_beta", ctypes.c_void_p),
                ("conv2", ctypes.c_void_p), ("conv2_bias", ctypes.c_void_p),
                ("skip", ctypes.c_void_p), ("skip_bias", ctypes.c_void_p)]


class NsplitDesc(ctypes.Structure):
    _fields_ = [("lin", LinearDesc), ("y_peers", ctypes.POINTER(ctypes.c_void_p)), ("npeers", ctypes.c_int),
                ("y_multicast", ctypes.c_void_p), ("ldy", ctypes.c_int64), ("col0", ctypes.c_int64)]


class Stats(ctypes.Structure):
    _fields_ = [("calls", ctypes.c_uint64), ("kernel_launches", ctypes.c_uint64), ("flops", ctypes.c_double),
                ("h2d_bytes", ctypes.c_double), ("d2h_bytes", ctypes.c_double), ("weight_bytes", ctypes.c_uint64),
                ("workspace_bytes", ctypes.c_uint64), ("device", ctypes.c_int32), ("last_status", ctypes.c_int32)]


_lib = None
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_ci = ctypes.c_int


def lib():
    """Load libenvgemm.so (fails loudly when it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise EnvgError(ERR_STATE, f"{LIB_PATH} not built: run `python -c 'import __graft_entry__ as g; g.build()'`")
        L = ctypes.CDLL(LIB_PATH)
        L.envg_version.restype = ctypes.c_char_p
        L.envg_last_error.restype = ctypes.c_char_p
        L.envg_init.argtypes = [_ci, ctypes.POINTER(_ci)]
        L.envg_weight_upload.argtypes = [_vp, _vp, _i64, _i64, _ci, ctypes.POINTER(_vp)]
        L.envg_weight_upload_shard.argtypes = [_vp, _vp, _i64, _i64, _i64, _i64, _ci, ctypes.POINTER(_vp)]
        L.envg_conv_weight_upload.argtypes = [_vp, _vp, _ci, _ci, _ci, _ci, ctypes.POINTER(_vp)]
        L.envg_weight_free.argtypes = [_vp]
        L.envg_safetensors_tensor_info.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(TensorInfo)]
        L.envg_safetensors_read_f32.argtypes = [ctypes.c_char_p, ctypes.c_char_p, _vp, _i64]
        L.envg_weight_upload_safetensors.argtypes = [ctypes.c_char_p, ctypes.c_char_p, _ci, _i64, _i64,
                                                     ctypes.POINTER(_vp)]
        L.envg_linear.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _ci, _vp, _ci]
        L.envg_linear_noalloc.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _ci, _vp, _ci]
        L.envg_linear_batch.argtypes = [ctypes.POINTER(LinearDesc), _ci, _ci]
        L.envg_linear_nsplit_batch.argtypes = [ctypes.POINTER(NsplitDesc), _ci, _ci]
        L.envg_linear_adaln.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _ci, _vp, _ci]
        L.envg_linear_rmsnorm.argtypes = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _ci, _vp, _ci]
        L.envg_linear_nsplit.argtypes = [_vp, ctypes.POINTER(_vp), _ci, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _i64,
                                         _i64, _ci, _vp, _ci]
        L.envg_conv2d.argtypes = [_vp, _vp, _vp, _vp] + [_ci] * 11
        L.envg_group_norm.argtypes = [_vp, _vp, _vp, _vp] + [_ci] * 7
        L.envg_attention.argtypes = [_vp, _vp, _vp, _vp] + [_ci] * 5 + [_i64] * 4 + [ctypes.c_float, _ci, _vp, _ci]
        L.envg_vae_resblock.argtypes = [_vp, _vp, ctypes.POINTER(ResBlockDesc), _ci, _ci, _ci, _ci, _ci]
        L.envg_sgemm.argtypes = [_ci, _ci, _ci, _i64, _i64, _i64, ctypes.c_float, _vp, _i64, _vp, _i64,
                                 ctypes.c_float, _vp, _i64]
        L.envg_set_stream.argtypes = [_vp]
        L.envg_get_stats.argtypes = [ctypes.POINTER(Stats)]
        L.envg_set_wait_cap_ns.argtypes = [ctypes.c_uint64]
        L.envg_selftest_wait_timeout.argtypes = [ctypes.c_uint64]
        L.envg_profile.argtypes = [_ci]
        L.envg_profile_read.argtypes = [ctypes.POINTER(KernelStat), _ci, ctypes.POINTER(_ci)]
        _lib = L
    return _lib


def header_symbols():
    """Names of every entry point declared in include/envgemm.h."""
    with open(HEADER_PATH) as f:
        txt = f.read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(envg_\w+)\s*\(", txt, re.M)))


def last_error():
    return lib().envg_last_error().decode()


def version():
    return lib().envg_version().decode()


def _check(rc):
    if rc != OK:
        raise EnvgError(rc, last_error())
    return rc


def init(device=0):
    ids = (_ci * 1)(device)
    return _check(lib().envg_init(1, ids))


def shutdown():
    return _check(lib().envg_shutdown())


def sync():
    return _check(lib().envg_sync())


def stats():
    s = Stats()
    _check(lib().envg_get_stats(ctypes.byref(s)))
    return {f: getattr(s, f) for f, _ in Stats._fields_}


def profile(enable):
    """Start (resetting the counters) or stop per-launch CUDA-event timing inside the library."""
    return _check(lib().envg_profile(1 if enable else 0))


def profile_read():
    """{kernel family: {launches, ms, flops, bytes}} accumulated since profile(True)."""
    arr = (KernelStat * 32)()
    n = _ci(0)
    _check(lib().envg_profile_read(arr, 32, ctypes.byref(n)))
    return {arr[i].name.decode(): {"launches": arr[i].launches, "ms": arr[i].ms, "flops": arr[i].flops,
                                   "bytes": arr[i].bytes} for i in range(n.value)}


def set_stream(stream_handle):
    """Launch on a caller stream (an int cudaStream_t, e.g. torch.cuda.Stream().cuda_stream) or,
    with None, on the library's own stream."""
    return _check(lib().envg_set_stream(_vp(stream_handle) if stream_handle is not None else None))


def set_wait_cap_ns(ns):
    return _check(lib().envg_set_wait_cap_ns(int(ns)))


def selftest_wait_timeout(cap_ns):
    """Return code of the bounded-wait self-test (ERR_TIMEOUT when the bound works)."""
    return lib().envg_selftest_wait_timeout(int(cap_ns))


def _is_torch(t):
    return type(t).__module__.startswith("torch")


def _ptr(a):
    if a is None:
        return None
    if _is_torch(a):
        return a.data_ptr()
    return a.ctypes.data


def _host_f32(a, name):
    if not (isinstance(a, np.ndarray) and a.dtype == np.float32 and a.flags.c_contiguous):
        raise TypeError(f"{name}: expected a C-contiguous float32 numpy array")
    return a


_follow_torch_stream = True


def follow_torch_stream(on):
    """Device-pointer calls launch on torch's current stream (default) or on whatever stream
    set_stream() selected (on=False)."""
    global _follow_torch_stream
    _follow_torch_stream = bool(on)


def _mode(*arrays):
    """HOST_PTRS for numpy operands, DEVICE_PTRS for torch CUDA tensors (never mixed)."""
    kinds = {(_is_torch(a)) for a in arrays if a is not None}
    if len(kinds) != 1:
        raise TypeError("operands must be all numpy (host) or all torch CUDA tensors (device)")
    if kinds.pop():
        import torch

        for a in arrays:
            if a is None:
                continue
            if not (a.is_cuda and a.dtype == torch.float32 and a.is_contiguous()):
                raise TypeError("device operands must be contiguous float32 CUDA tensors")
        if _follow_torch_stream:
            h = torch.cuda.current_stream().cuda_stream
            # torch's default stream has handle 0, which the C ABI reads as "the library's own
            # stream"; name it as cudaStreamLegacy (0x1) so both order on the same stream.
            lib().envg_set_stream(_vp(h if h else CUDA_STREAM_LEGACY))
        return DEVICE_PTRS
    for a in arrays:
        if a is not None:
            _host_f32(a, "operand")
    return HOST_PTRS


class Weight:
    """A device-resident bf16 weight (envg_weight handle).

    ``w`` is W[N, K] row-major as numpy uint16 (raw bf16 bits) or float32.  A float32 weight
    whose values are all bf16 numbers is stored as bf16; any other keeps its precision as a
    bf16x3 split (hi / lo parts, three times the tensor-core work), unless ``layout`` has
    ``LAYOUT_ROUND_BF16`` OR-ed in, which rounds it to bf16 (RNE).  ``shard=(n0, n1)`` uploads only
    output rows [n0, n1)
    (for GATE_UP: gate rows [n0, n1) and the same up rows).  ``conv=(out_ch, in_ch, kH, kW)``
    uploads a convolution weight [out_ch, in_ch, kH, kW].
    """

    def __init__(self, w, layout=LAYOUT_PLAIN, shard=None, conv=None):
        self.h = None
        if w is None:  # filled in by from_safetensors
            return
        w = np.ascontiguousarray(w)
        if w.dtype == np.uint16:
            pb, pf = w.ctypes.data, None
        elif w.dtype == np.float32:
            pb, pf = None, w.ctypes.data
        else:
            raise TypeError("weight must be uint16 (bf16 bits) or float32")
        h = _vp()
        L = lib()
        kind = layout & ~LAYOUT_ROUND_BF16
        if conv is not None:
            O, C, kH, kW = conv
            assert w.size == O * C * kH * kW, "ERROR : conv weight size mismatch"
            _check(L.envg_conv_weight_upload(pb, pf, O, C, kH, kW, ctypes.byref(h)))
            self.N, self.K = O, C * kH * kW
        else:
            N, K = w.shape
            if shard is None:
                _check(L.envg_weight_upload(pb, pf, N, K, layout, ctypes.byref(h)))
                self.N = N
            else:
                n0, n1 = shard
                _check(L.envg_weight_upload_shard(pb, pf, N, K, n0, n1, layout, ctypes.byref(h)))
                self.N = (n1 - n0) * (2 if kind == LAYOUT_GATE_UP else 1)
            self.K = K
        self.layout = kind
        self.conv = conv
        self.h = h

    @classmethod
    def from_safetensors(cls, path, name, layout=LAYOUT_PLAIN, shard=None):
        """Upload tensor ``name`` of a ``.safetensors`` file (envg_weight_upload_safetensors).

        A 2-D tensor [N, K] becomes a linear weight (``layout``, ``shard`` as in the constructor);
        a 4-D tensor [out_ch, in_ch, kH, kW] a convolution weight."""
        info = safetensors_tensor_info(path, name)
        n0, n1 = shard if shard is not None else (0, 0)
        h = _vp()
        _check(lib().envg_weight_upload_safetensors(os.fsencode(path), name.encode(), layout, n0, n1,
                                                    ctypes.byref(h)))
        self = cls(None)
        shape = info["shape"]
        if len(shape) == 4:
            self.conv = tuple(shape)
            self.N, self.K = shape[0], shape[1] * shape[2] * shape[3]
        else:
            self.conv = None
            rows = shape[0] if shard is None else (n1 - n0) * (2 if layout & 3 == LAYOUT_GATE_UP else 1)
            self.N, self.K = rows, shape[1]
        self.layout = layout & ~LAYOUT_ROUND_BF16
        self.h = h
        return self

    def free(self):
        if self.h is not None and self.h.value:
            _check(lib().envg_weight_free(self.h))
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def safetensors_tensor_info(path, name):
    """Header entry of tensor ``name`` (envg_safetensors_tensor_info; needs no GPU)."""
    info = TensorInfo()
    _check(lib().envg_safetensors_tensor_info(os.fsencode(path), name.encode(), ctypes.byref(info)))
    return {"dtype": info.dtype, "dtype_name": info.dtype_name.decode(), "shape": [info.shape[i] for i in range(info.ndim)],
            "offset": info.offset, "nbytes": info.nbytes}


def safetensors_read_f32(path, name):
    """Tensor ``name`` widened to fp32 on the host (envg_safetensors_read_f32; needs no GPU)."""
    shape = safetensors_tensor_info(path, name)["shape"]
    out = np.empty(shape, dtype=np.float32)
    _check(lib().envg_safetensors_read_f32(os.fsencode(path), name.encode(), out.ctypes.data, out.size))
    return out


def linear(dst, x, W, bias=None, epilogue=None, gate=None, sync=True):
    """dst = epilogue(x . W^T): envg_linear.  x [M, K]; dst [M, N] (N/2 for SILU_GATE)."""
    if epilogue is None:
        epilogue = EPI_SILU_GATE if W.layout == LAYOUT_GATE_UP else (EPI_BIAS if bias is not None else EPI_NONE)
    flags = _mode(dst, x, bias, gate)
    if flags == DEVICE_PTRS and not sync:
        flags |= ASYNC
    M, K = x.shape
    return _check(lib().envg_linear(_ptr(dst), _ptr(x), W.h, _ptr(bias), M, K, W.N, epilogue, _ptr(gate), flags))


def linear_adaln(dst, x, shift, scale, W, bias=None, epilogue=None, gate=None, sync=True):
    """dst = epilogue(AdaLN(x; shift, scale) . W^T): envg_linear_adaln (QNNAdaLN fused into the cast)."""
    if epilogue is None:
        epilogue = EPI_SILU_GATE if W.layout == LAYOUT_GATE_UP else (EPI_BIAS if bias is not None else EPI_NONE)
    flags = _mode(dst, x, shift, scale, bias, gate)
    if flags == DEVICE_PTRS and not sync:
        flags |= ASYNC
    M, K = x.shape
    return _check(lib().envg_linear_adaln(_ptr(dst), _ptr(x), _ptr(shift), _ptr(scale), W.h, _ptr(bias), M, K, W.N,
                                          epilogue, _ptr(gate), flags))


def linear_rmsnorm(dst, x, W, weight=None, bias=None, epilogue=None, gate=None, sync=True):
    """dst = epilogue(RMSNorm(x; weight) . W^T): envg_linear_rmsnorm (QNNRMSNormRows fused into the
    cast); weight None normalises without a per-column scale."""
    if epilogue is None:
        epilogue = EPI_SILU_GATE if W.layout == LAYOUT_GATE_UP else (EPI_BIAS if bias is not None else EPI_NONE)
    flags = _mode(dst, x, weight, bias, gate)
    if flags == DEVICE_PTRS and not sync:
        flags |= ASYNC
    M, K = x.shape
    return _check(lib().envg_linear_rmsnorm(_ptr(dst), _ptr(x), _ptr(weight), W.h, _ptr(bias), M, K, W.N, epilogue,
                                            _ptr(gate), flags))


def linear_noalloc(dst, x, W, bias=None, epilogue=None, gate=None, sync=True):
    """dst = epilogue(x . W^T) through envg_linear_noalloc, which allocates no device memory (its
    scratch is a fixed array in the library).  Torch CUDA tensors only; M <= 64."""
    if epilogue is None:
        epilogue = EPI_SILU_GATE if W.layout == LAYOUT_GATE_UP else (EPI_BIAS if bias is not None else EPI_NONE)
    flags = _mode(dst, x, bias, gate)
    if flags != DEVICE_PTRS:
        raise TypeError("linear_noalloc takes torch CUDA tensors (device pointers) only")
    if not sync:
        flags |= ASYNC
    M, K = x.shape
    return _check(lib().envg_linear_noalloc(_ptr(dst), _ptr(x), W.h, _ptr(bias), M, K, W.N, epilogue, _ptr(gate),
                                            flags))


def linear_batch(calls, sync=True):
    """Several linears in one envg_linear_batch call.  `calls` is a list of dicts with keys dst,
    x, W and optionally bias, epilogue, gate, all torch CUDA tensors (each distinct x is cast once
    and the casts overlap the previous GEMM on a second stream) or all numpy arrays (host
    pointers: the linears' copies in and out overlap one another and the GEMMs; synchronous)."""
    arr = (LinearDesc * len(calls))()
    keep = []
    modes = set()
    for i, c in enumerate(calls):
        W = c["W"]
        bias, gate = c.get("bias"), c.get("gate")
        epi = c.get("epilogue")
        if epi is None:
            epi = EPI_SILU_GATE if W.layout == LAYOUT_GATE_UP else (EPI_BIAS if bias is not None else EPI_NONE)
        modes.add(_mode(c["dst"], c["x"], bias, gate))
        M, K = c["x"].shape
        arr[i] = LinearDesc(_ptr(c["dst"]), _ptr(c["x"]), W.h, _ptr(bias), M, K, W.N, epi, _ptr(gate))
        keep.append(c)
    if len(modes) > 1:
        raise TypeError("a batch's operands must be all numpy (host) or all torch CUDA tensors (device)")
    if modes == {HOST_PTRS}:
        return _check(lib().envg_linear_batch(arr, len(calls), HOST_PTRS))
    flags = DEVICE_PTRS | (0 if sync else ASYNC)
    return _check(lib().envg_linear_batch(arr, len(calls), flags))


def linear_nsplit_batch(calls, sync=True):
    """Several N-split shards in one envg_linear_nsplit_batch call.  `calls`: dicts with keys
    y (this rank's copy of Y), x, W (the shard), col0 and peers (list of int pointers) or
    multicast, plus optional bias, epilogue, gate.  Synchronise the ranks before reading Y."""
    arr = (NsplitDesc * len(calls))()
    keep = []
    for i, c in enumerate(calls):
        W = c["W"]
        bias, gate = c.get("bias"), c.get("gate")
        epi = c.get("epilogue")
        if epi is None:
            epi = EPI_SILU_GATE if W.layout == LAYOUT_GATE_UP else (EPI_BIAS if bias is not None else EPI_NONE)
        _mode(c["y"], c["x"], bias, gate)
        M, K = c["x"].shape
        plist = list(c.get("peers") or [])
        parr = (_vp * max(1, len(plist)))(*[_vp(p) for p in plist]) if plist else None
        mc = c.get("multicast") or 0
        arr[i] = NsplitDesc(LinearDesc(_ptr(c["y"]), _ptr(c["x"]), W.h, _ptr(bias), M, K, W.N, epi, _ptr(gate)),
                            ctypes.cast(parr, ctypes.POINTER(ctypes.c_void_p)) if parr is not None else None,
                            len(plist), _vp(mc) if mc else None, c["y"].shape[1], c["col0"])
        keep.append((c, parr))
    flags = DEVICE_PTRS | (0 if sync else ASYNC)
    return _check(lib().envg_linear_nsplit_batch(arr, len(calls), flags))


def linear_nsplit(y_local, x, W, col0, peers=None, multicast=0, bias=None, epilogue=None, gate=None, sync=True):
    """This rank's shard of an N-split linear, writing its columns [col0, col0 + width) into every
    rank's copy of Y (torch CUDA tensors; `peers` = list of int device pointers of all ranks' Y,
    `multicast` = NVLS multicast address or 0).  Synchronise the ranks before reading Y."""
    if epilogue is None:
        epilogue = EPI_SILU_GATE if W.layout == LAYOUT_GATE_UP else (EPI_BIAS if bias is not None else EPI_NONE)
    _mode(y_local, x, bias, gate)
    M, K = x.shape
    ldy = y_local.shape[1]
    plist = list(peers or [])
    arr = (_vp * max(1, len(plist)))(*[_vp(p) for p in plist]) if plist else None
    flags = DEVICE_PTRS | (0 if sync else ASYNC)
    return _check(lib().envg_linear_nsplit(_ptr(y_local), arr, len(plist), _vp(multicast) if multicast else None, ldy,
                                           col0, _ptr(x), W.h, _ptr(bias), M, K, W.N, epilogue, _ptr(gate), flags))


def conv2d(dst, src, W, bias, stride, pad, epilogue=None, sync=True):
    """dst[B, O, outH, outW] = conv(src[B, C, H, W]) + bias (NCHW): envg_conv2d."""
    if epilogue is None:
        epilogue = EPI_BIAS if bias is not None else EPI_NONE
    flags = _mode(dst, src, bias)
    if flags == DEVICE_PTRS and not sync:
        flags |= ASYNC
    B, C, H, Wd = src.shape
    O, C2, kH, kW = W.conv
    return _check(lib().envg_conv2d(_ptr(dst), _ptr(src), W.h, _ptr(bias), C, O, H, Wd, kH, kW, stride, pad, B,
                                    epilogue, flags))


def group_norm(dst, src, gamma, beta, num_groups, silu=False, sync=True):
    """dst = GroupNorm(src) (+ SiLU), NCHW [B, C, H, W]: envg_group_norm (dst may be src)."""
    flags = _mode(dst, src, gamma, beta)
    if flags == DEVICE_PTRS and not sync:
        flags |= ASYNC
    B, C, H, Wd = src.shape
    return _check(lib().envg_group_norm(_ptr(dst), _ptr(src), _ptr(gamma), _ptr(beta), B, C, H, Wd, num_groups,
                                        1 if silu else 0, flags))


def attention(dst, q, k, v, heads, kv_heads, head_dim=128, scale=None, causal=False, key_mask=None, sync=True):
    """dst[seq_q, heads*hd] = per-head softmax(scale Q K^T (+ masks)) V: envg_attention.

    q [seq_q, >= heads*hd], k / v [seq_k, >= kv_heads*hd] fp32 (row strides = their widths);
    key_mask: int32 [seq_k] (numpy for host calls, CUDA tensor for device calls) or None."""
    if scale is None:
        scale = 1.0 / float(np.sqrt(head_dim))
    flags = _mode(dst, q, k, v)
    if flags == DEVICE_PTRS and not sync:
        flags |= ASYNC
    mp = None
    if key_mask is not None:
        if _is_torch(key_mask):
            import torch

            if not (key_mask.is_cuda and key_mask.dtype == torch.int32 and key_mask.is_contiguous()):
                raise TypeError("key_mask must be a contiguous int32 CUDA tensor")
            mp = key_mask.data_ptr()
        else:
            key_mask = np.ascontiguousarray(key_mask, dtype=np.int32)
            mp = key_mask.ctypes.data
    seq_q, seq_k = q.shape[0], k.shape[0]
    return _check(lib().envg_attention(_ptr(dst), _ptr(q), _ptr(k), _ptr(v), seq_q, seq_k, heads, kv_heads, head_dim,
                                       q.shape[1], k.shape[1], v.shape[1], dst.shape[1], float(scale),
                                       1 if causal else 0, mp, flags))


class ResBlock:
    """One VAE ResBlock (TVAEResBlock, quicknn_vae.pas:164-187) with device-resident conv weights.

    ``p`` holds norm1_gamma/beta [in_ch], conv1_w [out, in, 3, 3], conv1_b, norm2_gamma/beta
    [out_ch], conv2_w [out, out, 3, 3], conv2_b and, when in_ch != out_ch, skip_w [out, in, 1, 1]
    and skip_b.  Conv weights are numpy uint16 (bf16 bits) or float32 (rounded RNE at upload);
    the vectors are float32 numpy arrays (host calls) or CUDA tensors (device calls)."""

    def __init__(self, p):
        self.p = p
        w1 = p["conv1_w"]
        self.out_ch, self.in_ch = w1.shape[0], w1.shape[1]
        self.conv1 = Weight(w1.reshape(self.out_ch, -1), conv=tuple(w1.shape))
        w2 = p["conv2_w"]
        self.conv2 = Weight(w2.reshape(w2.shape[0], -1), conv=tuple(w2.shape))
        ws = p.get("skip_w")
        self.skip = Weight(ws.reshape(ws.shape[0], -1), conv=tuple(ws.shape)) if ws is not None else None

    def desc(self, vecs=None):
        v = vecs or self.p
        d = ResBlockDesc()
        d.in_ch, d.out_ch = self.in_ch, self.out_ch
        d.norm1_gamma, d.norm1_beta = _ptr(v.get("norm1_gamma")), _ptr(v.get("norm1_beta"))
        d.conv1, d.conv1_bias = self.conv1.h, _ptr(v.get("conv1_b"))
        d.norm2_gamma, d.norm2_beta = _ptr(v.get("norm2_gamma")), _ptr(v.get("norm2_beta"))
        d.conv2, d.conv2_bias = self.conv2.h, _ptr(v.get("conv2_b"))
        d.skip = self.skip.h if self.skip is not None else None
        d.skip_bias = _ptr(v.get("skip_b"))
        return d

    def forward(self, dst, src, num_groups, vecs=None, sync=True):
        """dst = skip(src) + conv2(SiLU(GN2(conv1(SiLU(GN1(src)))))): envg_vae_resblock.
        ``vecs`` overrides the vectors of ``p`` (e.g. CUDA tensors for a device call)."""
        v = vecs or self.p
        flags = _mode(dst, src, *[v.get(k) for k in ("norm1_gamma", "norm1_beta", "conv1_b", "norm2_gamma",
                                                      "norm2_beta", "conv2_b", "skip_b")])
        if flags == DEVICE_PTRS and not sync:
            flags |= ASYNC
        B, C, H, Wd = src.shape
        d = self.desc(v)
        return _check(lib().envg_vae_resblock(_ptr(dst), _ptr(src), ctypes.byref(d), B, H, Wd, num_groups, flags))


def sgemm(order, transA, transB, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc):
    """cblas_sgemm-compatible call on host numpy buffers (envg_sgemm)."""
    for a in (A, B, C):
        _host_f32(a, "sgemm operand")
    return _check(lib().envg_sgemm(order, transA, transB, M, N, K, alpha, A.ctypes.data, lda, B.ctypes.data, ldb,
                                   beta, C.ctypes.data, ldc))


# ---------------------------------------------------------------------------------------------
# Mirror of Envision's QNN operator surface for this path (src/quicknn_kernels.pas).  The
# weight argument is a device-resident Weight in place of the fp32/bf16 TMemoryBlock.
# ---------------------------------------------------------------------------------------------

def _assert(cond, msg):
    if not cond:
        raise AssertionError(msg)


def QNNLinear(dst, x, W, B, seqLen, inDIM, outDIM):
    """quicknn_kernels.pas:897-911 -> quicknncpu.pas:1807-1820: dst = x.W^T (+ B per row)."""
    _assert(W.N == outDIM and W.K == inDIM, "ERROR : QNNLinear weight shape mismatch")
    _assert(x.shape[0] >= seqLen and dst.shape[0] >= seqLen, "ERROR : QNNLinear out of bound")
    xs, ds = x[:seqLen], dst[:seqLen]
    return linear(ds, xs, W, bias=B, epilogue=EPI_BIAS if B is not None else EPI_NONE)


def QNNLinearNoBias(dst, x, W, seqLen, inDIM, outDIM):
    """quicknn_kernels.pas:913-927 -> quicknncpu.pas:1822-1828."""
    return QNNLinear(dst, x, W, None, seqLen, inDIM, outDIM)


def QNNLINEAR_BF16_OR_F32(dst, src, weight, weight_bf16, seq, srcDim, dstDim):
    """quicknn_kernels.pas:2093-2103 -> quicknncpu.pas:3062-3071: picks the bf16 weight if set."""
    w = weight_bf16 if weight_bf16 is not None else weight
    _assert(w is not None, "ERROR QNNLINEAR_BF16_OR_F32 : no weight or weight_16 assigned!")
    return QNNLinearNoBias(dst, src, w, seq, srcDim, dstDim)


def QNNMatMulNT(C, A, B, M, K, N):
    """quicknn_kernels.pas:847-861 -> quicknncpu.pas:1773-1784: C[M, N] = A[M, K] . B[N, K]^T.
    B is a device-resident Weight [N, K] (the Z-Image linears' use), or a host fp32 array [N, K],
    which goes through the cblas_gemm slot (envg_sgemm) with the reference's arguments."""
    if isinstance(B, Weight):
        _assert(B.N == N and B.K == K, "ERROR : QNNMatMul out of bound [B]")
        return linear(C[:M], A[:M], B, epilogue=EPI_NONE)
    _assert(A.size >= M * K, "ERROR : QNNMatMul out of bound [A]")
    _assert(B.size >= N * K, "ERROR : QNNMatMul out of bound [B]")
    _assert(C.size >= M * N, "ERROR : QNNMatMul out of bound [C]")
    return sgemm(ROW_MAJOR, NO_TRANS, TRANS, M, N, K, 1.0, A, K, B, K, 0.0, C, N)


def QNNMatMulNN(C, A, B, M, K, N):
    """quicknncpu.pas:1760-1771: C[M, N] = A[M, K] . B[K, N] through the cblas_gemm slot."""
    _assert(A.size >= M * K, "ERROR : QNNMatMul out of bound [A]")
    _assert(B.size >= K * N, "ERROR : QNNMatMul out of bound [B]")
    _assert(C.size >= M * N, "ERROR : QNNMatMul out of bound [C]")
    return sgemm(ROW_MAJOR, NO_TRANS, NO_TRANS, M, N, K, 1.0, A, K, B, N, 0.0, C, N)


def QNNMatMulTN(C, A, B, M, K, N):
    """quicknncpu.pas:1786-1797: C[M, N] = A^T . B with A stored [K, M] and B [K, N], called with
    the reference's leading dimensions lda = K and ldb = K (right when M = K = N, the square
    products it is used for; envg_sgemm refuses a leading dimension below the row length)."""
    _assert(A.size >= K * M, "ERROR : QNNMatMul out of bound [A]")
    _assert(B.size >= N * K, "ERROR : QNNMatMul out of bound [B]")
    _assert(C.size >= M * N, "ERROR : QNNMatMul out of bound [C]")
    return sgemm(ROW_MAJOR, TRANS, NO_TRANS, M, N, K, 1.0, A, K, B, K, 0.0, C, N)


def QNNLinearSiluMul(dst, x, W_gate_up, seqLen, inDIM, mlpDIM):
    """Fused QNNLinearNoBias into [gate | up] then QNNSiluMul(gate, up) (quicknncpu.pas:2404-2419),
    as the FLUX FFN does (quicknn_transformers.pas:1331-1341); dst is [seqLen, mlpDIM]."""
    _assert(W_gate_up.layout == LAYOUT_GATE_UP and W_gate_up.N == 2 * mlpDIM, "ERROR : gate/up weight mismatch")
    return linear(dst[:seqLen], x[:seqLen], W_gate_up, epilogue=EPI_SILU_GATE)


def QNNLinearGatedAdd(h, x, W, gate, seqLen, inDIM, outDIM, B=None):
    """Fused QNNLinear then QNNGatedAdd(h, gate, proj, seq, hidden) (quicknncpu.pas:853-859):
    h += gate (.) (x.W^T + B)."""
    _assert(W.N == outDIM and W.K == inDIM, "ERROR : QNNLinear weight shape mismatch")
    return linear(h[:seqLen], x[:seqLen], W, bias=B, epilogue=EPI_GATED_RESIDUAL, gate=gate)


def QNNAdaLNLinear(dst, src, shift, scale, W, B, seqLen, inDIM, outDIM):
    """QNNAdaLN(norm, src, shift, scale, seq, hidden) (quicknncpu.pas:3042-3060) followed by
    QNNLinear(dst, norm, W, B, seq, hidden, outDIM), fused: the normalised input never leaves the
    GPU as fp32."""
    _assert(W.N == outDIM and W.K == inDIM, "ERROR : QNNLinear weight shape mismatch")
    return linear_adaln(dst[:seqLen], src[:seqLen], shift, scale, W, bias=B,
                        epilogue=EPI_BIAS if B is not None else EPI_NONE)


def QNNRMSNormLinear(dst, src, norm_weight, W, B, seqLen, inDIM, outDIM):
    """QNNRMSNormRows(norm, src, norm_weight, seq, hidden) (quicknncpu.pas:2159-2198) followed by
    QNNLinear(dst, norm, W, B, seq, hidden, outDIM), fused as in the Qwen3 layer
    (quicknn_qwen3.pas:802, 817); a GATE_UP weight gives the SiLU-gated MLP input."""
    _assert(W.K == inDIM and (W.N == outDIM or (W.layout == LAYOUT_GATE_UP and W.N == 2 * outDIM)),
            "ERROR : QNNLinear weight shape mismatch")
    return linear_rmsnorm(dst[:seqLen], src[:seqLen], W, weight=norm_weight, bias=B)


def QNNGroupNorm(dst, src, gamma, beta, batch, channels, H, W, num_groups):
    """quicknncpu.pas:2259-2313 (NCHW)."""
    _assert(channels % num_groups == 0, "ERROR [GroupNorm] : channels not divisible by groups")
    return group_norm(dst.reshape(batch, channels, H, W), src.reshape(batch, channels, H, W), gamma, beta,
                      num_groups)


def QNNFlashAttention(dst, Q, K, V, heads, seq_q, seq_k, head_dim, scale):
    """quicknncpu.pas:2763-2860: Q/K/V/dst [seq, heads*head_dim] (head h at column h*head_dim)."""
    _assert(head_dim == 128, "ERROR [FlashAttention] : head_dim must be 128 on this device")
    return attention(dst.reshape(seq_q, heads * head_dim), Q.reshape(seq_q, heads * head_dim),
                     K.reshape(seq_k, heads * head_dim), V.reshape(seq_k, heads * head_dim), heads, heads,
                     head_dim, scale)


def QNNConv2d(dst, src, weights, bias, in_ch, out_ch, H, W, kH, kW, stride, padding, batch):
    """quicknn_kernels.pas:990-1010 -> quicknncpu.pas:1958-2132 (NCHW)."""
    _assert(weights.conv == (out_ch, in_ch, kH, kW), "ERROR [Conv2D] : weight geometry mismatch")
    outH = (H + 2 * padding - kH) // stride + 1
    outW = (W + 2 * padding - kW) // stride + 1
    _assert(dst.size >= batch * out_ch * outH * outW, "ERROR [Conv2D] : Incorrect destination size")
    return conv2d(dst.reshape(batch, out_ch, outH, outW), src.reshape(batch, in_ch, H, W), weights, bias, stride,
                  padding)
