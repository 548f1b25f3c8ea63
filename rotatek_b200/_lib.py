"""Loader and thin ctypes binding of librotatek_b200.so (the C ABI in
include/rotatek_b200.h).

The library is loaded on first use.  If it is missing or the tensors are not
CUDA tensors, calls raise -- there is no CPU fallback.  Build it with
``python -m rotatek_b200.csrc.build``.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "librotatek_b200.so")

RTK_OK, RTK_ERR_INVALID, RTK_ERR_UNSUPPORTED, RTK_ERR_WORKSPACE, RTK_ERR_CUDA = range(5)
RTK_DEVICE_TIMEOUT = 1

_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2, torch.uint8: 3}


class RtkTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("shape", ctypes.c_int64 * 4), ("stride", ctypes.c_int64 * 4)]


_P = ctypes.POINTER(RtkTensor)

# (name, restype, argtypes) of every exported entry point
SIGNATURES = {
    "rtk_abi_version": (ctypes.c_int, []),
    "rtk_last_error": (ctypes.c_char_p, []),
    "rtk_decode_set_sm_reserve": (ctypes.c_int, [ctypes.c_int]),
    "rtk_rotatek_decode_workspace_size": (ctypes.c_size_t, [ctypes.c_int32] + [ctypes.c_int64] * 7 + [ctypes.c_int32]),
    "rtk_decode_workspace_counter_bytes": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64]),
    "rtk_rotatek_decode": (ctypes.c_int, [_P] * 8 + [ctypes.c_int64, _P, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "rtk_rotatek_decode_static": (ctypes.c_int, [_P] * 8 + [ctypes.c_int64, _P, ctypes.c_void_p]),
    "rtk_rotatek_decode_fp8": (ctypes.c_int, [_P] * 10 + [ctypes.c_int64, _P, ctypes.c_void_p, ctypes.c_size_t,
                                                          ctypes.c_void_p]),
    "rtk_quantize_visual_fp8": (ctypes.c_int, [_P] * 6 + [ctypes.c_void_p]),
    "rtk_full_channel_decode_workspace_size": (ctypes.c_size_t, [ctypes.c_int32] + [ctypes.c_int64] * 5 + [ctypes.c_int32]),
    "rtk_full_channel_decode": (ctypes.c_int, [_P] * 3 + [ctypes.c_int64, _P, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "rtk_spark_decode": (ctypes.c_int, [_P] * 8 + [ctypes.c_int64, _P, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "rtk_spark_pack": (ctypes.c_int, [_P, _P, ctypes.c_void_p, ctypes.c_void_p]),
    "rtk_key_covariance": (ctypes.c_int, [_P, _P, _P, ctypes.c_void_p]),
    "rtk_rotate_keys": (ctypes.c_int, [_P, _P, _P, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "rtk_eigh_topk_workspace_size": (ctypes.c_size_t, [ctypes.c_int64]),
    "rtk_eigh_topk": (ctypes.c_int, [_P, ctypes.c_int64, _P, _P, ctypes.c_void_p, ctypes.c_size_t,
                                     ctypes.c_void_p]),
    "rtk_build_rotation_workspace_size": (ctypes.c_size_t, [ctypes.c_int64] * 3),
    "rtk_build_rotation": (ctypes.c_int, [_P, _P, ctypes.c_int64, ctypes.c_int64, _P, _P, _P, _P,
                                          ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "rtk_key_projection_workspace_size": (ctypes.c_size_t, [ctypes.c_int64] * 5 + [ctypes.c_int32]),
    "rtk_build_rotation_projected_workspace_size": (ctypes.c_size_t, [ctypes.c_int64] * 5 + [ctypes.c_int32]),
    "rtk_key_projection": (ctypes.c_int, [_P] * 5 + [ctypes.c_int64, ctypes.c_int64] + [_P] * 3 +
                           [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "rtk_build_rotation_projected": (ctypes.c_int, [_P] * 5 + [ctypes.c_int64, ctypes.c_int64, _P,
                                                              ctypes.c_int64, ctypes.c_int64] + [_P] * 5 +
                                     [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "rtk_read_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
    "rtk_read_static_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
    "rtk_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]),
}

_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH):
    """The loaded library (ctypes.CDLL) with typed entry points."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise RuntimeError(
                    f"rotatek_b200: {path} is missing; build it with "
                    "`python -m rotatek_b200.csrc.build` (there is no CPU fallback)")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def describe(t: Optional[torch.Tensor]):
    """rtk_tensor descriptor of a CUDA tensor (None -> NULL pointer)."""
    if t is None:
        return None
    nd = t.dim()
    if nd > 4:
        raise ValueError("tensors of more than 4 dimensions are not supported")
    d = RtkTensor()
    d.data = t.data_ptr()
    d.dtype = _DTYPES.get(t.dtype, -1)
    d.ndim = nd
    for i, (n, s) in enumerate(zip(t.shape, t.stride())):
        d.shape[i] = n
        d.stride[i] = s
    return ctypes.byref(d)


def check(code: int):
    if code == RTK_OK:
        return
    msg = load().rtk_last_error().decode()
    if code == RTK_ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(f"rotatek_b200 (status {code}): {msg}")


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("rotatek_b200 runs on CUDA tensors only (no CPU fallback)")


# ------------------------------------------------------------------ workspace
_ws_lock = threading.Lock()
_workspaces = {}     # device index -> uint8 buffer
_zero_prefix = {}    # device index -> leading bytes known to read zero


def workspace(device: torch.device, nbytes: int, counter_bytes: int) -> torch.Tensor:
    """Scratch of at least `nbytes` for `device` whose first `counter_bytes`
    read zero, as the decode kernels require before a call.

    One buffer per device, grown on demand and shared by every call on that
    device.  The kernels leave the counter bytes zero and dirty what follows,
    so the buffer is re-zeroed only when a call needs a longer zero prefix than
    the last one left (a larger batch * q_heads).  Calls are ordered on the
    current stream; callers that launch on several streams at once must
    synchronise them, as for the reference's shape-keyed scratch cache
    (rotatek/kernels/fused_decode.py:47-70)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _ws_lock:
        buf = _workspaces.get(idx)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 1 << 20)
            buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
            _workspaces[idx] = buf
            _zero_prefix[idx] = size
        if _zero_prefix[idx] < counter_bytes:
            buf[:counter_bytes].zero_()
        _zero_prefix[idx] = counter_bytes     # what follows is scratch after the call
        return buf


def read_status(device: Optional[torch.device] = None) -> int:
    """Device-status bits (RTK_DEVICE_TIMEOUT) recorded since the last read; clears them."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    buf = _workspaces.get(idx)
    if buf is None:
        return 0
    out = ctypes.c_uint32(0)
    stream = torch.cuda.current_stream(buf.device).cuda_stream
    check(load().rtk_read_status(ctypes.c_void_p(buf.data_ptr()), ctypes.c_void_p(stream),
                                 ctypes.byref(out)))
    return out.value


def read_static_status() -> int:
    """Device-status bits that rtk_rotatek_decode_static's calls on the current
    device set since the last read (its fixed scratch's status word); clears them."""
    out = ctypes.c_uint32(0)
    stream = torch.cuda.current_stream().cuda_stream
    check(load().rtk_read_static_status(ctypes.c_void_p(stream), ctypes.byref(out)))
    return out.value


def selftest_wait_timeout(limit_ns: int = 1_000_000, device: Optional[torch.device] = None) -> None:
    """Run the bounded-wait self-test kernel against this device's decode
    workspace: its wait on a barrier nothing arrives on gives up after
    ``limit_ns`` and sets RTK_DEVICE_TIMEOUT, which ``read_status`` then reports."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    buf = workspace(dev, 1 << 20, 256)
    stream = torch.cuda.current_stream(buf.device).cuda_stream
    check(load().rtk_selftest_wait_timeout(ctypes.c_void_p(buf.data_ptr()), ctypes.c_uint64(limit_ns),
                                           ctypes.c_void_p(stream)))


def set_decode_sm_reserve(sms: int) -> None:
    """Leave ``sms`` SMs free of the persistent decode kernels (process-wide),
    for a collective that runs beside them; 0 restores one CTA per SM."""
    check(load().rtk_decode_set_sm_reserve(int(sms)))
