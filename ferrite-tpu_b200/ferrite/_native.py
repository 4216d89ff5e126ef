"""ctypes binding of ``libferrite_b200.so``, the C ABI declared in ``include/ferrite_b200.h``.

This is the only place Python touches the native library.  Every entry point
takes device pointers, sizes and a ``cudaStream_t`` and returns a status code;
:func:`check` turns a non-zero status into :class:`FerriteError` carrying the
library's thread-local error string.

There is deliberately no fallback: if the library is missing, or a tensor is not
on a CUDA device, the call raises.  The library is built in-tree by
``ferrite-tpu_b200/build.py`` (``__graft_entry__.build()`` runs it).
"""

from __future__ import annotations

import ctypes
import functools
import itertools
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libferrite_b200.so")

OK = 0
BAD_SHAPE = 1
UNSUPPORTED_DTYPE = 2
LAUNCH_FAILED = 3
DEVICE_TIMEOUT = 4
BAD_ALIGNMENT = 5
WORKSPACE_TOO_SMALL = 6
INJECTED_FAULT = 7

STATUS_NAMES = {
    OK: "OK",
    BAD_SHAPE: "BAD_SHAPE",
    UNSUPPORTED_DTYPE: "UNSUPPORTED_DTYPE",
    LAUNCH_FAILED: "LAUNCH_FAILED",
    DEVICE_TIMEOUT: "DEVICE_TIMEOUT",
    BAD_ALIGNMENT: "BAD_ALIGNMENT",
    WORKSPACE_TOO_SMALL: "WORKSPACE_TOO_SMALL",
    INJECTED_FAULT: "INJECTED_FAULT",
}

F32, BF16, F16 = 0, 1, 2
_DTYPE_CODES = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t



class AttnStrides(ctypes.Structure):
    """``ferrite_attn_strides``: (batch, head, sequence) element strides of each
    [b, h, s, d] attention operand (d unit-stride)."""

    _fields_ = [(n, _i64 * 3) for n in ("q", "k", "v", "o", "dout", "dq", "dk", "dv")]


def attn_strides(**tensors: torch.Tensor) -> AttnStrides:
    """Strides of the named [b, h, s, d] views (``q=..., o=...``); unnamed fields are 0."""
    st = AttnStrides()
    for name, t in tensors.items():
        if t.stride(3) != 1:
            raise ValueError(f"{name}: head_dim must be unit-stride")
        getattr(st, name)[:] = (t.stride(0), t.stride(1), t.stride(2))
    return st


_sp = ctypes.POINTER(AttnStrides)

# name -> (restype, argtypes).  Must match include/ferrite_b200.h.
SIGNATURES: dict[str, tuple] = {
    "ferrite_last_error": (ctypes.c_char_p, []),
    "ferrite_version": (ctypes.c_char_p, []),
    "ferrite_device_status": (_i32, [_vp, _i32]),
    "ferrite_wait_probe": (_i32, [_vp, ctypes.c_uint64, _vp]),
    "ferrite_rmsnorm_fwd": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _f32, _i32, _i32]),
    "ferrite_add_rmsnorm_fwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _i32, _i32]),
    "ferrite_rmsnorm_bwd_workspace_size": (_sz, [_i64, _i64]),
    "ferrite_rmsnorm_bwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i64, _i64, _f32, _i32, _i32]),
    "ferrite_rmsnorm_bwd_noalloc": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _i32, _i32]),
    "ferrite_gemm": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _i32]),
    "ferrite_gemm_epilogue": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _vp, _i64]),
    "ferrite_gemm_rmsnorm": (_i32, [_vp, _vp, _vp, _vp, _f32, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _vp,
                                    _i64, _i32, _i32]),
    "ferrite_gemm_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64, _i32, _i32, _i32]),
    "ferrite_gemm_ws": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _i32, _vp, _sz]),
    "ferrite_attn_fwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _i32, _i32, _i32]),
    "ferrite_attn_bwd_prep": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32]),
    "ferrite_attn_bwd_dkv": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _i32, _i32, _i32]),
    "ferrite_attn_bwd_dq": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _i32, _i32, _i32]),
    "ferrite_adamw_workspace_size": (_sz, [_i64]),
    "ferrite_adamw_step": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _f32, _f32, _f32, _f32, _i64, _f32, _f32, _vp, _vp, _sz]),
    "ferrite_xent_fwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32]),
    "ferrite_xent_bwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _f32, _vp, _i64, _i64, _i64, _i64, _i32, _i32]),
    "ferrite_attn_bwd_ds_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64, _i32]),
    "ferrite_attn_bwd_ds": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sp, _vp, _sz, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _i32, _i32, _i32]),
    "ferrite_attn_bwd_dkv_ds": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _i32, _i32, _i32]),
    "ferrite_attn_bwd_dq_ds": (_i32, [_vp, _vp, _vp, _vp, _sp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _i32, _i32, _i32]),
    "ferrite_attn_fwd_strided": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _sp, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _i32, _i32, _i32]),
    "ferrite_attn_bwd_prep_strided": (_i32, [_vp, _vp, _vp, _vp, _sp, _i64, _i64, _i64, _i64, _i32]),
    "ferrite_attn_bwd_dkv_strided": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sp, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _i32, _i32, _i32]),
    "ferrite_attn_bwd_dq_strided": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sp, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _i32, _i32, _i32]),
    "ferrite_attn_decode": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _i32]),
    "ferrite_attn_decode_cluster": (_i32, [_i64, _i64, _i64, _i32, _i64]),
}


class FerriteError(RuntimeError):
    """A non-zero status from the native library."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"[{STATUS_NAMES.get(status, status)}] {message}")


class NativeLibraryMissing(RuntimeError):
    """The compiled library is absent: build it with ferrite-tpu_b200/build.py."""


_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library, with argtypes set."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryMissing(
                f"{LIB_PATH} not found; run `python ferrite-tpu_b200/build.py` (or __graft_entry__.build())"
            )
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().ferrite_last_error()
    return msg.decode() if msg else ""


def version() -> str:
    return lib().ferrite_version().decode()


def check(status: int) -> None:
    if status != OK:
        raise FerriteError(status, last_error())


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}; expected float32, bfloat16 or float16") from None


def require_cuda(*tensors: torch.Tensor) -> None:
    """The kernels only run on CUDA tensors; there is no host fallback."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "ferrite kernels run on CUDA tensors only (got a tensor on "
                f"{t.device}); there is no CPU fallback in the product path"
            )


def on_tensor_device(fn):
    """Decorator: run ``fn`` with the device of its first CUDA tensor argument
    current.  The library plans and launches on the current device (SM count,
    occupancy, kernel attributes, per-device caches) and the stream it is handed is
    that device's, so a call on tensors of another GPU must switch to it first."""

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        for a in itertools.chain(args, kwargs.values()):
            if isinstance(a, torch.Tensor) and a.is_cuda:
                if a.device.index == torch.cuda.current_device():
                    break
                with torch.cuda.device(a.device):
                    return fn(*args, **kwargs)
        return fn(*args, **kwargs)

    return wrapper


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_status(clear: bool = True) -> None:
    """Synchronise the current stream and raise if a device-side wait expired."""
    check(lib().ferrite_device_status(stream_ptr(), int(clear)))
