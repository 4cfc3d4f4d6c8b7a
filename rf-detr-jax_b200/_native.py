"""ctypes binding of ``librfdetr_b200.so`` (the C ABI declared in ``include/rfdetr_b200.h``).

Loading fails loudly when the library is missing: there is no CPU fallback.  Status codes from
the library become Python exceptions -- ``ValueError`` for bad arguments (as the reference
raises for bad shapes and names), ``RuntimeError`` for CUDA failures.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librfdetr_b200.so")

F32 = 0
BF16 = 1

OK = 0
ERR_SHAPE = 1
ERR_DTYPE = 2
ERR_ALIGN = 3
ERR_WORKSPACE = 4
ERR_CUDA = 5
ERR_LIMIT = 6
ERR_CAPACITY = 7

_lock = threading.Lock()
_lib = None

_c_int64_p = ctypes.POINTER(ctypes.c_int64)
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float

# name -> (restype, argtypes)
SIGNATURES = {
    "rfdetr_status_string": (ctypes.c_char_p, [_int]),
    "rfdetr_abi_version": (_int, []),
    "rfdetr_set_tuning": (_int, [ctypes.c_char_p, ctypes.c_char_p]),
    "rfdetr_take_device_fault": (_int, [_vp]),
    "rfdetr_selftest_bounded_wait": (_int, [_vp, _int, _vp]),
    "rfdetr_ipc_handle_bytes": (ctypes.c_size_t, []),
    "rfdetr_allreduce_flag_bytes": (ctypes.c_size_t, []),
    "rfdetr_ipc_get_handle": (_int, [_vp, _vp, ctypes.POINTER(ctypes.c_size_t)]),
    "rfdetr_ipc_open_handle": (_int, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "rfdetr_ipc_close_handle": (_int, [_vp]),
    "rfdetr_allreduce_sum_f32": (_int, [_vp, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), _int,
                                        _int, _i64, ctypes.c_uint32, _int, _vp]),
    "rfdetr_msda_forward": (_int, [_vp, _vp, _int, _c_int64_p, _c_int64_p, _vp, _vp, _int, _vp, _int,
                                   _i64, _i64, _i64, _i64, _i64, _i64]),
    "rfdetr_msda_backward_workspace_size": (ctypes.c_size_t, [_int, _i64, _i64, _i64, _i64]),
    "rfdetr_msda_backward_workspace_bytes": (ctypes.c_size_t, [_int, _int, _c_int64_p, _i64, _i64, _i64, _i64, _i64,
                                                               _i64]),
    "rfdetr_msda_backward": (_int, [_vp, _vp, _int, _c_int64_p, _c_int64_p, _vp, _vp, _int, _vp, _int,
                                    _vp, _vp, _vp, _vp, ctypes.c_size_t, _i64, _i64, _i64, _i64, _i64, _i64]),
    "rfdetr_msda_backward_noalloc": (_int, [_vp, _vp, _int, _c_int64_p, _c_int64_p, _vp, _vp, _int, _vp, _int,
                                            _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64]),
    "rfdetr_topk_select": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp]),
    "rfdetr_select_rows": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _vp, _vp]),
    "rfdetr_match_cost": (_int, [_vp, _vp, _int, _vp, _int, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                 _f32, _f32, _f32, _f32]),
    "rfdetr_lsap_batched": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp]),
    "rfdetr_msda_prologue": (_int, [_vp, _vp, _int, _vp, _vp, _vp, _i64, _c_int64_p, _vp, _vp, _vp, _i64, _i64,
                                    _i64, _i64, _i64, _i64]),
    "rfdetr_msda_prologue_backward": (_int, [_vp, _vp, _vp, _vp, _int, _vp, _i64, _vp, _c_int64_p, _vp, _int, _vp,
                                             _i64, _i64, _i64, _i64, _i64]),
    "rfdetr_match_stacked": (_int, [_vp, _vp, _int, _vp, _int, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                    _i64, _f32, _f32, _f32, _f32, _vp, _vp, _vp, _vp, _vp]),
    "rfdetr_set_losses": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                                 _f32, ctypes.c_int32, _vp, _vp, _vp, _vp]),
}


class NativeLibraryError(RuntimeError):
    """The native library is missing or unusable."""


def lib() -> ctypes.CDLL:
    """Load the library once (thread-safe) and declare every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise NativeLibraryError(
                    f"{LIB_PATH} is not built; run `python rf-detr-jax_b200/build.py` (needs nvcc)")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
    return _lib


def set_tuning(name: str, value: str | None) -> None:
    """Sets a process-wide tuning knob of the library (``rfdetr_set_tuning``): ``value`` is
    ``"a,b,..."`` (up to five integers) or ``None`` for the library's default.  Knob names are
    those of the environment variables the library reads once at its first launch, e.g.
    ``"RFDETR_LSAP_STAGE_KB"``."""
    status = lib().rfdetr_set_tuning(name.encode(), None if value is None else str(value).encode())
    if status != OK:
        raise ValueError(f"unknown tuning knob {name!r} or malformed value {value!r}")


def check_device_status(status: torch.Tensor, what: str = "device status") -> None:
    """Reads a device status word written by an entry point (synchronises its stream) and raises
    for a non-zero status."""
    check(int(status.reshape(-1)[0].item()), what)


def status_text(status: int) -> str:
    return lib().rfdetr_status_string(status).decode()


def check(status: int, what: str) -> None:
    """Raise for a non-zero status returned by ``what``."""
    if status == OK:
        return
    text = f"{what}: {status_text(status)} (status {status})"
    if status in (ERR_SHAPE, ERR_DTYPE, ERR_ALIGN, ERR_WORKSPACE, ERR_CAPACITY):
        raise ValueError(text)
    raise RuntimeError(text)


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return F32
    if dtype == torch.bfloat16:
        return BF16
    raise ValueError(f"unsupported dtype {dtype}; expected float32 or bfloat16")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    """The current torch stream of ``t``'s device, as a raw ``cudaStream_t``."""
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("the B200 backend takes CUDA tensors only (there is no CPU path)")
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError("all tensors must be on the same device")
    return device


def int64_array(values) -> ctypes.Array:
    values = [int(v) for v in values]
    return (ctypes.c_int64 * max(1, len(values)))(*values)
