"""ctypes binding of libscree_b200.so (the C ABI declared in include/scree_b200.h).

The library is loaded lazily on first use.  There is no fallback: if the shared
library is missing or cannot be loaded, every GPU entry point raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import os

# SCREE_B200_LIB points at another build of the library (benchmark A/B runs).
LIB_PATH = Path(os.environ.get("SCREE_B200_LIB", Path(__file__).resolve().parent / "libscree_b200.so"))

SCREE_OK = 0
SCREE_ERR_INVALID = 1
SCREE_ERR_UNSUPPORTED = 2
SCREE_ERR_CUDA = 3

F16, BF16, F32 = 0, 1, 2

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_F = ctypes.c_float
_S = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/scree_b200.h
_SIGNATURES = {
    "scree_last_error": (_I, [ctypes.c_char_p, _S]),
    "scree_version": (_I, []),
    "scree_device_status": (_I, [ctypes.POINTER(_I), _I]),
    "scree_launch_count": (ctypes.c_longlong, []),
    "scree_profile_enable": (_I, [_I]),
    "scree_profile_read": (_I, [_I, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong)]),
    "scree_attn_fwd_workspace_size": (_S, [_L, _L, _L, _I]),
    "scree_attn_fwd": (
        _I,
        [_P, _P, _P, _L, _L, _L, _L, _L, _L, _P, _I, _L, _L, _L, _I, _I, _I, _F, _L, _P, _L, _L, _P, _P, _S, _P],
    ),
    "scree_attn_fwd_noalloc": (
        _I,
        [_P, _P, _P, _L, _L, _L, _L, _L, _L, _P, _I, _L, _L, _L, _I, _I, _I, _F, _L, _P, _L, _L, _P, _P],
    ),
    "scree_attn_bwd_workspace_size": (_S, [_L, _L, _L, _I]),
    "scree_attn_bwd": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _I, _L, _L, _L, _I, _I, _I, _F, _L, _P, _P, _P, _P, _S, _P],
    ),
    "scree_rmsnorm_fwd": (_I, [_P, _L, _P, _I, _P, _L, _P, _L, _L, _I, _F, _P]),
    "scree_norm_bwd_workspace_size": (_S, [_L, _L]),
    "scree_rmsnorm_bwd": (_I, [_P, _P, _P, _I, _P, _P, _P, _L, _L, _I, _P, _S, _P]),
    "scree_layernorm_fwd": (_I, [_P, _L, _P, _P, _I, _P, _L, _P, _P, _L, _L, _I, _F, _P]),
    "scree_layernorm_bwd": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _L, _L, _I, _P, _S, _P]),
    "scree_softmax_fwd": (_I, [_P, _P, _I, _L, _L, _L, _I, _P, _P]),
    "scree_softmax_bwd": (_I, [_P, _P, _P, _I, _L, _L, _L, _I, _P, _P]),
    "scree_pack": (_I, [_P, _P, _I, _L, _L, _L, _L, _L, _P, _P]),
    "scree_to_padded": (_I, [_P, _P, _I, _L, _L, _L, _L, _P, _I, _P, _P, _P]),
    "scree_padded_lengths": (_I, [_P, _L, _L, _P, _P]),
    "scree_from_padded": (_I, [_P, _P, _L, _L, _L, _L, _P, _P]),
}

EXPORTED = tuple(_SIGNATURES)

_lib = None
_lock = threading.Lock()


class ScreeError(RuntimeError):
    """A CUDA-side failure reported by libscree_b200."""


def load() -> ctypes.CDLL:
    """Load (once) and return the native library; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"libscree_b200.so not found at {LIB_PATH}; build it with "
                    "`python -m scree_b200.build` (scree_b200 has no CPU fallback)"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().scree_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Map a scree_status to the exception the reference raises for it."""
    if rc == SCREE_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == SCREE_ERR_INVALID:
        raise ValueError(msg)
    if rc == SCREE_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise ScreeError(msg)


def device_status(reset: bool = True) -> int:
    """Device status word (0 = ok).  Synchronises with the device."""
    v = ctypes.c_int(0)
    check(load().scree_device_status(ctypes.byref(v), 1 if reset else 0), "scree_device_status")
    return v.value


PROF_ATTN_FWD, PROF_ATTN_BWD, PROF_NORM_FWD, PROF_NORM_BWD, PROF_GATHER = 0, 1, 2, 3, 4


def profile_enable(on: bool) -> None:
    load().scree_profile_enable(1 if on else 0)


def profile_read(kernel: int) -> tuple[float, int]:
    """(total milliseconds, launches) of one kernel kind since the last read."""
    ms = ctypes.c_double(0.0)
    n = ctypes.c_longlong(0)
    check(load().scree_profile_read(kernel, ctypes.byref(ms), ctypes.byref(n)), "scree_profile_read")
    return ms.value, n.value


def launch_count() -> int:
    return int(load().scree_launch_count())


def dtype_code(dtype) -> int:
    import torch

    if dtype == torch.float16:
        return F16
    if dtype == torch.bfloat16:
        return BF16
    if dtype == torch.float32:
        return F32
    raise TypeError(f"unsupported dtype {dtype} (float16, bfloat16, float32)")


def stream_ptr(device=None) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream
