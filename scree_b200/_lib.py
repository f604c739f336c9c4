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
_ALT_LIB = "SCREE_B200_LIB" in os.environ

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
    "scree_validate_offsets": (_I, [_P, _I, _L, _L, _P]),
    "scree_selftest_wait_timeout": (_I, [ctypes.c_longlong, _P, _P]),
    "scree_attn_fwd_workspace_size": (_S, [_L, _L, _L, _I]),
    "scree_attn_fwd": (
        _I,
        [_P, _P, _P, _L, _L, _L, _L, _L, _L, _P, _I, _L, _L, _L, _I, _I, _I, _F, _L, _P, _L, _L, _P, _P, _S, _P],
    ),
    "scree_attn_fwd_gqa": (
        _I,
        [_P, _P, _P, _L, _L, _L, _L, _L, _L, _P, _I, _L, _L, _L, _L, _I, _I, _I, _F, _L, _P, _L, _L, _P, _P, _S, _P],
    ),
    "scree_attn_bwd_gqa": (
        _I,
        [_P, _P, _P, _P, _P, _P, _P, _I, _L, _L, _L, _L, _I, _I, _I, _F, _L, _P, _P, _P, _P, _S, _P],
    ),
    "scree_attn_fwd_kv": (
        _I,
        [_P, _P, _P, _L, _L, _L, _L, _L, _L, _P, _P, _I, _L, _L, _L, _L, _L, _I, _I, _I, _F, _P, _L, _L, _P, _P, _S, _P],
    ),
    "scree_kv_append": (_I, [_P, _P, _P, _P, _I, _L, _L, _L, _L, _L, _P, _P, _P]),
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
    "scree_rmsnorm_qkv_workspace_size": (_S, [_L, _L, _L]),
    "scree_rmsnorm_qkv_fwd": (_I, [_P, _L, _P, _I, _P, _P, _P, _L, _L, _L, _I, _F, _P, _S, _P]),
    "scree_softmax_fwd": (_I, [_P, _P, _I, _L, _L, _L, _I, _P, _P]),
    "scree_softmax_bwd": (_I, [_P, _P, _P, _I, _L, _L, _L, _I, _P, _P]),
    "scree_pack": (_I, [_P, _P, _I, _L, _L, _L, _L, _L, _P, _P]),
    "scree_to_padded": (_I, [_P, _P, _I, _L, _L, _L, _L, _P, _I, _P, _P, _P]),
    "scree_padded_lengths": (_I, [_P, _L, _L, _P, _P]),
    "scree_padded_lengths_ex": (_I, [_P, _I, _L, _L, _P, _P]),
    "scree_to_padded_ex": (_I, [_P, _P, _I, _L, _L, _L, _L, _P, _I, _P, _P, _I, _P]),
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
                if _ALT_LIB and not hasattr(lib, name):
                    continue  # an older build under A/B comparison may lack newer entry points
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


DEVERR_WAIT_TIMEOUT = 1
DEVERR_BAD_INPUT = 2
_DEVERR_NAMES = {DEVERR_WAIT_TIMEOUT: "a bounded wait timed out", DEVERR_BAD_INPUT: "invalid input (offsets)"}


def describe_status(status: int) -> str:
    code, site = status >> 16, status & 0xFFFF
    return f"{_DEVERR_NAMES.get(code, f'error code {code}')} at site {site}"


def raise_device_status(reset: bool = True) -> None:
    """Raise ScreeError if a kernel recorded an error in the device status word
    (synchronises); clears the word when ``reset``."""
    st = device_status(reset)
    if st != 0:
        raise ScreeError(f"libscree_b200 device status {st:#x}: {describe_status(st)}")


def validate_offsets(offsets, total: int, stream=None) -> None:
    """Enqueue the device-side offsets check (offsets[0] == 0, non-decreasing,
    offsets[-1] == total); a violation shows up in the device status word."""
    import torch

    assert offsets.is_cuda and offsets.ndim == 1 and offsets.dtype in (torch.int32, torch.int64)
    cu = offsets.contiguous()
    s = stream if stream is not None else stream_ptr(cu.device)
    with torch.cuda.device(cu.device):
        rc = load().scree_validate_offsets(cu.data_ptr(), 1 if cu.dtype == torch.int64 else 0,
                                           cu.numel() - 1, int(total), s)
    check(rc, "scree_validate_offsets")


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
