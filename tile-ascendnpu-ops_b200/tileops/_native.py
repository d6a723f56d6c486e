"""ctypes binding of the C ABI in ``include/tileops_c.h``.

``libtileops_b200.so`` (built by ``csrc/build.py``) is loaded from this
package directory the first time a kernel runs.  Every entry point is
declared here with the argument types of the header; ``call`` turns a
non-zero status into a Python exception:

* ``TILEOPS_EBADDTYPE`` / ``EBADSHAPE`` / ``EALIGN`` / ``EINVAL`` -> ``ValueError``
* ``TILEOPS_ELAUNCH`` / ``ETIMEOUT`` -> ``RuntimeError``

There is no fallback: if the library is missing or cannot be loaded, the
call raises ``NativeLibraryError`` naming the build command.
"""

from __future__ import annotations

import ctypes
import re
import threading
from pathlib import Path
from typing import Optional

import torch

__all__ = [
    "NativeLibraryError",
    "LIB_PATH",
    "call",
    "declared_entry_points",
    "dtype_code",
    "lib",
    "stream_handle",
]

LIB_PATH = Path(__file__).resolve().parent / "libtileops_b200.so"
_HEADER = Path(__file__).resolve().parents[2] / "include" / "tileops_c.h"

OK = 0
EBADDTYPE = -1
EBADSHAPE = -2
EALIGN = -3
ELAUNCH = -4
ETIMEOUT = -5
EINVAL = -6
GDN_QK_L2NORM = 1  # TILEOPS_GDN_QK_L2NORM

_DTYPE_CODES = {
    torch.float32: 0,
    torch.float16: 1,
    torch.bfloat16: 2,
    torch.bool: 3,
    torch.uint8: 4,
    torch.int8: 5,
    torch.int16: 6,
    torch.int32: 7,
    torch.int64: 8,
}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i = ctypes.c_int
_d = ctypes.c_double

# name -> argument types, in header order.
_SIGNATURES: dict[str, list] = {
    "tileops_hardswish_fwd": [_p, _p, _i64, _i, _p],
    "tileops_hardsigmoid_fwd": [_p, _p, _i64, _i, _p],
    "tileops_clamp_scalar_fwd": [_p, _p, _i64, _i, _i, _d, _i, _d, _p],
    "tileops_isnan_fwd": [_p, _p, _i64, _i, _p],
    "tileops_isinf_fwd": [_p, _p, _i64, _i, _p],
    "tileops_isfinite_fwd": [_p, _p, _i64, _i, _p],
    "tileops_bitwise_not_fwd": [_p, _p, _i64, _i, _p],
    "tileops_gelu_and_mul_fwd": [_p, _p, _i64, _i64, _i, _p],
    "tileops_gelu_tanh_and_mul_fwd": [_p, _p, _i64, _i64, _i, _p],
    "tileops_fused_add_layer_norm_fwd": [_p, _p, _p, _p, _p, _p, _i64, _i64, _d, _i, _i, _p],
    "tileops_conv1d_depthwise_fwd": [_p, _p, _p, _p] + [_i64] * 8 + [_i, _i, _i, _p],
    "tileops_conv1d_direct_fwd": [_p, _p, _p, _p] + [_i64] * 10 + [_i, _p],
    "tileops_mha_fwd": [_p, _p, _p, _p, _p] + [_i64] * 6 + [_i, _d, _i, _p],
    "tileops_gdn_prefill_fwd": [_p] * 9 + [_i64] * 6 + [_d, _i, _p],
    "tileops_gdn_workspace_bytes": [_i64] * 5,
    "tileops_gdn_prefill_fwd_noalloc": [_p] * 8 + [_i64] * 6 + [_d, _i, _p],
    "tileops_gdn_varlen_workspace_bytes": [_i64] * 5,
    "tileops_gdn_prefill_varlen_fwd": [_p] * 6 + [_i64] + [_p] * 4 + [_i64] * 5 + [_d, _i, _i, _p],
    "tileops_gla_decode_fwd": [_p] * 7 + [_i64] * 4 + [_d, _i, _p],
    "tileops_ssd_chunk_scan_fwd": [_p] * 7 + [_i64] * 7 + [_i, _p],
    "tileops_device_error_flag": [_p, _i],
    "tileops_selftest_wait_timeout": [_p, _i64, _i64, _p, _p],
    "tileops_abi_version": [],
    "tileops_status_string": [_i],
}


class NativeLibraryError(RuntimeError):
    """The CUDA kernel library is missing or failed to load."""


_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise NativeLibraryError(
                    f"{LIB_PATH.name} is not built; run "
                    "`python tile-ascendnpu-ops_b200/csrc/build.py` (or __graft_entry__.build())"
                )
            try:
                handle = ctypes.CDLL(str(LIB_PATH))
            except OSError as e:  # pragma: no cover - depends on the machine
                raise NativeLibraryError(f"cannot load {LIB_PATH}: {e}") from e
            for name, argtypes in _SIGNATURES.items():
                fn = getattr(handle, name, None)
                if fn is None:
                    continue  # reported by declared_entry_points() checks
                fn.argtypes = argtypes
                fn.restype = {
                    "tileops_status_string": ctypes.c_char_p,
                    "tileops_gdn_workspace_bytes": ctypes.c_int64,
                    "tileops_gdn_varlen_workspace_bytes": ctypes.c_int64,
                }.get(name, ctypes.c_int)
            _lib = handle
    return _lib


def declared_entry_points() -> list[str]:
    """Names of every function the C header declares."""
    text = _HEADER.read_text()
    return sorted(
        set(re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(tileops_\w+)\s*\(", text, re.M))
    )


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"dtype {dtype} has no native code") from None


def stream_handle(device: torch.device) -> ctypes.c_void_p:
    """The current torch stream of ``device`` as a ``cudaStream_t``."""
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def status_string(status: int) -> str:
    return lib().tileops_status_string(status).decode()


def call(name: str, *args) -> None:
    """Invoke entry point ``name``; raise on a non-zero status."""
    fn = getattr(lib(), name, None)
    if fn is None:
        raise NativeLibraryError(f"{LIB_PATH.name} does not export {name}")
    status = fn(*args)
    if status == OK:
        return
    msg = f"{name} failed: {status_string(status)} (status {status})"
    if status in (EBADDTYPE, EBADSHAPE, EALIGN, EINVAL):
        raise ValueError(msg)
    raise RuntimeError(msg)


def ptr(t: Optional[torch.Tensor]) -> ctypes.c_void_p:
    """Device pointer of a tensor (NULL for None)."""
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def launch(name: str, device: torch.device, *args) -> None:
    """Call ``name(*args, stream)`` on ``device``'s current torch stream.

    The library links its own CUDA runtime, which launches into the context
    current on the calling thread; the guard makes that ``device``'s context
    when the caller's current device differs.
    """
    if device.type != "cuda":
        raise ValueError(f"{name}: tensors must be on a cuda device, got {device}")
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx != torch.cuda.current_device():
        with torch.cuda.device(idx):
            call(name, *args, stream_handle(device))
    else:
        call(name, *args, stream_handle(device))
