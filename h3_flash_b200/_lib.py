"""ctypes binding of libh3b.so (C ABI declared in include/h3b.h).

The library is loaded lazily on first use. A missing or stale library is an
error, never a silent fallback: every GPU op of this package runs through it.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path
from typing import Any

from . import _build

_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None

H3B_OK = 0
H3B_ERR_VALUE = 1
H3B_ERR_CUDA = 2
H3B_ERR_UNSUPPORTED = 3
ABI_VERSION = 8
IPC_HANDLE_BYTES = 64

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_f32 = ctypes.c_float

# name -> argument types (the trailing stream is a void*), mirrors include/h3b.h
SIGNATURES: dict[str, list[Any]] = {
    "h3b_rmsnorm_modulate": [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                             _f32, _p],
    "h3b_residual_gate_rmsnorm_modulate": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64,
                                           _i64, _i64, _i64, _i64, _i64, _f32, _p],
    "h3b_modulate": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p],
    "h3b_gated_residual": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p],
    "h3b_swiglu": [_p, _p, _i64, _i64, _i64, _i64, _p],
    "h3b_gelu_tanh": [_p, _p, _i64, _i64, _i64, _i64, _p],
    "h3b_qknorm_rope": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _f32, _p],
    "h3b_qknorm_rope_pack": [_p, _p, _p, _p, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _i64,
                             _i64, _i64, _i64, _f32, _f32, _p],
    "h3b_pack_qkv": [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                     _i64, _p],
    "h3b_merge_heads": [_p, _p, _i64, _i64, _i64, _p],
    "h3b_attention": [_p, _p, _p, _p] + [_i64] * 17 + [_f32, _p, _i64, _p],
    "h3b_attention_workspace_size": [_i64, _i64, _i64, _i64, _i64, ctypes.POINTER(_i64)],
    "h3b_attention_noalloc": [_p, _p, _p, _p] + [_i64] * 17 + [_f32, _p],
    "h3b_clear_device_status": [_p],
    "h3b_qknorm_rope_pack_p2p": [_p, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _p, _p, _p,
                                 _p, _i64, _i64, _i64, _i64, _f32, _f32, _p],
    "h3b_scatter_heads_p2p": [_p, _p, _p, _i64, _i64, _i64, _i64, _p],
    "h3b_qkv_gemm_pack": [_p, _i64, _p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64,
                          _i64, _f32, _f32, _p, _i64, _p],
    "h3b_qkv_gemm_pack_workspace_size": [_i64, _i64, ctypes.POINTER(_i64)],
    "h3b_qkv_gemm_pack_p2p": [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p,
                              _i64, _i64, _i64, _f32, _f32, _p, _i64, _p],
    "h3b_gemm": [_p, _i64, _p, _i64, _i64, _i64, _p, _i64, _p, _i64, _p],
    "h3b_gemm_swiglu": [_p, _i64, _p, _i64, _i64, _i64, _p, _i64, _p, _p],
    "h3b_gemm_gated_residual": [_p, _i64, _p, _i64, _i64, _i64, _p, _i64, _p, _p, _i64, _p, _i64, _p, _i64,
                                _p],
    "h3b_attention_p2p": [_p, _p, _i64, _i64, _p, _i64, _i64, _f32, _p, _i64, _p],
    "h3b_peer_barrier": [_p, _i64, _i64, _p],
    "h3b_ipc_handle": [_p, _p, ctypes.POINTER(_i64)],
    "h3b_ipc_open": [_p, _i64, ctypes.POINTER(_p)],
    "h3b_ipc_close": [_p, _i64],
}


def library_path() -> Path:
    override = os.environ.get("H3B_LIBRARY")
    return Path(override) if override else _build.LIB_PATH


def load() -> ctypes.CDLL:
    """Load libh3b.so (building it first if this checkout has nvcc and it is stale)."""

    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = library_path()
        if os.environ.get("H3B_LIBRARY") is None and _build.is_stale():
            try:
                _build.build()
            except Exception as error:  # pragma: no cover - depends on toolchain
                if not path.exists():
                    raise RuntimeError(
                        f"h3b CUDA extension missing at {path} and could not be built: {error}"
                    ) from error
        if not path.exists():
            raise RuntimeError(f"h3b CUDA extension missing at {path}; run h3_flash_b200._build")
        lib = ctypes.CDLL(str(path))
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
        lib.h3b_abi_version.restype = ctypes.c_int
        lib.h3b_last_error.restype = ctypes.c_char_p
        lib.h3b_device_status.argtypes = [ctypes.POINTER(ctypes.c_int)]
        lib.h3b_device_status.restype = ctypes.c_int
        lib.h3b_peer_flags_bytes.argtypes = []
        lib.h3b_peer_flags_bytes.restype = ctypes.c_int64
        lib.h3b_kernel_launches.argtypes = []
        lib.h3b_kernel_launches.restype = ctypes.c_int64
        lib.h3b_reset_kernel_launches.argtypes = []
        lib.h3b_reset_kernel_launches.restype = None
        version = lib.h3b_abi_version()
        if version != ABI_VERSION:
            raise RuntimeError(f"libh3b.so ABI {version} != expected {ABI_VERSION}")
        _LIB = lib
        return lib


def exported_symbols() -> list[str]:
    return sorted(SIGNATURES) + ["h3b_abi_version", "h3b_last_error", "h3b_device_status",
                                 "h3b_peer_flags_bytes", "h3b_kernel_launches",
                                 "h3b_reset_kernel_launches"]


def check(code: int, what: str) -> None:
    """Map a C status code to the Python exception the reference raises."""

    if code == H3B_OK:
        return
    message = load().h3b_last_error().decode(errors="replace") or what
    if code == H3B_ERR_VALUE:
        raise ValueError(message)
    raise RuntimeError(message)


def call(name: str, *args: Any) -> None:
    """Call an entry point and raise on a failing status."""

    check(getattr(load(), name)(*args), name)


def reset_launch_count() -> None:
    load().h3b_reset_kernel_launches()


def launch_count() -> int:
    """h3b kernels launched by this process since the last reset, counted by the
    library at each launch (an attention call with a split tail launches two)."""

    return int(load().h3b_kernel_launches())


def device_status() -> int:
    value = ctypes.c_int(0)
    check(load().h3b_device_status(ctypes.byref(value)), "h3b_device_status")
    return value.value


def clear_device_status(stream: int) -> None:
    call("h3b_clear_device_status", stream)
