"""ctypes binding of ``libtrntensor_b200.so`` (declared in include/trntensor_b200.h).

There is no fallback: if the library is missing or cannot be loaded, every
device entry point raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libtrntensor_b200.so"
_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

TT_OK = 0
TT_ERR_NULL = 1
TT_ERR_SHAPE = 2
TT_ERR_ALIGN = 3
TT_ERR_WORKSPACE = 4
TT_ERR_DEVICE = 5
TT_ERR_CUDA = 6
TT_ERR_TMA = 7

_P = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); must match include/trntensor_b200.h
SIGNATURES: dict[str, tuple] = {
    "tt_status_string": (ctypes.c_char_p, [_I]),
    "tt_version": (_I, []),
    "tt_device_check": (_I, []),
    "tt_last_cuda_error": (ctypes.c_char_p, []),
    "tt_mp2_num_pairs": (_LL, [_I]),
    "tt_mp2_workspace_bytes": (_SZ, [_I, _I, _I]),
    "tt_mp2_tf32_workspace_bytes": (_SZ, [_I, _I, _I]),
    "tt_split_tf32": (_I, [_P, _P, _P, _LL, _I, _I, _P]),
    "tt_split_i8": (_I, [_P, _P, _P, _LL, _I, _I, _P]),
    "tt_mp2_range_stats_f32": (_I, [_P, _LL, _I, _P, _P]),
    "tt_split_i8_rows": (_I, [_P, _P, _P, _LL, _LL, _LL, _I, _I, _P]),
    "tt_mp2_energy_f32": (_I, [_P, _P, _P, _I, _I, _I, _LL, _LL, _P, _SZ, _P, _P, _P, _P]),
    "tt_mp2_energy_presplit_i8": (_I, [_P, _P, _I, _P, _P, _I, _I, _LL, _LL, _P, _P, _P, _P]),
    "tt_mp2_energy_f32_noalloc": (_I, [_P, _P, _P, _I, _I, _I, _P, _P, _P, _P]),
    "tt_mp2_energy_tf32x3": (_I, [_P, _P, _I, _P, _P, _I, _I, _LL, _LL, _P, _P, _P, _P]),
    "tt_mp2_energy_f64": (_I, [_P, _P, _P, _I, _I, _I, _LL, _LL, _P, _P, _P]),
    "tt_mp2_f64_workspace_bytes": (_SZ, [_I, _I, _I]),
    "tt_mp2_energy_f64_tc": (_I, [_P, _P, _P, _I, _I, _I, _LL, _LL, _P, _SZ, _P, _P, _P, _P]),
    "tt_mp2_energy_simt_f32": (_I, [_P, _P, _P, _I, _I, _I, _LL, _LL, _P, _P, _P]),
    "tt_ao2mo_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "tt_ao2mo_f32": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _SZ, _P, _P, _P]),
    "tt_ao2mo_f32_slab": (_I, [_P, _LL, _LL, _P, _P, _I, _I, _I, _I, _P, _SZ, _P, _P, _P]),
    "tt_ao2mo_simt_f32": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _SZ, _P, _P]),
    "tt_ao2mo_f64": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _SZ, _P, _P]),
    "tt_ao2mo_f64_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "tt_ao2mo_f64_tc": (_I, [_P, _P, _P, _I, _I, _I, _I, _P, _SZ, _P, _P, _P]),
    "tt_mp2_dd_workspace_bytes": (_SZ, [_I, _I, _I]),
    "tt_mp2_energy_dd": (_I, [_P, _P, _P, _I, _I, _I, _LL, _LL, _P, _SZ, _P, _P, _P]),
    "tt_gemm_dd": (_I, [_P, _P, _I, _LL, _P, _P, _I, _LL, _P, _P, _LL, _I, _I, _I, _I, _P]),
    "tt_debug_wait_timeout": (_I, [_P, _LL, _P, _P]),
    "tt_gemm_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "tt_gemm_f32": (_I, [_P, _I, _LL, _P, _I, _LL, _P, _LL, _I, _I, _I, _I, _P, _SZ, _P, _P]),
}


def library_path() -> Path:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load the device library once (thread-safe) and bind its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = os.environ.get("TRNTENSOR_B200_LIB", str(_LIB_PATH))
        if not Path(path).exists():
            raise RuntimeError(
                f"trntensor_b200 device library not found at {path}; build it with "
                "`python -m trntensor_b200._build` (nvcc, sm_100a). There is no CPU fallback."
            )
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


class DeviceError(RuntimeError):
    """A device-side wait ran out (the kernel recorded a status code)."""


def check(status: int, what: str) -> None:
    """Turn a C-ABI status code into the matching Python exception."""
    if status == TT_OK:
        return
    lib = load()
    msg = lib.tt_status_string(status).decode()
    if status == TT_ERR_CUDA:
        msg += f" ({lib.tt_last_cuda_error().decode()})"
    if status in (TT_ERR_SHAPE, TT_ERR_NULL, TT_ERR_ALIGN, TT_ERR_WORKSPACE):
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg}")
