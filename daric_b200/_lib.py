"""ctypes binding of ``libdaric_b200.so`` (C ABI in include/daric_b200.h).

The shared library is the product: there is no Python or CPU implementation
behind these calls. Loading fails loudly when the library is missing.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

_LIB_PATH = Path(__file__).resolve().parent / "libdaric_b200.so"

OK = 0
ERR_INVALID = 1
ERR_CUDA = 2
ERR_STATE = 3
ERR_DEVICE = 4

DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_BF16 = 2
DTYPE_FP8_E4M3 = 3

ROPE_NONE = 0
ROPE_FLEXIBLE = 1
ROPE_DELTA = 2

SELECT_TOPK = 0
SELECT_THRESHOLD = 1

# int64 host arrays pass as addresses (numpy's ctypes.data): building a
# POINTER(c_int64) object per array costs more than the call's C side
_i64p = C.c_void_p
_i32p = C.POINTER(C.c_int32)
_vp = C.c_void_p

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "daric_last_error": (C.c_char_p, []),
    "daric_version": (C.c_int, []),
    "daric_device_sm_count": (C.c_int, [C.c_int, C.POINTER(C.c_int)]),
    "daric_device_errors": (C.c_int, [C.c_int, C.POINTER(C.c_int)]),
    "daric_copier_create": (C.c_int, [C.POINTER(_vp)]),
    "daric_copier_destroy": (None, [_vp]),
    "daric_copier_register_layer": (
        C.c_int, [_vp, C.c_char_p, _vp, C.c_int, C.c_int, _i64p, _i64p, C.c_int64, C.c_int]),
    "daric_copier_register_store": (C.c_int, [_vp, _vp, C.c_int64, C.c_int]),
    "daric_copier_register_rotary": (
        C.c_int, [_vp, C.c_char_p, C.c_int, _vp, C.c_int, C.c_int64, C.c_int64, C.c_int]),
    "daric_copier_gather_pages": (
        C.c_int, [_vp, C.c_int64, C.POINTER(C.c_char_p), _i64p, _i64p, _vp, C.c_int64, C.c_int, _i64p, _vp]),
    "daric_copier_scatter_pages": (
        C.c_int, [_vp, C.c_int64, C.POINTER(C.c_char_p), _i64p, _i64p, _vp, C.c_int64, C.c_int, _i64p, _vp]),
    "daric_copier_rerotate_scatter_pages": (
        C.c_int, [_vp, C.c_int64, C.POINTER(C.c_char_p), _i64p, _i64p, _vp, C.c_int64, C.c_int, _i64p,
                  _i64p, C.c_int, C.c_int64, _i64p, _i64p, _i64p, _vp, C.c_int64, _i64p, _i64p, _vp]),
    "daric_copier_load_chunks": (
        C.c_int, [_vp, C.c_int64, C.POINTER(C.c_char_p), C.c_int64, C.c_int64, C.c_int64, _i64p, _i64p, _i64p,
                  _vp, C.c_int64, C.c_int, C.c_int, _i64p, _i64p, _i64p, _vp, C.c_int64, _i64p, _vp]),
    "daric_copier_rerotate_inplace": (
        C.c_int, [_vp, C.c_int64, C.POINTER(C.c_char_p), C.c_int, C.c_int64, _vp, C.c_int64,
                  _i64p, _i64p, _i64p, _i64p, _i64p, _vp]),
    "daric_batched_memcpy_d2h": (C.c_int, [_vp, _vp, C.c_int64, _i64p, _i64p, _i64p, C.c_int, _vp]),
    "daric_batched_memcpy_h2d": (C.c_int, [_vp, _vp, C.c_int64, _i64p, _i64p, _i64p, C.c_int, _vp]),
    "daric_score_select": (
        C.c_int, [_vp, C.c_int64, C.c_int64, C.c_int64, _i64p, _i64p, _i64p, _i64p, C.c_int, C.c_float,
                  _vp, C.c_int64, _i64p, C.c_int64, _vp, _vp, _vp, C.c_int64, _i64p, C.c_int, _vp]),
    "daric_score_select_noalloc": (
        C.c_int, [_vp, C.c_int64, C.c_int64, C.c_int64, _i64p, _i64p, _i64p, _i64p, C.c_int, C.c_float,
                  _vp, C.c_int64, _i64p, C.c_int64, _vp, _vp, _vp, C.c_int64, _i64p, C.c_int, _vp]),
    "daric_ptrs_to_slots": (
        C.c_int, [C.c_int64, _i64p, _i64p, _i64p, _vp, C.c_int64, C.c_int64, _vp, _vp, C.c_int, _vp]),
}

_lib = None


def lib_path() -> Path:
    return _LIB_PATH


def load() -> C.CDLL:
    """Loads the native library (once). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        raise ImportError(
            f"daric_b200 native library not found at {_LIB_PATH}; build it with "
            "`python -m daric_b200.build` (nvcc, sm_100a). There is no fallback implementation.")
    lib = C.CDLL(str(_LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class DaricError(RuntimeError):
    """Error reported by the native library (reference: TORCH_CHECK / CUDA_CHECK)."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def check(status: int) -> None:
    if status != OK:
        msg = load().daric_last_error().decode(errors="replace")
        raise DaricError(status, msg)


def i64(values) -> tuple[np.ndarray, int]:
    """int64 host array + its address (keep the array alive while the address is used)."""
    a = values
    if not (type(a) is np.ndarray and a.dtype == np.int64 and a.ndim == 1 and a.flags.c_contiguous):
        a = np.ascontiguousarray(np.asarray(values, dtype=np.int64).reshape(-1))
    return a, a.ctypes.data


def names_array(names) -> C.Array:
    """char* array of layer names; an already-built array is passed through.
    Repeated names share one encoded buffer (the library caches lookups by
    pointer within a call)."""
    if isinstance(names, C.Array):
        return names
    cache: dict[str, bytes] = {}
    enc = [cache.setdefault(n, n.encode()) if isinstance(n, str) else bytes(n) for n in names]
    return (C.c_char_p * len(enc))(*enc)


def device_errors(device: int) -> int:
    """Reads and clears the device error bits (1 block id, 2 table position, 4 block table,
    8 a bounded wait in the bulk pipeline timed out)."""
    v = C.c_int(0)
    check(load().daric_device_errors(int(device), C.byref(v)))
    return v.value


def sm_count(device: int) -> int:
    v = C.c_int(0)
    check(load().daric_device_sm_count(int(device), C.byref(v)))
    return v.value
