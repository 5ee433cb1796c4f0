"""The C-ABI library loads and exports every symbol its header declares; host
argument checks report errors without touching a GPU."""
import ctypes as C
import re
from pathlib import Path

import pytest

from daric_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "daric_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"DARIC_API\s+[\w\s\*]+?\b(daric_\w+)\s*\(", text)))


def test_i64_passes_int64_arrays_by_address():
    """Host int64 arrays reach the C ABI as addresses: a contiguous int64
    vector is used as is, anything else is converted to one first."""
    import numpy as np
    a = np.arange(5, dtype=np.int64)
    arr, addr = _lib.i64(a)
    assert arr is a and addr == a.ctypes.data
    for src in ([3, 1, 2], np.arange(6, dtype=np.int64)[::2], np.arange(3, dtype=np.int32), np.ones((2, 2), np.int64)):
        arr, addr = _lib.i64(src)
        assert arr.dtype == np.int64 and arr.ndim == 1 and arr.flags.c_contiguous
        assert addr == arr.ctypes.data
        np.testing.assert_array_equal(arr, np.asarray(src).reshape(-1))
        assert np.ctypeslib.as_array((C.c_int64 * arr.size).from_address(addr)).tolist() == arr.tolist()


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "daric_copier_scatter_pages" in syms and "daric_score_select" in syms
    assert len(syms) >= 17


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for s in declared_symbols():
        assert hasattr(lib, s), s
    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_exports_are_only_the_c_abi():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.lib_path())], capture_output=True, text=True).stdout
    names = [l.split()[-1] for l in out.splitlines() if " T " in l]
    assert names and all(n.startswith("daric_") for n in names), names


def test_host_errors_without_gpu():
    lib = _lib.load()
    h = C.c_void_p()
    _lib.check(lib.daric_copier_create(C.byref(h)))
    try:
        sizes, sp = _lib.i64([2, 4, 16, 8, 128])
        strides, tp = _lib.i64([65536, 16384, 1024, 128, 1])
        rc = lib.daric_copier_register_layer(h, b"l0", C.c_void_p(0x1000), -1, 5, sp, tp, 2, 0)
        assert rc == _lib.ERR_INVALID and b"must be on GPU" in lib.daric_last_error()
        # scatter before register_store -> reference message (copier.cpp:83)
        names = _lib.names_array(["l0"])
        off, op = _lib.i64([0])
        rc = lib.daric_copier_scatter_pages(h, 1, names, op, op, None, 0, 0, op, None)
        assert rc == _lib.ERR_INVALID
        assert b"store buffer not registered" in lib.daric_last_error()
        with pytest.raises(_lib.DaricError, match="store buffer not registered"):
            _lib.check(rc)
    finally:
        lib.daric_copier_destroy(h)


def test_register_layer_shape_checks_without_gpu():
    lib = _lib.load()
    h = C.c_void_p()
    _lib.check(lib.daric_copier_create(C.byref(h)))
    try:
        # holes in the page span are rejected as in helpers.cu:49-59
        sizes, sp = _lib.i64([2, 4, 16, 8, 128])
        strides, tp = _lib.i64([4 * 16 * 8 * 256, 16 * 8 * 256, 8 * 256, 256, 1])
        rc = lib.daric_copier_register_layer(h, b"l0", C.c_void_p(0x1000), 0, 5, sp, tp, 2, 0)
        assert rc == _lib.ERR_INVALID and b"dense physical span" in lib.daric_last_error()
        strides, tp = _lib.i64([4 * 16 * 8 * 128, 16 * 8 * 128, 8 * 128, 128, 1])
        _lib.check(lib.daric_copier_register_layer(h, b"l0", C.c_void_p(0x1000), 0, 5, sp, tp, 2, 0))
    finally:
        lib.daric_copier_destroy(h)
