"""The C-ABI shared library: loads without a GPU, exports every function the
header declares (and the Python binding covers exactly those), and rejects
bad arguments on the host before touching the device."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

from yanah_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "yanah_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(yn_\w+)\s*\(", text, flags=re.M)))


def test_header_declarations_parsed():
    names = declared_functions()
    assert "yn_stack_decode" in names and "yn_moe_layer_noalloc" in names
    assert len(names) >= 25


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_the_header():
    assert set(_lib.exported_symbols()) | {"yn_last_error", "yn_version"} == set(declared_functions())


def test_host_only_calls():
    lib = _lib.lib()
    lib.yn_version.restype = C.c_char_p
    assert b"sm_100a" in lib.yn_version()
    d = _lib.Dims(2048, 512, 10, 512, 512, 1, 1e-6)
    assert lib.yn_workspace_bytes(C.byref(d)) == 538_624
    assert lib.yn_stack_table_bytes(48) > 0


def test_argument_checks_before_any_device_work():
    lib = _lib.lib()
    lib.yn_last_error.restype = C.c_char_p
    d = _lib.Dims(2048, 512, 10, 512, 512, 1, 1e-6)
    layer = _lib.Layer()
    buf = (C.c_uint8 * 16)()
    p = C.cast(buf, C.c_void_p)
    # row count outside [1, YN_MAX_ROWS]
    for T in (0, 9):
        assert lib.yn_moe_layer(C.byref(d), C.byref(layer), p, T, None, 0, p, p, None) == _lib.YN_E_UNSUPPORTED
    # unsupported shapes
    bad = _lib.Dims(2048, 2048, 10, 512, 512, 1, 1e-6)
    assert lib.yn_moe_layer(C.byref(bad), C.byref(layer), p, 1, None, 0, p, p, None) == _lib.YN_E_UNSUPPORTED
    # aliasing input/output
    assert lib.yn_moe_layer(C.byref(d), C.byref(layer), p, 1, None, 0, p, p, None) == _lib.YN_E_INVALID
    assert b"alias" in lib.yn_last_error()
    # the static-workspace variant refuses a workspace above its fixed size
    big = _lib.Dims(4096, 512, 16, 2048, 2048, 1, 1e-6)
    q = C.cast((C.c_uint8 * 16)(), C.c_void_p)
    assert lib.yn_moe_layer_noalloc(C.byref(big), C.byref(layer), p, 1, None, 0, q, None, None) == \
        _lib.YN_E_UNSUPPORTED
    assert b"static scratch" in lib.yn_last_error()
