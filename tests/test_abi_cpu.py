"""CPU checks of the native boundary: the library loads and exports exactly the
functions that include/tcst_b200.h declares; host-side argument validation
rejects bad calls before any device work."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tcst_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tcst_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from torchcst_b200 import _native
    if not os.path.exists(_native.LIB_PATH):
        from torchcst_b200 import build
        build.build()
    return _native.load()


def test_header_matches_binding_table():
    from torchcst_b200 import _native
    assert declared_functions() == sorted(_native.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert b"sm_100a" in lib.tcst_version()


def test_struct_layouts_match_header():
    from torchcst_b200 import _native as N
    assert ctypes.sizeof(N.Axis) == 32
    assert ctypes.sizeof(N.Coordinates) == 8 + 8 * 8 + 64
    assert N.AdamW.field_ratio.offset == 32


def test_argument_errors_without_device(lib):
    from torchcst_b200 import _native as N
    ax = N.Axis(12, 5, 2, 8, 1.0, 0.0)  # 12/5 is not a merge power
    rc = lib.tcst_decode_route(None, 0, ctypes.byref(ax), ctypes.byref(ax),
                               ctypes.byref(N.Coordinates()), None, None, None, None, None)
    assert rc == 1
    assert b"base_tile_sites" in lib.tcst_last_error()
    ax = N.Axis(16, 1, 2, 32, 1.0, 0.0)
    rc = lib.tcst_atom_energies(None, 0, ctypes.byref(ax), ctypes.byref(ax), None, None)
    assert rc == 3  # modes above the build limit
    rc = lib.tcst_gemm_tf32x3(-1, 1, 1, None, None, 4, 0, None, None, 4, 0, None, 4, 1, 0,
                              None, None)
    assert rc == 1
    with pytest.raises(ValueError):
        N.check(1, "probe")
