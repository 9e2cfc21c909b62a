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


def _declarations():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    return text, dict(re.findall(r"\b(tcst_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text))


def test_header_argument_counts_match_binding_table():
    """Every declared function takes as many parameters as its ctypes binding."""
    from torchcst_b200 import _native
    _, decls = _declarations()
    for name, params in decls.items():
        params = params.strip()
        count = 0 if params in ("", "void") else len(params.split(","))
        assert count == len(_native.SIGNATURES[name][1]), name


def test_adamw_struct_matches_header():
    """tcst_adamw (all 4-byte members) has the ctypes mirror's size and order."""
    from torchcst_b200 import _native as N
    text, _ = _declarations()
    body = re.search(r"typedef struct tcst_adamw \{(.*?)\} tcst_adamw;", text, re.S).group(1)
    names = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        for item in decl.split(None, 1)[1].split(","):
            m = re.match(r"\s*(\w+)\s*(?:\[(\d+)\])?", item)
            names += [m.group(1)] * int(m.group(2) or 1)
    mirror = []
    for fname, ftype in N.AdamW._fields_:
        mirror += [fname] * (ctypes.sizeof(ftype) // 4)
    assert names == mirror
    assert ctypes.sizeof(N.AdamW) == 4 * len(names)


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
    # Atom counts whose scratch byte count would overflow 64 bits are refused
    # before any size arithmetic or device call.
    ax = N.Axis(1024, 1, 2, 8, 1.0, 0.0)
    for atoms in (1 << 62, (1 << 63) - 1, 32769):
        rc = lib.tcst_assemble_weight_static(None, atoms, ctypes.byref(ax), ctypes.byref(ax),
                                             None, 0, None, None, 0, None)
        assert rc == 3, atoms
        assert b"more than the built-in" in lib.tcst_last_error()
    rc = lib.tcst_assemble_weight_static(None, -1, ctypes.byref(ax), ctypes.byref(ax),
                                         None, 0, None, None, 0, None)
    assert rc == 1
