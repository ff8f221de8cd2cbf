"""CPU checks of the C-ABI library: it builds, loads, exports every symbol the public header declares,
and its argument validation rejects bad calls with a status and a message (no kernel is launched)."""
import ctypes
import os
import re

import pytest

from openattention_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    names = []
    inc = os.path.join(ROOT, "include")
    for f in sorted(os.listdir(inc)):
        if f.endswith(".h"):
            src = open(os.path.join(inc, f)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names += re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(oa_\w+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = header_functions()
    assert "oa_flash_qhead_proxies" in names and "oa_version" in names and len(names) >= 4


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in header_functions():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def header_arities():
    """Parameter count of every oa_* function the public header declares."""
    out = {}
    inc = os.path.join(ROOT, "include")
    for f in sorted(os.listdir(inc)):
        if f.endswith(".h"):
            src = re.sub(r"/\*.*?\*/", "", open(os.path.join(inc, f)).read(), flags=re.S)
            for name, params in re.findall(r"\b(oa_\w+)\s*\(([^;{]*?)\)\s*;", src, flags=re.S):
                params = params.strip()
                out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_ctypes_signatures_match_the_header():
    """A ctypes argument list longer or shorter than the C declaration would pass garbage silently."""
    arities = header_arities()
    assert set(arities) == set(header_functions())
    for name, n in arities.items():
        assert len(_lib.SIGNATURES[name][1]) == n, f"{name}: header has {n} parameters, ctypes table " \
                                                   f"{len(_lib.SIGNATURES[name][1])}"


def test_version_and_error_path():
    lib = _lib.load()
    assert b"sm_100a" in lib.oa_version()
    # BQ = 0 fails validation before any device work
    st = lib.oa_flash_qhead_proxies(None, 0, None, None, 0, 0, None, 0, None, 0, None, None, 0, 0, None, 0, None, 0,
                                    0, 0, 0, 0, 0, ctypes.c_float(1.0), 0, None, 0, None)
    assert st == 1
    assert b"BQ" in lib.oa_last_error_string()
    with pytest.raises(RuntimeError, match="status 1"):
        _lib.call("oa_flash_qhead_proxies", None, 0, None, None, 0, 0, None, 0, None, 0, None, None, 0, 0, None, 0,
                  None, 0, 0, 0, 0, 0, 0, ctypes.c_float(1.0), 0, None, 0, None)


def test_workspace_sizing():
    lib = _lib.load()
    assert lib.oa_flash_workspace_bytes(1024, 15, 216, 64, 0) == 0          # enough rows: no split
    w = lib.oa_flash_workspace_bytes(32, 15, 216, 64, 0)                      # B=1: split-K
    assert w >= 32 * 2 * (128 * 4 + 8)
