"""The C ABI library loads, exports every symbol include/jasper_b200.h declares,
and reports host-side errors without touching a GPU."""
import ctypes as C
import re
from pathlib import Path

import pytest

from jasper_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    hdr = (ROOT / "include" / "jasper_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+char\*|int)\s+(jb_\w+)\s*\(", hdr, re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "jb_graph_search" in syms and "jb_graph_construct" in syms and len(syms) >= 15


@pytest.mark.parametrize("sym", declared_symbols())
def test_library_exports_symbol(sym):
    L = _lib.lib()
    assert hasattr(L, sym), sym


def test_python_signatures_cover_header():
    assert set(declared_symbols()) - {"jb_last_error"} <= set(_lib.SIGNATURES)


def test_abi_version():
    assert _lib.lib().jb_abi_version() == 1


def test_invalid_handle_is_reported():
    L = _lib.lib()
    info = _lib.GraphInfo()
    rc = L.jb_graph_get_info(987654, C.byref(info))
    assert rc == _lib.JB_ERR_INVALID_HANDLE
    assert b"Invalid handle" in L.jb_last_error()
    with pytest.raises(_lib.JasperError):
        _lib.call("jb_graph_free", 987654)


def test_bad_metric_is_invalid_argument():
    h = C.c_int64(-1)
    with pytest.raises(ValueError):
        _lib.call("jb_graph_load", b"/nonexistent", 128, 32, 7, 0, C.byref(h))


def test_null_out_pointer_is_invalid_argument():
    with pytest.raises(ValueError):
        _lib.call("jb_graph_get_info", 0, None)
