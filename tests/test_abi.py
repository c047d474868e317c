"""CPU checks of the C-ABI library: it is built, loads, and exports every declared symbol."""
import ctypes
import pathlib
import re

from tt_atom import _lib

HEADER = pathlib.Path(__file__).resolve().parents[1] / "include" / "atom_b200.h"


def declared():
    src = HEADER.read_text()
    return sorted(set(re.findall(r"^int\s+(atom_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_entry_points():
    names = declared()
    assert "atom_gemm" in names and "atom_fused_rotate" in names and len(names) > 20


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib._LIB_PATH))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    assert set(declared()) <= set(_lib.declared_symbols()), \
        set(declared()) - set(_lib.declared_symbols())


def test_argument_errors_are_reported_without_a_gpu():
    lib = _lib.lib()
    # W not a multiple of 4 -> ATOM_ERR_ARG before any device work
    rc = lib.atom_fused_rotate(None, None, 1, 9, 9, 6, 1, None, None, None, None, None)
    assert rc == 1
    assert "multiple of 4" in _lib.last_error()
    g = _lib.GemmGroups()
    g.ngroups = 0
    assert lib.atom_gemm(None, 1, 1, ctypes.byref(g), None, 1, None, None, None, None, None, 0,
                         0, 0, 0, None) == 1
