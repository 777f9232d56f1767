"""The C-ABI library loads on a machine without a GPU and exports every symbol that
include/argus_b200.h declares (no compute calls are made here)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "argus_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(argus_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_header_symbols():
    from argus_b200 import _lib
    assert os.path.exists(_lib.LIB_PATH), "build the library first (python -m argus_b200.build)"
    L = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing
    assert L.argus_version() >= 100


def test_python_binding_covers_header():
    from argus_b200 import _lib, attention, paged
    from argus_b200.core import jl
    declared = set(declared_symbols())
    bound = (set(_lib.SIGNATURES) | set(attention.BOUND_SYMBOLS) | set(paged.BOUND_SYMBOLS) | set(jl.BOUND_SYMBOLS)
             | {"argus_status_string", "argus_last_error", "argus_version"})
    assert declared <= bound, sorted(declared - bound)


def test_status_strings():
    from argus_b200 import _lib
    assert _lib.status_string(0) == "ok"
    assert "misaligned" in _lib.status_string(_lib.ERR_MISALIGNED)
