"""CPU checks of the C-ABI library: it loads and exports every entry point include/qres.h declares (no compute:
there is no GPU here)."""
import ctypes
import os
import re

from tt_qwen_resident_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(ROOT, "include", "qres.h")).read()
    return sorted(set(re.findall(r"^QRES_API\s+\w+\s+(qres_\w+)\(", src, flags=re.M)))


def test_header_matches_binding_list():
    assert declared() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared():
        assert hasattr(L, name), name
    _lib.lib()  # the typed binding resolves too


def test_errors_without_gpu_are_reported_not_raised():
    L = _lib.lib()
    h = ctypes.c_void_p()
    cfg = _lib.Config(2, 2, 0, 9, 1, 1, 0, 0)  # rows 9 > QRES_MAX_ROWS
    assert L.qres_create(ctypes.byref(cfg), 0, 1, ctypes.byref(h)) == 1
    assert "rows" in _lib.last_error()
    cfg = _lib.Config(2, 2, 0, 1, 1, 1, 0, 0)
    assert L.qres_create(ctypes.byref(cfg), 3, 2, ctypes.byref(h)) == 1  # rank out of range
