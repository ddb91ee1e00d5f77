"""The C-ABI library loads without a GPU and exports every function that
include/toy_b200.h declares (no compute calls here)."""
import ctypes as C
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "toy_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = set(re.findall(r"\b((?:tnn|tb2)_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_functions()
    assert "tb2_gemm" in names and "tnn_compute_backward" in names and "tb2_llama_realize" in names


def test_library_loads_and_exports_all_declared_symbols():
    from toy_b200 import _lib
    L = _lib.lib()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing


def test_no_cpu_backend():
    """backend_kind 0 (CPU) is refused: there is no CPU fallback path."""
    from toy_b200 import _lib
    L = _lib.lib()
    assert L.tnn_link_check() == 73
    assert not L.tnn_session_new(0)
