"""ctypes binding of ``libtoyb200.so`` (the C ABI declared in include/toy_b200.h).

The library is the product; this module only declares argument types. It
fails loudly when the shared library is missing: there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtoyb200.so")


class Operand(C.Structure):
    _fields_ = [("hi", C.c_void_p), ("lo", C.c_void_p), ("mn_major", C.c_int), ("ld", C.c_longlong),
                ("rows", C.c_int), ("cols", C.c_int), ("batch_stride", C.c_longlong), ("nbatch", C.c_int),
                ("bdiv1", C.c_int), ("bmul1", C.c_int), ("bdiv2", C.c_int), ("bmul2", C.c_int)]


class Epilogue(C.Structure):
    _fields_ = [("mode", C.c_int), ("alpha", C.c_float), ("out", C.c_void_p), ("res", C.c_void_p),
                ("out_hi", C.c_void_p), ("out_lo", C.c_void_p), ("bstride", C.c_longlong), ("m_div", C.c_int),
                ("m_s1", C.c_longlong), ("m_s0", C.c_longlong), ("n_div", C.c_int), ("n_s1", C.c_longlong)]


_lib = None

# (name, restype, argtypes) for every exported symbol this module binds.
_SIGS = [
    ("tb2_gemm", C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(Operand), C.POINTER(Operand),
                           C.POINTER(Epilogue), C.c_void_p]),
    ("tb2_split_f32", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    ("tb2_device_error", C.c_int, []),
    ("tb2_version", C.c_char_p, []),
]


def lib() -> C.CDLL:
    """Load the shared library once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"toy_b200: {LIB_PATH} is missing; run `python toy_b200/build.py` "
                               "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, res, args in _SIGS:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"toy_b200: {what} failed with code {rc}")
