"""Host-side helpers of the reference's FFI module, over the toy_b200 C ABI.

Mirrors the TinyNN helpers toy's recipes call (lib/toy/ffi/tinynn.rb:1054-1100):
upload_int_array, upload_row_major, download_row_major. Arrays are numpy
arrays or Python sequences instead of Ruby Mats; numeric conventions are the
same (f64 on the host, narrowed to f32 / i32 by the library).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import check, lib


def _f64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64).reshape(-1))


def _i64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64).reshape(-1))


def upload_int_array(sess, tensor, values) -> None:
    """TinyNN.upload_int_array (tinynn.rb:1060) -> tnn_upload_from_int_array."""
    a = _i64(values)
    check(lib().tnn_upload_from_int_array(sess, tensor, a.ctypes.data_as(C.POINTER(C.c_long)), a.size),
          "tnn_upload_from_int_array")


def upload_row_major(sess, tensor, mat) -> None:
    """TinyNN.upload_row_major (tinynn.rb:1054) -> tnn_upload_from_float_array."""
    a = _f64(mat)
    check(lib().tnn_upload_from_float_array(sess, tensor, a.ctypes.data_as(C.POINTER(C.c_double)), a.size),
          "tnn_upload_from_float_array")


def upload_label_ids(sess, tensor, ids) -> None:
    """Index fast path for the labels tensor (one id per token, -1 = none)."""
    a = _i64(ids)
    check(lib().tb2_upload_label_ids(sess, tensor, a.ctypes.data_as(C.POINTER(C.c_long)), a.size),
          "tb2_upload_label_ids")


def download_row_major(sess, tensor, rows: int, cols: int) -> np.ndarray:
    """TinyNN.download_row_major (tinynn.rb:1090-1100) -> tnn_download_to_f64_array."""
    out = np.empty(rows * cols, dtype=np.float64)
    check(lib().tnn_download_to_f64_array(sess, tensor, out.ctypes.data_as(C.POINTER(C.c_double)), out.size),
          "tnn_download_to_f64_array")
    return out.reshape(rows, cols)
