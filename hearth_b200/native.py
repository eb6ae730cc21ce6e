"""GPU counterparts of the reference's ``hearth._native`` kernel entry points
(python/hearth/_native.py:222-263): same names, argument meaning and error behaviour, computed by
the sm_100a kernels through include/hearth_b200.h."""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import last_error, lib


def _as_ptr(buf):
    if isinstance(buf, np.ndarray):
        a = np.ascontiguousarray(buf)
        return C.c_void_p(a.ctypes.data), a
    if isinstance(buf, (bytes, bytearray, memoryview)):
        a = np.frombuffer(buf, dtype=np.uint8)
        return C.c_void_p(a.ctypes.data), a
    raise TypeError(f"expected bytes or ndarray, got {type(buf).__name__}")


def row_bytes(dtype: int, n: int) -> int:
    return int(lib().hxb_row_bytes(int(dtype), int(n)))


def dequantize(dtype: int, buf, rows: int, cols: int) -> np.ndarray:
    """hearth_dequantize on the GPU."""
    ptr, keep = _as_ptr(buf)
    if keep.nbytes < rows * row_bytes(dtype, cols):
        raise ValueError("buffer too small")
    y = np.empty((rows, cols), dtype=np.float32)
    rc = lib().hxb_dequantize(int(dtype), ptr, int(rows), int(cols), C.c_void_p(y.ctypes.data))
    if rc != 0:
        raise RuntimeError(f"hxb_dequantize failed with {rc}: {last_error()}")
    return y


def matmul(dtype, W, rows, cols, X: np.ndarray, isa: int = 0) -> np.ndarray:
    """Y[T, rows] = X[T, cols] . W^T by the GPU kernels (NUMERICS §3, bit-identical to the
    reference's hearth_matmul). ``isa`` is accepted for signature compatibility and ignored."""
    if isa not in (0, 1, 2, 3):
        raise ValueError(f"isa must be 0 (auto), 1 (scalar), 2 (avx2) or 3 (avx512), got {isa!r}")
    X = np.ascontiguousarray(X, dtype=np.float32)
    if X.ndim == 1:
        X = X[None, :]
    if X.ndim != 2 or X.shape[1] != cols:
        raise ValueError(f"X must be [T, {cols}], got {X.shape}")
    rb = row_bytes(dtype, cols)
    if rb == 0:
        raise ValueError(f"dtype {dtype} cannot encode rows of {cols}")
    wptr, wkeep = _as_ptr(W)
    if wkeep.nbytes != rows * rb:
        raise ValueError(f"W has {wkeep.nbytes} bytes, expected {rows * rb}")
    T = X.shape[0]
    Y = np.empty((T, rows), dtype=np.float32)
    rc = lib().hxb_matmul(int(dtype), wptr, int(rows), int(cols), C.c_void_p(X.ctypes.data), int(T),
                          C.c_void_p(Y.ctypes.data))
    if rc != 0:
        raise RuntimeError(f"hxb_matmul(dtype={dtype}, {rows}x{cols}, T={T}) failed with {rc}: {last_error()}")
    return Y
