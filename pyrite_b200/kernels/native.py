"""ctypes shim over libpyrite_b200.so -- the reference kernel module's call surface.

Mirrors ``pyrite/kernels/native.py`` of the reference: the same functions
(``matvec``, ``dequantize_rows``, ``supports_native``, ``native_available``,
``native_type_ids``, ``sorted_native_types``), argument meaning and error
behaviour (``ValueError`` on a rejected shape or buffer), so an executor
written against the reference module can import this one instead.  The work
runs on the current CUDA device: the borrowed payload is copied to the device
for the call and decoded and accumulated in fp64 there.

The device-resident path (weights already in HBM, fp32 activations, the
caller's stream) is in :mod:`pyrite_b200.kernels.cuda`.

There is no CPU fallback: without the library or a CUDA device,
``native_available()`` is False and every compute call raises.
"""
from __future__ import annotations

import ctypes
from array import array
from collections.abc import Sequence

from .. import _lib
from ..ggml_types import type_name

#: GGML type ids with a kernel; must equal the library's table
#: (the reference keeps the same set in pyrite/kernels/native.py:31-53).
NATIVE_TYPES = frozenset({0, 1, 2, 3, 6, 7, 8, 9, 10, 11, 12, 13, 14, 20, 23, 24, 25, 26, 27, 28, 30})


class _PyBuffer(ctypes.Structure):
    """CPython's stable Py_buffer layout, used for a read-only simple view."""

    _fields_ = [
        ("buf", ctypes.c_void_p), ("obj", ctypes.c_void_p), ("length", ctypes.c_ssize_t),
        ("itemsize", ctypes.c_ssize_t), ("readonly", ctypes.c_int), ("ndim", ctypes.c_int),
        ("format", ctypes.c_void_p), ("shape", ctypes.c_void_p), ("strides", ctypes.c_void_p),
        ("suboffsets", ctypes.c_void_p), ("internal", ctypes.c_void_p),
    ]


_get_buffer = ctypes.pythonapi.PyObject_GetBuffer
_get_buffer.argtypes = (ctypes.py_object, ctypes.POINTER(_PyBuffer), ctypes.c_int)
_get_buffer.restype = ctypes.c_int
_release_buffer = ctypes.pythonapi.PyBuffer_Release
_release_buffer.argtypes = (ctypes.POINTER(_PyBuffer),)
_release_buffer.restype = None


def _library() -> ctypes.CDLL | None:
    lib = _lib.load()
    if lib is None:
        return None
    if frozenset(_lib.type_ids(lib)) != NATIVE_TYPES:
        # The two halves of the table drifted apart: refuse the library rather
        # than send a layout down the wrong kernel.
        return None
    return lib


def native_available() -> bool:
    """True when the library loaded and a CUDA device is usable."""
    return _library() is not None and _lib.device_count() > 0


def supports_native(ggml_type: int) -> bool:
    return ggml_type in NATIVE_TYPES and native_available()


def native_type_ids() -> tuple[int, ...]:
    lib = _library()
    return tuple(_lib.type_ids(lib)) if lib is not None else ()


def sorted_native_types() -> list[str]:
    return [type_name(t) for t in sorted(native_type_ids())]


def _with_buffer(payload, callback):
    view = _PyBuffer()
    _get_buffer(payload, ctypes.byref(view), 0)  # PyBUF_SIMPLE: contiguous bytes
    try:
        return callback(view.buf, view.length)
    finally:
        _release_buffer(ctypes.byref(view))


def _kernel_error(code: int, operation: str) -> None:
    if code == -4:
        raise RuntimeError(f"native {operation} failed on the CUDA device (error {code})")
    if code != 0:
        raise ValueError(f"native {operation} rejected the matrix buffer/shape (error {code})")


def _require(ggml_type: int) -> ctypes.CDLL:
    lib = _library()
    if ggml_type not in NATIVE_TYPES or lib is None or _lib.device_count() == 0:
        raise ValueError(f"no native kernel for GGML type {ggml_type}")
    return lib


def matvec(ggml_type: int, payload: bytes | bytearray | memoryview, vector: Sequence[float],
           rows: int, cols: int) -> list[float]:
    """Fused quantized matrix-vector product without a dequantized matrix."""
    lib = _require(ggml_type)
    if len(vector) != cols or rows <= 0 or cols <= 0:
        raise ValueError("matrix/vector shape mismatch")
    x = array("d", vector)
    result = array("d", [0.0]) * rows
    x_view = (ctypes.c_double * len(x)).from_buffer(x)
    out_view = (ctypes.c_double * len(result)).from_buffer(result)
    code = _with_buffer(payload, lambda address, length: lib.pyrite_matvec(
        ggml_type, address, length, x_view, out_view, rows, cols))
    _kernel_error(code, "matvec")
    return result.tolist()


def dequantize_rows(ggml_type: int, payload: bytes | bytearray | memoryview, rows: int,
                    cols: int) -> list[float]:
    """Dequantize a bounded row range (used for embedding lookups)."""
    lib = _require(ggml_type)
    if rows <= 0 or cols <= 0:
        raise ValueError("invalid or overflowing matrix shape")
    result = array("d", [0.0]) * (rows * cols)
    out_view = (ctypes.c_double * len(result)).from_buffer(result)
    code = _with_buffer(payload, lambda address, length: lib.pyrite_dequantize_rows(
        ggml_type, address, length, out_view, rows, cols))
    _kernel_error(code, "dequantize")
    return result.tolist()
