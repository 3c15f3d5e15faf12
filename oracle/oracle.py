"""TEST INFRASTRUCTURE ONLY: Python handle on the CPU oracle.

Loads ``_build/libggml_oracle.so`` (the fp64 restatement in ``ggml_oracle.c``)
and, when it was built, ``_ref/libpyrite_native.so`` (the reference's own C
kernel library compiled from ``pyrite/kernels/native.c``).  Only the test
suite, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
import this module; the product package never does.

Pinning: ``tests/test_oracle.py`` checks the restatement against the golden
vectors in ``tests/golden`` (made by the reference's Python decoders,
``pyrite/tensor_ops.py``) and, when the reference library is present, against
that library bit for bit.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libggml_oracle.so"
REF_SO = HERE / "_ref" / "libpyrite_native.so"

_PD = ctypes.POINTER(ctypes.c_double)


def build() -> None:
    """Compile the oracle (and the reference library when its source exists)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _bind(lib: ctypes.CDLL, prefix: str) -> ctypes.CDLL:
    mv = getattr(lib, f"{prefix}_matvec")
    mv.argtypes = (ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, _PD, _PD, ctypes.c_size_t, ctypes.c_size_t)
    mv.restype = ctypes.c_int
    dq = getattr(lib, f"{prefix}_dequantize_rows")
    dq.argtypes = (ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, _PD, ctypes.c_size_t, ctypes.c_size_t)
    dq.restype = ctypes.c_int
    ty = getattr(lib, f"{prefix}_types" if prefix == "oracle" else f"{prefix}_native_types")
    ty.argtypes = (ctypes.POINTER(ctypes.c_int), ctypes.c_size_t)
    ty.restype = ctypes.c_int
    return lib


_ORACLE: ctypes.CDLL | None = None
_REF: ctypes.CDLL | None = None


def oracle_lib() -> ctypes.CDLL:
    global _ORACLE
    if _ORACLE is None:
        if not ORACLE_SO.is_file():
            build()
        _ORACLE = _bind(ctypes.CDLL(str(ORACLE_SO)), "oracle")
        _ORACLE.oracle_geometry.argtypes = (
            ctypes.c_int, ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t))
        _ORACLE.oracle_geometry.restype = ctypes.c_int
    return _ORACLE


def reference_lib() -> ctypes.CDLL | None:
    """The reference's C library built from source, or None where it was not built."""
    global _REF
    if _REF is None and REF_SO.is_file():
        _REF = _bind(ctypes.CDLL(str(REF_SO)), "pyrite")
    return _REF


def type_ids() -> list[int]:
    lib = oracle_lib()
    n = lib.oracle_types(None, 0)
    buf = (ctypes.c_int * n)()
    lib.oracle_types(buf, n)
    return list(buf)


def geometry(type_id: int) -> tuple[int, int]:
    bs, bpb = ctypes.c_size_t(), ctypes.c_size_t()
    if oracle_lib().oracle_geometry(type_id, ctypes.byref(bs), ctypes.byref(bpb)) != 0:
        raise ValueError(f"unknown GGML type {type_id}")
    return bs.value, bpb.value


def row_bytes(type_id: int, cols: int) -> int:
    bs, bpb = geometry(type_id)
    return cols // bs * bpb


def _call_matvec(fn, type_id, payload, x, rows, cols):
    buf = np.ascontiguousarray(np.frombuffer(payload, dtype=np.uint8))
    xv = np.ascontiguousarray(x, dtype=np.float64)
    out = np.zeros(rows, dtype=np.float64)
    rc = fn(type_id, buf.ctypes.data, buf.nbytes, xv.ctypes.data_as(_PD), out.ctypes.data_as(_PD), rows, cols)
    if rc != 0:
        raise ValueError(f"oracle matvec rejected the matrix (error {rc})")
    return out


def matvec(type_id: int, payload, x, rows: int, cols: int) -> np.ndarray:
    """fp64 ``W @ x`` for ``rows`` quantized rows (oracle restatement)."""
    return _call_matvec(oracle_lib().oracle_matvec, type_id, payload, x, rows, cols)


def matvec_threaded(type_id: int, payload, x, rows: int, cols: int, threads: int | None = None) -> np.ndarray:
    """Same result as :func:`matvec`, row ranges split over host threads."""
    from concurrent.futures import ThreadPoolExecutor

    threads = threads or os.cpu_count() or 1
    buf = np.frombuffer(payload, dtype=np.uint8)
    rb = row_bytes(type_id, cols)
    bounds = [rows * i // threads for i in range(threads + 1)]
    with ThreadPoolExecutor(threads) as pool:
        parts = pool.map(
            lambda i: matvec(type_id, buf[bounds[i] * rb:bounds[i + 1] * rb], x, bounds[i + 1] - bounds[i], cols)
            if bounds[i + 1] > bounds[i] else np.zeros(0),
            range(threads))
        return np.concatenate(list(parts))


def dequantize_rows(type_id: int, payload, rows: int, cols: int) -> np.ndarray:
    lib = oracle_lib()
    buf = np.ascontiguousarray(np.frombuffer(payload, dtype=np.uint8))
    out = np.zeros(rows * cols, dtype=np.float64)
    rc = lib.oracle_dequantize_rows(type_id, buf.ctypes.data, buf.nbytes, out.ctypes.data_as(_PD), rows, cols)
    if rc != 0:
        raise ValueError(f"oracle dequantize rejected the matrix (error {rc})")
    return out.reshape(rows, cols)


def reference_matvec(type_id: int, payload, x, rows: int, cols: int) -> np.ndarray:
    lib = reference_lib()
    if lib is None:
        raise RuntimeError("reference library not built")
    return _call_matvec(lib.pyrite_matvec, type_id, payload, x, rows, cols)


def reference_matvec_threaded(type_id: int, payload, x, rows: int, cols: int, threads: int | None = None) -> np.ndarray:
    """The reference C kernel over row ranges on ``threads`` host threads."""
    from concurrent.futures import ThreadPoolExecutor

    threads = threads or os.cpu_count() or 1
    buf = np.frombuffer(payload, dtype=np.uint8)
    rb = row_bytes(type_id, cols)
    bounds = [rows * i // threads for i in range(threads + 1)]
    with ThreadPoolExecutor(threads) as pool:
        parts = pool.map(
            lambda i: reference_matvec(type_id, buf[bounds[i] * rb:bounds[i + 1] * rb], x,
                                       bounds[i + 1] - bounds[i], cols)
            if bounds[i + 1] > bounds[i] else np.zeros(0),
            range(threads))
        return np.concatenate(list(parts))


def reference_dequantize_rows(type_id: int, payload, rows: int, cols: int) -> np.ndarray:
    lib = reference_lib()
    if lib is None:
        raise RuntimeError("reference library not built")
    buf = np.ascontiguousarray(np.frombuffer(payload, dtype=np.uint8))
    out = np.zeros(rows * cols, dtype=np.float64)
    rc = lib.pyrite_dequantize_rows(type_id, buf.ctypes.data, buf.nbytes, out.ctypes.data_as(_PD), rows, cols)
    if rc != 0:
        raise ValueError(f"reference dequantize rejected the matrix (error {rc})")
    return out.reshape(rows, cols)


def moe_route(logits, top_k: int, norm_topk_prob: bool = True, scale: float = 1.0) -> tuple[list[int], list[float]]:
    """The reference's routing (pyrite/executor.py:757-772): fp64 softmax
    (pyrite/tensor_ops.py:513-521), experts ranked by (-p, e), the top_k
    weights renormalised to sum 1 when norm_topk_prob, then scaled."""
    import math
    values = [float(v) for v in logits]
    m = max(values)
    exps = [math.exp(v - m) for v in values]
    total = sum(exps)
    probs = [e / total for e in exps]
    chosen = sorted(range(len(probs)), key=lambda e: (-probs[e], e))[:top_k]
    weights = [probs[e] for e in chosen]
    if norm_topk_prob:
        t = sum(weights)
        if t > 0:
            weights = [w / t for w in weights]
    if scale != 1.0:
        weights = [w * scale for w in weights]
    return chosen, weights
