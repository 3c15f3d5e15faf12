"""GGML quantizers (host, multithreaded C++ in libpyrite_b200.so).

``quantize(type_id, values)`` returns the GGML payload bytes of ``values`` (a
flat float array whose length is a multiple of the block size).  Q8_0 / Q4_0
and Q2_K..Q6_K are byte-identical to the reference's fixture encoders
(``scripts/build_vocab_fixture.py`` and ``tests/k_quant.py``); Q4_1 / Q5_0 /
Q5_1 to the gguf package's quantizers, which the reference's tests use for
those formats; IQ4_NL / IQ4_XS use this package's own encoder.
"""
from __future__ import annotations

import numpy as np

from . import _lib
from .ggml_types import spec


def quantize_types() -> tuple[int, ...]:
    lib = _lib.require()
    n = lib.pyrite_quantize_types(None, 0)
    import ctypes
    buf = (ctypes.c_int * n)()
    lib.pyrite_quantize_types(buf, n)
    return tuple(buf)


def quantize(type_id: int, values, threads: int = 0) -> bytes:
    lib = _lib.require()
    t = spec(type_id)
    src = np.ascontiguousarray(np.asarray(values, dtype=np.float64).ravel())
    if src.size == 0 or src.size % t.block_size:
        raise ValueError(f"{t.name} needs a multiple of {t.block_size} values, got {src.size}")
    dst = np.empty(src.size // t.block_size * t.bytes_per_block, dtype=np.uint8)
    code = lib.pyrite_quantize(type_id, src.ctypes.data, src.size, dst.ctypes.data, dst.nbytes, threads)
    if code != 0:
        raise ValueError(f"quantize rejected the input (error {code}: {_lib.error_string(code)})")
    return dst.tobytes()


def gaussian_weights(rows: int, cols: int, seed: int, sigma: float = 0.02) -> np.ndarray:
    """Seeded N(0, sigma) float32 weights, ``numpy.random.default_rng(seed)``."""
    return np.random.default_rng(seed).normal(0.0, sigma, rows * cols).astype(np.float32)
