"""Seeded GGML payload generators for the tests and the benchmark inputs.

``random_payload`` follows the scheme of the reference's kernel test
(``tests/test_native_kernels.py:32-87``): pseudo-random bytes with every fp16
scale / min word of each block overwritten by a finite half, so the payload
exercises every code path of the decoders without NaN scales.  It is
vectorised with numpy so benchmark-size matrices take milliseconds.
"""
from __future__ import annotations

import numpy as np

from pyrite_b200.ggml_types import spec

#: byte offsets of fp16 scale words inside a block (the reference test's table)
SCALE_OFFSETS: dict[int, tuple[int, ...]] = {
    1: (0,), 2: (0,), 3: (0, 2), 6: (0,), 7: (0, 2), 8: (0,), 9: (0, 2), 10: (80, 82),
    11: (108,), 12: (0, 2), 13: (0, 2), 14: (208,), 20: (0,), 23: (0,), 30: (0,),
}
_FLOAT_LINEAR = {0: np.float32, 28: np.float64}


def random_payload(ggml_type: int, rows: int, cols: int, seed: int = 0, scale_half: float = 0.0078125) -> bytes:
    """``rows`` rows of ``cols`` values with finite scales (default scale 2^-7)."""
    rng = np.random.default_rng(seed)
    t = spec(ggml_type)
    if ggml_type in _FLOAT_LINEAR:
        return rng.uniform(-1.0, 1.0, rows * cols).astype(_FLOAT_LINEAR[ggml_type]).tobytes()
    nblocks = rows * (cols // t.block_size)
    raw = rng.integers(0, 256, size=(nblocks, t.bytes_per_block), dtype=np.uint8)
    if ggml_type in (1, 30):  # F16 / BF16: keep every value finite and modest
        vals = rng.uniform(-1.0, 1.0, nblocks).astype(np.float32)
        if ggml_type == 1:
            raw = vals.astype(np.float16).view(np.uint8).reshape(nblocks, 2)
        else:
            raw = (vals.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).reshape(nblocks, 2)
        return raw.tobytes()
    half = np.frombuffer(np.float16(scale_half).tobytes(), dtype=np.uint8)
    for off in SCALE_OFFSETS.get(ggml_type, ()):
        raw[:, off:off + 2] = half
    return raw.tobytes()


def row_bytes(ggml_type: int, cols: int) -> int:
    t = spec(ggml_type)
    return cols // t.block_size * t.bytes_per_block
