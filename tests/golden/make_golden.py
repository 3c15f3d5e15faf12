"""Generate the golden vectors under tests/golden from the reference itself.

Run where the reference tree is (``PYRITE_REF_ROOT``, default: a
``reference`` directory beside the repository); the GPU box and the test
suite never need it, they read the committed ``.npz`` files.

    python tests/golden/make_golden.py

Outputs
-------
decoders.npz
    For each of the 21 decodable GGML types: the deterministic pseudo-random
    payload of the reference's kernel test (``tests/test_native_kernels.py``
    ``_payload``: LCG seed 20240607, fp16 scale words patched to 1.0), the
    values decoded by the reference Python decoder
    (``pyrite.tensor_ops.decode_vector``), the probe vector
    ``x[i] = 0.4 cos(0.13 i)`` and the reference C kernel's ``matvec`` of the
    two (``pyrite.kernels.native.matvec``).  Two shapes: 2x512 (the
    reference's own) and 3x1024 (seed 777).
encoders.npz
    Bytes produced by the reference's fixture quantizers -- ``tests/k_quant.py``
    (Q2_K..Q6_K) and ``scripts/build_vocab_fixture.py`` (Q8_0, Q4_0) -- over
    (a) the smooth weights of ``test_native_kernels`` and (b) seeded
    N(0, 0.02) float32 weights, so the package's quantizers can be checked for
    byte identity.
"""
from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
REF = Path(os.environ.get("PYRITE_REF_ROOT", ROOT.parent / "reference"))
OUT = Path(__file__).resolve().parent


def _import_reference():
    sys.path.insert(0, str(REF))
    import pyrite.kernels.native as native  # noqa: E402
    from pyrite.tensor_ops import DECODABLE_TYPES, decode_vector  # noqa: E402
    from scripts import build_vocab_fixture as bvf  # noqa: E402
    from tests import k_quant  # noqa: E402
    from tests import test_native_kernels as tnk  # noqa: E402

    return native, DECODABLE_TYPES, decode_vector, tnk, k_quant, bvf


def decoders(native, types, decode_vector, tnk) -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    for rows, cols, seed in ((2, 512, 20240607), (3, 1024, 777)):
        x = [math.cos(i * 0.13) * 0.4 for i in range(cols)]
        out[f"x_{cols}"] = np.array(x, dtype=np.float64)
        for t in sorted(types):
            payload = tnk._payload(t, rows, cols, seed)
            decoded = decode_vector(t, payload, rows * cols)
            key = f"{t}_{rows}x{cols}"
            out[f"payload_{key}"] = np.frombuffer(payload, dtype=np.uint8).copy()
            out[f"decoded_{key}"] = np.array(decoded, dtype=np.float64)
            if all(math.isfinite(v) for v in decoded):
                out[f"matvec_{key}"] = np.array(native.matvec(t, payload, x, rows, cols), dtype=np.float64)
    return out


def encoders(k_quant, bvf) -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    smooth = [math.sin(i * 0.071) * 0.6 + math.cos(i * 0.019) * 0.2 for i in range(2 * 512)]
    gauss = np.random.default_rng(1234).normal(0.0, 0.02, 4 * 1024).astype(np.float32)
    # Edge blocks: an all-zero block, a constant block and a single spike.
    edge = np.zeros(3 * 256, dtype=np.float32)
    edge[256:512] = 0.125
    edge[600] = -0.75
    sets = {"smooth": [float(v) for v in smooth], "gauss": [float(v) for v in gauss],
            "edge": [float(v) for v in edge]}
    for name, values in sets.items():
        out[f"input_{name}"] = np.array(values, dtype=np.float64)
        for t, enc in sorted(k_quant.K_ENCODERS.items()):
            out[f"enc_{t}_{name}"] = np.frombuffer(enc(values), dtype=np.uint8).copy()
        for t, enc in sorted(bvf.QUANT_ENCODERS.items()):
            out[f"enc_{t}_{name}"] = np.frombuffer(enc(values), dtype=np.uint8).copy()
    return out


def main() -> None:
    native, types, decode_vector, tnk, k_quant, bvf = _import_reference()
    if not native.native_available():
        raise SystemExit("the reference C library did not build")
    np.savez_compressed(OUT / "decoders.npz", **decoders(native, types, decode_vector, tnk))
    np.savez_compressed(OUT / "encoders.npz", **encoders(k_quant, bvf))
    for name in ("decoders.npz", "encoders.npz"):
        print(name, (OUT / name).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
