"""Several columns at once: the tcgen05 tensor-core product (B200).

For ncols >= 2 the main formats (Q8_0, Q4_K, Q5_K, Q6_K, IQ4_XS) run on the
5th-generation tensor cores with a split-bf16 scheme (W X ~= Whi Xhi + Whi Xlo
+ Wlo Xhi, fp32 accumulation in tensor memory).  The bar is the north star's:
every output within 1e-4 of sum_k |W[r,k] X[c,k]| of the oracle's fp64
product -- checked column by column against the C oracle at small sizes and
against an fp64 product of the (bit-exact, separately tested) decoded weights
at the configs[1] sizes.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests.payloads import random_payload

pytestmark = pytest.mark.gpu

TC_TYPES = [8, 12, 13, 14, 23]
TOL = 1e-4


def _run(ggml_type, payload, x, rows, cols, offset=0):
    import torch

    from pyrite_b200.kernels import cuda as K
    host = np.zeros(len(payload) + offset, dtype=np.uint8)
    host[offset:] = np.frombuffer(payload, dtype=np.uint8)
    buf = torch.from_numpy(host).cuda()
    y = K.matvec(ggml_type, buf[offset:], torch.from_numpy(x).cuda(), rows, cols)
    torch.cuda.synchronize()
    assert K.status() == 0
    return y.cpu().numpy()


def _check_columns(ggml_type, payload, x, rows, cols, got):
    w = O.dequantize_rows(ggml_type, payload, rows, cols)
    x64 = x.astype(np.float64)
    want = x64 @ w.T
    absdot = np.abs(x64) @ np.abs(w).T
    err = np.abs(got.astype(np.float64) - want) / np.maximum(absdot, 1e-30)
    assert float(err.max()) <= TOL, f"max relative error {err.max():.3e}"


@pytest.mark.parametrize("ncols", [2, 8, 16, 17, 33, 64, 65, 130])
@pytest.mark.parametrize("ggml_type", TC_TYPES)
def test_tc_columns_match_oracle(cuda_device, ggml_type, ncols):
    rows, cols = 67, 1536  # one partial row tile, K split over a 2-CTA cluster
    payload = random_payload(ggml_type, rows, cols, seed=ncols + 100 * ggml_type)
    x = np.random.default_rng(ncols).normal(0, 1, (ncols, cols)).astype(np.float32)
    got = _run(ggml_type, payload, x, rows, cols)
    assert got.shape == (ncols, rows)
    _check_columns(ggml_type, payload, x, rows, cols, got)


@pytest.mark.parametrize("rows,cols", [(1, 256), (128, 256), (300, 4096), (513, 1024), (2, 14336), (1000, 2304)])
@pytest.mark.parametrize("ggml_type", TC_TYPES)
def test_tc_ragged_shapes(cuda_device, ggml_type, rows, cols):
    ncols = 8
    payload = random_payload(ggml_type, rows, cols, seed=rows + cols)
    x = np.random.default_rng(rows).normal(0, 1, (ncols, cols)).astype(np.float32)
    _check_columns(ggml_type, payload, x, rows, cols, _run(ggml_type, payload, x, rows, cols))


@pytest.mark.parametrize("offset", [2, 4, 8, 14])
@pytest.mark.parametrize("ggml_type", TC_TYPES)
def test_tc_unaligned_payloads(cuda_device, ggml_type, offset):
    rows, cols, ncols = 19, 2048, 8
    payload = random_payload(ggml_type, rows, cols, seed=offset)
    x = np.random.default_rng(offset).normal(0, 1, (ncols, cols)).astype(np.float32)
    _check_columns(ggml_type, payload, x, rows, cols, _run(ggml_type, payload, x, rows, cols, offset))


def test_tc_extreme_magnitudes(cuda_device):
    """Activations spanning many binades (the bf16 split keeps fp32's range)."""
    rows, cols, ncols = 40, 1024, 16
    rng = np.random.default_rng(5)
    x = (rng.normal(0, 1, (ncols, cols)) * 10.0 ** rng.integers(-20, 20, (ncols, cols))).astype(np.float32)
    for t in TC_TYPES:
        payload = random_payload(t, rows, cols, seed=t)
        _check_columns(t, payload, x, rows, cols, _run(t, payload, x, rows, cols))


@pytest.mark.parametrize("ncols", [8, 64])
@pytest.mark.parametrize("ggml_type", TC_TYPES)
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (14336, 4096), (4096, 14336)])
def test_tc_configs1_sizes(cuda_device, ggml_type, rows, cols, ncols):
    """configs[1] at batch 8 and 64: quantized seeded N(0, 0.02) weights against
    an fp64 product of the decoded weights (the decoder is bit-exact)."""
    import torch

    from pyrite_b200.kernels import cuda as K
    from pyrite_b200.quantize import gaussian_weights, quantize
    payload = quantize(ggml_type, gaussian_weights(rows, cols, 7 + rows + cols))
    w = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    x = torch.randn(ncols, cols, device="cuda", generator=torch.Generator("cuda").manual_seed(ncols))
    got = K.matvec(ggml_type, w, x, rows, cols).double()
    wd = K.dequantize_rows(ggml_type, w, rows, cols).double()
    want = x.double() @ wd.T
    absdot = x.double().abs() @ wd.abs().T
    torch.cuda.synchronize()
    assert K.status() == 0
    assert float(((got - want).abs() / absdot.clamp_min(1e-30)).max()) <= TOL


def test_tc_is_deterministic(cuda_device):
    import torch

    from pyrite_b200.kernels import cuda as K
    rows, cols, ncols = 4096, 4096, 64
    for t in TC_TYPES:
        w = torch.frombuffer(bytearray(random_payload(t, rows, cols, seed=t)), dtype=torch.uint8).cuda()
        x = torch.randn(ncols, cols, device="cuda")
        a = K.matvec(t, w, x, rows, cols)
        b = K.matvec(t, w, x, rows, cols)
        assert torch.equal(a, b)
