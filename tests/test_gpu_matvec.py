"""Parity of the CUDA path with the oracle, through the C ABI (B200).

Bars (north star): dequantized values bit-exact (fp64 entry points: equal to
the reference's doubles; fp32 entry points: equal to the reference's doubles
rounded to fp32); matvec rows within max relative error 1e-4 for the fp32
device path, measured against sum_k |W[r,k] x[k]| (so rows whose terms cancel
do not dominate); the fp64 reference-compatible entry point within the
reference's own 1e-11 (tests/test_native_kernels.py:105-126).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests.payloads import random_payload, row_bytes

pytestmark = pytest.mark.gpu

TYPES = [0, 1, 2, 3, 6, 7, 8, 9, 10, 11, 12, 13, 14, 20, 23, 24, 25, 26, 27, 28, 30]
FP32_MATVEC_TOL = 1e-4


def _torch():
    import torch
    return torch


def rel_err(got, want, absdot):
    return float(np.max(np.abs(np.asarray(got, dtype=np.float64) - want) / np.maximum(absdot, 1e-30)))


def abs_dot(ggml_type, payload, x, rows, cols):
    w = O.dequantize_rows(ggml_type, payload, rows, cols)
    return np.abs(w) @ np.abs(np.asarray(x, dtype=np.float64))


# ---- reference-compatible entry points (host fp64 buffers) -------------------

@pytest.mark.parametrize("shape", [(2, 512), (3, 1024)])
@pytest.mark.parametrize("ggml_type", TYPES)
def test_compat_matvec_and_dequantize_match_reference_golden(cuda_device, golden_decoders, ggml_type, shape):
    from pyrite_b200.kernels import native
    rows, cols = shape
    key = f"{ggml_type}_{rows}x{cols}"
    payload = golden_decoders[f"payload_{key}"].tobytes()
    decoded = golden_decoders[f"decoded_{key}"]
    got_rows = np.array(native.dequantize_rows(ggml_type, payload, rows, cols))
    finite = ~np.isnan(decoded)
    assert np.array_equal(got_rows[finite].view(np.uint64), decoded[finite].view(np.uint64))
    assert np.array_equal(np.isnan(got_rows), ~finite)
    if f"matvec_{key}" in golden_decoders.files:
        x = golden_decoders[f"x_{cols}"]
        got = native.matvec(ggml_type, payload, list(x), rows, cols)
        assert got == pytest.approx(list(golden_decoders[f"matvec_{key}"]), rel=1e-11, abs=1e-11)


def test_compat_rejects_bad_shapes_like_the_reference(cuda_device):
    from pyrite_b200.kernels import native
    with pytest.raises(ValueError):
        native.matvec(8, bytes(33), [0.0] * 32, 1, 32)
    with pytest.raises(ValueError):
        native.matvec(12, bytes(144), [0.0] * 255, 1, 255)
    with pytest.raises(ValueError):
        native.matvec(99, bytes(4), [0.0], 1, 1)


# ---- device-resident fp32 path ----------------------------------------------------

def _device_matvec(ggml_type, payload, x, rows, cols, offset=0):
    """Run pyrite_cuda_matvec with the payload placed `offset` bytes into a buffer."""
    torch = _torch()
    from pyrite_b200.kernels import cuda as K
    host = np.zeros(len(payload) + offset, dtype=np.uint8)
    host[offset:] = np.frombuffer(payload, dtype=np.uint8)
    buf = torch.from_numpy(host).cuda()
    w = buf[offset:]
    xt = torch.as_tensor(np.asarray(x, dtype=np.float32)).cuda()
    y = K.matvec(ggml_type, w, xt, rows, cols)
    torch.cuda.synchronize()
    assert K.status() == 0
    return y.cpu().numpy()


@pytest.mark.parametrize("ggml_type", TYPES)
def test_device_dequantize_is_the_rounded_reference_value(cuda_device, golden_decoders, ggml_type):
    torch = _torch()
    from pyrite_b200.kernels import cuda as K
    rows, cols = 3, 1024
    key = f"{ggml_type}_{rows}x{cols}"
    payload = golden_decoders[f"payload_{key}"].tobytes()
    want = golden_decoders[f"decoded_{key}"].astype(np.float32)
    w = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    got = K.dequantize_rows(ggml_type, w, rows, cols).cpu().numpy().ravel()
    finite = ~np.isnan(want)
    assert np.array_equal(got[finite].view(np.uint32), want[finite].view(np.uint32))


@pytest.mark.parametrize("ggml_type", TYPES)
def test_device_matvec_golden_payloads(cuda_device, golden_decoders, ggml_type):
    for rows, cols in [(2, 512), (3, 1024)]:
        key = f"{ggml_type}_{rows}x{cols}"
        if f"matvec_{key}" not in golden_decoders.files:
            continue
        payload = golden_decoders[f"payload_{key}"].tobytes()
        x = golden_decoders[f"x_{cols}"].astype(np.float32)
        got = _device_matvec(ggml_type, payload, x, rows, cols)
        want = O.matvec(ggml_type, payload, x.astype(np.float64), rows, cols)
        assert rel_err(got, want, abs_dot(ggml_type, payload, x, rows, cols)) <= FP32_MATVEC_TOL


# rows x cols cases that walk every tail of the streamed kernel: partial row
# groups, partial chunks (cols not a multiple of the chunk), single rows,
# more groups than warps.
# includes rows of at most 16 units (16-lane slots: 256..1024 columns of the
# 64-value K-quant units, the 2048 x 768 MoE expert down shape)
RAGGED = [(1, 256), (3, 768), (5, 1280), (37, 2304), (130, 4096), (513, 1024), (2, 14336), (2048, 768), (700, 512)]


@pytest.mark.parametrize("rows,cols", RAGGED)
@pytest.mark.parametrize("ggml_type", TYPES)
def test_device_matvec_ragged_shapes(cuda_device, ggml_type, rows, cols):
    payload = random_payload(ggml_type, rows, cols, seed=rows * 7 + cols + ggml_type)
    x = np.random.default_rng(rows + cols).normal(0, 1, cols).astype(np.float32)
    got = _device_matvec(ggml_type, payload, x, rows, cols)
    want = O.matvec(ggml_type, payload, x.astype(np.float64), rows, cols)
    assert rel_err(got, want, abs_dot(ggml_type, payload, x, rows, cols)) <= FP32_MATVEC_TOL


@pytest.mark.parametrize("offset", [2, 4, 8, 6, 14])
@pytest.mark.parametrize("ggml_type", [8, 12, 13, 14, 23, 2, 10, 11, 3, 6, 7, 9, 20])
def test_device_matvec_unaligned_payloads(cuda_device, ggml_type, offset):
    rows, cols = 19, 2048
    payload = random_payload(ggml_type, rows, cols, seed=offset)
    x = np.random.default_rng(offset).normal(0, 1, cols).astype(np.float32)
    got = _device_matvec(ggml_type, payload, x, rows, cols, offset=offset)
    want = O.matvec(ggml_type, payload, x.astype(np.float64), rows, cols)
    assert rel_err(got, want, abs_dot(ggml_type, payload, x, rows, cols)) <= FP32_MATVEC_TOL


@pytest.mark.parametrize("ncols", [2, 3, 8, 11])
@pytest.mark.parametrize("ggml_type", [8, 12, 13, 14, 23, 0, 30])
def test_device_matvec_several_columns(cuda_device, ggml_type, ncols):
    torch = _torch()
    from pyrite_b200.kernels import cuda as K
    rows, cols = 67, 1536
    payload = random_payload(ggml_type, rows, cols, seed=ncols)
    x = np.random.default_rng(ncols).normal(0, 1, (ncols, cols)).astype(np.float32)
    w = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    got = K.matvec(ggml_type, w, torch.from_numpy(x).cuda(), rows, cols).cpu().numpy()
    assert got.shape == (ncols, rows)
    for c in range(ncols):
        want = O.matvec(ggml_type, payload, x[c].astype(np.float64), rows, cols)
        assert rel_err(got[c], want, abs_dot(ggml_type, payload, x[c], rows, cols)) <= FP32_MATVEC_TOL


def test_device_row_ranges_are_independent(cuda_device):
    """Any row partition gives bit-identical rows (the sharding property)."""
    torch = _torch()
    from pyrite_b200.kernels.cuda import QuantMatrix
    rows, cols = 1000, 4096
    for t in (8, 12, 14, 23):
        m = QuantMatrix.from_bytes(t, random_payload(t, rows, cols, seed=t), rows, cols)
        x = torch.randn(cols, device="cuda")
        full = m.matvec(x)
        parts = torch.cat([m.matvec(x, a, b - a) for a, b in [(0, 333), (333, 334), (334, 1000)]])
        assert torch.equal(full, parts)


@pytest.mark.parametrize("ggml_type", [8, 12, 13, 14, 23, 2, 30, 3, 6, 7, 9, 20])
def test_prepared_x_path_matches_one_shot_matvec(cuda_device, ggml_type):
    """One encoding of x shared by several matrices gives the one-shot results."""
    torch = _torch()
    from pyrite_b200.kernels import cuda as K
    cols = 4096
    x = torch.randn(cols, device="cuda")
    px = K.prepare_x(x)
    for rows, seed in [(300, 1), (4096, 2), (7, 3)]:
        payload = random_payload(ggml_type, rows, cols, seed=seed)
        w = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
        a = K.matvec(ggml_type, w, x, rows, cols)
        b = K.matvec_prepared(ggml_type, w, px, rows, cols)
        assert torch.equal(a, b)
        want = O.matvec(ggml_type, payload, x.double().cpu().numpy(), rows, cols)
        got = b.cpu().numpy()
        assert rel_err(got, want, abs_dot(ggml_type, payload, x.cpu().numpy(), rows, cols)) <= FP32_MATVEC_TOL
