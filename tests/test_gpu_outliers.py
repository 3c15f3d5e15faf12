"""Batch-1 matvec parity when the activation has outlier channels (B200).

LLM activations carry a few channels far larger than the rest.  The batch-1
kernels re-encode x per 32-value block as int8 digits scaled by the block's
largest magnitude; a block holding one outlier keeps its other values only to
a precision set by the outlier, so such "wide" blocks carry a third digit.
These tests put one 10^3 outlier (random sign) in every 32-value block, give
the weights zero fp32 values on those columns, and compare every batch-1 entry
point with the fp64 oracle (restating pyrite/kernels/native.c:518-555, exact
products over exact x).  The bound is 1e-4 relative to sum |w x| over the
columns WITHOUT outliers: the outlier columns then cannot inflate the
denominator, so the small values' precision is what is measured.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O


TOL = 1e-4
TYPES = [8, 12, 13, 14, 23]  # Q8_0, Q4_K, Q5_K, Q6_K, IQ4_XS
OUTLIER = 1000.0


def outlier_x(cols: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """N(0, 1) fp32 values with one +-1000 outlier per 32-value block; returns (x, outlier columns)."""
    rng = np.random.default_rng(seed)
    x = rng.normal(0.0, 1.0, cols).astype(np.float32)
    cols_o = np.arange(0, cols, 32) + rng.integers(0, 32, cols // 32)
    x[cols_o] = (OUTLIER * np.where(rng.random(cols_o.size) < 0.5, -1.0, 1.0)).astype(np.float32)
    return x, cols_o


def payload_zero_on(ggml_type: int, rows: int, cols: int, zero_cols: np.ndarray, seed: int) -> bytes:
    from pyrite_b200.quantize import gaussian_weights, quantize
    w = gaussian_weights(rows, cols, seed).reshape(rows, cols)
    w[:, zero_cols] = 0.0
    return quantize(ggml_type, w.ravel())


def check(ggml_type, payload, x_used, y_gpu, rows, cols, outlier_cols, what):
    """y_gpu within TOL of the oracle on x_used, relative to sum |w x| off the outlier columns."""
    x64 = np.asarray(x_used, dtype=np.float64)
    want = O.matvec(ggml_type, payload, x64, rows, cols)
    w = O.dequantize_rows(ggml_type, payload, rows, cols)
    keep = np.ones(cols, dtype=bool)
    keep[outlier_cols] = False
    bound = np.abs(w[:, keep]) @ np.abs(x64[keep])
    err = float(np.max(np.abs(np.asarray(y_gpu, dtype=np.float64) - want) / np.maximum(bound, 1e-30)))
    assert err <= TOL, f"{what}, type {ggml_type}, {rows}x{cols}: max relative error {err:.3e}"
    return err


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def _ws(cols: int):
    import torch

    from pyrite_b200.kernels import cuda as K
    buf = torch.empty(K.workspace_size(0, cols) + 256, dtype=torch.uint8, device="cuda")
    off = (-buf.data_ptr()) % 256
    return buf, buf.data_ptr() + off, buf.numel() - off


SHAPES = [(256, 4096), (128, 14336), (96, 768), (64, 1024)]


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("ggml_type", TYPES)
def test_matvec_and_prepared_with_outlier_channels(cuda_device, ggml_type, rows, cols):
    """pyrite_cuda_matvec and pyrite_cuda_prepare_x + pyrite_cuda_matvec_prepared."""
    import torch

    from pyrite_b200.kernels import cuda as K
    x, oc = outlier_x(cols, seed=cols + ggml_type)
    payload = payload_zero_on(ggml_type, rows, cols, oc, seed=rows * 7 + cols)
    w = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    xd = torch.from_numpy(x).cuda()
    y = K.matvec(ggml_type, w, xd, rows, cols)
    px = K.prepare_x(xd)
    y2 = K.matvec_prepared(ggml_type, w, px, rows, cols)
    torch.cuda.synchronize()
    assert K.status() == 0
    check(ggml_type, payload, x, y.cpu().numpy(), rows, cols, oc, "pyrite_cuda_matvec")
    check(ggml_type, payload, x, y2.cpu().numpy(), rows, cols, oc, "pyrite_cuda_matvec_prepared")


# the other formats of the batch-1 tile kernel: Q4_0, Q4_1, Q5_0, Q5_1, Q8_1,
# Q2_K, Q3_K, IQ4_NL
MORE_TILE_TYPES = [2, 3, 6, 7, 9, 10, 11, 20]


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(256, 4096), (128, 14336), (96, 768)])
@pytest.mark.parametrize("ggml_type", MORE_TILE_TYPES)
def test_more_tile_formats_with_outlier_channels(cuda_device, ggml_type, rows, cols):
    """The other formats of the batch-1 tile kernel, whose wide-block pass
    multiplies the third digits by the code part without the block's offset
    (-8, -16, -4, m or dmin*m, applied to the exact fp32 sums of x).  Q4_0,
    Q2_K, Q3_K and IQ4_NL weights come from the package's quantizers with the
    outlier columns zeroed; the formats without an encoder use seeded random
    blocks (non-zero weights on the outlier columns, whose digits the encoding
    carries exactly)."""
    import torch

    from pyrite_b200.kernels import cuda as K
    from pyrite_b200.quantize import quantize_types
    from tests.payloads import random_payload
    x, oc = outlier_x(cols, seed=5 * cols + ggml_type)
    if ggml_type in quantize_types():
        payload = payload_zero_on(ggml_type, rows, cols, oc, seed=rows * 3 + cols)
    else:
        payload = random_payload(ggml_type, rows, cols, seed=rows * 3 + cols)
    w = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    xd = torch.from_numpy(x).cuda()
    y = K.matvec(ggml_type, w, xd, rows, cols)
    y2 = K.matvec_prepared(ggml_type, w, K.prepare_x(xd), rows, cols)
    torch.cuda.synchronize()
    assert K.status() == 0
    check(ggml_type, payload, x, y.cpu().numpy(), rows, cols, oc, "pyrite_cuda_matvec")
    check(ggml_type, payload, x, y2.cpu().numpy(), rows, cols, oc, "pyrite_cuda_matvec_prepared")


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(256, 4096), (128, 14336), (64, 1024)])
@pytest.mark.parametrize("ggml_type", TYPES)
def test_noalloc_with_outlier_channels(cuda_device, ggml_type, rows, cols):
    """pyrite_cuda_matvec_noalloc (the encoding in the library's fixed array)."""
    import torch

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K
    lib = _lib.require()
    x, oc = outlier_x(cols, seed=3 * cols + ggml_type)
    payload = payload_zero_on(ggml_type, rows, cols, oc, seed=rows + cols)
    w = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    xd = torch.from_numpy(x).cuda()
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    assert lib.pyrite_cuda_matvec_noalloc(ggml_type, w.data_ptr(), w.numel(), xd.data_ptr(), y.data_ptr(), rows,
                                          cols, 0, _stream()) == 0
    torch.cuda.synchronize()
    assert K.status() == 0
    check(ggml_type, payload, x, y.cpu().numpy(), rows, cols, oc, "pyrite_cuda_matvec_noalloc")


def _transformed(lib, ggml_type, w, x, x_op, norm, x_out, ws_ptr, ws_len, y, rows, cols):
    import torch
    code = lib.pyrite_cuda_matvec_transformed(ggml_type, w.data_ptr(), w.numel(), x.data_ptr(), x_op,
                                              norm.data_ptr() if norm is not None else None, 1e-6,
                                              x_out.data_ptr(), ws_ptr, ws_len, y.data_ptr(), rows, cols, 0,
                                              _stream())
    assert code == 0, code
    torch.cuda.synchronize()


def _form(lib, ggml_type, w, x, x_op, norm, x_out, rows, cols):
    return lib.pyrite_cuda_matvec_transformed_form(ggml_type, w.data_ptr(), w.numel(), x.data_ptr(), x_op,
                                                   norm.data_ptr() if norm is not None else None,
                                                   x_out.data_ptr() if x_out is not None else None, rows, cols)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(256, 2048), (256, 4096), (128, 14336)])
@pytest.mark.parametrize("given_ws", [False, True])
@pytest.mark.parametrize("ggml_type", TYPES)
def test_transformed_rmsnorm_with_outlier_channels(cuda_device, ggml_type, rows, cols, given_ws):
    """pyrite_cuda_matvec_transformed with RMSNorm: the prologue form (no
    workspace) and, at 2048 values with a workspace, the form with the
    operation's own kernel.  The kernel's fp32 x' (x_out) is the oracle's input;
    x_out itself is checked against an fp64 RMSNorm."""
    import torch

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K
    lib = _lib.require()
    x, oc = outlier_x(cols, seed=5 * cols + ggml_type)
    payload = payload_zero_on(ggml_type, rows, cols, oc, seed=rows * 3 + cols)
    w = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    xd = torch.from_numpy(x).cuda()
    norm = torch.ones(cols, device="cuda")
    x_out = torch.empty(cols, device="cuda")
    y = torch.empty(rows, device="cuda")
    buf, ptr, ln = _ws(cols)
    if not given_ws:
        ptr, ln = None, 0
    form = _form(lib, ggml_type, w, xd, _lib.X_RMSNORM, norm, x_out if given_ws else None, rows, cols)
    assert form == (1 if (not given_ws or cols >= 4096) else 0)
    _transformed(lib, ggml_type, w, xd, _lib.X_RMSNORM, norm, x_out, ptr, ln, y, rows, cols)
    assert K.status() == 0
    xs = x_out.cpu().numpy()
    x64 = x.astype(np.float64)
    want_x = x64 / np.sqrt(np.mean(x64 * x64) + 1e-6)
    assert np.allclose(xs, want_x, rtol=1e-6, atol=0)
    check(ggml_type, payload, xs, y.cpu().numpy(), rows, cols, oc, f"transformed RMSNorm (form {form})")


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(256, 4096), (128, 14336)])
@pytest.mark.parametrize("given_ws", [False, True])
@pytest.mark.parametrize("ggml_type", TYPES)
def test_transformed_silu_with_outlier_channels(cuda_device, ggml_type, rows, cols, given_ws):
    """pyrite_cuda_matvec_transformed with SiLU(gate) * up, gate ~ 8 (silu close
    to the identity there) and up = x / 8, so x' carries the outliers: the
    prologue form (no workspace) and the form with the operation's own kernel."""
    import torch

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K
    lib = _lib.require()
    x, oc = outlier_x(cols, seed=7 * cols + ggml_type)
    payload = payload_zero_on(ggml_type, rows, cols, oc, seed=rows * 5 + cols)
    w = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    gate = np.full(cols, 8.0, dtype=np.float32) + np.random.default_rng(cols).uniform(-0.5, 0.5, cols).astype(np.float32)
    gu = torch.from_numpy(np.concatenate([gate, (x / 8.0).astype(np.float32)])).cuda()
    x_out = torch.empty(cols, device="cuda")
    y = torch.empty(rows, device="cuda")
    buf, ptr, ln = _ws(cols)
    if not given_ws:
        ptr, ln = None, 0
    form = _form(lib, ggml_type, w, gu, _lib.X_SILU_MUL, None, x_out if given_ws else None, rows, cols)
    assert form == (0 if given_ws else 1)
    _transformed(lib, ggml_type, w, gu, _lib.X_SILU_MUL, None, x_out, ptr, ln, y, rows, cols)
    assert K.status() == 0
    xs = x_out.cpu().numpy()
    g64, u64 = gate.astype(np.float64), (x / 8.0).astype(np.float32).astype(np.float64)
    assert np.allclose(xs, g64 / (1.0 + np.exp(-g64)) * u64, rtol=1e-5, atol=0)
    check(ggml_type, payload, xs, y.cpu().numpy(), rows, cols, oc, f"transformed SiLU*up (form {form})")


def test_two_digit_encoding_alone_would_miss_the_bar():
    """The reason for the third digit, on the CPU: a numpy model of the
    encoding shows that two digits alone exceed the bar on these inputs while
    the three-digit form used for wide blocks stays far inside it."""
    rng = np.random.default_rng(11)
    cols, rows = 4096, 64
    x, oc = outlier_x(cols, seed=1)
    w = rng.normal(0, 1, (rows, cols))
    w[:, oc] = 0.0
    xb = x.reshape(-1, 32).astype(np.float32)
    amax = np.abs(xb).max(1, keepdims=True)
    t = (xb * (np.float32(127) / amax)).astype(np.float32)
    d0 = np.rint(t)
    u = ((t - d0) * np.float32(254)).astype(np.float32)
    d1 = np.rint(u)
    d2 = np.rint(((u - d1) * np.float32(254)).astype(np.float32))
    s = amax.astype(np.float64) / 127
    two = (s * (d0 + d1 / 254)).ravel()
    three = (s * (d0 + d1 / 254 + d2 / 254**2)).ravel()
    keep = np.ones(cols, dtype=bool)
    keep[oc] = False
    bound = np.abs(w[:, keep]) @ np.abs(x[keep].astype(np.float64))
    exact = w @ x.astype(np.float64)
    e2 = np.max(np.abs(w @ two - exact) / bound)
    e3 = np.max(np.abs(w @ three - exact) / bound)
    assert e2 > TOL > 10 * e3
