"""pyrite_cuda_matvec_noalloc: the matvec for callers that cannot allocate.

Some hosts own all device memory themselves (their pool, their budget) or call
through an FFI with no device allocator, so they cannot hand the library a
workspace.  The no-allocation entry point keeps the activation's encoding in a
fixed array inside the library.  These checks call it through the C ABI,
several times in a row on different shapes (so each call runs over what the
previous one left in the shared array), and compare each result with the fp64
oracle (pyrite/kernels/native.c:518-555) and with the regular
pyrite_cuda_matvec entry point's, within the suite's matvec tolerance.  The
shapes include the widest activation the batch-1 kernel takes (32768 values,
the array's size) and one past it (65536 values, the generic kernel, which
reads x directly).  The file sorts last so that a failing run here has
already run every other test; it also passes on its own in a fresh process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests.payloads import random_payload

pytestmark = pytest.mark.gpu

TOL = 1e-4  # relative to sum_k |W[r,k] x[k]|, as in test_gpu_matvec.py


def _abs_dot(torch, K, t, w, x, rows, cols):
    full = K.dequantize_rows(t, w, rows, cols)
    return full.abs().double() @ x.abs().double()


def _noalloc(lib, t, w, x, y, rows, cols, stream):
    return lib.pyrite_cuda_matvec_noalloc(t, w.data_ptr(), w.numel(), x.data_ptr(), y.data_ptr(), rows, cols, 0,
                                          stream)


def test_noalloc_matches_the_workspace_entry_point_twice_in_a_row(cuda_device):
    import torch

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K

    lib = _lib.require()
    stream = torch.cuda.current_stream().cuda_stream
    cases = [(12, 777, 4096, 1), (8, 1000, 14336, 2), (14, 64, 2048, 3), (23, 300, 1024, 4), (13, 48, 32768, 5),
             (8, 32, 65536, 6)]
    outs = []
    for t, rows, cols, seed in cases:  # consecutive calls share the fixed array
        w = torch.frombuffer(bytearray(random_payload(t, rows, cols, seed=seed)), dtype=torch.uint8).cuda()
        x = torch.from_numpy(np.random.default_rng(seed).normal(0, 1, cols).astype(np.float32)).cuda()
        y = torch.empty(rows, dtype=torch.float32, device="cuda")
        assert _noalloc(lib, t, w, x, y, rows, cols, stream) == 0
        outs.append((t, w, x, y, rows, cols))
    torch.cuda.synchronize()
    assert K.status() == 0
    for t, w, x, y, rows, cols in outs:
        ref = K.matvec(t, w, x, rows, cols)
        bound = _abs_dot(torch, K, t, w, x, rows, cols)
        err = ((y.double() - ref.double()).abs() / bound.clamp_min(1e-30)).max().item()
        assert err <= TOL, f"type {t}: {err} against pyrite_cuda_matvec"
        want = O.matvec(t, w.cpu().numpy().tobytes(), x.cpu().double().numpy(), rows, cols)
        err = float(np.max(np.abs(y.cpu().double().numpy() - want) / np.maximum(bound.cpu().numpy(), 1e-30)))
        assert err <= TOL, f"type {t}, {rows}x{cols}: {err} against the oracle"


def test_noalloc_rejects_activations_beyond_its_fixed_scratch(cuda_device):
    from pyrite_b200 import _lib

    lib = _lib.require()
    cols = 65536 + 256
    dev = ctypes.c_void_p(1 << 20)  # never dereferenced: the size check comes first
    assert lib.pyrite_cuda_matvec_noalloc(12, dev, 144 * (cols // 256), dev, dev, 1, cols, 0, None) == -2
