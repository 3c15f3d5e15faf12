"""The matrices and kernel launches the benchmark times, checked against the oracle (B200).

bench.py times 15 batch-1 products: {Q8_0, Q4_K, Q5_K, Q6_K, IQ4_XS} x
{4096x4096, 14336x4096, 4096x14336}, built from its own seeds
(bench.build_payloads / bench.x_vectors) and launched as prepare_x +
matvec_prepared with static weights, which is what picks the kernel
instantiations (rows per stage, units per lane) the timing covers.  Here the
same payloads go through the same calls, and every row is compared with the
fp64 oracle (pyrite/kernels/native.c:518-555) within 1e-4 relative to
sum |w x|.  The same products at 8 and 64 columns (the tensor-core leg) are
covered by tests/test_gpu_tc.py.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-4


@pytest.fixture(scope="module")
def bench_inputs():
    import bench
    return bench.build_payloads(), bench.x_vectors(), bench.workload()


def test_every_bench_matrix_matches_the_oracle(cuda_device, bench_inputs):
    import torch

    from pyrite_b200.kernels import cuda as K
    payloads, xs, wl = bench_inputs
    assert len(wl) == 15
    X = {c: torch.from_numpy(v).cuda() for c, v in xs.items()}
    px = {c: K.prepare_x(X[c]) for c in X}
    worst = {}
    for name, t, r, c in wl:
        w = torch.frombuffer(bytearray(payloads[(t, r, c)]), dtype=torch.uint8).cuda()
        y = K.matvec_prepared(t, w, px[c], r, c, static_weights=True)
        torch.cuda.synchronize()
        assert K.status() == 0
        want = O.matvec_threaded(t, payloads[(t, r, c)], xs[c].astype(np.float64), r, c)
        dense = K.dequantize_rows(t, w, r, c)  # each value the rounded reference fp64 value
        bound = (dense.abs().double() @ X[c].abs().double()).cpu().numpy()
        err = float(np.max(np.abs(y.cpu().numpy().astype(np.float64) - want) / np.maximum(bound, 1e-30)))
        worst[f"{name} {r}x{c}"] = err
        del w, dense
        torch.cuda.empty_cache()
    bad = {k: v for k, v in worst.items() if v > TOL}
    assert not bad, f"rows beyond {TOL}: {bad}"

