"""bench.py's workload and byte accounting, on CPU.

The roofline figure of the JSON line divides algorithmic bytes by the measured
launch time, so the byte count per matrix is pinned here against the GGML
block geometry: rows x (cols / block) x bytes per block of weights, plus the
fp32 x and y once each.
"""
from __future__ import annotations

import pytest

import bench

# weight bytes of one matrix of the configs[1] microbench (GGML block geometry)
WEIGHT_BYTES = {
    (4096, 4096): {"Q8_0": 17_825_792, "Q4_K": 9_437_184, "Q5_K": 11_534_336, "Q6_K": 13_762_560,
                   "IQ4_XS": 8_912_896},
    (14336, 4096): {"Q8_0": 62_390_272, "Q4_K": 33_030_144, "Q5_K": 40_370_176, "Q6_K": 48_168_960,
                    "IQ4_XS": 31_195_136},
}


def test_workload_is_the_fifteen_matrices():
    wl = bench.workload()
    assert len(wl) == 15
    assert {(r, c) for _, _, r, c in wl} == set(bench.SHAPES)
    assert {n for n, _, _, _ in wl} == set(bench.TYPES)


@pytest.mark.parametrize("shape", list(WEIGHT_BYTES))
def test_algorithmic_bytes_follow_the_block_geometry(shape):
    rows, cols = shape
    for name, want in WEIGHT_BYTES[shape].items():
        t = bench.TYPES[name]
        assert rows * bench.row_bytes(t, cols) == want
        assert bench.algo_bytes(t, rows, cols) == want + (rows + cols) * 4
        # the transposed shape streams the same weight bytes
        assert cols * bench.row_bytes(t, rows) == want


def test_step_bytes():
    assert sum(bench.algo_bytes(t, r, c) for _, t, r, c in bench.workload()) == 492_683_264


def test_other_type_payloads_have_the_row_geometry():
    for name, t in bench.OTHER_TYPES.items():
        p = bench.other_payload(t, 8, 512, seed=1)
        assert len(p) == 8 * bench.row_bytes(t, 512), name
