"""The routing comparison of the MoE decode tests, on CPU.

Over long windows the decode's fp32 hidden states and the reference's fp64
ones may order two experts whose router logits nearly tie differently.  The
GPU test accepts such a difference only where the reference's own golden file
shows the tie (tests/test_gpu_moe.py::_tie_flip); these cases pin that rule
with hand-made golden records.
"""
from __future__ import annotations

import pytest

from tests.test_gpu_moe import ROUTER_TIE, _tie_flip

WANT = [[5, 3, 9, 1], [7, 2, 4, 8]]


def golden(boundary=(0.5, 0.5), order=(0.5, 0.5), runner_up=(6, 0)):
    return {"experts": [WANT], "router_margin": [list(boundary)], "router_order_margin": [list(order)],
            "runner_up": [list(runner_up)]}


def test_equal_routing_passes():
    assert _tie_flip([list(r) for r in WANT], golden(), 0) is False


def test_order_only_difference_needs_a_tie_inside_the_top_k():
    swapped = [[3, 5, 9, 1], WANT[1]]
    assert _tie_flip(swapped, golden(order=(ROUTER_TIE / 2, 0.5)), 0) is False
    with pytest.raises(AssertionError):
        _tie_flip(swapped, golden(order=(10 * ROUTER_TIE, 0.5)), 0)


def test_boundary_swap_needs_a_tie_with_the_runner_up():
    flipped = [[5, 3, 9, 6], WANT[1]]  # last chosen expert 1 replaced by runner-up 6
    assert _tie_flip(flipped, golden(boundary=(ROUTER_TIE / 2, 0.5)), 0) is True
    with pytest.raises(AssertionError):  # no tie there in the reference
        _tie_flip(flipped, golden(boundary=(10 * ROUTER_TIE, 0.5)), 0)
    with pytest.raises(AssertionError):  # a tie, but another expert came in
        _tie_flip([[5, 3, 9, 11], WANT[1]], golden(boundary=(ROUTER_TIE / 2, 0.5)), 0)


def test_a_tie_flip_ends_the_comparison_of_the_later_layers():
    # layer 0 took the runner-up; layer 1 then saw another input and ordered
    # (or chose) its experts differently, which is no longer compared
    later = [[5, 3, 9, 6], [8, 4, 2, 7]]
    assert _tie_flip(later, golden(boundary=(ROUTER_TIE / 2, 0.5)), 0) is True
    # an order-only tie in layer 0 keeps the state: layer 1 is still compared
    with pytest.raises(AssertionError):
        _tie_flip([[3, 5, 9, 1], [8, 4, 2, 7]], golden(order=(ROUTER_TIE / 2, 0.5)), 0)


def test_golden_files_without_margins_accept_no_difference():
    with pytest.raises(AssertionError):
        _tie_flip([[3, 5, 9, 1], WANT[1]], {"experts": [WANT]}, 0)
