"""Tensor-parallel shard plan: which bytes of which tensor each GPU holds.

The path shards by independent rows (``pyrite/executor.py:481-509``: any row
range of a GGML matrix is one contiguous byte span).  For a decode step across
``world`` GPUs of one box the layout follows the two-collective scheme:

* attention by heads: rank g computes q heads ``[g nq/W, (g+1) nq/W)`` and the
  kv heads they read (its own kv heads when ``nkv % W == 0``, else the one kv
  head its q heads share, replicated); Q/K/V are row ranges of their matrices;
* the output projection by input columns: rank g multiplies its heads' slice
  of every row of ``attn_output`` (block-aligned), giving a partial residual
  update that one allreduce sums;
* the SwiGLU feed-forward: gate/up by rows, down by input columns, one
  allreduce;
* routed experts by id: rank g owns experts ``{e : e % W == g}``; the router is
  replicated, every rank combines the selected experts it owns and the same
  allreduce sums the partial updates;
* the LM head by rows, then an allgather of the logits.

Norm weights, the embedding and the router are replicated.  Everything here is
host-side slicing of GGML payload bytes (numpy), testable without a GPU.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .ggml_types import spec as ggml_spec


def row_bytes(ggml_type: int, cols: int) -> int:
    s = ggml_spec(ggml_type)
    if cols % s.block_size:
        raise ValueError(f"{cols} columns is not a whole number of {s.block_size}-value blocks")
    return cols // s.block_size * s.bytes_per_block


def slice_rows(payload: bytes, ggml_type: int, cols: int, r0: int, r1: int) -> bytes:
    """Rows [r0, r1) of a GGML matrix: one contiguous byte span."""
    rb = row_bytes(ggml_type, cols)
    return payload[r0 * rb:r1 * rb]


def slice_cols(payload: bytes, ggml_type: int, rows: int, cols: int, c0: int, c1: int) -> bytes:
    """Columns [c0, c1) of every row (block-aligned): the rows of a rows x (c1-c0) matrix."""
    s = ggml_spec(ggml_type)
    if c0 % s.block_size or c1 % s.block_size:
        raise ValueError(f"column range [{c0}, {c1}) is not aligned to {s.block_size}-value blocks")
    rb = row_bytes(ggml_type, cols)
    a = np.frombuffer(payload, dtype=np.uint8).reshape(rows, rb)
    b0, b1 = c0 // s.block_size * s.bytes_per_block, c1 // s.block_size * s.bytes_per_block
    return np.ascontiguousarray(a[:, b0:b1]).tobytes()


@dataclass(frozen=True)
class HeadShard:
    """Attention heads of one rank."""

    q0: int      # first q head
    nq: int      # q heads
    kv0: int     # first kv head
    nkv: int     # kv heads


def head_shard(nq: int, nkv: int, world: int, rank: int) -> HeadShard:
    if nq % world:
        raise ValueError(f"{nq} q heads do not split over {world} GPUs")
    group = nq // nkv
    per = nq // world
    q0 = rank * per
    if nkv % world == 0:
        kper = nkv // world
        return HeadShard(q0, per, rank * kper, kper)
    if group % per:
        raise ValueError(f"{per} q heads per GPU do not tile GQA groups of {group}")
    return HeadShard(q0, per, q0 // group, 1)


def even_range(n: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """[a, b) of an even split of n items, boundaries multiples of `align`."""
    if n % (world * align):
        raise ValueError(f"{n} does not split into {world} ranges aligned to {align}")
    per = n // world
    return rank * per, (rank + 1) * per


def owned_experts(n_experts: int, world: int, rank: int) -> list[int]:
    """Global ids of the experts rank `rank` holds, in local order (local i = global e // world)."""
    return [e for e in range(n_experts) if e % world == rank]
