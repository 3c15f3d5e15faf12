"""Shard plan on the CPU: the tensor-parallel split of a decode step
(pyrite_b200.shard) reproduces the unsharded products -- column shards of the
output / down projections summed by an allreduce over world_size-2 gloo ranks,
row shards of Q/K/V, gate/up and the LM head concatenated -- with the oracle's
fp64 matvec standing in for the GPU kernel."""
from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import oracle as O
from pyrite_b200.shard import even_range, head_shard, owned_experts, slice_cols, slice_rows
from tests.payloads import random_payload


def test_head_shards_cover_every_head_once():
    for nq, nkv, world in [(32, 8, 8), (32, 4, 8), (16, 8, 2), (32, 4, 2), (64, 4, 8), (4, 2, 2)]:
        shards = [head_shard(nq, nkv, world, r) for r in range(world)]
        assert sorted(q for s in shards for q in range(s.q0, s.q0 + s.nq)) == list(range(nq))
        group = nq // nkv
        for s in shards:  # every q head's kv head is local
            assert all(s.kv0 <= q // group < s.kv0 + s.nkv for q in range(s.q0, s.q0 + s.nq))
    with pytest.raises(ValueError):
        head_shard(30, 5, 4, 0)


def test_slices_reassemble():
    t, rows, cols = 12, 6, 1024
    p = random_payload(t, rows, cols, seed=1)
    assert slice_rows(p, t, cols, 0, 3) + slice_rows(p, t, cols, 3, 6) == p
    left, right = slice_cols(p, t, rows, cols, 0, 512), slice_cols(p, t, rows, cols, 512, 1024)
    w = O.dequantize_rows(t, p, rows, cols)
    assert np.array_equal(O.dequantize_rows(t, left, rows, 512), w[:, :512])
    assert np.array_equal(O.dequantize_rows(t, right, rows, 512), w[:, 512:])
    with pytest.raises(ValueError):
        slice_cols(p, t, rows, cols, 0, 100)
    assert owned_experts(8, 3, 1) == [1, 4, 7]
    assert even_range(1792 * 8, 8, 3, 256) == (5376, 7168)


def _rank(rank: int, world: int, port: int, q: "object") -> None:
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    t, h, qd = 14, 512, 1024  # an output projection h x qd (Q6_K) by input columns
    payload = random_payload(t, h, qd, seed=3)
    x = np.random.default_rng(4).normal(0, 1, qd)
    c0, c1 = even_range(qd, world, rank, 256)
    part = O.matvec(t, slice_cols(payload, t, h, qd, c0, c1), x[c0:c1], h, c1 - c0)
    buf = torch.from_numpy(part.copy())
    dist.all_reduce(buf)
    full = O.matvec(t, payload, x, h, qd)
    # LM head by rows + allgather
    v, vrows = 12, 64
    lm = random_payload(v, vrows, h, seed=5)
    xh = np.random.default_rng(6).normal(0, 1, h)
    r0, r1 = even_range(vrows, world, rank)
    mine = torch.from_numpy(O.matvec(v, slice_rows(lm, v, h, r0, r1), xh, r1 - r0, h).copy())
    gathered = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(gathered, mine)
    lm_ok = np.allclose(torch.cat(gathered).numpy(), O.matvec(v, lm, xh, vrows, h), rtol=1e-12, atol=1e-12)
    q.put((rank, float(np.max(np.abs(buf.numpy() - full))), bool(lm_ok)))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gloo_column_shards_and_allreduce():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, err, lm_ok in results:
        assert err < 1e-9 and lm_ok


def test_chunked_expert_subset_equals_slices_of_full_stack():
    """A GPU drawing only its experts of a chunked-weight checkpoint gets the
    very bytes of those experts' slices of the full stacked tensors."""
    from dataclasses import replace

    from pyrite_b200.synthetic import MoESpec, moe_tensors
    spec = replace(MoESpec.c5(), num_hidden_layers=1, hidden_size=256, moe_intermediate_size=256, num_experts=8,
                   vocab_size=512, num_attention_heads=4, num_key_value_heads=2)
    full = {n: (d, p) for n, d, _, p in moe_tensors(spec)}
    mine = owned_experts(8, 4, 3)
    for n, d, _, p in moe_tensors(spec, experts=mine):
        fd, fp = full[n]
        assert d == fd
        if len(d) == 3:
            per = len(fp) // 8
            assert p == b"".join(fp[e * per:(e + 1) * per] for e in mine)
        else:
            assert p == fp


@pytest.mark.parametrize("which", ["c3", "c4", "c5"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_model_configs_shard_over_one_box(which, world):
    """configs[2]-[4] split over 2, 4 and 8 GPUs (bench.py's tensor-parallel
    legs): every rank gets whole heads, block-aligned column ranges, an even
    vocabulary range and E / world experts, and the ranks cover everything once."""
    from pyrite_b200.synthetic import DenseSpec, MoESpec
    spec = {"c3": DenseSpec.c3, "c4": MoESpec.c4, "c5": MoESpec.c5}[which]()
    q_seen, e_seen, v_seen = [], [], []
    for rank in range(world):
        hs = head_shard(spec.num_attention_heads, spec.num_key_value_heads, world, rank)
        q_seen += list(range(hs.q0, hs.q0 + hs.nq))
        group = spec.num_attention_heads // spec.num_key_value_heads
        assert all(hs.kv0 <= q // group < hs.kv0 + hs.nkv for q in range(hs.q0, hs.q0 + hs.nq))
        assert (hs.q0 * spec.head_dim) % 256 == 0  # output-projection columns stay super-block aligned
        v0, v1 = even_range(spec.vocab_size, world, rank)
        v_seen += [v0, v1]
        if isinstance(spec, MoESpec):
            e_seen += owned_experts(spec.num_experts, world, rank)
        else:
            f0, f1 = even_range(spec.intermediate_size, world, rank)
            assert f0 % 256 == 0 and f1 % 256 == 0
    assert sorted(q_seen) == list(range(spec.num_attention_heads))
    assert v_seen[0] == 0 and v_seen[-1] == spec.vocab_size
    if e_seen:
        assert sorted(e_seen) == list(range(spec.num_experts))
