"""Routed experts (Qwen3-MoE feed-forward) on the B200, through the C ABI.

* routing: softmax top-k with the reference's (-p, e) order and weight
  renormalisation (oracle.moe_route, executor.py:757-772);
* the expert matvec over a stacked tensor with device-side ids (batch-1
  kernel and the generic kernel) against the oracle's fp64 product of each
  selected slice (qwen3_moe.py:364-398);
* a whole synthetic Qwen3-MoE model (Q4_K_M mix) decoding greedily with the
  reference executor's token ids and routed experts
  (tests/golden/moe_tiny.json, made by tests/golden/make_moe_golden.py).
"""
from __future__ import annotations

import json
from dataclasses import fields
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests.payloads import random_payload

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("n,k,norm", [(128, 8, True), (16, 4, True), (64, 6, False), (5, 5, True)])
def test_route_matches_reference_order_and_weights(cuda_device, n, k, norm):
    import torch

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K
    lib = _lib.require()
    rng = np.random.default_rng(n + k)
    for trial in range(5):
        logits = rng.normal(0, 1.5, n).astype(np.float32)
        if trial == 1:
            logits[1] = logits[n - 1] = logits.max() + 1.0  # a tie: the lower id ranks first
        x = torch.from_numpy(logits).cuda()
        ids = torch.zeros(k, dtype=torch.int32, device="cuda")
        w = torch.zeros(k, device="cuda")
        want_ids, want_w = O.moe_route(logits.astype(np.float64), k, norm)
        for shards in (1, 3):
            for index in range(shards):
                gids = torch.zeros(k, dtype=torch.int32, device="cuda")
                assert lib.pyrite_cuda_moe_route(x.data_ptr(), n, k, 1 if norm else 0, 1.0, shards, index,
                                                 ids.data_ptr(), w.data_ptr(), gids.data_ptr(),
                                                 torch.cuda.current_stream().cuda_stream) == 0
                torch.cuda.synchronize()
                assert K.status() == 0
                assert gids.cpu().tolist() == want_ids
                assert ids.cpu().tolist() == [e // shards if e % shards == index else -1 for e in want_ids]
                wl = np.asarray([v if e % shards == index else 0.0 for e, v in zip(want_ids, want_w)],
                                dtype=np.float32)
                assert np.allclose(w.cpu().numpy(), wl, rtol=1e-6, atol=0)


@pytest.mark.parametrize("ggml_type,cols", [(12, 2048), (14, 768), (14, 2048), (8, 1024), (23, 512), (2, 512)])
def test_expert_matvec_matches_each_slice(cuda_device, ggml_type, cols):
    import torch

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K
    lib = _lib.require()
    rows, n_experts, sel = 96, 12, [7, 0, 11, 3, 3]
    payload = random_payload(ggml_type, rows * n_experts, cols, seed=cols + ggml_type)
    w = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    k = len(sel)
    ids = torch.tensor(sel, dtype=torch.int32, device="cuda")
    rng = np.random.default_rng(1)
    for shared_x in (True, False):
        xs = rng.normal(0, 1, (1 if shared_x else k, cols)).astype(np.float32)
        x = torch.from_numpy(xs).cuda()
        per = int(lib.pyrite_cuda_workspace_size(0, cols, 1))
        ws = torch.empty(per * xs.shape[0] + 256, dtype=torch.uint8, device="cuda")
        off = (-ws.data_ptr()) % 256
        assert lib.pyrite_cuda_prepare_x(x.data_ptr(), cols, cols, xs.shape[0], ws.data_ptr() + off, ws.numel() - off,
                                         torch.cuda.current_stream().cuda_stream) == 0
        y = torch.full((k, rows + 5), -7.0, device="cuda")
        code = lib.pyrite_cuda_matvec_experts(ggml_type, w.data_ptr(), w.numel(), n_experts, ids.data_ptr(), k,
                                              x.data_ptr(), 0 if shared_x else cols, ws.data_ptr() + off,
                                              ws.numel() - off, 0 if shared_x else per, y.data_ptr(), rows + 5,
                                              rows, cols, 0, torch.cuda.current_stream().cuda_stream)
        assert code == 0
        torch.cuda.synchronize()
        assert K.status() == 0
        got = y.cpu().numpy()
        rb = O.row_bytes(ggml_type, cols)
        for j, e in enumerate(sel):
            sl = payload[e * rows * rb:(e + 1) * rows * rb]
            xj = xs[0 if shared_x else j].astype(np.float64)
            want = O.matvec(ggml_type, sl, xj, rows, cols)
            absdot = np.abs(O.dequantize_rows(ggml_type, sl, rows, cols)) @ np.abs(xj)
            assert np.max(np.abs(got[j, :rows] - want) / np.maximum(absdot, 1e-30)) <= 1e-4
            assert np.all(got[j, rows:] == -7.0)  # nothing written past the slice's rows



@pytest.mark.parametrize("ggml_type,cols", [(12, 2048), (14, 768), (8, 1024), (2, 512)])
@pytest.mark.parametrize("groups", [2, 3])
def test_expert_groups_equal_one_call_per_stack(cuda_device, ggml_type, cols, groups):
    """pyrite_cuda_matvec_expert_groups over `groups` stacks stored back to back
    (gate | up) gives, bit for bit, what one pyrite_cuda_matvec_experts call
    per stack gives; ids of -1 (experts held elsewhere) leave their rows of
    every group untouched."""
    import torch

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K
    lib = _lib.require()
    rows, n_experts, sel = 64, 6, [5, -1, 0, 5]
    k = len(sel)
    payload = random_payload(ggml_type, rows * n_experts * groups, cols, seed=7 * cols + groups)
    w = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    ids = torch.tensor(sel, dtype=torch.int32, device="cuda")
    x = torch.from_numpy(np.random.default_rng(groups).normal(0, 1, cols).astype(np.float32)).cuda()
    per = int(lib.pyrite_cuda_workspace_size(0, cols, 1))
    ws = torch.empty(per + 256, dtype=torch.uint8, device="cuda")
    off = (-ws.data_ptr()) % 256
    s = torch.cuda.current_stream().cuda_stream
    assert lib.pyrite_cuda_prepare_x(x.data_ptr(), cols, cols, 1, ws.data_ptr() + off, ws.numel() - off, s) == 0
    y = torch.full((groups * k, rows), -3.0, device="cuda")
    assert lib.pyrite_cuda_matvec_expert_groups(ggml_type, w.data_ptr(), w.numel(), n_experts, groups,
                                                ids.data_ptr(), k, x.data_ptr(), 0, ws.data_ptr() + off,
                                                ws.numel() - off, 0, y.data_ptr(), rows, rows, cols, 0, s) == 0
    one = w.numel() // groups
    for g in range(groups):
        yg = torch.full((k, rows), -3.0, device="cuda")
        assert lib.pyrite_cuda_matvec_experts(ggml_type, w.data_ptr() + g * one, one, n_experts, ids.data_ptr(), k,
                                              x.data_ptr(), 0, ws.data_ptr() + off, ws.numel() - off, 0,
                                              yg.data_ptr(), rows, rows, cols, 0, s) == 0
        torch.cuda.synchronize()
        assert torch.equal(y[g * k:(g + 1) * k], yg)
        assert bool((yg[1] == -3.0).all())
    assert K.status() == 0
    # a stack length that is not groups * n_experts matrices is refused
    assert lib.pyrite_cuda_matvec_expert_groups(ggml_type, w.data_ptr(), w.numel() - one, n_experts, groups,
                                                ids.data_ptr(), k, x.data_ptr(), 0, ws.data_ptr() + off,
                                                ws.numel() - off, 0, y.data_ptr(), rows, rows, cols, 0, s) == -3


@pytest.mark.parametrize("E,h,k,shards,index", [(128, 2048, 8, 1, 0), (16, 256, 4, 2, 1), (60, 1024, 6, 4, 3)])
def test_router_route_equals_matvec_then_route(cuda_device, E, h, k, shards, index):
    """pyrite_cuda_moe_router_route (one launch): logits within fp32 rounding
    of the fp64 product, and the ids, weights and global ids that
    pyrite_cuda_moe_route gives for those logits; the ticket is left at zero."""
    import torch

    from pyrite_b200 import _lib
    lib = _lib.require()
    g = torch.Generator("cuda").manual_seed(E * h + k)
    router = torch.randn(E, h, device="cuda", generator=g) * 0.02
    s = torch.cuda.current_stream().cuda_stream
    ticket = torch.zeros(1, dtype=torch.int32, device="cuda")
    for rep in range(3):
        x = torch.randn(h, device="cuda", generator=g)
        got_l = torch.empty(E, device="cuda")
        got = [torch.full((k,), -5, dtype=torch.int32, device="cuda"), torch.zeros(k, device="cuda"),
               torch.zeros(k, dtype=torch.int32, device="cuda")]
        assert lib.pyrite_cuda_moe_router_route(0, router.data_ptr(), router.numel() * 4, h, x.data_ptr(),
                                                got_l.data_ptr(), E, k, 1, 1.0, shards, index, got[0].data_ptr(),
                                                got[1].data_ptr(), got[2].data_ptr(), ticket.data_ptr(), s) == 0
        exact = (router.double() @ x.double()).float()
        assert torch.allclose(got_l, exact, rtol=2e-7, atol=1e-9)
        want_l = got_l.clone()
        want = [torch.full((k,), -5, dtype=torch.int32, device="cuda"), torch.zeros(k, device="cuda"),
                torch.zeros(k, dtype=torch.int32, device="cuda")]
        assert lib.pyrite_cuda_moe_route(want_l.data_ptr(), E, k, 1, 1.0, shards, index, want[0].data_ptr(),
                                         want[1].data_ptr(), want[2].data_ptr(), s) == 0
        torch.cuda.synchronize()
        for a, b in zip(got, want):
            assert torch.equal(a, b)
        assert int(ticket.item()) == 0
    # quantized routers are not taken
    assert lib.pyrite_cuda_moe_router_route(8, router.data_ptr(), router.numel(), h, x.data_ptr(), got_l.data_ptr(),
                                            E, k, 1, 1.0, 1, 0, got[0].data_ptr(), got[1].data_ptr(), None,
                                            ticket.data_ptr(), s) == -1


@pytest.mark.parametrize("E,h,k", [(128, 2048, 8), (16, 256, 4)])
def test_norm_router_route_equals_norm_then_router_route(cuda_device, E, h, k):
    """pyrite_cuda_moe_norm_router_route (RMSNorm in the routing launch) writes
    the same normed vector, encoding, logits and routing as
    pyrite_cuda_rmsnorm_encode followed by pyrite_cuda_moe_router_route."""
    import torch

    from pyrite_b200 import _lib
    lib = _lib.require()
    g = torch.Generator("cuda").manual_seed(h + k)
    router = torch.randn(E, h, device="cuda", generator=g) * 0.02
    nw = torch.rand(h, device="cuda", generator=g) + 0.5
    x = torch.randn(h, device="cuda", generator=g) * 3
    s = torch.cuda.current_stream().cuda_stream
    per = int(lib.pyrite_cuda_workspace_size(0, h, 1))

    def ws():
        b = torch.zeros(per + 256, dtype=torch.uint8, device="cuda")
        off = (-b.data_ptr()) % 256
        return b, b.data_ptr() + off, b.numel() - off, off

    def outs():
        return (torch.empty(E, device="cuda"), torch.full((k,), -5, dtype=torch.int32, device="cuda"),
                torch.zeros(k, device="cuda"), torch.zeros(k, dtype=torch.int32, device="cuda"))

    ticket = torch.zeros(1, dtype=torch.int32, device="cuda")
    nb, nptr, nlen, noff = ws()
    normed = torch.empty(h, device="cuda")
    got = outs()
    assert lib.pyrite_cuda_moe_norm_router_route(0, router.data_ptr(), router.numel() * 4, h, x.data_ptr(),
                                                 nw.data_ptr(), 1e-6, normed.data_ptr(), nptr, nlen,
                                                 got[0].data_ptr(), E, k, 1, 1.0, 1, 0, got[1].data_ptr(),
                                                 got[2].data_ptr(), got[3].data_ptr(), ticket.data_ptr(), s) == 0
    rb, rptr, rlen, roff = ws()
    ref_n = torch.empty(h, device="cuda")
    assert lib.pyrite_cuda_rmsnorm_encode(x.data_ptr(), nw.data_ptr(), h, 1e-6, ref_n.data_ptr(), rptr, rlen, s) == 0
    want = outs()
    assert lib.pyrite_cuda_moe_router_route(0, router.data_ptr(), router.numel() * 4, h, ref_n.data_ptr(),
                                            want[0].data_ptr(), E, k, 1, 1.0, 1, 0, want[1].data_ptr(),
                                            want[2].data_ptr(), want[3].data_ptr(), ticket.data_ptr(), s) == 0
    torch.cuda.synchronize()
    # the same fp64 statistics up to summation order: equal to within an ulp
    assert torch.allclose(normed, ref_n, rtol=2e-7, atol=0)
    assert np.mean((nb[noff:noff + per] == rb[roff:roff + per]).cpu().numpy()) > 0.999
    assert torch.allclose(got[0], want[0], rtol=1e-6, atol=1e-7)
    for a, b in zip(got[1:], want[1:]):
        assert torch.equal(a, b)
    assert int(ticket.item()) == 0

def _moe_spec(d):
    from pyrite_b200.synthetic import MoESpec
    names = {f.name for f in fields(MoESpec)}
    return MoESpec(**{k: v for k, v in d["spec"].items() if k in names})


# Router-logit gap under which the reference's last chosen expert and its
# runner-up are a tie at fp32 precision: the decode's hidden states differ from
# the reference's fp64 ones by ~1e-5 relative, router logits are O(1).
ROUTER_TIE = 1e-3


def _tie_flip(route, g, step) -> bool:
    """Compare one pass's routed experts with the reference's.  Equal lists
    pass.  The same experts in another order must be a tie inside the top k
    (the reference's smallest gap between consecutive chosen experts at most
    ROUTER_TIE; the weighted sum is the same) and pass.  Any other difference
    must be a tie at the top-k boundary -- the reference's margin between its
    last chosen expert and the runner-up at most ROUTER_TIE, and the two
    swapped -- and returns True: from there on (the later layers of the same
    pass included, whose input the other experts changed) the two decodes
    legitimately follow different branches, so the comparison stops (the
    greedy ids of the whole window were compared already).  The margins come
    from golden files that record them (``router_margin``,
    ``router_order_margin``); without them any difference fails."""
    want = g["experts"][step]
    for layer, (a, b) in enumerate(zip(route, want)):
        if a == b:
            continue
        assert "router_margin" in g, f"routing differs at pass {step}, layer {layer}: {a} vs {b}"
        if sorted(a) == sorted(b):
            gap = g["router_order_margin"][step][layer]
            assert gap <= ROUTER_TIE, f"pass {step}, layer {layer}: order {a} vs {b} with a reference gap of {gap}"
            continue
        gap = g["router_margin"][step][layer]
        assert gap <= ROUTER_TIE, f"routing differs at pass {step}, layer {layer} with a reference margin of {gap}"
        assert sorted(a) == sorted(b[:-1] + [g["runner_up"][step][layer]]), \
            f"pass {step}, layer {layer}: {a} is not the reference's choice {b} with its tie swapped"
        return True
    return False


@pytest.mark.parametrize("golden", ["moe_tiny.json", "moe_c4_2l.json", "moe_c5_2l.json", "moe_c4_2l_w128.json",
                                    "moe_c5_2l_w128.json"])
def test_moe_decode_matches_reference(cuda_device, golden):
    """Greedy ids, routed experts of every layer of every pass and top logits;
    moe_c4_2l is configs[3] at full width (hidden 2048, 128 experts top-8,
    expert ffn 768, vocab 151936) with 2 layers, moe_c5_2l configs[4] at full
    width (hidden 4096, 64 q / 4 kv heads, 128 experts top-8, expert ffn 1536)
    with 2 layers; the _w128 files decode the same checkpoints over a
    128-position window (120-token prompt, 8 greedy tokens)."""
    import torch

    from pyrite_b200.kernels import cuda as K
    from pyrite_b200.model import MixedDecoder
    g = json.loads((GOLDEN / golden).read_text())
    dec = MixedDecoder.synthetic(_moe_spec(g), device=cuda_device, max_ctx=128)
    prompt, want = g["prompt"], g["generated"]
    got = dec.generate(prompt, len(want))
    assert K.status() == 0
    assert got[len(prompt):] == want
    # pass by pass: routed experts of every layer and the top logits
    dec.reset(prompt)
    worst = 0.0
    for step, top in enumerate(g["top_logits"][: len(prompt) + len(want) - 1]):
        dec.run_steps(1)
        torch.cuda.synchronize()
        if _tie_flip(dec.route_log.cpu().tolist(), g, step):
            break  # the state follows the other branch of a tie from here on
        logits = dec.logits.double().cpu()
        ids = [i for i, _ in top]
        vals = torch.tensor([v for _, v in top], dtype=torch.float64)
        assert int(torch.argmax(logits)) == ids[0]
        worst = max(worst, float((logits[ids] - vals).abs().max()))
    # the dense decoders' bound (tests/test_gpu_decode.py: the two-digit
    # activation encoding carried through two layers of a 4096-wide model)
    from tests.test_gpu_decode import LOGIT_TOL
    assert worst <= LOGIT_TOL, f"max |logit - reference| = {worst}"
