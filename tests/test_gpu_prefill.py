"""Batched prefill (MixedDecoder.prefill) against the reference and the one-position path (B200).

The reference runs a prompt one position per forward pass
(pyrite/executor.py:920-923).  The batched prefill runs blocks of positions:
every projection as one multi-column product on the tensor cores, the glue
per row (pyrite_cuda_embed_rows / rmsnorm_rows / qk_rope_kv_rows /
attention_rows / silu_mul_rows).  Checked here: each row kernel against its
one-position kernel (bit-exact where the arithmetic is the same), the causal
block attention against an fp64 restatement of executor.py:733-755, and the
greedy ids of the goldens (made by the reference executor) after a block
prefill, with block sizes that put block edges inside the prompt.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def _dense_spec(g):
    from dataclasses import fields

    from pyrite_b200.synthetic import DenseSpec
    return DenseSpec(**{k: v for k, v in g["spec"].items() if k in {f.name for f in fields(DenseSpec)}})


@pytest.mark.parametrize("golden", ["c1_small.json", "llama_tiny.json", "c3_2l.json", "c3_2l_w128.json"])
@pytest.mark.parametrize("block", [64, 5, 1])
def test_prefilled_decode_matches_reference_greedy_ids(cuda_device, golden, block):
    import torch

    from pyrite_b200.kernels import cuda as K
    from pyrite_b200.model import MixedDecoder
    from tests.test_gpu_decode import LOGIT_TOL
    g = json.loads((GOLDEN / golden).read_text())
    dec = MixedDecoder.synthetic(_dense_spec(g), device=cuda_device, max_ctx=512)
    prompt, want = g["prompt"], g["generated"]
    got = dec.generate(prompt, len(want), prefill_block=block)
    assert K.status() == 0
    assert got[len(prompt):] == want, f"greedy ids differ after a {block}-position prefill"
    # the first generated token's logits (position len(prompt) - 1)
    dec.prefill(prompt, block)
    dec.run_steps(1)
    top = g["top_logits"][len(prompt) - 1]
    logits = dec.logits.double().cpu()
    ids = [i for i, _ in top]
    err = float((logits[ids] - torch.tensor([v for _, v in top], dtype=torch.float64)).abs().max())
    assert err <= LOGIT_TOL


def test_prefill_fills_the_cache_like_one_position_steps(cuda_device):
    """KV cache rows after a block prefill against the rows the one-position
    step writes: the same values up to the products' rounding (tensor-core
    product of split bf16 planes vs the batch-1 kernel's digit encoding)."""
    import torch

    from pyrite_b200.model import MixedDecoder
    g = json.loads((GOLDEN / "llama_tiny.json").read_text())
    dec = MixedDecoder.synthetic(_dense_spec(g), device=cuda_device, max_ctx=128)
    prompt = g["prompt"] + g["generated"][:5]
    dec.reset(prompt)
    dec.capture()
    dec.reset(prompt)
    dec.run_steps(len(prompt) - 1)
    torch.cuda.synchronize()
    n = len(prompt) - 1
    k_seq, v_seq = dec.kcache[:, :n].clone(), dec.vcache[:, :n].clone()
    dec.prefill(prompt, 4)
    assert int(dec.pos) == n
    k_pre, v_pre = dec.kcache[:, :n], dec.vcache[:, :n]
    for a, b in ((k_pre, k_seq), (v_pre, v_seq)):
        scale = b.abs().amax(dim=-1, keepdim=True).clamp_min(1e-6)
        assert float(((a - b).abs() / scale).max()) < 2e-3


def test_row_kernels_equal_the_one_position_kernels(cuda_device):
    import torch

    from pyrite_b200 import _lib
    lib = _lib.require()
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator("cuda").manual_seed(5)
    n, c = 2048, 7
    x = torch.randn(c, n, device="cuda", generator=g) * 3
    w = torch.rand(n, device="cuda", generator=g) + 0.5
    out = torch.empty(c, n, device="cuda")
    assert lib.pyrite_cuda_rmsnorm_rows(x.data_ptr(), n, w.data_ptr(), n, c, 1e-6, out.data_ptr(), n, st) == 0
    ws = torch.zeros(int(lib.pyrite_cuda_workspace_size(0, n, 1)) + 256, dtype=torch.uint8, device="cuda")
    off = (-ws.data_ptr()) % 256
    for j in range(c):
        ref = torch.empty(n, device="cuda")
        assert lib.pyrite_cuda_rmsnorm_encode(x[j].data_ptr(), w.data_ptr(), n, 1e-6, ref.data_ptr(), ws.data_ptr() + off,
                                              ws.numel() - off, st) == 0
        torch.cuda.synchronize()
        assert torch.allclose(out[j], ref, rtol=1e-6, atol=0)  # same fp64 statistics, other summation order
    # SiLU(gate) * up: elementwise, bit-exact
    f = 1536
    gu = torch.randn(c, 2 * f, device="cuda", generator=g) * 4
    act = torch.empty(c, f, device="cuda")
    assert lib.pyrite_cuda_silu_mul_rows(gu.data_ptr(), 2 * f, f, c, act.data_ptr(), f, st) == 0
    for j in range(c):
        ref = torch.empty(f, device="cuda")
        wsa = torch.zeros(int(lib.pyrite_cuda_workspace_size(0, f, 1)) + 256, dtype=torch.uint8, device="cuda")
        o2 = (-wsa.data_ptr()) % 256
        assert lib.pyrite_cuda_silu_mul_encode(gu[j].data_ptr(), f, ref.data_ptr(), wsa.data_ptr() + o2,
                                               wsa.numel() - o2, st) == 0
        torch.cuda.synchronize()
        assert torch.equal(act[j], ref)


@pytest.mark.parametrize("nq,nkv,first,count", [(32, 8, 0, 37), (16, 4, 100, 64), (8, 8, 3000, 20), (64, 4, 8100, 33)])
def test_qk_rope_kv_rows_and_causal_attention(cuda_device, nq, nkv, first, count):
    """qk_rope_kv_rows equals qk_rope_kv position by position (same fp64 per-head
    arithmetic: bit-exact); attention_rows equals an fp64 restatement of the
    reference's attention for each position of the block within 1e-4 of
    sum_t p_t |v_t|."""
    import torch

    from pyrite_b200 import _lib
    from tests.test_gpu_attention_long import HD, rope_table
    lib = _lib.require()
    st = torch.cuda.current_stream().cuda_stream
    max_ctx, theta, eps = first + count + 3, 1e6, 1e-6
    rng = np.random.default_rng(first + nq)
    qkv = torch.from_numpy(rng.normal(0, 1, (count, (nq + 2 * nkv) * HD)).astype(np.float32)).cuda()
    qn = torch.from_numpy((rng.random(HD) + 0.5).astype(np.float32)).cuda()
    kn = torch.from_numpy((rng.random(HD) + 0.5).astype(np.float32)).cuda()
    kc = torch.from_numpy(rng.normal(0, 1, (max_ctx, nkv * HD)).astype(np.float32)).cuda()
    vc = torch.from_numpy(rng.normal(0, 1, (max_ctx, nkv * HD)).astype(np.float32)).cuda()
    kc2, vc2 = kc.clone(), vc.clone()
    rope = torch.from_numpy(rope_table(max_ctx, theta)).cuda()
    qr = torch.empty(count, nq * HD, device="cuda")
    assert lib.pyrite_cuda_qk_rope_kv_rows(qkv.data_ptr(), (nq + 2 * nkv) * HD, qn.data_ptr(), kn.data_ptr(), nq, nkv,
                                           HD, eps, first, None, 1, 0, count, rope.data_ptr(), max_ctx, qr.data_ptr(),
                                           nq * HD, kc.data_ptr(), vc.data_ptr(), st) == 0
    qref = torch.empty(nq * HD, device="cuda")
    for j in range(count):
        p = torch.tensor([first + j], dtype=torch.int32, device="cuda")
        assert lib.pyrite_cuda_qk_rope_kv(qkv[j].data_ptr(), qn.data_ptr(), kn.data_ptr(), nq, nkv, HD, eps,
                                          p.data_ptr(), rope.data_ptr(), max_ctx, qref.data_ptr(), kc2.data_ptr(),
                                          vc2.data_ptr(), st) == 0
        torch.cuda.synchronize()
        assert torch.equal(qr[j], qref)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    out = torch.empty(count, nq * HD, device="cuda")
    assert lib.pyrite_cuda_attention_rows(qr.data_ptr(), nq * HD, kc.data_ptr(), vc.data_ptr(), 0, first, None, 1, count,
                                          nq, nkv, HD, max_ctx, out.data_ptr(), nq * HD, st) == 0
    torch.cuda.synchronize()
    K, V, Q, O = (t.double().cpu().numpy() for t in (kc, vc, qr, out))
    grp = nq // nkv
    for j in range(0, count, max(1, count // 6)):
        T = first + j + 1
        for h in range(0, nq, max(1, nq // 4)):
            kk = K[:T, (h // grp) * HD:(h // grp + 1) * HD]
            vv = V[:T, (h // grp) * HD:(h // grp + 1) * HD]
            sc = kk @ Q[j, h * HD:(h + 1) * HD] / np.sqrt(HD)
            pr = np.exp(sc - sc.max())
            pr /= pr.sum()
            want, bound = pr @ vv, pr @ np.abs(vv)
            got = O[j, h * HD:(h + 1) * HD]
            assert float((np.abs(got - want) / bound).max()) <= 1e-4
