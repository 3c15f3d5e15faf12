"""Post ops: a batch-1 matvec that also runs the next decode-step operation on
its whole output in its last CTA (pyrite_cuda_matvec_prepared_post), through
the C ABI (B200).

Each fused call must give exactly what the product followed by the operation's
own kernel gives: RMSNorm + encoding (executor.py:621-624), SiLU * up +
encoding (dense.py:491-494) and the greedy argmax (sampler.py:12-15), for a
format with the batch-1 kernel (fused in the last CTA) and one without (the
product, then the operation's kernel).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from tests.payloads import random_payload

pytestmark = pytest.mark.gpu


def _setup(ggml_type, rows, cols, seed):
    import torch

    from pyrite_b200.kernels import cuda as K
    payload = random_payload(ggml_type, rows, cols, seed=seed)
    w = torch.frombuffer(bytearray(payload), dtype=torch.uint8).cuda()
    x = torch.randn(cols, device="cuda", generator=torch.Generator("cuda").manual_seed(seed))
    px = K.prepare_x(x)
    return w, x, px


def _ws(n):
    import torch

    from pyrite_b200 import _lib
    lib = _lib.require()
    need = int(lib.pyrite_cuda_workspace_size(0, n, 1))
    buf = torch.zeros(need + 256, dtype=torch.uint8, device="cuda")
    off = (-buf.data_ptr()) % 256
    return buf, buf.data_ptr() + off, buf.numel() - off, off, need


def _run_post(ggml_type, w, x, px, y, rows, cols, post):
    import torch

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K
    lib = _lib.require()
    code = lib.pyrite_cuda_matvec_prepared_post(ggml_type, w.data_ptr(), w.numel(), x.data_ptr(), px.ptr, px.nbytes,
                                                y.data_ptr(), rows, cols, 0, ctypes.byref(post),
                                                torch.cuda.current_stream().cuda_stream)
    assert code == 0, code
    torch.cuda.synchronize()
    assert K.status() == 0


@pytest.mark.parametrize("ggml_type", [8, 12, 14, 23, 2])
def test_post_rmsnorm_encode_equals_separate_kernel(cuda_device, ggml_type):
    import torch

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K
    lib = _lib.require()
    rows, cols = 1024, 2048
    w, x, px = _setup(ggml_type, rows, cols, 3)
    norm_w = torch.rand(rows, device="cuda") + 0.5
    y = torch.empty(rows, device="cuda")
    out = torch.empty(rows, device="cuda")
    ticket = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws_buf, ws_ptr, ws_len, ws_off, need = _ws(rows)
    p = _lib.PostOp()
    p.op, p.eps, p.weight, p.out = _lib.POST_RMSNORM_ENCODE, 1e-6, norm_w.data_ptr(), out.data_ptr()
    p.workspace, p.workspace_len, p.ticket = ws_ptr, ws_len, ticket.data_ptr()
    for _ in range(3):  # repeated: the ticket must come back to zero
        _run_post(ggml_type, w, x, px, y, rows, cols, p)
        assert int(ticket.item()) == 0
    want_y = K.matvec_prepared(ggml_type, w, px, rows, cols)
    assert torch.equal(y, want_y)
    ref_out = torch.empty(rows, device="cuda")
    ref_buf, ref_ptr, ref_len, ref_off, _ = _ws(rows)
    assert lib.pyrite_cuda_rmsnorm_encode(y.data_ptr(), norm_w.data_ptr(), rows, 1e-6, ref_out.data_ptr(), ref_ptr,
                                          ref_len, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    # same fp64 statistics up to the summation order of a 256- vs 1024-thread CTA
    assert torch.allclose(out, ref_out, rtol=1e-6, atol=0)
    a = ws_buf[ws_off:ws_off + need].cpu().numpy()
    b = ref_buf[ref_off:ref_off + need].cpu().numpy()
    assert np.mean(a == b) > 0.999


@pytest.mark.parametrize("ggml_type", [8, 12, 2])
def test_post_silu_mul_encode_equals_separate_kernel(cuda_device, ggml_type):
    import torch

    from pyrite_b200 import _lib
    lib = _lib.require()
    f, cols = 1536, 1024
    rows = 2 * f
    w, x, px = _setup(ggml_type, rows, cols, 5)
    y = torch.empty(rows, device="cuda")
    act = torch.empty(f, device="cuda")
    ticket = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws_buf, ws_ptr, ws_len, ws_off, need = _ws(f)
    p = _lib.PostOp()
    p.op, p.out, p.workspace, p.workspace_len, p.ticket = (_lib.POST_SILU_MUL_ENCODE, act.data_ptr(), ws_ptr, ws_len,
                                                           ticket.data_ptr())
    _run_post(ggml_type, w, x, px, y, rows, cols, p)
    assert int(ticket.item()) == 0
    ref = torch.empty(f, device="cuda")
    ref_buf, ref_ptr, ref_len, ref_off, _ = _ws(f)
    assert lib.pyrite_cuda_silu_mul_encode(y.data_ptr(), f, ref.data_ptr(), ref_ptr, ref_len,
                                           torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(act, ref)
    assert torch.equal(ws_buf[ws_off:ws_off + need], ref_buf[ref_off:ref_off + need])


@pytest.mark.parametrize("ggml_type", [8, 12, 2])
@pytest.mark.parametrize("rows", [151936, 4096, 7])
def test_post_argmax_picks_first_maximum(cuda_device, ggml_type, rows):
    import torch

    from pyrite_b200 import _lib
    lib = _lib.require()
    cols = 1024
    w, x, px = _setup(ggml_type, rows, cols, rows)
    y = torch.empty(rows, device="cuda")
    ticket = torch.zeros(1, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(int(lib.pyrite_cuda_post_scratch_size()), dtype=torch.uint8, device="cuda")
    tokens = torch.zeros(16, dtype=torch.int32, device="cuda")
    pos = torch.tensor([5], dtype=torch.int32, device="cuda")
    p = _lib.PostOp()
    p.op, p.ticket, p.scratch, p.scratch_len = _lib.POST_ARGMAX, ticket.data_ptr(), scratch.data_ptr(), scratch.numel()
    p.tokens, p.pos, p.prompt_len, p.max_ctx = tokens.data_ptr(), pos.data_ptr(), 3, 16
    _run_post(ggml_type, w, x, px, y, rows, cols, p)
    ys = y.cpu().numpy()
    want = int(np.flatnonzero(ys == ys.max())[0])
    assert int(tokens[6].item()) == want
    assert int(pos.item()) == 6
    assert int(ticket.item()) == 0
    # a prompt position is never overwritten
    pos.fill_(0)
    tokens.fill_(-1)
    _run_post(ggml_type, w, x, px, y, rows, cols, p)
    assert int(tokens[1].item()) == -1 and int(pos.item()) == 1


@pytest.mark.parametrize("max_ctx,pos", [(512, 0), (512, 17), (512, 511), (4096, 2500), (4096, 63), (4096, 64)])
def test_split_attention_step_equals_separate_kernels(cuda_device, max_ctx, pos):
    """The context-split fused attention step (per-chunk partials merged by the
    last CTA) against qk_rope_kv + attention over the same cache."""
    import numpy as np
    import torch

    from pyrite_b200 import _lib
    lib = _lib.require()
    nq, nkv, hd = 16, 4, 128
    g = torch.Generator("cuda").manual_seed(pos)
    qkv = torch.randn((nq + 2 * nkv) * hd, device="cuda", generator=g)
    qn = torch.rand(hd, device="cuda", generator=g) + 0.5
    kn = torch.rand(hd, device="cuda", generator=g) + 0.5
    ang = np.arange(max_ctx)[:, None] * (1e6 ** (-2.0 * np.arange(hd // 2) / hd))[None, :]
    rope = torch.from_numpy(np.ascontiguousarray(np.stack([np.cos(ang), np.sin(ang)], -1))).cuda()
    kc = torch.randn(max_ctx, nkv * hd, device="cuda", generator=g)
    vc = torch.randn(max_ctx, nkv * hd, device="cuda", generator=g)
    kc2, vc2 = kc.clone(), vc.clone()
    p = torch.tensor([pos], dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    # separate kernels
    q = torch.empty(nq * hd, device="cuda")
    ref = torch.empty(nq * hd, device="cuda")
    assert lib.pyrite_cuda_qk_rope_kv(qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), nq, nkv, hd, 1e-6, p.data_ptr(),
                                      rope.data_ptr(), max_ctx, q.data_ptr(), kc2.data_ptr(), vc2.data_ptr(), s) == 0
    assert lib.pyrite_cuda_attention(q.data_ptr(), kc2.data_ptr(), vc2.data_ptr(), p.data_ptr(), nq, nkv, hd,
                                     max_ctx, ref.data_ptr(), s) == 0 or max_ctx * 4 > 48 * 1024
    # fused, split
    out = torch.empty(nq * hd, device="cuda")
    per = int(lib.pyrite_cuda_workspace_size(0, nq * hd, 1))
    ws = torch.zeros(per + 256, dtype=torch.uint8, device="cuda")
    off = (-ws.data_ptr()) % 256
    scratch = torch.zeros(int(lib.pyrite_cuda_attention_scratch_size(nq, max_ctx)), dtype=torch.uint8, device="cuda")
    for _ in range(2):  # the tickets come back to zero
        assert lib.pyrite_cuda_attention_step(qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), nq, nkv, hd, 1e-6,
                                              p.data_ptr(), rope.data_ptr(), max_ctx, kc.data_ptr(), vc.data_ptr(),
                                              out.data_ptr(), ws.data_ptr() + off, ws.numel() - off,
                                              scratch.data_ptr(), scratch.numel(), s) == 0
    torch.cuda.synchronize()
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert int(scratch[: 4 * nq].view(torch.int32).abs().sum()) == 0
    if max_ctx * 4 <= 48 * 1024:
        assert torch.allclose(out, ref, rtol=1e-4, atol=1e-5)
    else:  # beyond the one-CTA kernel's shared memory: an fp64 softmax in torch
        qh = q.view(nq, hd).double()
        k = kc2[: pos + 1].view(pos + 1, nkv, hd).double()
        v = vc2[: pos + 1].view(pos + 1, nkv, hd).double()
        grp = nq // nkv
        want = []
        for h in range(nq):
            sc = (k[:, h // grp] @ qh[h]) / np.sqrt(hd)
            w = torch.softmax(sc, 0)
            want.append(w @ v[:, h // grp])
        want = torch.cat(want).float()
        assert torch.allclose(out, want, rtol=1e-4, atol=1e-5)


def _transformed(lib, ggml_type, w, x, x_op, norm, x_out, ws_ptr, ws_len, y, rows, cols, flags=0):
    import torch

    code = lib.pyrite_cuda_matvec_transformed(ggml_type, w.data_ptr(), w.numel(), x.data_ptr(), x_op,
                                              norm.data_ptr() if norm is not None else None, 1e-6,
                                              x_out.data_ptr() if x_out is not None else None, ws_ptr, ws_len,
                                              y.data_ptr(), rows, cols, flags,
                                              torch.cuda.current_stream().cuda_stream)
    assert code == 0, code
    torch.cuda.synchronize()


@pytest.mark.parametrize("ggml_type", [8, 12, 13, 14, 23, 2])
@pytest.mark.parametrize("rows,cols", [(1024, 2048), (7, 4096), (3000, 14336), (64, 1024)])
@pytest.mark.parametrize("given_ws", [True, False])
def test_matvec_rmsnorm_prologue_equals_separate_kernels(cuda_device, ggml_type, rows, cols, given_ws):
    """RMSNorm computed with the matvec (pyrite_cuda_matvec_transformed; in its
    prologue when no workspace is given, else in the form the library picks)
    against pyrite_cuda_rmsnorm_encode + pyrite_cuda_matvec_prepared: the same
    fp64 statistics up to summation order, so the same product within 1e-5 of
    sum |w x|; accumulate adds to y."""
    if ggml_type == 2 and not given_ws:
        pytest.skip("formats without the batch-1 kernel need the workspace")
    import torch

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K
    lib = _lib.require()
    w, x, _ = _setup(ggml_type, rows, cols, rows + cols)
    x = x * 3.0
    norm_w = torch.rand(cols, device="cuda") + 0.5
    s = torch.cuda.current_stream().cuda_stream
    ref_x = torch.empty(cols, device="cuda")
    ref_buf, ref_ptr, ref_len, _, _ = _ws(cols)
    assert lib.pyrite_cuda_rmsnorm_encode(x.data_ptr(), norm_w.data_ptr(), cols, 1e-6, ref_x.data_ptr(), ref_ptr,
                                          ref_len, s) == 0
    ref_y = torch.empty(rows, device="cuda")
    assert lib.pyrite_cuda_matvec_prepared(ggml_type, w.data_ptr(), w.numel(), ref_x.data_ptr(), ref_ptr, ref_len,
                                           ref_y.data_ptr(), rows, cols, 0, s) == 0
    dense = K.dequantize_rows(ggml_type, w, rows, cols).double().abs()
    bound = (dense @ ref_x.double().abs()).float() * 1e-5 + 1e-6
    x_out = torch.full((cols,), float("nan"), device="cuda")
    y = torch.full((rows,), float("nan"), device="cuda")
    buf, ptr, ln, _, _ = _ws(cols)
    if not given_ws:
        ptr, ln = None, 0
    _transformed(lib, ggml_type, w, x, _lib.X_RMSNORM, norm_w, x_out, ptr, ln, y, rows, cols)
    assert K.status() == 0
    assert torch.allclose(x_out, ref_x, rtol=1e-6, atol=0)
    assert bool(((y - ref_y).abs() <= bound).all())
    base = torch.randn(rows, device="cuda")
    y2 = base.clone()
    _transformed(lib, ggml_type, w, x, _lib.X_RMSNORM, norm_w, x_out if given_ws else None, ptr, ln, y2, rows,
                 cols, 2)  # PYRITE_F_ACCUMULATE
    assert bool(((y2 - (base + ref_y)).abs() <= bound + 1e-6 * base.abs()).all())


@pytest.mark.parametrize("ggml_type", [8, 12, 14, 2])
@pytest.mark.parametrize("rows,f", [(4096, 14336), (5, 1024)])
@pytest.mark.parametrize("given_ws", [True, False])
def test_matvec_silu_prologue_equals_separate_kernels(cuda_device, ggml_type, rows, f, given_ws):
    """SiLU(gate) * up computed with the down projection (in its prologue when
    no workspace is given): elementwise, so the encoded activation and the
    product are identical to pyrite_cuda_silu_mul_encode +
    pyrite_cuda_matvec_prepared."""
    if ggml_type == 2 and not given_ws:
        pytest.skip("formats without the batch-1 kernel need the workspace")
    import torch

    from pyrite_b200 import _lib
    lib = _lib.require()
    w, _, _ = _setup(ggml_type, rows, f, rows ^ f)
    gu = torch.randn(2 * f, device="cuda", generator=torch.Generator("cuda").manual_seed(f)) * 4
    s = torch.cuda.current_stream().cuda_stream
    ref_act = torch.empty(f, device="cuda")
    ref_buf, ref_ptr, ref_len, _, _ = _ws(f)
    assert lib.pyrite_cuda_silu_mul_encode(gu.data_ptr(), f, ref_act.data_ptr(), ref_ptr, ref_len, s) == 0
    ref_y = torch.empty(rows, device="cuda")
    assert lib.pyrite_cuda_matvec_prepared(ggml_type, w.data_ptr(), w.numel(), ref_act.data_ptr(), ref_ptr, ref_len,
                                           ref_y.data_ptr(), rows, f, 0, s) == 0
    act = torch.empty(f, device="cuda")
    y = torch.empty(rows, device="cuda")
    buf, ptr, ln, _, _ = _ws(f)
    if not given_ws:
        ptr, ln = None, 0
    _transformed(lib, ggml_type, w, gu, _lib.X_SILU_MUL, None, act, ptr, ln, y, rows, f)
    assert torch.equal(act, ref_act)
    assert torch.equal(y, ref_y)


def test_matvec_transformed_rejects_bad_arguments(cuda_device):
    import torch

    from pyrite_b200 import _lib
    lib = _lib.require()
    w, x, _ = _setup(8, 64, 256, 1)
    y = torch.empty(64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    # unknown operation, RMSNorm without a weight, a format without the batch-1
    # kernel given no workspace
    assert lib.pyrite_cuda_matvec_transformed(8, w.data_ptr(), w.numel(), x.data_ptr(), 3, None, 1e-6, None, None, 0,
                                              y.data_ptr(), 64, 256, 0, s) == -3
    assert lib.pyrite_cuda_matvec_transformed(8, w.data_ptr(), w.numel(), x.data_ptr(), 1, None, 1e-6, None, None, 0,
                                              y.data_ptr(), 64, 256, 0, s) == -3
    w2, _, _ = _setup(1, 64, 256, 1)  # F16: the warp-per-row kernel only
    assert lib.pyrite_cuda_matvec_transformed(1, w2.data_ptr(), w2.numel(), x.data_ptr(), 2, None, 1e-6, None, None,
                                              0, y.data_ptr(), 64, 256, 0, s) == -3


@pytest.mark.parametrize("n_slices,vocab", [(2, 4096), (8, 151936), (4, 128256)])
def test_argmax_pairs_over_a_split_vocabulary(cuda_device, n_slices, vocab):
    """pyrite_cuda_argmax_local on each slice of a vocabulary (as each GPU of a
    vocabulary-sharded LM head would), the pairs concatenated (the all-gather),
    then pyrite_cuda_argmax_pick: the first index of the global maximum
    (sampler.py:12-15), with the maximum planted in several slices so the
    lowest id must win the tie."""
    import torch

    from pyrite_b200 import _lib
    lib = _lib.require()
    s = torch.cuda.current_stream().cuda_stream
    g = torch.Generator("cuda").manual_seed(vocab + n_slices)
    logits = torch.randn(vocab, device="cuda", generator=g)
    per = vocab // n_slices
    top = float(logits.max()) + 1.0
    planted = [per * k + 17 * k + 3 for k in range(1, n_slices)]  # in slices 1.. (not 0)
    logits[planted] = top
    pairs = torch.zeros(2 * n_slices, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    for k in range(n_slices):
        sl = logits[per * k: per * (k + 1)]
        assert lib.pyrite_cuda_argmax_local(sl.data_ptr(), per, per * k, scratch.data_ptr(), scratch.numel(),
                                            pairs[2 * k:].data_ptr(), s) == 0
    tokens = torch.full((8,), -1, dtype=torch.int32, device="cuda")
    pos = torch.tensor([3], dtype=torch.int32, device="cuda")
    assert lib.pyrite_cuda_argmax_pick(pairs.data_ptr(), n_slices, tokens.data_ptr(), pos.data_ptr(), 0, 8, s) == 0
    torch.cuda.synchronize()
    assert int(tokens[4]) == min(planted) == int(torch.argmax(logits)) and int(pos) == 4
    v = pairs.view(-1, 2)
    for k in range(n_slices):  # each pair: the slice's maximum and its global id
        sl = logits[per * k: per * (k + 1)]
        assert int(v[k, 1]) == per * k + int(torch.argmax(sl))
        assert float(v[k, 0:1].view(torch.float32)) == float(sl.max())
