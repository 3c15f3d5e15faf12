"""The decode step's attention at long context against an fp64 restatement (B200).

The reference's attention for one new position (pyrite/executor.py:685-755):
per-head RMSNorm of q and k when the model has QK-norm weights
(executor.py:621-624), NEOX RoPE with angle pos * theta^(-2i/head_dim)
(executor.py:626-644), k and v appended to the fp32 cache (LayerKV,
executor.py:78-140), then for every q head a softmax over the scores
q . k_t / sqrt(head_dim) of all cached positions t <= pos of its kv group and
the probability-weighted sum of the values, in fp64.  restate() below is that
computation in numpy fp64; pyrite_cuda_attention_step (the context split over
several CTAs per head, partials merged by the last one) must match it within
1e-4 relative to sum_t p_t |v_t| at the geometries of configs[2]
(Llama-3-8B: 32 q / 8 kv heads, no QK norm, KV ctx 4096), configs[3]
(Qwen3-30B-A3B: 32 q / 4 kv heads, QK norm) and configs[4]
(Qwen3-235B-A22B: 64 q / 4 kv heads, QK norm, KV ctx 8192).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HD = 128
TOL = 1e-4


def rope_table(max_ctx: int, theta: float) -> np.ndarray:
    """(cos, sin) of pos * theta^(-2i/HD) for i < HD/2, fp64, as the reference computes them."""
    freq = np.array([theta ** (-2.0 * i / HD) for i in range(HD // 2)])
    ang = np.arange(max_ctx, dtype=np.float64)[:, None] * freq[None, :]
    return np.ascontiguousarray(np.stack([np.cos(ang), np.sin(ang)], -1))


def prep_head(v: np.ndarray, norm: np.ndarray | None, pos: int, theta: float, eps: float) -> np.ndarray:
    v = v.astype(np.float64)
    if norm is not None:
        v = v / np.sqrt(np.sum(v * v) / v.size + eps) * norm.astype(np.float64)
    half = HD // 2
    i = np.arange(half)
    ang = pos * theta ** (-2.0 * i / HD)
    c, s = np.cos(ang), np.sin(ang)
    x0, x1 = v[:half].copy(), v[half:].copy()
    out = v.copy()
    out[:half] = x0 * c - x1 * s
    out[half:] = x0 * s + x1 * c
    return out


def restate(qkv, q_norm, k_norm, nq, nkv, pos, theta, eps, k_cache, v_cache):
    """fp64 attention output of position pos, and the fp32 k / v rows it appends."""
    q = qkv[: nq * HD].reshape(nq, HD)
    k = qkv[nq * HD:(nq + nkv) * HD].reshape(nkv, HD)
    v = qkv[(nq + nkv) * HD:].reshape(nkv, HD)
    qh = np.stack([prep_head(q[h], q_norm, pos, theta, eps) for h in range(nq)])
    kh = np.stack([prep_head(k[h], k_norm, pos, theta, eps) for h in range(nkv)])
    k_row = kh.reshape(-1).astype(np.float32)  # the cache is fp32 (array('f'))
    v_row = v.reshape(-1).astype(np.float32)
    keys = np.concatenate([k_cache[:pos], k_row[None]]).astype(np.float64).reshape(pos + 1, nkv, HD)
    vals = np.concatenate([v_cache[:pos], v_row[None]]).astype(np.float64).reshape(pos + 1, nkv, HD)
    grp = nq // nkv
    out, scale = np.empty((nq, HD)), np.empty(nq * HD)
    for h in range(nq):
        sc = keys[:, h // grp] @ qh[h] / np.sqrt(HD)
        p = np.exp(sc - sc.max())
        p /= p.sum()
        out[h] = p @ vals[:, h // grp]
        scale[h * HD:(h + 1) * HD] = p @ np.abs(vals[:, h // grp])
    return out.reshape(-1), k_row, v_row, scale


CASES = [  # (name, n_q, n_kv, qk_norm, theta, max_ctx, pos)
    ("configs[2]", 32, 8, False, 5e5, 4096, 63),
    ("configs[2]", 32, 8, False, 5e5, 4096, 64),
    ("configs[2]", 32, 8, False, 5e5, 4096, 2500),
    ("configs[2]", 32, 8, False, 5e5, 4096, 4095),
    ("configs[3]", 32, 4, True, 1e6, 1024, 1023),
    ("configs[4]", 64, 4, True, 1e6, 8192, 8191),
    ("configs[4]", 64, 4, True, 1e6, 8192, 3000),
]


@pytest.mark.parametrize("name,nq,nkv,qk_norm,theta,max_ctx,pos", CASES)
def test_attention_step_matches_fp64_restatement(cuda_device, name, nq, nkv, qk_norm, theta, max_ctx, pos):
    import torch

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K
    lib = _lib.require()
    rng = np.random.default_rng(pos * 31 + nq)
    eps = 1e-6
    qkv = rng.normal(0, 1, (nq + 2 * nkv) * HD).astype(np.float32)
    q_norm = (rng.random(HD) + 0.5).astype(np.float32) if qk_norm else None
    k_norm = (rng.random(HD) + 0.5).astype(np.float32) if qk_norm else None
    k_cache = rng.normal(0, 1, (max_ctx, nkv * HD)).astype(np.float32)
    v_cache = rng.normal(0, 1, (max_ctx, nkv * HD)).astype(np.float32)
    want, k_row, v_row, scale = restate(qkv, q_norm, k_norm, nq, nkv, pos, theta, eps, k_cache, v_cache)

    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    d_qkv, d_kc, d_vc = dev(qkv), dev(k_cache), dev(v_cache)
    d_qn = dev(q_norm) if qk_norm else None
    d_kn = dev(k_norm) if qk_norm else None
    rope = dev(rope_table(max_ctx, theta))
    p = torch.tensor([pos], dtype=torch.int32, device="cuda")
    out = torch.empty(nq * HD, device="cuda")
    per = int(lib.pyrite_cuda_workspace_size(0, nq * HD, 1))
    ws = torch.zeros(per + 256, dtype=torch.uint8, device="cuda")
    off = (-ws.data_ptr()) % 256
    scratch = torch.zeros(int(lib.pyrite_cuda_attention_scratch_size(nq, max_ctx)), dtype=torch.uint8, device="cuda")
    code = lib.pyrite_cuda_attention_step(d_qkv.data_ptr(), d_qn.data_ptr() if qk_norm else None,
                                          d_kn.data_ptr() if qk_norm else None, nq, nkv, HD, eps, p.data_ptr(),
                                          rope.data_ptr(), max_ctx, d_kc.data_ptr(), d_vc.data_ptr(), out.data_ptr(),
                                          ws.data_ptr() + off, ws.numel() - off, scratch.data_ptr(), scratch.numel(),
                                          torch.cuda.current_stream().cuda_stream)
    assert code == 0, code
    torch.cuda.synchronize()
    assert K.status() == 0
    got_k, got_v = d_kc[pos].cpu().numpy(), d_vc[pos].cpu().numpy()
    assert np.array_equal(got_v, v_row)
    assert np.allclose(got_k, k_row, rtol=1e-6, atol=1e-7)
    others = np.ones(max_ctx, dtype=bool)
    others[pos] = False
    assert np.array_equal(d_kc.cpu().numpy()[others], k_cache[others])  # only row pos is written
    err = np.abs(out.cpu().numpy().astype(np.float64) - want) / (scale + 1e-30)
    assert float(err.max()) <= TOL, f"{name} pos {pos}: max relative error {err.max():.3e}"
