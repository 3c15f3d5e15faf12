"""Device-resident batch-1 decode of ``qwen3moe`` checkpoints (routed experts).

The B200 counterpart of the reference's ``Qwen3MoEExecutor``
(``pyrite/executor.py:685-939``): per layer RMSNorm, Q/K/V projections,
per-head QK RMSNorm, NEOX RoPE, fp32 KV cache, grouped-query attention, output
projection and residual, RMSNorm, then the routed feed-forward -- router
matvec, softmax top-k (``executor.py:757-793``), for every selected expert the
gate/up/down products over its slice of the stacked expert tensors
(``executor.py:672-683``, ``qwen3_moe.py:364-398``), SiLU, the weighted sum
in rank order and the residual; final RMSNorm, LM head, greedy argmax.

Every weight stays in HBM in its GGML bytes (the checkpoint's Q4_K_M mix:
one GGML type per tensor).  The expert ids are computed on the device and
read by the expert matvecs there, so one decode step is a fixed launch
sequence captured in one CUDA graph.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .kernels.cuda import STATIC_WEIGHTS, _check
from .synthetic import F32, MoESpec, moe_tensors

ACCUMULATE = 2  # PYRITE_F_ACCUMULATE


@dataclass
class _Mat:
    ggml_type: int
    data: torch.Tensor  # uint8, GGML bytes
    rows: int
    cols: int


@dataclass
class _MoELayer:
    attn_norm: torch.Tensor
    ffn_norm: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    qk: _Mat       # [q | k] rows (one GGML type)
    v: _Mat
    o: _Mat
    router: _Mat
    gate_exps: _Mat  # stacked: rows = moe ff, E matrices
    up_exps: _Mat
    down_exps: _Mat


class MoEDecoder:
    """One sequence, batch 1, every weight in HBM; greedy decoding."""

    def __init__(self, spec: MoESpec, tensors: dict[str, tuple[tuple[int, ...], int, bytes]],
                 device: torch.device | str = "cuda", max_ctx: int = 512):
        self.spec = spec
        self.dev = d = torch.device(device)
        self.max_ctx = max_ctx
        self.lib = L = _lib.require()
        h, ff, E, k = spec.hidden_size, spec.moe_intermediate_size, spec.num_experts, spec.num_experts_per_tok

        def mat(name: str) -> _Mat:
            dims, t, payload = tensors[name]
            rows = int(np.prod(dims[1:]))
            return _Mat(t, torch.frombuffer(bytearray(payload), dtype=torch.uint8).to(d), rows, dims[0])

        def stacked(name: str) -> _Mat:
            dims, t, payload = tensors[name]
            return _Mat(t, torch.frombuffer(bytearray(payload), dtype=torch.uint8).to(d), dims[1], dims[0])

        def f32(name: str) -> torch.Tensor:
            dims, t, payload = tensors[name]
            if t != F32:
                raise ValueError(f"{name} must be F32")
            return torch.frombuffer(bytearray(payload), dtype=torch.float32).to(d)

        self.embd = mat("token_embd.weight")
        self.lm_head = self.embd if spec.tied_embeddings else mat("output.weight")
        self.out_norm = f32("output_norm.weight")
        self.layers: list[_MoELayer] = []
        for i in range(spec.num_hidden_layers):
            p = f"blk.{i}."
            q, kk = mat(p + "attn_q.weight"), mat(p + "attn_k.weight")
            if q.ggml_type != kk.ggml_type:
                raise ValueError(f"{p}attn_q and attn_k must share a GGML type")
            qk = _Mat(q.ggml_type, torch.cat([q.data, kk.data]), q.rows + kk.rows, q.cols)
            self.layers.append(_MoELayer(
                attn_norm=f32(p + "attn_norm.weight"), ffn_norm=f32(p + "ffn_norm.weight"),
                q_norm=f32(p + "attn_q_norm.weight"), k_norm=f32(p + "attn_k_norm.weight"),
                qk=qk, v=mat(p + "attn_v.weight"), o=mat(p + "attn_output.weight"),
                router=mat(p + "ffn_gate_inp.weight"), gate_exps=stacked(p + "ffn_gate_exps.weight"),
                up_exps=stacked(p + "ffn_up_exps.weight"), down_exps=stacked(p + "ffn_down_exps.weight")))

        # activations and state
        q_dim, kv_dim = spec.q_dim, spec.kv_dim
        z = lambda *shape, dt=torch.float32: torch.zeros(*shape, dtype=dt, device=d)  # noqa: E731
        self.hidden, self.normed = z(h), z(h)
        self.qkv, self.attn = z(q_dim + 2 * kv_dim), z(q_dim)
        self.router_logits = z(E)
        self.expert_ids, self.expert_w = z(k, dt=torch.int32), z(k)
        self.gate, self.up, self.act, self.down = z(k, ff), z(k, ff), z(k, ff), z(k, h)
        self.logits = z(spec.vocab_size)
        self.kcache = z(spec.num_hidden_layers, max_ctx, kv_dim)
        self.vcache = torch.zeros_like(self.kcache)
        self.tokens, self.pos = z(max_ctx, dt=torch.int32), z(1, dt=torch.int32)
        self.argmax_scratch = z(int(L.pyrite_cuda_post_scratch_size()) + 256, dt=torch.uint8)
        self.ticket = z(1, dt=torch.int32)
        # the experts each layer routed to in the latest step (rank order)
        self.route_log = z(spec.num_hidden_layers, k, dt=torch.int32)

        def ws(n: int, copies: int = 1) -> tuple[torch.Tensor, int, int]:
            per = int(L.pyrite_cuda_workspace_size(0, n, 1))
            buf = torch.empty(per * copies + 256, dtype=torch.uint8, device=d)
            return buf, (-buf.data_ptr()) % 256, per

        self.ws_h, self.ws_q, self.ws_act = ws(h), ws(q_dim), ws(ff, k)
        half = spec.head_dim // 2
        inv = spec.rope_theta ** (-2.0 * np.arange(half, dtype=np.float64) / spec.head_dim)
        ang = np.arange(max_ctx, dtype=np.float64)[:, None] * inv[None, :]
        self.rope = torch.from_numpy(np.ascontiguousarray(np.stack([np.cos(ang), np.sin(ang)], axis=-1))).to(d)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.prompt_len = 0

    @classmethod
    def synthetic(cls, spec: MoESpec, device="cuda", max_ctx: int = 512) -> "MoEDecoder":
        tensors = {name: (dims, t, payload) for name, dims, t, payload in moe_tensors(spec)}
        return cls(spec, tensors, device=device, max_ctx=max_ctx)

    # ------------------------------------------------------------------ helpers
    @staticmethod
    def _wsp(ws: tuple[torch.Tensor, int, int]) -> tuple[int, int]:
        buf, off, _ = ws
        return buf.data_ptr() + off, buf.numel() - off

    def _mv(self, m: _Mat, x: torch.Tensor, ws, y: torch.Tensor, flags: int, stream: int, post=None) -> None:
        wptr, wlen = self._wsp(ws)
        if post is None:
            code = self.lib.pyrite_cuda_matvec_prepared(m.ggml_type, m.data.data_ptr(), m.data.numel(), x.data_ptr(),
                                                        wptr, wlen, y.data_ptr(), m.rows, m.cols,
                                                        flags | STATIC_WEIGHTS, stream)
        else:
            code = self.lib.pyrite_cuda_matvec_prepared_post(m.ggml_type, m.data.data_ptr(), m.data.numel(),
                                                             x.data_ptr(), wptr, wlen, y.data_ptr(), m.rows, m.cols,
                                                             flags | STATIC_WEIGHTS, ctypes.byref(post), stream)
        _check(code, "matvec")

    def _experts(self, m: _Mat, x: torch.Tensor, x_stride: int, ws, ws_stride: int, y: torch.Tensor,
                 stream: int) -> None:
        wptr, wlen = self._wsp(ws)
        E, k = self.spec.num_experts, self.spec.num_experts_per_tok
        code = self.lib.pyrite_cuda_matvec_experts(m.ggml_type, m.data.data_ptr(), m.data.numel(), E,
                                                   self.expert_ids.data_ptr(), k, x.data_ptr(), x_stride, wptr, wlen,
                                                   ws_stride, y.data_ptr(), y.shape[1], m.rows, m.cols, 0, stream)
        _check(code, "expert matvec")

    def _norm(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, ws, stream: int) -> None:
        wptr, wlen = self._wsp(ws)
        _check(self.lib.pyrite_cuda_rmsnorm_encode(x.data_ptr(), w.data_ptr(), x.numel(), float(self.spec.rms_norm_eps),
                                                   out.data_ptr(), wptr, wlen, stream), "rmsnorm")

    # ------------------------------------------------------------------ one step
    def _step(self, stream: int) -> None:
        s, L = self.spec, self.lib
        h, ff, k = s.hidden_size, s.moe_intermediate_size, s.num_experts_per_tok
        eps = float(s.rms_norm_eps)
        qk_rows = s.q_dim + s.kv_dim
        _check(L.pyrite_cuda_embed(self.embd.ggml_type, self.embd.data.data_ptr(), s.vocab_size, h,
                                   self.tokens.data_ptr(), self.pos.data_ptr(), self.hidden.data_ptr(), stream), "embed")
        for li, ly in enumerate(self.layers):
            self._norm(self.hidden, ly.attn_norm, self.normed, self.ws_h, stream)
            self._mv(ly.qk, self.normed, self.ws_h, self.qkv, 0, stream)
            self._mv(ly.v, self.normed, self.ws_h, self.qkv[qk_rows:], 0, stream)
            wq, wql = self._wsp(self.ws_q)
            _check(L.pyrite_cuda_attention_step(
                self.qkv.data_ptr(), ly.q_norm.data_ptr(), ly.k_norm.data_ptr(), s.num_attention_heads,
                s.num_key_value_heads, s.head_dim, eps, self.pos.data_ptr(), self.rope.data_ptr(), self.max_ctx,
                self.kcache[li].data_ptr(), self.vcache[li].data_ptr(), self.attn.data_ptr(), wq, wql, stream),
                "attention_step")
            self._mv(ly.o, self.attn, self.ws_q, self.hidden, ACCUMULATE, stream)
            self._norm(self.hidden, ly.ffn_norm, self.normed, self.ws_h, stream)
            # routed feed-forward
            self._mv(ly.router, self.normed, self.ws_h, self.router_logits, 0, stream)
            _check(L.pyrite_cuda_moe_route(self.router_logits.data_ptr(), s.num_experts, k,
                                           1 if s.norm_topk_prob else 0, 1.0, self.expert_ids.data_ptr(),
                                           self.expert_w.data_ptr(), stream), "route")
            self.route_log[li].copy_(self.expert_ids)
            self._experts(ly.gate_exps, self.normed, 0, self.ws_h, 0, self.gate, stream)
            self._experts(ly.up_exps, self.normed, 0, self.ws_h, 0, self.up, stream)
            wa, wal = self._wsp(self.ws_act)
            _check(L.pyrite_cuda_moe_silu_mul_encode(self.gate.data_ptr(), self.up.data_ptr(), ff, k,
                                                     self.act.data_ptr(), wa, wal, stream), "moe silu")
            self._experts(ly.down_exps, self.act, ff, self.ws_act, self.ws_act[2], self.down, stream)
            _check(L.pyrite_cuda_moe_combine(self.down.data_ptr(), self.expert_w.data_ptr(), k, h,
                                             self.hidden.data_ptr(), stream), "combine")
        self._norm(self.hidden, self.out_norm, self.normed, self.ws_h, stream)
        post = _lib.PostOp()
        post.op = _lib.POST_ARGMAX
        post.ticket = self.ticket.data_ptr()
        post.scratch = self.argmax_scratch.data_ptr()
        post.scratch_len = self.argmax_scratch.numel()
        post.tokens, post.pos = self.tokens.data_ptr(), self.pos.data_ptr()
        post.prompt_len, post.max_ctx = self.prompt_len, self.max_ctx
        self._mv(self.lm_head, self.normed, self.ws_h, self.logits, 0, stream, post=post)

    # ------------------------------------------------------------------ public
    def reset(self, prompt: list[int]) -> None:
        if not prompt or any(not 0 <= t < self.spec.vocab_size for t in prompt):
            raise ValueError("prompt token ids must be non-empty and inside the vocabulary")
        if len(prompt) >= self.max_ctx:
            raise ValueError("prompt does not fit the KV cache")
        if self.graph is not None and len(prompt) != self.prompt_len:
            self.graph = None
        self.prompt_len = len(prompt)
        self.tokens.zero_()
        self.tokens[: len(prompt)] = torch.tensor(prompt, dtype=torch.int32, device=self.dev)
        self.pos.zero_()
        self.kcache.zero_()
        self.vcache.zero_()

    def capture(self) -> None:
        stream = torch.cuda.Stream(device=self.dev)
        saved = self.pos.clone()
        with torch.cuda.stream(stream):
            self._step(stream.cuda_stream)
            torch.cuda.synchronize(self.dev)
            self.pos.copy_(saved)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                self._step(stream.cuda_stream)
        torch.cuda.synchronize(self.dev)
        self.pos.copy_(saved)
        self.graph = g

    def run_steps(self, n: int) -> None:
        if self.graph is None:
            self.capture()
        for _ in range(n):
            self.graph.replay()

    def generate(self, prompt: list[int], max_new_tokens: int) -> list[int]:
        """Greedy continuation, the reference's ``generate(..., temperature=0)``."""
        if len(prompt) + max_new_tokens > self.max_ctx:
            raise ValueError("prompt + new tokens exceed the KV cache")
        if max_new_tokens == 0:
            return list(prompt)
        if self.graph is None or self.prompt_len != len(prompt):
            self.reset(prompt)
            self.capture()
        self.reset(prompt)
        self.run_steps(len(prompt) + max_new_tokens - 1)
        torch.cuda.synchronize(self.dev)
        return [int(t) for t in self.tokens[: len(prompt) + max_new_tokens].cpu()]
