"""Device-resident batch-1 decode of mixed-type checkpoints: dense
``llama`` / ``qwen3`` models in a K-quant mix (configs[2], the
Llama-3-8B-shaped Q4_K_M model) and ``qwen3moe`` models with routed experts
(configs[3] and [4]).

The B200 counterpart of the reference's executors (``pyrite/dense.py:440-513``
and ``pyrite/executor.py:685-939``): per layer RMSNorm, Q/K/V projections,
per-head QK RMSNorm where the checkpoint has it, NEOX RoPE, fp32 KV cache,
grouped-query attention, output projection and residual, RMSNorm, then the
feed-forward -- SwiGLU, or for MoE the router matvec, softmax top-k
(``executor.py:757-793``), for every selected expert the gate/up/down products
over its slice of the stacked expert tensors (``executor.py:672-683``,
``qwen3_moe.py:364-398``), SiLU, the weighted sum in rank order -- and the
residual; final RMSNorm, LM head, greedy argmax.

Every weight stays in HBM in its GGML bytes, one GGML type per tensor.  The
expert ids are computed on the device and read by the expert matvecs there,
so one decode step is a fixed launch sequence captured in one CUDA graph.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .kernels.cuda import STATIC_WEIGHTS, _check
from .synthetic import F32, DenseSpec, MoESpec, dense_tensors, moe_tensors

ACCUMULATE = 2  # PYRITE_F_ACCUMULATE


@dataclass
class _Mat:
    ggml_type: int
    data: torch.Tensor  # uint8, GGML bytes
    rows: int
    cols: int


@dataclass
class _Layer:
    attn_norm: torch.Tensor
    ffn_norm: torch.Tensor
    q_norm: torch.Tensor | None
    k_norm: torch.Tensor | None
    qk: _Mat       # [q | k] rows (one GGML type)
    v: _Mat
    o: _Mat
    # dense feed-forward
    gate_up: _Mat | None = None  # [gate | up] rows when both share a type
    gate: _Mat | None = None
    up: _Mat | None = None
    down: _Mat | None = None
    # routed experts
    router: _Mat | None = None
    gate_exps: _Mat | None = None  # stacked: rows = moe ff, E matrices
    up_exps: _Mat | None = None
    down_exps: _Mat | None = None
    gate_up_exps: _Mat | None = None  # [gate stack | up stack] when both share a type (one launch for both)


class MixedDecoder:
    """One sequence, batch 1, every weight in HBM; greedy decoding.

    ``replicate``: the checkpoint's tensors hold layers 0 and 1 only; layer i
    gets its own device copy of layer i % 2's bytes (a full-depth model for
    throughput runs without generating every layer's weights on the host).
    """

    def __init__(self, spec: DenseSpec | MoESpec, tensors: dict[str, tuple[tuple[int, ...], int, bytes]],
                 device: torch.device | str = "cuda", max_ctx: int = 512, replicate: bool = False):
        self.spec = spec
        self.moe = isinstance(spec, MoESpec)
        self.dev = d = torch.device(device)
        self.max_ctx = max_ctx
        self.lib = L = _lib.require()
        h = spec.hidden_size
        first: dict[str, torch.Tensor] = {}  # replicate: the uploaded layer-0/1 tensors

        def raw(name: str) -> torch.Tensor:
            if replicate and name.startswith("blk."):
                parts = name.split(".")
                parts[1] = str(int(parts[1]) % 2)
                src = ".".join(parts)
                if src not in first:  # first use: upload; later layers: a device copy of their own
                    first[src] = torch.frombuffer(bytearray(tensors[src][2]), dtype=torch.uint8).to(d)
                    return first[src]
                return first[src].clone()
            return torch.frombuffer(bytearray(tensors[name][2]), dtype=torch.uint8).to(d)

        def meta(name: str) -> tuple[tuple[int, ...], int]:
            if replicate and name.startswith("blk."):
                parts = name.split(".")
                parts[1] = str(int(parts[1]) % 2)
                name = ".".join(parts)
            dims, t, _ = tensors[name]
            return dims, t

        def mat(name: str) -> _Mat:
            dims, t = meta(name)
            return _Mat(t, raw(name), int(np.prod(dims[1:])), dims[0])

        def stacked(name: str) -> _Mat:
            dims, t = meta(name)
            return _Mat(t, raw(name), dims[1], dims[0])

        def f32(name: str) -> torch.Tensor | None:
            if not replicate and name not in tensors:
                return None
            dims, t = meta(name)
            if t != F32:
                raise ValueError(f"{name} must be F32")
            return raw(name).view(torch.float32)

        def has(name: str) -> bool:
            if replicate and name.startswith("blk."):
                parts = name.split(".")
                parts[1] = str(int(parts[1]) % 2)
                name = ".".join(parts)
            return name in tensors

        def cat(a: _Mat, b: _Mat) -> _Mat | None:
            if a.ggml_type != b.ggml_type or a.cols != b.cols:
                return None
            return _Mat(a.ggml_type, torch.cat([a.data, b.data]), a.rows + b.rows, a.cols)

        self.embd = mat("token_embd.weight")
        tied = spec.tied_embeddings or "output.weight" not in tensors
        self.lm_head = self.embd if tied else mat("output.weight")
        self.out_norm = f32("output_norm.weight")
        self.layers: list[_Layer] = []
        for i in range(spec.num_hidden_layers):
            p = f"blk.{i}."
            q, kk = mat(p + "attn_q.weight"), mat(p + "attn_k.weight")
            qk = cat(q, kk)
            if qk is None:
                raise ValueError(f"{p}attn_q and attn_k must share a GGML type")
            ly = _Layer(attn_norm=f32(p + "attn_norm.weight"), ffn_norm=f32(p + "ffn_norm.weight"),
                        q_norm=f32(p + "attn_q_norm.weight") if has(p + "attn_q_norm.weight") else None,
                        k_norm=f32(p + "attn_k_norm.weight") if has(p + "attn_k_norm.weight") else None,
                        qk=qk, v=mat(p + "attn_v.weight"), o=mat(p + "attn_output.weight"))
            if self.moe:
                ly.router = mat(p + "ffn_gate_inp.weight")
                ly.gate_exps = stacked(p + "ffn_gate_exps.weight")
                ly.up_exps = stacked(p + "ffn_up_exps.weight")
                ly.down_exps = stacked(p + "ffn_down_exps.weight")
            else:
                g, u = mat(p + "ffn_gate.weight"), mat(p + "ffn_up.weight")
                ly.gate_up = cat(g, u)
                if ly.gate_up is None:
                    ly.gate, ly.up = g, u
                ly.down = mat(p + "ffn_down.weight")
            self.layers.append(ly)
        first.clear()
        self.n_stack_experts = spec.num_experts if self.moe else 0
        self._pair_expert_stacks()

        # activations and state
        q_dim, kv_dim = spec.q_dim, spec.kv_dim
        z = lambda *shape, dt=torch.float32: torch.zeros(*shape, dtype=dt, device=d)  # noqa: E731
        self.hidden, self.normed = z(h), z(h)
        self.qkv, self.attn = z(q_dim + 2 * kv_dim), z(q_dim)
        if self.moe:
            ff, E, k = spec.moe_intermediate_size, spec.num_experts, spec.num_experts_per_tok
            self.router_logits = z(E)
            self.route_ticket = z(1, dt=torch.int32)
            self.expert_ids, self.expert_w = z(k, dt=torch.int32), z(k)
            self.gate_up_out = z(2 * k, ff)  # [gate_j | up_j] of the selected experts
            self.gate, self.up = self.gate_up_out[:k], self.gate_up_out[k:]
            self.act, self.down = z(k, ff), z(k, h)
        else:
            ff, k = spec.intermediate_size, 1
            self.gu, self.act = z(2 * ff), z(ff)
        self.ff = ff
        self.logits = z(spec.vocab_size)
        self.kcache = z(spec.num_hidden_layers, max_ctx, kv_dim)
        self.vcache = torch.zeros_like(self.kcache)
        self.tokens, self.pos = z(max_ctx, dt=torch.int32), z(1, dt=torch.int32)
        self.argmax_scratch = z(int(L.pyrite_cuda_post_scratch_size()) + 256, dt=torch.uint8)
        self.ticket = z(1, dt=torch.int32)
        self.expert_shards, self.expert_shard = 1, 0  # experts by id over GPUs (sharded subclass)
        self.attn_scratch = z(int(L.pyrite_cuda_attention_scratch_size(spec.num_attention_heads, max_ctx)),
                              dt=torch.uint8)
        # the experts each layer routed to in the latest step (rank order)
        self.route_log = z(spec.num_hidden_layers, k, dt=torch.int32) if self.moe else None

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
    def synthetic(cls, spec: DenseSpec | MoESpec, device="cuda", max_ctx: int = 512,
                  replicate: bool = False) -> "MixedDecoder":
        """The seeded synthetic checkpoint of ``spec`` (pyrite_b200.synthetic);
        ``replicate`` generates layers 0 and 1 only (see the class)."""
        gen_spec = spec
        if replicate:
            from dataclasses import replace
            gen_spec = replace(spec, num_hidden_layers=min(2, spec.num_hidden_layers))
        gen = moe_tensors if isinstance(spec, MoESpec) else dense_tensors
        tensors = {name: (dims, t, payload) for name, dims, t, payload in gen(gen_spec)}
        return cls(spec, tensors, device=device, max_ctx=max_ctx, replicate=replicate)

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

    def _mvx(self, m: _Mat, x: torch.Tensor, x_op: int, norm: torch.Tensor | None, x_out: torch.Tensor, ws,
             y: torch.Tensor, flags: int, stream: int) -> None:
        """y (+)= W x' with x' = RMSNorm(x) or SiLU(gate) * up computed inside the matvec."""
        wptr, wlen = self._wsp(ws)
        code = self.lib.pyrite_cuda_matvec_transformed(
            m.ggml_type, m.data.data_ptr(), m.data.numel(), x.data_ptr(), x_op,
            norm.data_ptr() if norm is not None else None, float(self.spec.rms_norm_eps), x_out.data_ptr(), wptr,
            wlen, y.data_ptr(), m.rows, m.cols, flags | STATIC_WEIGHTS, stream)
        _check(code, "matvec+x")

    def _x_in_workspace(self, m: _Mat, x: torch.Tensor, x_op: int, norm: torch.Tensor | None,
                        x_out: torch.Tensor) -> bool:
        """Whether ``_mvx(m, x, ...)`` runs the operation's own kernel first, so
        that its workspace and ``x_out`` hold x' for further matrices."""
        form = self.lib.pyrite_cuda_matvec_transformed_form(
            m.ggml_type, m.data.data_ptr(), m.data.numel(), x.data_ptr(), x_op,
            norm.data_ptr() if norm is not None else None, x_out.data_ptr(), m.rows, m.cols)
        _check(min(form, 0), "matvec+x form")
        return form == 0

    def _mvx2(self, a: _Mat, b: _Mat, x: torch.Tensor, norm: torch.Tensor, ws, ya: torch.Tensor,
              yb: torch.Tensor, stream: int) -> None:
        """ya = A RMSNorm(x), yb = B RMSNorm(x): the norm runs once when the
        library computes it in a kernel of its own, else in both prologues."""
        X = _lib.X_RMSNORM
        self._mvx(a, x, X, norm, self.normed, ws, ya, 0, stream)
        if self._x_in_workspace(a, x, X, norm, self.normed):
            self._mv(b, self.normed, ws, yb, 0, stream)
        else:
            self._mvx(b, x, X, norm, self.normed, ws, yb, 0, stream)

    def _pair_expert_stacks(self) -> None:
        """Store ffn_gate_exps and ffn_up_exps back to back when they share a
        type and shape, so one launch multiplies both for every selected expert."""
        for ly in self.layers:
            g, u = ly.gate_exps, ly.up_exps
            if g is None or u is None or g.ggml_type != u.ggml_type or (g.rows, g.cols) != (u.rows, u.cols):
                continue
            ly.gate_up_exps = _Mat(g.ggml_type, torch.cat([g.data, u.data]), g.rows, g.cols)
            ly.gate_exps = ly.up_exps = None

    def _experts(self, m: _Mat, x: torch.Tensor, x_stride: int, ws, ws_stride: int, y: torch.Tensor,
                 stream: int, groups: int = 1) -> None:
        """y[j] = stack (j // k) expert ids[j % k] times activation j % k, for
        j < groups * k, in one launch."""
        wptr, wlen = self._wsp(ws)
        k = self.spec.num_experts_per_tok
        code = self.lib.pyrite_cuda_matvec_expert_groups(
            m.ggml_type, m.data.data_ptr(), m.data.numel(), self.n_stack_experts, groups, self.expert_ids.data_ptr(),
            k, x.data_ptr(), x_stride, wptr, wlen, ws_stride, y.data_ptr(), y.shape[-1], m.rows, m.cols, 0, stream)
        _check(code, "expert matvec")

    def _route(self, ly: _Layer, li: int, stream: int) -> None:
        """ffn RMSNorm of the residual (into ``normed`` and its encoding), router
        logits and top-k routing: one launch for an F32 router."""
        s, L = self.spec, self.lib
        k, norm = s.num_experts_per_tok, 1 if s.norm_topk_prob else 0
        if ly.router.ggml_type == F32:
            wptr, wlen = self._wsp(self.ws_h)
            _check(L.pyrite_cuda_moe_norm_router_route(
                F32, ly.router.data.data_ptr(), ly.router.data.numel(), ly.router.cols, self.hidden.data_ptr(),
                ly.ffn_norm.data_ptr(), float(s.rms_norm_eps), self.normed.data_ptr(), wptr, wlen,
                self.router_logits.data_ptr(), s.num_experts, k, norm, 1.0, self.expert_shards, self.expert_shard,
                self.expert_ids.data_ptr(), self.expert_w.data_ptr(), self.route_log[li].data_ptr(),
                self.route_ticket.data_ptr(), stream), "norm+router+route")
            return
        self._norm(self.hidden, ly.ffn_norm, self.normed, self.ws_h, stream)
        self._mv(ly.router, self.normed, self.ws_h, self.router_logits, 0, stream)
        _check(L.pyrite_cuda_moe_route(self.router_logits.data_ptr(), s.num_experts, k, norm, 1.0, self.expert_shards,
                                       self.expert_shard, self.expert_ids.data_ptr(), self.expert_w.data_ptr(),
                                       self.route_log[li].data_ptr(), stream), "route")

    def _down_combine(self, ly: _Layer, target: torch.Tensor, stream: int) -> None:
        """target += sum_j w_j down_j over the selected experts.  (The combine as
        a post op in the last CTA of the down projection was measured 12%
        slower per step than this separate 8-CTA kernel.)"""
        k = self.spec.num_experts_per_tok
        self._experts(ly.down_exps, self.act, self.ff, self.ws_act, self.ws_act[2], self.down, stream)
        _check(self.lib.pyrite_cuda_moe_combine(self.down.data_ptr(), self.expert_w.data_ptr(), k,
                                                self.spec.hidden_size, target.data_ptr(), stream), "combine")

    def _gate_up_experts(self, ly: _Layer, stream: int) -> None:
        if ly.gate_up_exps is not None:
            self._experts(ly.gate_up_exps, self.normed, 0, self.ws_h, 0, self.gate_up_out, stream, groups=2)
        else:
            self._experts(ly.gate_exps, self.normed, 0, self.ws_h, 0, self.gate, stream)
            self._experts(ly.up_exps, self.normed, 0, self.ws_h, 0, self.up, stream)

    def _norm(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, ws, stream: int) -> None:
        wptr, wlen = self._wsp(ws)
        _check(self.lib.pyrite_cuda_rmsnorm_encode(x.data_ptr(), w.data_ptr(), x.numel(), float(self.spec.rms_norm_eps),
                                                   out.data_ptr(), wptr, wlen, stream), "rmsnorm")

    # ------------------------------------------------------------------ one step
    def _step(self, stream: int) -> None:
        s, L = self.spec, self.lib
        h, ff = s.hidden_size, self.ff
        eps = float(s.rms_norm_eps)
        qk_rows = s.q_dim + s.kv_dim
        _check(L.pyrite_cuda_embed(self.embd.ggml_type, self.embd.data.data_ptr(), s.vocab_size, h,
                                   self.tokens.data_ptr(), self.pos.data_ptr(), self.hidden.data_ptr(), stream), "embed")
        for li, ly in enumerate(self.layers):
            self._mvx2(ly.qk, ly.v, self.hidden, ly.attn_norm, self.ws_h, self.qkv, self.qkv[qk_rows:], stream)
            wq, wql = self._wsp(self.ws_q)
            _check(L.pyrite_cuda_attention_step(
                self.qkv.data_ptr(), ly.q_norm.data_ptr() if ly.q_norm is not None else None,
                ly.k_norm.data_ptr() if ly.k_norm is not None else None, s.num_attention_heads,
                s.num_key_value_heads, s.head_dim, eps, self.pos.data_ptr(), self.rope.data_ptr(), self.max_ctx,
                self.kcache[li].data_ptr(), self.vcache[li].data_ptr(), self.attn.data_ptr(), wq, wql, self.attn_scratch.data_ptr(),
                self.attn_scratch.numel(), stream),
                "attention_step")
            self._mv(ly.o, self.attn, self.ws_q, self.hidden, ACCUMULATE, stream)
            if not self.moe:  # SwiGLU feed-forward, norm and SiLU in the projections' prologues
                if ly.gate_up is not None:
                    self._mvx(ly.gate_up, self.hidden, _lib.X_RMSNORM, ly.ffn_norm, self.normed, self.ws_h, self.gu, 0,
                              stream)
                else:
                    self._mvx2(ly.gate, ly.up, self.hidden, ly.ffn_norm, self.ws_h, self.gu[:ff], self.gu[ff:], stream)
                self._mvx(ly.down, self.gu, _lib.X_SILU_MUL, None, self.act, self.ws_act, self.hidden, ACCUMULATE,
                          stream)
                continue
            # routed feed-forward (the norm runs inside the routing launch)
            k = s.num_experts_per_tok
            self._route(ly, li, stream)
            self._gate_up_experts(ly, stream)
            wa, wal = self._wsp(self.ws_act)
            _check(L.pyrite_cuda_moe_silu_mul_encode(self.gate.data_ptr(), self.up.data_ptr(), ff, k,
                                                     self.act.data_ptr(), wa, wal, stream), "moe silu")
            self._down_combine(ly, self.hidden, stream)
        self._norm(self.hidden, self.out_norm, self.normed, self.ws_h, stream)
        post = _lib.PostOp()
        post.op = _lib.POST_ARGMAX
        post.ticket = self.ticket.data_ptr()
        post.scratch = self.argmax_scratch.data_ptr()
        post.scratch_len = self.argmax_scratch.numel()
        post.tokens, post.pos = self.tokens.data_ptr(), self.pos.data_ptr()
        post.prompt_len, post.max_ctx = self.prompt_len, self.max_ctx
        self._mv(self.lm_head, self.normed, self.ws_h, self.logits, 0, stream, post=post)

    # ------------------------------------------------------------------ batched prefill
    @property
    def batched_prefill(self) -> bool:
        """Whether :meth:`prefill` runs blocks of positions (dense checkpoints on
        one GPU) or the one-position step."""
        return not self.moe

    def _mm(self, m: _Mat, x: torch.Tensor, ldx: int, y: torch.Tensor, ldy: int, ncols: int, ws: torch.Tensor,
            flags: int, stream: int) -> None:
        """Y[j] (+)= W X[j] for ncols rows of X (row-major, ldx / ldy floats
        apart): the tensor-core product where the format has one."""
        off = (-ws.data_ptr()) % 256
        code = self.lib.pyrite_cuda_matvec(m.ggml_type, m.data.data_ptr(), m.data.numel(), x.data_ptr(), ldx,
                                           y.data_ptr(), ldy, m.rows, m.cols, ncols, flags | STATIC_WEIGHTS,
                                           ws.data_ptr() + off, ws.numel() - off, stream)
        _check(code, "multi-column matvec")

    def prefill(self, prompt: list[int], block: int = 64) -> None:
        """Reset to ``prompt`` and run positions 0 .. len(prompt) - 2 through
        the model in blocks of up to ``block`` positions, so that the next
        decode step (position len(prompt) - 1) yields the first new token.

        The reference runs the prompt one position per forward pass
        (executor.py:920-923); here every projection of a block is one
        multi-column product on the tensor cores (pyrite_cuda_matvec with
        ncols > 1), the glue runs per row (pyrite_cuda_*_rows) and attention is
        causal inside the block.  Each position gets the arithmetic of the
        one-token step up to fp32 summation order; the last layer's
        feed-forward is skipped (it feeds only the logits of prompt positions,
        which greedy decoding never reads).  Dense checkpoints; MoE
        checkpoints run their prompt through the one-token step."""
        self.reset(prompt)
        n = len(prompt) - 1
        if n <= 0:
            return
        if not self.batched_prefill:
            self.run_steps(n)
            return
        s, L, d = self.spec, self.lib, self.dev
        h, ff, q, kv = s.hidden_size, self.ff, s.q_dim, s.kv_dim
        B = max(1, min(block, n))
        z = lambda *shape: torch.empty(*shape, dtype=torch.float32, device=d)  # noqa: E731
        hid, nrm, qkv, qr, att = z(B, h), z(B, h), z(B, q + 2 * kv), z(B, q), z(B, q)
        gu, act = z(B, 2 * ff), z(B, ff)
        mats = [m for ly in self.layers for m in (ly.qk, ly.v, ly.o, ly.gate_up, ly.gate, ly.up, ly.down) if m is not None]
        need = max(int(L.pyrite_cuda_workspace_size(m.ggml_type, m.cols, c)) for m in mats for c in {1, B})
        ws = torch.empty(need + 256, dtype=torch.uint8, device=d)
        st = torch.cuda.current_stream(d).cuda_stream
        eps = float(s.rms_norm_eps)
        last = len(self.layers) - 1
        for p0 in range(0, n, B):
            c = min(B, n - p0)
            _check(L.pyrite_cuda_embed_rows(self.embd.ggml_type, self.embd.data.data_ptr(), s.vocab_size, h,
                                            self.tokens[p0:].data_ptr(), 1, None, c, hid.data_ptr(), h, st),
                   "embed rows")
            for li, ly in enumerate(self.layers):
                _check(L.pyrite_cuda_rmsnorm_rows(hid.data_ptr(), h, ly.attn_norm.data_ptr(), h, c, eps,
                                                  nrm.data_ptr(), h, st), "rmsnorm rows")
                self._mm(ly.qk, nrm, h, qkv, q + 2 * kv, c, ws, 0, st)
                self._mm(ly.v, nrm, h, qkv[:, q + kv:], q + 2 * kv, c, ws, 0, st)
                _check(L.pyrite_cuda_qk_rope_kv_rows(
                    qkv.data_ptr(), q + 2 * kv, ly.q_norm.data_ptr() if ly.q_norm is not None else None,
                    ly.k_norm.data_ptr() if ly.k_norm is not None else None, s.num_attention_heads,
                    s.num_key_value_heads, s.head_dim, eps, p0, None, 1, 0, c, self.rope.data_ptr(), self.max_ctx,
                    qr.data_ptr(), q, self.kcache[li].data_ptr(), self.vcache[li].data_ptr(), st), "qk rope kv rows")
                _check(L.pyrite_cuda_attention_rows(qr.data_ptr(), q, self.kcache[li].data_ptr(),
                                                    self.vcache[li].data_ptr(), 0, p0, None, 1, c,
                                                    s.num_attention_heads, s.num_key_value_heads, s.head_dim,
                                                    self.max_ctx, att.data_ptr(), q, st), "attention rows")
                self._mm(ly.o, att, q, hid, h, c, ws, ACCUMULATE, st)
                if li == last:
                    continue
                _check(L.pyrite_cuda_rmsnorm_rows(hid.data_ptr(), h, ly.ffn_norm.data_ptr(), h, c, eps,
                                                  nrm.data_ptr(), h, st), "rmsnorm rows")
                if ly.gate_up is not None:
                    self._mm(ly.gate_up, nrm, h, gu, 2 * ff, c, ws, 0, st)
                else:
                    self._mm(ly.gate, nrm, h, gu, 2 * ff, c, ws, 0, st)
                    self._mm(ly.up, nrm, h, gu[:, ff:], 2 * ff, c, ws, 0, st)
                _check(L.pyrite_cuda_silu_mul_rows(gu.data_ptr(), 2 * ff, ff, c, act.data_ptr(), ff, st), "silu rows")
                self._mm(ly.down, act, ff, hid, h, c, ws, ACCUMULATE, st)
        self.pos.fill_(n)
        torch.cuda.synchronize(d)
        del hid, nrm, qkv, qr, att, gu, act, ws

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

    def generate(self, prompt: list[int], max_new_tokens: int, prefill_block: int = 0) -> list[int]:
        """Greedy continuation, the reference's ``generate(..., temperature=0)``.
        ``prefill_block`` > 0: the prompt in blocks of that many positions
        (:meth:`prefill`); 0: one position per step, as the reference."""
        if len(prompt) + max_new_tokens > self.max_ctx:
            raise ValueError("prompt + new tokens exceed the KV cache")
        if max_new_tokens == 0:
            return list(prompt)
        if self.graph is None or self.prompt_len != len(prompt):
            self.reset(prompt)
            self.capture()
        if prefill_block > 0:
            self.prefill(prompt, prefill_block)
            self.run_steps(max_new_tokens)
        else:
            self.reset(prompt)
            self.run_steps(len(prompt) + max_new_tokens - 1)
        torch.cuda.synchronize(self.dev)
        self.check_status()
        return [int(t) for t in self.tokens[: len(prompt) + max_new_tokens].cpu()]

    def check_status(self) -> None:
        """Raise if a kernel of the steps run so far gave up a bounded wait (a
        copy that never landed, or, across GPUs, a peer of the NVLink sum that
        never arrived: its partials were then not added and the ranks' tokens
        are no longer valid).  Reads and clears the device status word; call
        after a synchronize."""
        code = int(self.lib.pyrite_cuda_status(1))
        if code != 0:
            raise RuntimeError(f"decode step failed on the device (status word {code:#x}): a bounded wait timed out "
                               "or an expert id was out of range; the generated tokens are not valid")
