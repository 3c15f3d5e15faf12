"""Device-resident batch-1 decode of dense ``qwen3`` / ``llama`` checkpoints.

The B200 counterpart of the reference's dense executor
(``pyrite/dense.py:440-513`` on top of ``pyrite/executor.py:621-939``): the
same forward pass -- embedding lookup, per layer RMSNorm, Q/K/V projections,
per-head QK RMSNorm, NEOX RoPE, fp32 KV cache, grouped-query attention, output
projection, residual, RMSNorm, SwiGLU MLP, residual; final RMSNorm, LM head
over the (tied) embedding matrix, greedy sampling -- with every weight
resident in HBM and every projection a fused dequantize x matvec from
libpyrite_b200.so.

B200 layout choices:
  * Q, K and V rows are stored back to back as one matrix (they share their
    input), gate and up likewise: two fewer launches per layer, one activation
    encoding each.
  * The residual adds are fused into the output and down projections
    (``y += W x``).
  * The token id and the position live in device memory: one step is a fixed
    sequence of launches, captured once in a CUDA graph and replayed for the
    whole prompt (processed one token at a time, as the reference does) and
    every generated token, with no host synchronisation in between.
  * Fused step (default): the RMSNorm before a projection and the SwiGLU
    before the down projection go through ``pyrite_cuda_matvec_transformed``,
    which computes them in the projection's own prologue (every CTA encodes
    its copy of the activation in shared memory) where that is faster than a
    kernel of their own (norms over 4096 values and more); q/k norm, RoPE, KV
    append, attention and the encoding of its output run as one kernel; the
    greedy argmax runs in the last CTA of the LM-head matvec (a post op).
    (The norms as post ops in the last CTA of their producer were measured
    slower than their own kernels: one CTA serialises the work.)
    ``fused=False`` keeps one launch per operation (same results up to fp32
    rounding).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .ggml_types import spec as ggml_spec
from .kernels.cuda import STATIC_WEIGHTS, _check
from .synthetic import DenseSpec, dense_tensors

ACCUMULATE = 2  # PYRITE_F_ACCUMULATE


def _aligned(nbytes: int, device) -> tuple[torch.Tensor, int]:
    buf = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
    return buf, (-buf.data_ptr()) % 256


@dataclass
class _Layer:
    attn_norm: torch.Tensor
    ffn_norm: torch.Tensor
    q_norm: torch.Tensor | None
    k_norm: torch.Tensor | None
    qkv: torch.Tensor      # [q | k | v] rows, GGML bytes
    o: torch.Tensor
    gate_up: torch.Tensor  # [gate | up] rows
    down: torch.Tensor


class DenseDecoder:
    """One sequence, batch 1, weights in HBM; greedy decoding."""

    def __init__(self, spec: DenseSpec, tensors: dict[str, tuple[tuple[int, ...], int, bytes]],
                 device: torch.device | str = "cuda", max_ctx: int = 512, fused: bool = True):
        self.spec = spec
        self.dev = torch.device(device)
        self.max_ctx = max_ctx
        self.fused = fused
        self.lib = _lib.require()
        h, f = spec.hidden_size, spec.intermediate_size
        self.wtype = spec.weight_type

        def upload(name: str) -> torch.Tensor:
            dims, t, payload = tensors[name]
            if t != self.wtype and t != 0:
                raise ValueError(f"{name}: mixed weight types are not supported yet")
            return torch.frombuffer(bytearray(payload), dtype=torch.uint8).to(self.dev)

        def f32(name: str) -> torch.Tensor:
            dims, t, payload = tensors[name]
            if t != 0:
                raise ValueError(f"{name} must be F32")
            return torch.frombuffer(bytearray(payload), dtype=torch.float32).to(self.dev)

        def cat(*names: str) -> torch.Tensor:
            return torch.cat([upload(n) for n in names])

        self.embd = upload("token_embd.weight")
        self.lm_head = self.embd if spec.tied_embeddings else upload("output.weight")
        self.out_norm = f32("output_norm.weight")
        self.layers: list[_Layer] = []
        for i in range(spec.num_hidden_layers):
            p = f"blk.{i}."
            self.layers.append(_Layer(
                attn_norm=f32(p + "attn_norm.weight"), ffn_norm=f32(p + "ffn_norm.weight"),
                q_norm=f32(p + "attn_q_norm.weight") if spec.qk_norm else None,
                k_norm=f32(p + "attn_k_norm.weight") if spec.qk_norm else None,
                qkv=cat(p + "attn_q.weight", p + "attn_k.weight", p + "attn_v.weight"),
                o=upload(p + "attn_output.weight"),
                gate_up=cat(p + "ffn_gate.weight", p + "ffn_up.weight"),
                down=upload(p + "ffn_down.weight")))

        # activations and state
        d = self.dev
        qkv_rows = spec.q_dim + 2 * spec.kv_dim
        self.hidden = torch.zeros(h, dtype=torch.float32, device=d)
        self.normed = torch.zeros(h, dtype=torch.float32, device=d)
        self.qkv = torch.zeros(qkv_rows, dtype=torch.float32, device=d)
        self.q = torch.zeros(spec.q_dim, dtype=torch.float32, device=d)
        self.attn = torch.zeros(spec.q_dim, dtype=torch.float32, device=d)
        self.gu = torch.zeros(2 * f, dtype=torch.float32, device=d)
        self.act = torch.zeros(f, dtype=torch.float32, device=d)
        self.logits = torch.zeros(spec.vocab_size, dtype=torch.float32, device=d)
        self.kcache = torch.zeros(spec.num_hidden_layers, max_ctx, spec.kv_dim, dtype=torch.float32, device=d)
        self.vcache = torch.zeros_like(self.kcache)
        self.tokens = torch.zeros(max_ctx, dtype=torch.int32, device=d)
        self.pos = torch.zeros(1, dtype=torch.int32, device=d)
        self.argmax_scratch = torch.zeros(max(2048, int(self.lib.pyrite_cuda_post_scratch_size())),
                                          dtype=torch.uint8, device=d)
        self.attn_scratch = torch.zeros(int(self.lib.pyrite_cuda_attention_scratch_size(spec.num_attention_heads,
                                                                                           max_ctx)),
                                        dtype=torch.uint8, device=d)
        # one ticket counter per fused call site (three per layer + the LM head)
        self.tickets = torch.zeros(3 * spec.num_hidden_layers + 1, dtype=torch.int32, device=d)
        ws = lambda n: _aligned(int(self.lib.pyrite_cuda_workspace_size(0, n, 1)), d)  # noqa: E731
        self.ws_h, self.ws_h_off = ws(h)
        self.ws_q, self.ws_q_off = ws(spec.q_dim)
        self.ws_f, self.ws_f_off = ws(f)
        # NEOX RoPE table, fp64 like the reference: angle = pos * theta^(-2i/n_rot)
        half = spec.head_dim // 2
        inv = spec.rope_theta ** (-2.0 * np.arange(half, dtype=np.float64) / spec.head_dim)
        ang = np.arange(max_ctx, dtype=np.float64)[:, None] * inv[None, :]
        table = np.stack([np.cos(ang), np.sin(ang)], axis=-1).astype(np.float64)
        self.rope = torch.from_numpy(np.ascontiguousarray(table)).to(d)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.prompt_len = 0

    @classmethod
    def synthetic(cls, spec: DenseSpec, device="cuda", max_ctx: int = 512, fused: bool = True) -> "DenseDecoder":
        tensors = {name: (dims, t, payload) for name, dims, t, payload in dense_tensors(spec)}
        return cls(spec, tensors, device=device, max_ctx=max_ctx, fused=fused)

    # ------------------------------------------------------------------ one step
    def _ws(self, which: str) -> tuple[int, int]:
        buf, off = {"h": (self.ws_h, self.ws_h_off), "q": (self.ws_q, self.ws_q_off),
                    "f": (self.ws_f, self.ws_f_off)}[which]
        return buf.data_ptr() + off, buf.numel() - off

    def _matvec(self, w: torch.Tensor, x: torch.Tensor, ws: str, y: torch.Tensor, rows: int, cols: int,
                flags: int, stream: int) -> None:
        wptr, wlen = self._ws(ws)
        code = self.lib.pyrite_cuda_matvec_prepared(self.wtype, w.data_ptr(), w.numel(), x.data_ptr(), wptr, wlen,
                                                    y.data_ptr(), rows, cols, flags | STATIC_WEIGHTS, stream)
        _check(code, "matvec")

    def _post(self, op: int, ticket: int, *, weight=None, out=None, ws: str | None = None) -> _lib.PostOp:
        p = _lib.PostOp()
        p.op = op
        p.eps = float(self.spec.rms_norm_eps)
        p.weight = weight.data_ptr() if weight is not None else None
        p.out = out.data_ptr() if out is not None else None
        if ws is not None:
            p.workspace, p.workspace_len = self._ws(ws)
        p.ticket = self.tickets.data_ptr() + 4 * ticket
        p.scratch = self.argmax_scratch.data_ptr()
        p.scratch_len = self.argmax_scratch.numel()
        p.tokens = self.tokens.data_ptr()
        p.pos = self.pos.data_ptr()
        p.prompt_len = self.prompt_len
        p.max_ctx = self.max_ctx
        return p

    def _matvec_post(self, w: torch.Tensor, x: torch.Tensor, ws: str, y: torch.Tensor, rows: int, cols: int,
                     flags: int, post: _lib.PostOp, stream: int) -> None:
        wptr, wlen = self._ws(ws)
        code = self.lib.pyrite_cuda_matvec_prepared_post(self.wtype, w.data_ptr(), w.numel(), x.data_ptr(), wptr, wlen,
                                                         y.data_ptr(), rows, cols, flags | STATIC_WEIGHTS,
                                                         ctypes.byref(post), stream)
        _check(code, "matvec+post")

    def _matvec_x(self, w: torch.Tensor, x: torch.Tensor, x_op: int, norm: torch.Tensor | None, ws: str,
                  x_out: torch.Tensor, y: torch.Tensor, rows: int, cols: int, flags: int, stream: int) -> None:
        """y (+)= W x' with x' = RMSNorm(x) or SiLU(gate) * up computed inside the matvec."""
        wptr, wlen = self._ws(ws)
        code = self.lib.pyrite_cuda_matvec_transformed(
            self.wtype, w.data_ptr(), w.numel(), x.data_ptr(), x_op, norm.data_ptr() if norm is not None else None,
            float(self.spec.rms_norm_eps), x_out.data_ptr(), wptr, wlen, y.data_ptr(), rows, cols,
            flags | STATIC_WEIGHTS, stream)
        _check(code, "matvec+x")

    def _step_fused(self, stream: int) -> None:
        s, L = self.spec, self.lib
        h, f = s.hidden_size, s.intermediate_size
        eps = float(s.rms_norm_eps)
        nl = len(self.layers)
        _check(L.pyrite_cuda_embed(self.wtype, self.embd.data_ptr(), s.vocab_size, h, self.tokens.data_ptr(),
                                   self.pos.data_ptr(), self.hidden.data_ptr(), stream), "embed")
        for li, ly in enumerate(self.layers):
            self._matvec_x(ly.qkv, self.hidden, _lib.X_RMSNORM, ly.attn_norm, "h", self.normed, self.qkv,
                           s.q_dim + 2 * s.kv_dim, h, 0, stream)
            wq, wql = self._ws("q")
            _check(L.pyrite_cuda_attention_step(
                self.qkv.data_ptr(), ly.q_norm.data_ptr() if ly.q_norm is not None else None,
                ly.k_norm.data_ptr() if ly.k_norm is not None else None, s.num_attention_heads,
                s.num_key_value_heads, s.head_dim, eps, self.pos.data_ptr(), self.rope.data_ptr(), self.max_ctx,
                self.kcache[li].data_ptr(), self.vcache[li].data_ptr(), self.attn.data_ptr(), wq, wql,
                self.attn_scratch.data_ptr(), self.attn_scratch.numel(), stream), "attention_step")
            self._matvec(ly.o, self.attn, "q", self.hidden, h, s.q_dim, ACCUMULATE, stream)
            self._matvec_x(ly.gate_up, self.hidden, _lib.X_RMSNORM, ly.ffn_norm, "h", self.normed, self.gu,
                           2 * f, h, 0, stream)
            self._matvec_x(ly.down, self.gu, _lib.X_SILU_MUL, None, "f", self.act, self.hidden, h, f, ACCUMULATE,
                           stream)
        wh, whl = self._ws("h")
        _check(L.pyrite_cuda_rmsnorm_encode(self.hidden.data_ptr(), self.out_norm.data_ptr(), h, eps,
                                            self.normed.data_ptr(), wh, whl, stream), "rmsnorm")
        self._matvec_post(self.lm_head, self.normed, "h", self.logits, s.vocab_size, h, 0,
                          self._post(_lib.POST_ARGMAX, 3 * nl), stream)

    def _step(self, stream: int) -> None:
        if self.fused:
            self._step_fused(stream)
            return
        s, L = self.spec, self.lib
        h, f = s.hidden_size, s.intermediate_size
        eps = float(s.rms_norm_eps)
        _check(L.pyrite_cuda_embed(self.wtype, self.embd.data_ptr(), s.vocab_size, h, self.tokens.data_ptr(),
                                   self.pos.data_ptr(), self.hidden.data_ptr(), stream), "embed")
        for li, ly in enumerate(self.layers):
            wh, whl = self._ws("h")
            _check(L.pyrite_cuda_rmsnorm_encode(self.hidden.data_ptr(), ly.attn_norm.data_ptr(), h, eps,
                                                self.normed.data_ptr(), wh, whl, stream), "rmsnorm")
            self._matvec(ly.qkv, self.normed, "h", self.qkv, s.q_dim + 2 * s.kv_dim, h, 0, stream)
            kc, vc = self.kcache[li], self.vcache[li]
            _check(L.pyrite_cuda_qk_rope_kv(
                self.qkv.data_ptr(), ly.q_norm.data_ptr() if ly.q_norm is not None else None,
                ly.k_norm.data_ptr() if ly.k_norm is not None else None, s.num_attention_heads,
                s.num_key_value_heads, s.head_dim, eps, self.pos.data_ptr(), self.rope.data_ptr(), self.max_ctx,
                self.q.data_ptr(), kc.data_ptr(), vc.data_ptr(), stream), "qk_rope_kv")
            _check(L.pyrite_cuda_attention(self.q.data_ptr(), kc.data_ptr(), vc.data_ptr(), self.pos.data_ptr(),
                                           s.num_attention_heads, s.num_key_value_heads, s.head_dim, self.max_ctx,
                                           self.attn.data_ptr(), stream), "attention")
            wq, wql = self._ws("q")
            _check(L.pyrite_cuda_prepare_x(self.attn.data_ptr(), s.q_dim, s.q_dim, 1, wq, wql, stream), "prepare")
            self._matvec(ly.o, self.attn, "q", self.hidden, h, s.q_dim, ACCUMULATE, stream)
            _check(L.pyrite_cuda_rmsnorm_encode(self.hidden.data_ptr(), ly.ffn_norm.data_ptr(), h, eps,
                                                self.normed.data_ptr(), wh, whl, stream), "rmsnorm")
            self._matvec(ly.gate_up, self.normed, "h", self.gu, 2 * f, h, 0, stream)
            wf, wfl = self._ws("f")
            _check(L.pyrite_cuda_silu_mul_encode(self.gu.data_ptr(), f, self.act.data_ptr(), wf, wfl, stream), "silu")
            self._matvec(ly.down, self.act, "f", self.hidden, h, f, ACCUMULATE, stream)
        wh, whl = self._ws("h")
        _check(L.pyrite_cuda_rmsnorm_encode(self.hidden.data_ptr(), self.out_norm.data_ptr(), h, eps,
                                            self.normed.data_ptr(), wh, whl, stream), "rmsnorm")
        self._matvec(self.lm_head, self.normed, "h", self.logits, s.vocab_size, h, 0, stream)
        _check(L.pyrite_cuda_argmax_step(self.logits.data_ptr(), s.vocab_size, self.argmax_scratch.data_ptr(),
                                         self.argmax_scratch.numel(), self.tokens.data_ptr(), self.pos.data_ptr(),
                                         self.prompt_len, self.max_ctx, stream), "argmax")

    # ------------------------------------------------------------------ public
    def reset(self, prompt: list[int]) -> None:
        if not prompt or any(not 0 <= t < self.spec.vocab_size for t in prompt):
            raise ValueError("prompt token ids must be non-empty and inside the vocabulary")
        if len(prompt) >= self.max_ctx:
            raise ValueError("prompt does not fit the KV cache")
        if self.graph is not None and len(prompt) != self.prompt_len:
            self.graph = None  # the prompt length is a launch argument
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
            self._step(stream.cuda_stream)      # warm: sets kernel attributes before capture
            torch.cuda.synchronize(self.dev)
            self.pos.copy_(saved)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                self._step(stream.cuda_stream)
        torch.cuda.synchronize(self.dev)
        self.pos.copy_(saved)
        self.graph = g

    def run_steps(self, n: int) -> None:
        """Replay ``n`` decode steps (enqueued on the current stream)."""
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
            self.capture()  # its warm-up step dirties the state; reset again below
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
