"""Several sequences decoded together (multi-sequence decode, e.g. batch 16).

The reference decodes one sequence per ``generate`` call
(pyrite/executor.py:878-939); serving 16 prompts means 16 independent runs.
:class:`BatchDecoder` advances ``batch`` sequences of equal prompt length by
one position per step, all in one CUDA graph:

* the weights are read once per step for all sequences: every projection
  (Q|K, V, O, the dense feed-forward, the LM head) is one multi-column product
  over the sequences' rows (tensor cores where the format has them);
* each sequence has its own KV cache; QK-norm / RoPE / KV append and the
  attention run per row at the shared position (pyrite_cuda_*_rows with
  pos_step 0 and a per-row cache stride);
* routed experts (qwen3moe): the router is one multi-column product, the
  top-k routing one launch over the rows (pyrite_cuda_moe_route_rows, the
  reference's softmax / (-p, e) order / renormalisation, executor.py:757-772),
  the gate|up products of every (sequence, selected expert) pair one launch
  (pyrite_cuda_matvec_expert_rows: each selection reads its sequence's
  encoded activation), SiLU * up and the down products likewise, and the
  weighted combine per row in rank order (executor.py:786-792);
* greedy argmax per row (sampler.py:12-15) into each sequence's tokens.

Each sequence gets the arithmetic of the one-sequence decoder
(:class:`pyrite_b200.model.MixedDecoder`) up to the products' summation
order (multi-column products instead of batch-1 kernels), so the oracle is
one :meth:`MixedDecoder.generate` per prompt -- which itself matches the
reference executor's greedy ids.
"""
from __future__ import annotations

import torch

from . import _lib
from .kernels.cuda import STATIC_WEIGHTS, _check
from .model import ACCUMULATE, MixedDecoder, _Mat


class BatchDecoder(MixedDecoder):
    """``batch`` sequences of one checkpoint, decoded greedily together."""

    def __init__(self, spec, tensors, device="cuda", max_ctx: int = 512, batch: int = 16, replicate: bool = False):
        super().__init__(spec, tensors, device=device, max_ctx=max_ctx, replicate=replicate)
        if not 1 <= batch <= 128:
            raise ValueError("batch must be 1..128")
        s, L, d = self.spec, self.lib, self.dev
        self.batch = B = batch
        h, q, kv, V = s.hidden_size, s.q_dim, s.kv_dim, s.vocab_size
        z = lambda *shape, dt=torch.float32: torch.zeros(*shape, dtype=dt, device=d)  # noqa: E731
        self.btokens, self.bpos = z(B, max_ctx, dt=torch.int32), z(1, dt=torch.int32)
        self.bk = z(s.num_hidden_layers, B, max_ctx, kv)
        self.bv = torch.zeros_like(self.bk)
        self.bhid, self.bnrm = z(B, h), z(B, h)
        self.bqkv, self.bq, self.batt = z(B, q + 2 * kv), z(B, q), z(B, q)
        self.blogits = z(B, V)
        mats = [self.lm_head] + [m for ly in self.layers for m in (ly.qk, ly.v, ly.o, ly.gate_up, ly.gate, ly.up,
                                                                    ly.down, ly.router) if m is not None]
        need = max(int(L.pyrite_cuda_workspace_size(m.ggml_type, m.cols, c)) for m in mats for c in {1, B})
        if self.moe:
            k, ff, E = s.num_experts_per_tok, self.ff, s.num_experts
            self.brlog = z(B, E)
            self.bids, self.bw = z(B * k, dt=torch.int32), z(B * k)
            self.bgu = z(2 * B * k, ff)  # [gate rows | up rows] of the B k selections
            self.bact, self.bdown = z(B * k, ff), z(B * k, h)
            self.per_h = int(L.pyrite_cuda_workspace_size(0, h, 1))
            self.per_ff = int(L.pyrite_cuda_workspace_size(0, ff, 1))
            self.bws_h = torch.empty(self.per_h * B + 256, dtype=torch.uint8, device=d)
            self.bws_act = torch.empty(self.per_ff * B * k + 256, dtype=torch.uint8, device=d)
        else:
            self.bgu, self.bact = z(B, 2 * self.ff), z(B, self.ff)
        self.bws = torch.empty(need + 256, dtype=torch.uint8, device=d)
        self.bgraph: torch.cuda.CUDAGraph | None = None
        self.bprompt_len = 0

    @classmethod
    def synthetic(cls, spec, device="cuda", max_ctx: int = 512, batch: int = 16,
                  replicate: bool = False) -> "BatchDecoder":
        """The seeded synthetic checkpoint of ``spec``; ``replicate``: layers 0
        and 1 generated, deeper layers their own device copies of those bytes."""
        from dataclasses import replace

        from .synthetic import MoESpec, dense_tensors, moe_tensors
        gen_spec = replace(spec, num_hidden_layers=min(2, spec.num_hidden_layers)) if replicate else spec
        gen = moe_tensors if isinstance(spec, MoESpec) else dense_tensors
        tensors = {name: (dims, t, payload) for name, dims, t, payload in gen(gen_spec)}
        return cls(spec, tensors, device=device, max_ctx=max_ctx, batch=batch, replicate=replicate)

    @staticmethod
    def _aligned(buf: torch.Tensor) -> tuple[int, int]:
        off = (-buf.data_ptr()) % 256
        return buf.data_ptr() + off, buf.numel() - off

    def _bmm(self, m: _Mat, x: torch.Tensor, ldx: int, y: torch.Tensor, ldy: int, flags: int, stream: int) -> None:
        wp, wl = self._aligned(self.bws)
        _check(self.lib.pyrite_cuda_matvec(m.ggml_type, m.data.data_ptr(), m.data.numel(), x.data_ptr(), ldx,
                                           y.data_ptr(), ldy, m.rows, m.cols, self.batch, flags | STATIC_WEIGHTS, wp,
                                           wl, stream), "multi-column matvec")

    # ------------------------------------------------------------------ one step of every sequence
    def _bstep(self, st: int) -> None:
        s, L, B = self.spec, self.lib, self.batch
        h, q, kv, ff, mc = s.hidden_size, s.q_dim, s.kv_dim, self.ff, self.max_ctx
        eps = float(s.rms_norm_eps)
        pos = self.bpos.data_ptr()
        _check(L.pyrite_cuda_embed_rows(self.embd.ggml_type, self.embd.data.data_ptr(), s.vocab_size, h,
                                        self.btokens.data_ptr(), mc, pos, B, self.bhid.data_ptr(), h, st), "embed rows")
        for li, ly in enumerate(self.layers):
            _check(L.pyrite_cuda_rmsnorm_rows(self.bhid.data_ptr(), h, ly.attn_norm.data_ptr(), h, B, eps,
                                              self.bnrm.data_ptr(), h, st), "rmsnorm rows")
            self._bmm(ly.qk, self.bnrm, h, self.bqkv, q + 2 * kv, 0, st)
            self._bmm(ly.v, self.bnrm, h, self.bqkv[:, q + kv:], q + 2 * kv, 0, st)
            _check(L.pyrite_cuda_qk_rope_kv_rows(
                self.bqkv.data_ptr(), q + 2 * kv, ly.q_norm.data_ptr() if ly.q_norm is not None else None,
                ly.k_norm.data_ptr() if ly.k_norm is not None else None, s.num_attention_heads,
                s.num_key_value_heads, s.head_dim, eps, 0, pos, 0, mc * kv, B, self.rope.data_ptr(), mc,
                self.bq.data_ptr(), q, self.bk[li].data_ptr(), self.bv[li].data_ptr(), st), "qk rope kv rows")
            _check(L.pyrite_cuda_attention_rows(self.bq.data_ptr(), q, self.bk[li].data_ptr(), self.bv[li].data_ptr(),
                                                mc * kv, 0, pos, 0, B, s.num_attention_heads, s.num_key_value_heads,
                                                s.head_dim, mc, self.batt.data_ptr(), q, st), "attention rows")
            self._bmm(ly.o, self.batt, q, self.bhid, h, ACCUMULATE, st)
            _check(L.pyrite_cuda_rmsnorm_rows(self.bhid.data_ptr(), h, ly.ffn_norm.data_ptr(), h, B, eps,
                                              self.bnrm.data_ptr(), h, st), "rmsnorm rows")
            if not self.moe:
                if ly.gate_up is not None:
                    self._bmm(ly.gate_up, self.bnrm, h, self.bgu, 2 * ff, 0, st)
                else:
                    self._bmm(ly.gate, self.bnrm, h, self.bgu, 2 * ff, 0, st)
                    self._bmm(ly.up, self.bnrm, h, self.bgu[:, ff:], 2 * ff, 0, st)
                _check(L.pyrite_cuda_silu_mul_rows(self.bgu.data_ptr(), 2 * ff, ff, B, self.bact.data_ptr(), ff, st),
                       "silu rows")
                self._bmm(ly.down, self.bact, ff, self.bhid, h, ACCUMULATE, st)
                continue
            self._moe_rows(ly, st)
        _check(L.pyrite_cuda_rmsnorm_rows(self.bhid.data_ptr(), h, self.out_norm.data_ptr(), h, B, eps,
                                          self.bnrm.data_ptr(), h, st), "rmsnorm rows")
        self._bmm(self.lm_head, self.bnrm, h, self.blogits, s.vocab_size, 0, st)
        _check(L.pyrite_cuda_argmax_rows(self.blogits.data_ptr(), s.vocab_size, s.vocab_size, B,
                                         self.btokens.data_ptr(), mc, pos, self.bprompt_len, mc, st), "argmax rows")
        _check(L.pyrite_cuda_advance_pos(pos, st), "advance")

    def _moe_rows(self, ly, st: int) -> None:
        """The routed feed-forward of every sequence (the normed rows in bnrm)."""
        s, L, B = self.spec, self.lib, self.batch
        h, ff, k, E = s.hidden_size, self.ff, s.num_experts_per_tok, s.num_experts
        r = ly.router
        if r.ggml_type == 0:  # F32: fp64 accumulation, as the one-sequence routing launch
            _check(L.pyrite_cuda_moe_router_rows(0, r.data.data_ptr(), r.data.numel(), h, self.bnrm.data_ptr(), h, B,
                                                 self.brlog.data_ptr(), E, E, st), "router rows")
        else:
            self._bmm(r, self.bnrm, h, self.brlog, E, 0, st)
        _check(L.pyrite_cuda_moe_route_rows(self.brlog.data_ptr(), E, B, E, k, 1 if s.norm_topk_prob else 0, 1.0,
                                            self.bids.data_ptr(), self.bw.data_ptr(), st), "route rows")
        wh, whl = self._aligned(self.bws_h)
        _check(L.pyrite_cuda_prepare_x(self.bnrm.data_ptr(), h, h, B, wh, whl, st), "prepare x rows")

        def experts(m: _Mat, groups: int, y: torch.Tensor) -> None:
            _check(L.pyrite_cuda_matvec_expert_rows(
                m.ggml_type, m.data.data_ptr(), m.data.numel(), self.n_stack_experts, groups, self.bids.data_ptr(), B,
                k, self.bnrm.data_ptr(), h, wh, whl, self.per_h, y.data_ptr(), ff, m.rows, m.cols, 0, st),
                "expert rows")

        if ly.gate_up_exps is not None:
            experts(ly.gate_up_exps, 2, self.bgu)
        else:
            experts(ly.gate_exps, 1, self.bgu[: B * k])
            experts(ly.up_exps, 1, self.bgu[B * k:])
        wa, wal = self._aligned(self.bws_act)
        _check(L.pyrite_cuda_moe_silu_mul_encode(self.bgu[: B * k].data_ptr(), self.bgu[B * k:].data_ptr(), ff, B * k,
                                                 self.bact.data_ptr(), wa, wal, st), "moe silu rows")
        dn = ly.down_exps
        _check(L.pyrite_cuda_matvec_expert_groups(dn.ggml_type, dn.data.data_ptr(), dn.data.numel(),
                                                  self.n_stack_experts, 1, self.bids.data_ptr(), B * k,
                                                  self.bact.data_ptr(), ff, wa, wal, self.per_ff,
                                                  self.bdown.data_ptr(), h, dn.rows, dn.cols, 0, st), "expert down")
        _check(L.pyrite_cuda_moe_combine_rows(self.bdown.data_ptr(), self.bw.data_ptr(), k, h, B, self.bhid.data_ptr(),
                                              h, st), "combine rows")

    # ------------------------------------------------------------------ public
    def breset(self, prompts: list[list[int]]) -> None:
        """``batch`` prompts of equal length; caches and positions cleared."""
        if len(prompts) != self.batch:
            raise ValueError(f"{self.batch} prompts expected, got {len(prompts)}")
        n = len(prompts[0])
        if n == 0 or n >= self.max_ctx or any(len(p) != n for p in prompts):
            raise ValueError("prompts must be non-empty, of equal length and fit the KV cache")
        if any(not 0 <= t < self.spec.vocab_size for p in prompts for t in p):
            raise ValueError("prompt token ids must lie inside the vocabulary")
        if self.bgraph is not None and n != self.bprompt_len:
            self.bgraph = None
        self.bprompt_len = n
        self.btokens.zero_()
        self.btokens[:, :n] = torch.tensor(prompts, dtype=torch.int32, device=self.dev)
        self.bpos.zero_()
        self.bk.zero_()
        self.bv.zero_()

    def bcapture(self) -> None:
        stream = torch.cuda.Stream(device=self.dev)
        saved = self.bpos.clone()
        with torch.cuda.stream(stream):
            self._bstep(stream.cuda_stream)  # warm: kernel attributes are set before capture
            torch.cuda.synchronize(self.dev)
            self.bpos.copy_(saved)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                self._bstep(stream.cuda_stream)
        torch.cuda.synchronize(self.dev)
        self.bpos.copy_(saved)
        self.bgraph = g

    def brun_steps(self, n: int) -> None:
        if self.bgraph is None:
            self.bcapture()
        for _ in range(n):
            self.bgraph.replay()

    def bgenerate(self, prompts: list[list[int]], max_new_tokens: int) -> list[list[int]]:
        """Greedy continuations of all prompts (each as ``generate(..., temperature=0)``)."""
        n = len(prompts[0]) if prompts else 0
        if n + max_new_tokens > self.max_ctx:
            raise ValueError("prompt + new tokens exceed the KV cache")
        if self.bgraph is None or self.bprompt_len != n:
            self.breset(prompts)
            self.bcapture()
        self.breset(prompts)
        self.brun_steps(n + max_new_tokens - 1)
        torch.cuda.synchronize(self.dev)
        self.check_status()
        return [[int(t) for t in row] for row in self.btokens[:, : n + max_new_tokens].cpu()]
