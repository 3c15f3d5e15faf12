"""Tensor-parallel batch-1 decode across the GPUs of one box (NVLink).

One process per GPU (``torchrun``); rank g holds the shard of every tensor that
:mod:`pyrite_b200.shard` assigns it and runs the same decode step as
:class:`pyrite_b200.model.MixedDecoder` on its shard, with two collectives
per layer, both inside the step's CUDA graph:

* after the attention output projection (rank g multiplied its heads' columns):
  ``allreduce`` of the partial residual update (hidden size floats);
* after the feed-forward down projection (its rows of gate/up, its columns of
  down; or, for MoE, the selected experts it owns): the same ``allreduce``;

each one kernel (``pyrite_cuda_allreduce_sum``: every rank publishes its
partial in a buffer the others map by CUDA IPC, raises a flag in every peer's
buffer and sums all partials over NVLink in rank order; ``p2p=False`` uses
NCCL instead), and for the greedy token one NCCL ``all_gather`` of 8 bytes per
GPU: each rank's best (logit, id) over its slice of the vocabulary (the LM
head's rows are sharded by vocabulary), from which every rank picks the same
token (the largest logit, the lowest id on ties).  Norms, the
embedding lookup and the router are replicated.  Sums across GPUs change the
fp32 summation order only; greedy ids are checked against the reference's.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .kernels.cuda import _check
from .model import _Layer, _Mat, MixedDecoder
from .shard import even_range, head_shard, owned_experts, row_bytes, slice_cols, slice_rows
from .synthetic import F32, DenseSpec, MoESpec, dense_tensors, moe_tensors


class ShardedDecoder(MixedDecoder):
    """``MixedDecoder`` split over ``world`` GPUs (this process: ``rank``)."""

    def __init__(self, spec: DenseSpec | MoESpec, tensors: dict[str, tuple[tuple[int, ...], int, bytes]],
                 rank: int, world: int, device: torch.device | str = "cuda", max_ctx: int = 512,
                 replicate: bool = False, group=None, p2p: bool = True):
        self.spec = spec
        self.moe = isinstance(spec, MoESpec)
        self.dev = d = torch.device(device)
        self.max_ctx = max_ctx
        self.lib = L = _lib.require()
        self.rank, self.world, self.group = rank, world, group
        h, hd = spec.hidden_size, spec.head_dim
        hs = head_shard(spec.num_attention_heads, spec.num_key_value_heads, world, rank)
        self.heads = hs

        def src(name: str) -> str:
            if replicate and name.startswith("blk."):
                parts = name.split(".")
                parts[1] = str(int(parts[1]) % 2)
                return ".".join(parts)
            return name

        def dev(b: bytes) -> torch.Tensor:
            return torch.frombuffer(bytearray(b), dtype=torch.uint8).to(d)

        def full(name: str) -> _Mat:
            dims, t, payload = tensors[src(name)]
            return _Mat(t, dev(payload), int(np.prod(dims[1:])), dims[0])

        def rows(name: str, r0: int, r1: int) -> _Mat:
            dims, t, payload = tensors[src(name)]
            return _Mat(t, dev(slice_rows(payload, t, dims[0], r0, r1)), r1 - r0, dims[0])

        def cols(name: str, c0: int, c1: int) -> _Mat:
            dims, t, payload = tensors[src(name)]
            return _Mat(t, dev(slice_cols(payload, t, dims[1], dims[0], c0, c1)), dims[1], c1 - c0)

        def f32(name: str) -> torch.Tensor:
            dims, t, payload = tensors[src(name)]
            if t != F32:
                raise ValueError(f"{name} must be F32")
            return dev(payload).view(torch.float32)

        def has(name: str) -> bool:
            return src(name) in tensors

        def cat(a: _Mat, b: _Mat) -> _Mat:
            if a.ggml_type != b.ggml_type or a.cols != b.cols:
                raise ValueError("concatenated matrices must share a GGML type and width")
            return _Mat(a.ggml_type, torch.cat([a.data, b.data]), a.rows + b.rows, a.cols)

        self.embd = full("token_embd.weight")
        tied = spec.tied_embeddings or "output.weight" not in tensors
        v0, v1 = even_range(spec.vocab_size, world, rank)
        self.vocab_rows = (v0, v1)
        self.lm_head = rows("token_embd.weight" if tied else "output.weight", v0, v1)
        self.out_norm = f32("output_norm.weight")
        q0, q1 = hs.q0 * hd, (hs.q0 + hs.nq) * hd
        k0, k1 = hs.kv0 * hd, (hs.kv0 + hs.nkv) * hd
        self.layers: list[_Layer] = []
        for i in range(spec.num_hidden_layers):
            p = f"blk.{i}."
            ly = _Layer(attn_norm=f32(p + "attn_norm.weight"), ffn_norm=f32(p + "ffn_norm.weight"),
                        q_norm=f32(p + "attn_q_norm.weight") if has(p + "attn_q_norm.weight") else None,
                        k_norm=f32(p + "attn_k_norm.weight") if has(p + "attn_k_norm.weight") else None,
                        qk=cat(rows(p + "attn_q.weight", q0, q1), rows(p + "attn_k.weight", k0, k1)),
                        v=rows(p + "attn_v.weight", k0, k1), o=cols(p + "attn_output.weight", q0, q1))
            if self.moe:
                E = spec.num_experts
                mine = owned_experts(E, world, rank)
                ly.router = full(p + "ffn_gate_inp.weight")
                for comp in ("gate", "up", "down"):
                    dims, t, payload = tensors[src(p + f"ffn_{comp}_exps.weight")]
                    per = dims[1] * row_bytes(t, dims[0])
                    if len(payload) == len(mine) * per:  # drawn for this GPU only (chunked specs)
                        local = payload
                    else:
                        local = b"".join(payload[e * per:(e + 1) * per] for e in mine)
                    setattr(ly, f"{comp}_exps", _Mat(t, dev(local), dims[1], dims[0]))
            else:
                f0, f1 = even_range(spec.intermediate_size, world, rank)
                ly.gate_up = cat(rows(p + "ffn_gate.weight", f0, f1), rows(p + "ffn_up.weight", f0, f1))
                ly.down = cols(p + "ffn_down.weight", f0, f1)
            self.layers.append(ly)
        self.n_stack_experts = len(owned_experts(spec.num_experts, world, rank)) if self.moe else 0
        self._pair_expert_stacks()

        z = lambda *shape, dt=torch.float32: torch.zeros(*shape, dtype=dt, device=d)  # noqa: E731
        nq_l, nkv_l = hs.nq * hd, hs.nkv * hd
        self.hidden, self.normed, self.part = z(h), z(h), z(h)
        self.qkv, self.attn = z(nq_l + 2 * nkv_l), z(nq_l)
        if self.moe:
            ff, k = spec.moe_intermediate_size, spec.num_experts_per_tok
            self.router_logits = z(spec.num_experts)
            self.route_ticket = z(1, dt=torch.int32)
            self.expert_ids, self.expert_w = z(k, dt=torch.int32), z(k)
            self.gate_up_out = z(2 * k, ff)
            self.gate, self.up = self.gate_up_out[:k], self.gate_up_out[k:]
            self.act, self.down = z(k, ff), z(k, h)
        else:
            ff, k = spec.intermediate_size // world, 1
            self.gu, self.act = z(2 * ff), z(ff)
        self.ff = ff
        self.logits_local = z(v1 - v0)
        self.logits = z(spec.vocab_size)  # filled only with gather_logits (the greedy step exchanges pairs)
        self.gather_logits = False
        self.pair_local = torch.zeros(2, dtype=torch.int32, device=d)  # {float value, int32 id}
        self.pairs = torch.zeros(2 * world, dtype=torch.int32, device=d)
        self.kcache = z(spec.num_hidden_layers, max_ctx, nkv_l)
        self.vcache = torch.zeros_like(self.kcache)
        self.tokens, self.pos = z(max_ctx, dt=torch.int32), z(1, dt=torch.int32)
        self.argmax_scratch = z(max(2048, int(L.pyrite_cuda_post_scratch_size())), dt=torch.uint8)
        self.ticket = z(1, dt=torch.int32)
        self.attn_scratch = z(int(L.pyrite_cuda_attention_scratch_size(hs.nq, max_ctx)), dt=torch.uint8)
        self.expert_shards, self.expert_shard = world, rank
        self.route_log = z(spec.num_hidden_layers, k, dt=torch.int32) if self.moe else None

        def ws(n: int, copies: int = 1) -> tuple[torch.Tensor, int, int]:
            per = int(L.pyrite_cuda_workspace_size(0, n, 1))
            buf = torch.empty(per * copies + 256, dtype=torch.uint8, device=d)
            return buf, (-buf.data_ptr()) % 256, per

        self.ws_h, self.ws_q, self.ws_act = ws(h), ws(nq_l), ws(ff, k)
        half = hd // 2
        inv = spec.rope_theta ** (-2.0 * np.arange(half, dtype=np.float64) / hd)
        ang = np.arange(max_ctx, dtype=np.float64)[:, None] * inv[None, :]
        self.rope = torch.from_numpy(np.ascontiguousarray(np.stack([np.cos(ang), np.sin(ang)], axis=-1))).to(d)
        self.graph = None
        self.prompt_len = 0
        # the communicator is set up (and warmed) before any graph capture
        dist.all_reduce(self.part, group=self.group)
        torch.cuda.synchronize(d)
        self._ipc_owned: int | None = None
        self._ipc_opened: list[int] = []
        self.peer_buffers = None
        if p2p and world > 1:
            self._setup_p2p()

    def _setup_p2p(self) -> None:
        """The one-shot NVLink sum (pyrite_cuda_allreduce_sum): a zeroed buffer
        per rank shared by CUDA IPC handles, the device array of every rank's
        buffer address and this rank's call counter."""
        L, d, h = self.lib, self.dev, self.spec.hidden_size
        ptr, handle = ctypes.c_void_p(), (ctypes.c_ubyte * 64)()
        self.ar_buffer_len = int(L.pyrite_cuda_allreduce_buffer_size(h))
        _check(L.pyrite_cuda_ipc_buffer_create(self.ar_buffer_len, ctypes.byref(ptr), handle), "ipc buffer")
        self._ipc_owned = ptr.value
        handles: list[bytes | None] = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        ptrs = []
        for r, hb in enumerate(handles):
            if r == self.rank:
                ptrs.append(ptr.value)
                continue
            p = ctypes.c_void_p()
            _check(L.pyrite_cuda_ipc_buffer_open(hb, ctypes.byref(p)), "ipc open")
            self._ipc_opened.append(p.value)
            ptrs.append(p.value)
        self.peer_buffers = torch.tensor(ptrs, dtype=torch.int64, device=d)
        self.ar_epoch = torch.zeros(1, dtype=torch.int32, device=d)
        torch.cuda.synchronize(d)
        dist.barrier(group=self.group)  # every buffer is zeroed before any flag is raised

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after every rank's
        last step: call it on all ranks after a barrier)."""
        torch.cuda.synchronize(self.dev)
        for p in self._ipc_opened:
            self.lib.pyrite_cuda_ipc_buffer_close(p, 0)
        self._ipc_opened = []
        if self._ipc_owned is not None:
            self.lib.pyrite_cuda_ipc_buffer_close(self._ipc_owned, 1)
            self._ipc_owned = None
        self.peer_buffers = None

    @property
    def batched_prefill(self) -> bool:
        """Tensor-parallel prompts run through the one-position step (its
        projections' partials are summed across GPUs after each block's
        products, which the batched path does not do)."""
        return False

    def capture(self) -> None:
        dist.barrier(group=self.group)  # the ranks' first steps start together
        super().capture()

    @classmethod
    def synthetic(cls, spec: DenseSpec | MoESpec, rank: int, world: int, device="cuda", max_ctx: int = 512,
                  replicate: bool = False, group=None) -> "ShardedDecoder":
        gen_spec = spec
        if replicate:
            from dataclasses import replace
            gen_spec = replace(spec, num_hidden_layers=min(2, spec.num_hidden_layers))
        if isinstance(spec, MoESpec):  # chunked specs draw only this GPU's experts
            subset = owned_experts(spec.num_experts, world, rank) if spec.chunked_weights else None
            items = moe_tensors(gen_spec, experts=subset)
        else:
            items = dense_tensors(gen_spec)
        tensors = {name: (dims, t, payload) for name, dims, t, payload in items}
        return cls(spec, tensors, rank, world, device=device, max_ctx=max_ctx, replicate=replicate, group=group)

    # ------------------------------------------------------------------ one step
    def _allreduce_into_hidden(self, stream: int) -> None:
        """hidden += sum over ranks of part: one kernel over NVLink peer
        memory (pyrite_cuda_allreduce_sum), or NCCL when p2p is off."""
        if self.peer_buffers is not None:
            _check(self.lib.pyrite_cuda_allreduce_sum(self.part.data_ptr(), self.hidden.data_ptr(), self.part.numel(),
                                                      self.peer_buffers.data_ptr(), self.ar_buffer_len, self.world,
                                                      self.rank,
                                                      self.ar_epoch.data_ptr(), stream), "allreduce")
            return
        dist.all_reduce(self.part, group=self.group)
        self.hidden.add_(self.part)

    def _step(self, stream: int) -> None:
        s, L, hs = self.spec, self.lib, self.heads
        h, ff, hd = s.hidden_size, self.ff, s.head_dim
        eps = float(s.rms_norm_eps)
        qk_rows = (hs.nq + hs.nkv) * hd
        _check(L.pyrite_cuda_embed(self.embd.ggml_type, self.embd.data.data_ptr(), s.vocab_size, h,
                                   self.tokens.data_ptr(), self.pos.data_ptr(), self.hidden.data_ptr(), stream), "embed")
        for li, ly in enumerate(self.layers):
            self._mvx2(ly.qk, ly.v, self.hidden, ly.attn_norm, self.ws_h, self.qkv, self.qkv[qk_rows:], stream)
            wq, wql = self._wsp(self.ws_q)
            _check(L.pyrite_cuda_attention_step(
                self.qkv.data_ptr(), ly.q_norm.data_ptr() if ly.q_norm is not None else None,
                ly.k_norm.data_ptr() if ly.k_norm is not None else None, hs.nq, hs.nkv, hd, eps,
                self.pos.data_ptr(), self.rope.data_ptr(), self.max_ctx, self.kcache[li].data_ptr(),
                self.vcache[li].data_ptr(), self.attn.data_ptr(), wq, wql, self.attn_scratch.data_ptr(),
                self.attn_scratch.numel(), stream), "attention_step")
            self._mv(ly.o, self.attn, self.ws_q, self.part, 0, stream)
            self._allreduce_into_hidden(stream)
            if not self.moe:
                self._mvx(ly.gate_up, self.hidden, _lib.X_RMSNORM, ly.ffn_norm, self.normed, self.ws_h, self.gu, 0,
                          stream)
                self._mvx(ly.down, self.gu, _lib.X_SILU_MUL, None, self.act, self.ws_act, self.part, 0, stream)
            else:
                k = s.num_experts_per_tok
                self._route(ly, li, stream)
                self._gate_up_experts(ly, stream)
                wa, wal = self._wsp(self.ws_act)
                _check(L.pyrite_cuda_moe_silu_mul_encode(self.gate.data_ptr(), self.up.data_ptr(), ff, k,
                                                         self.act.data_ptr(), wa, wal, stream), "moe silu")
                self.part.zero_()
                self._down_combine(ly, self.part, stream)
            self._allreduce_into_hidden(stream)
        self._norm(self.hidden, self.out_norm, self.normed, self.ws_h, stream)
        self._mv(self.lm_head, self.normed, self.ws_h, self.logits_local, 0, stream)
        # greedy over the split vocabulary: this GPU's best (value, id) pair, an
        # all-gather of 8 bytes per GPU, then the same pick on every rank
        _check(L.pyrite_cuda_argmax_local(self.logits_local.data_ptr(), self.logits_local.numel(), self.vocab_rows[0],
                                          self.argmax_scratch.data_ptr(), self.argmax_scratch.numel(),
                                          self.pair_local.data_ptr(), stream), "argmax local")
        dist.all_gather_into_tensor(self.pairs, self.pair_local, group=self.group)
        _check(L.pyrite_cuda_argmax_pick(self.pairs.data_ptr(), self.world, self.tokens.data_ptr(),
                                         self.pos.data_ptr(), self.prompt_len, self.max_ctx, stream), "argmax pick")
        if self.gather_logits:  # the whole vocabulary's logits, for inspection only
            dist.all_gather_into_tensor(self.logits, self.logits_local, group=self.group)
