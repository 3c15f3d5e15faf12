"""Seeded synthetic checkpoints of the benchmarked model shapes (no public weights exist for them).

``dense_tensors(spec)`` yields every tensor of a dense ``qwen3`` / ``llama``
GGUF checkpoint -- name, GGML dims, GGML type and payload bytes -- in the
tensor contract the reference's dense executor validates
(``pyrite/dense.py:349-395``): matrices are seeded N(0, 0.02) float32 weights
quantized by :mod:`pyrite_b200.quantize` (byte-identical to the reference's
own encoders), norm weights are F32 ones.  The same bytes feed both the GGUF
file the reference runs on and the B200 executor, so the two see identical
weights without shipping the file.

GGML dims are ``(cols, rows)``: ``attn_q.weight`` of a model with hidden size
h and q dimension q has dims ``(h, q)`` and q rows of h values.
"""
from __future__ import annotations

import zlib
from collections.abc import Iterator
from dataclasses import dataclass

import numpy as np

from .quantize import quantize


@dataclass(frozen=True)
class DenseSpec:
    architecture: str = "qwen3"
    hidden_size: int = 1024
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 3072
    vocab_size: int = 151936
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-6
    qk_norm: bool = True
    tied_embeddings: bool = True
    weight_type: int = 8  # Q8_0
    context_length: int = 40960
    seed: int = 20240607
    mix: str = ""         # "q4_k_m": one type per tensor (dense_tensor_type), else weight_type

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @classmethod
    def c1(cls) -> "DenseSpec":
        """Qwen3-0.6B-shaped, all matrices Q8_0."""
        return cls()

    @classmethod
    def c3(cls) -> "DenseSpec":
        """Llama-3-8B-shaped, Q4_K_M mix."""
        return cls(architecture="llama", hidden_size=4096, num_hidden_layers=32, num_attention_heads=32,
                   num_key_value_heads=8, head_dim=128, intermediate_size=14336, vocab_size=128256,
                   rope_theta=500_000.0, rms_norm_eps=1e-5, qk_norm=False, tied_embeddings=False,
                   weight_type=12, context_length=8192, mix="q4_k_m")


def _weights(name: str, count: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng((zlib.crc32(name.encode()) ^ seed) & 0xFFFFFFFF)
    return rng.normal(0.0, 0.02, count).astype(np.float32)


def _weights_chunked(name: str, count: int, seed: int, chunk: int = 1 << 22) -> np.ndarray:
    """Seeded N(0, 0.02) float32 weights drawn in independently seeded chunks
    on all host cores (the ~10^10-value checkpoints of configs[4]): chunk i of
    tensor `name` comes from default_rng([crc32(name), seed, i])."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    out = np.empty(count, dtype=np.float32)
    key = zlib.crc32(name.encode())

    def fill(i: int) -> None:
        part = out[i * chunk:(i + 1) * chunk]
        np.random.default_rng([key, seed & 0xFFFFFFFF, i]).standard_normal(part.shape[0], dtype=np.float32, out=part)
        part *= np.float32(0.02)

    with ThreadPoolExecutor(max(1, os.cpu_count() or 1)) as ex:
        list(ex.map(fill, range((count + chunk - 1) // chunk)))
    return out


def _weights_chunked_ranges(name: str, count: int, seed: int, ranges: list[tuple[int, int]],
                            chunk: int = 1 << 22) -> np.ndarray:
    """Values [a, b) for each (a, b) of ``ranges``, concatenated, of
    ``_weights_chunked(name, count, seed)``, drawing only the chunks they
    touch (one GPU's experts of a configs[4] stack)."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    key = zlib.crc32(name.encode())
    need = sorted({i for a, b in ranges for i in range(a // chunk, (b - 1) // chunk + 1)})

    def draw(i: int) -> np.ndarray:
        n = min(chunk, count - i * chunk)
        part = np.random.default_rng([key, seed & 0xFFFFFFFF, i]).standard_normal(n, dtype=np.float32)
        part *= np.float32(0.02)
        return part

    with ThreadPoolExecutor(max(1, os.cpu_count() or 1)) as ex:
        chunks = dict(zip(need, ex.map(draw, need)))
    out = np.empty(sum(b - a for a, b in ranges), dtype=np.float32)
    o = 0
    for a, b in ranges:
        for i in range(a // chunk, (b - 1) // chunk + 1):
            lo, hi = max(a, i * chunk), min(b, (i + 1) * chunk)
            out[o:o + hi - lo] = chunks[i][lo - i * chunk:hi - i * chunk]
            o += hi - lo
    return out


def metadata(spec: DenseSpec) -> dict[str, object]:
    """GGUF metadata keys the reference reads (``dense.py:113-186``)."""
    a = spec.architecture
    return {
        f"{a}.embedding_length": spec.hidden_size,
        f"{a}.block_count": spec.num_hidden_layers,
        f"{a}.feed_forward_length": spec.intermediate_size,
        f"{a}.attention.head_count": spec.num_attention_heads,
        f"{a}.attention.head_count_kv": spec.num_key_value_heads,
        f"{a}.attention.key_length": spec.head_dim,
        f"{a}.attention.value_length": spec.head_dim,
        f"{a}.attention.layer_norm_rms_epsilon": float(spec.rms_norm_eps),
        f"{a}.rope.freq_base": float(spec.rope_theta),
        f"{a}.context_length": spec.context_length,
        f"{a}.tied_word_embeddings": bool(spec.tied_embeddings),
        f"{a}.attention.qk_norm": bool(spec.qk_norm),
    }


def layer_matrices(spec: DenseSpec) -> list[tuple[str, int, int]]:
    """(suffix, rows, cols) of each per-layer matrix."""
    h, q, kv, f = spec.hidden_size, spec.q_dim, spec.kv_dim, spec.intermediate_size
    return [("attn_q.weight", q, h), ("attn_k.weight", kv, h), ("attn_v.weight", kv, h),
            ("attn_output.weight", h, q), ("ffn_gate.weight", f, h), ("ffn_up.weight", f, h),
            ("ffn_down.weight", h, f)]


def dense_tensor_type(spec: DenseSpec, name: str) -> int:
    """GGML type of a matrix: ``weight_type``, or for the Q4_K_M mix Q6_K for
    attn_v, ffn_down of the even layers (half of them) and the output
    projection, Q4_K for the rest."""
    if spec.mix != "q4_k_m":
        return spec.weight_type
    if name == "output.weight" or name.endswith("attn_v.weight"):
        return 14
    if name.endswith("ffn_down.weight"):
        return 14 if int(name.split(".")[1]) % 2 == 0 else 12
    return 12


def dense_tensors(spec: DenseSpec) -> Iterator[tuple[str, tuple[int, ...], int, bytes]]:
    """(name, GGML dims, GGML type, payload) for every tensor of the checkpoint."""
    ones = lambda n: np.ones(n, dtype=np.float32).tobytes()  # noqa: E731
    t = dense_tensor_type(spec, "token_embd.weight")
    yield ("token_embd.weight", (spec.hidden_size, spec.vocab_size), t,
           quantize(t, _weights("token_embd.weight", spec.hidden_size * spec.vocab_size, spec.seed)))
    yield ("output_norm.weight", (spec.hidden_size,), 0, ones(spec.hidden_size))
    if not spec.tied_embeddings:
        t = dense_tensor_type(spec, "output.weight")
        yield ("output.weight", (spec.hidden_size, spec.vocab_size), t,
               quantize(t, _weights("output.weight", spec.hidden_size * spec.vocab_size, spec.seed)))
    for layer in range(spec.num_hidden_layers):
        p = f"blk.{layer}."
        yield (p + "attn_norm.weight", (spec.hidden_size,), 0, ones(spec.hidden_size))
        if spec.qk_norm:
            yield (p + "attn_q_norm.weight", (spec.head_dim,), 0, ones(spec.head_dim))
            yield (p + "attn_k_norm.weight", (spec.head_dim,), 0, ones(spec.head_dim))
        yield (p + "ffn_norm.weight", (spec.hidden_size,), 0, ones(spec.hidden_size))
        for suffix, rows, cols in layer_matrices(spec):
            t = dense_tensor_type(spec, p + suffix)
            yield (p + suffix, (cols, rows), t, quantize(t, _weights(p + suffix, rows * cols, spec.seed)))


def prompt_ids(spec: DenseSpec, n: int = 16, seed: int = 7) -> list[int]:
    """The benchmark prompt: ``n`` seeded uniform token ids."""
    return [int(v) for v in np.random.default_rng(seed).integers(0, spec.vocab_size, n)]


# ---------------------------------------------------------------- MoE (qwen3moe)
@dataclass(frozen=True)
class MoESpec:
    """A ``qwen3moe`` checkpoint: configs[3] (Qwen3-30B-A3B-shaped)
    and smaller variants for parity runs."""

    architecture: str = "qwen3moe"
    hidden_size: int = 2048
    num_hidden_layers: int = 48
    num_attention_heads: int = 32
    num_key_value_heads: int = 4
    head_dim: int = 128
    intermediate_size: int = 6144      # dense feed-forward length (metadata only)
    moe_intermediate_size: int = 768
    num_experts: int = 128
    num_experts_per_tok: int = 8
    vocab_size: int = 151936
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-6
    norm_topk_prob: bool = True
    tied_embeddings: bool = False
    context_length: int = 40960
    seed: int = 20240607
    qk_norm: bool = True
    chunked_weights: bool = False  # weights from _weights_chunked (configs[4] sizes)

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @classmethod
    def c4(cls) -> "MoESpec":
        """Qwen3-30B-A3B-shaped, Q4_K_M mix."""
        return cls()

    @classmethod
    def c5(cls) -> "MoESpec":
        """Qwen3-235B-A22B-shaped, Q4_K_M mix (~142 GB)."""
        return cls(hidden_size=4096, num_hidden_layers=94, num_attention_heads=64, num_key_value_heads=4,
                   intermediate_size=12288, moe_intermediate_size=1536, chunked_weights=True)

    @classmethod
    def tiny(cls) -> "MoESpec":
        """A two-layer model small enough for the reference to run in seconds."""
        return cls(hidden_size=512, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                   intermediate_size=1024, moe_intermediate_size=256, num_experts=16, num_experts_per_tok=4,
                   vocab_size=2048)


#: The Q4_K_M mix: Q4_K for most tensors, Q6_K for attn_v,
#: half of ffn_down (the even layers) and the output projection; the router
#: (ffn_gate_inp) stays F32 as llama.cpp keeps it.
Q4_K, Q6_K, F32 = 12, 14, 0


def moe_tensor_type(spec: MoESpec, name: str) -> int:
    if name == "output.weight":
        return Q6_K
    if name.endswith("attn_v.weight"):
        return Q6_K
    if name.endswith("ffn_down_exps.weight"):
        layer = int(name.split(".")[1])
        return Q6_K if layer % 2 == 0 else Q4_K
    if name.endswith("ffn_gate_inp.weight") or name.endswith("norm.weight"):
        return F32
    return Q4_K


def moe_metadata(spec: MoESpec) -> dict[str, object]:
    """GGUF metadata keys the reference reads (``qwen3_moe.py:148-254``)."""
    a = spec.architecture
    return {
        f"{a}.embedding_length": spec.hidden_size,
        f"{a}.block_count": spec.num_hidden_layers,
        f"{a}.feed_forward_length": spec.intermediate_size,
        f"{a}.expert_feed_forward_length": spec.moe_intermediate_size,
        f"{a}.expert_count": spec.num_experts,
        f"{a}.expert_used_count": spec.num_experts_per_tok,
        f"{a}.expert_weights_norm": bool(spec.norm_topk_prob),
        f"{a}.attention.head_count": spec.num_attention_heads,
        f"{a}.attention.head_count_kv": spec.num_key_value_heads,
        f"{a}.attention.key_length": spec.head_dim,
        f"{a}.attention.value_length": spec.head_dim,
        f"{a}.attention.layer_norm_rms_epsilon": float(spec.rms_norm_eps),
        f"{a}.rope.freq_base": float(spec.rope_theta),
        f"{a}.context_length": spec.context_length,
        f"{a}.tied_word_embeddings": bool(spec.tied_embeddings),
    }


def moe_tensors(spec: MoESpec, experts: list[int] | None = None) -> Iterator[tuple[str, tuple[int, ...], int, bytes]]:
    """(name, GGML dims, GGML type, payload) of every tensor of the checkpoint.
    A stacked expert tensor ``(cols, rows, E)`` is E matrices back to back.
    ``experts`` (chunked-weight specs only): the stacked tensors' payloads hold
    just those experts, in that order (the bytes of the full tensor's slices),
    and only their values are drawn."""
    ones = lambda n: np.ones(n, dtype=np.float32).tobytes()  # noqa: E731
    h, q, kv, ff, E = spec.hidden_size, spec.q_dim, spec.kv_dim, spec.moe_intermediate_size, spec.num_experts

    gen = _weights_chunked if spec.chunked_weights else _weights

    if experts is not None and not spec.chunked_weights:
        raise ValueError("expert subsets need a chunked-weight spec")

    def mat(name: str, dims: tuple[int, ...]) -> tuple[str, tuple[int, ...], int, bytes]:
        t = moe_tensor_type(spec, name)
        count = int(np.prod(dims))
        if experts is not None and len(dims) == 3:  # one GPU's experts of a stack
            per = dims[0] * dims[1]
            w = _weights_chunked_ranges(name, count, spec.seed, [(e * per, (e + 1) * per) for e in experts])
        else:
            w = gen(name, count, spec.seed)
        return name, dims, t, (w.tobytes() if t == F32 else quantize(t, w))

    yield mat("token_embd.weight", (h, spec.vocab_size))
    yield ("output_norm.weight", (h,), F32, ones(h))
    if not spec.tied_embeddings:
        yield mat("output.weight", (h, spec.vocab_size))
    for layer in range(spec.num_hidden_layers):
        p = f"blk.{layer}."
        yield (p + "attn_norm.weight", (h,), F32, ones(h))
        yield mat(p + "attn_q.weight", (h, q))
        yield mat(p + "attn_k.weight", (h, kv))
        yield mat(p + "attn_v.weight", (h, kv))
        yield mat(p + "attn_output.weight", (q, h))
        yield (p + "attn_q_norm.weight", (spec.head_dim,), F32, ones(spec.head_dim))
        yield (p + "attn_k_norm.weight", (spec.head_dim,), F32, ones(spec.head_dim))
        yield (p + "ffn_norm.weight", (h,), F32, ones(h))
        yield mat(p + "ffn_gate_inp.weight", (h, E))
        yield mat(p + "ffn_gate_exps.weight", (h, ff, E))
        yield mat(p + "ffn_up_exps.weight", (h, ff, E))
        yield mat(p + "ffn_down_exps.weight", (ff, h, E))
