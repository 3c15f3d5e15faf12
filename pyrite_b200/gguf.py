"""GGUF checkpoint -> HBM: the file's tensors uploaded as-is, ready for the decoders.

``read(path)`` parses a GGUF v2/v3 file with the validation rules of the
reference's reader (pyrite/adapters/gguf.py:209-326): magic, version 2..3,
safety limits on counts, unique metadata keys and tensor names, names shorter
than GGML_MAX_NAME (64), at most 4 dimensions, no zero dimension, a
power-of-two ``general.alignment`` (default 32), aligned tensor offsets, every
payload inside the file and none overlapping another; and each tensor's byte
size from its GGML geometry (a row of dims[0] values is dims[0] / block_size
blocks, pyrite/ggml_types.py:117-136), which rejects a row that is not a whole
number of blocks.  Tensor payloads are not read here: they are views into a
read-only memory map of the file.

``spec_from_metadata`` builds the decoder's model description from the
``{arch}.*`` keys the reference reads (pyrite/dense.py:103-186 for ``llama``
/ ``qwen3``, pyrite/qwen3_moe.py:148-254 for ``qwen3moe``), and ``load``
returns a :class:`pyrite_b200.model.MixedDecoder` whose weights are the
file's GGML blocks copied to HBM unchanged (no repacking: a row range of a
matrix stays one contiguous byte range, as the kernels expect).
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

from .ggml_types import spec as ggml_spec


class GGUFError(ValueError):
    """A malformed or unsupported GGUF file."""


MAGIC = b"GGUF"
DEFAULT_ALIGNMENT = 32
MAX_DIMS = 4
MAX_NAME = 64
MIN_VERSION, MAX_VERSION = 2, 3
MAX_TENSORS = 10_000_000
MAX_METADATA = 1_000_000
MAX_ARRAY = 100_000_000

# metadata value types (GGUF)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", U64: "<Q", I64: "<q",
           F64: "<d"}


@dataclass(frozen=True)
class GGUFTensor:
    name: str
    dims: tuple[int, ...]   # GGML order: dims[0] = values per row
    ggml_type: int
    offset: int             # absolute byte offset in the file
    nbytes: int


@dataclass
class GGUFFile:
    path: Path
    version: int
    alignment: int
    data_offset: int
    metadata: dict[str, Any]
    tensors: dict[str, GGUFTensor]
    _map: mmap.mmap | None = field(default=None, repr=False)

    def payload(self, name: str) -> memoryview:
        """The tensor's bytes: a read-only view into the mapped file."""
        t = self.tensors[name]
        if self._map is None:
            with self.path.open("rb") as fh:
                self._map = mmap.mmap(fh.fileno(), 0, access=mmap.ACCESS_READ)
        return memoryview(self._map)[t.offset:t.offset + t.nbytes]

    def close(self) -> None:
        """Unmap the file (views handed out by payload() must be released first)."""
        if self._map is not None:
            try:
                self._map.close()
            except BufferError:  # a payload view is still alive: the map goes with it
                pass
            self._map = None


class _Reader:
    """Bounded little-endian reads from the open file (never past its end)."""

    def __init__(self, fh, size: int):
        self.fh, self.size = fh, size

    @property
    def pos(self) -> int:
        return self.fh.tell()

    @property
    def remaining(self) -> int:
        return self.size - self.fh.tell()

    def take(self, n: int) -> bytes:
        if n < 0 or n > self.remaining:
            raise GGUFError(f"GGUF file truncated: needs {n} bytes at offset {self.pos}, {self.remaining} remain")
        return self.fh.read(n)

    def scalar(self, fmt: str):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self, label: str) -> str:
        n = self.scalar("<Q")
        if n > self.remaining:
            raise GGUFError(f"GGUF {label} declares {n} bytes but only {self.remaining} remain")
        try:
            return self.take(n).decode("utf-8")
        except UnicodeDecodeError as exc:
            raise GGUFError(f"invalid UTF-8 in GGUF {label}") from exc


def _value(r: _Reader, kind: int, key: str) -> Any:
    if kind in _SCALAR:
        return r.scalar(_SCALAR[kind])
    if kind == BOOL:
        v = r.scalar("<B")
        if v not in (0, 1):
            raise GGUFError(f"invalid GGUF boolean value {v} for {key!r}")
        return bool(v)
    if kind == STRING:
        return r.string(f"metadata value for {key!r}")
    if kind == ARRAY:
        etype, count = r.scalar("<I"), r.scalar("<Q")
        if count > MAX_ARRAY:
            raise GGUFError(f"GGUF metadata array {key!r} declares {count} elements, above the {MAX_ARRAY} limit")
        if count > r.remaining:
            raise GGUFError(f"GGUF metadata array {key!r} declares {count} elements but only "
                            f"{r.remaining} bytes remain")
        return tuple(_value(r, etype, key) for _ in range(count))
    raise GGUFError(f"unsupported GGUF metadata value type {kind} for key {key!r}")


def tensor_bytes(dims: tuple[int, ...], ggml_type: int, name: str = "") -> int:
    """Payload size of a tensor: rows of dims[0] values, each a whole number of blocks."""
    try:
        s = ggml_spec(ggml_type)
    except (KeyError, ValueError) as exc:
        raise GGUFError(f"tensor {name!r}: unknown GGML type {ggml_type}") from exc
    if not dims:
        dims = (1,)
    if dims[0] % s.block_size:
        raise GGUFError(f"tensor {name!r}: a row of {dims[0]} values is not a whole number of "
                        f"{s.block_size}-value {s.name} blocks")
    rows = 1
    for d in dims[1:]:
        rows *= d
    return dims[0] // s.block_size * s.bytes_per_block * rows


def read(path: str | Path) -> GGUFFile:
    """Parse and validate a GGUF v2/v3 file (the tensor payloads stay on disk)."""
    path = Path(path)
    if not path.is_file():
        raise FileNotFoundError(path)
    size = path.stat().st_size
    if size < 24:
        raise GGUFError(f"not a GGUF checkpoint: {path.name} is {size} bytes")
    with path.open("rb") as fh:
        r = _Reader(fh, size)
        if r.take(4) != MAGIC:
            raise GGUFError(f"not a GGUF checkpoint: bad magic in {path.name}")
        version = r.scalar("<I")
        if not MIN_VERSION <= version <= MAX_VERSION:
            raise GGUFError(f"unsupported GGUF version {version}: v{MIN_VERSION}-v{MAX_VERSION} are read "
                            "(v1 used 32-bit counts)")
        n_tensors, n_meta = r.scalar("<Q"), r.scalar("<Q")
        if n_tensors > MAX_TENSORS or n_meta > MAX_METADATA:
            raise GGUFError(f"GGUF header declares {n_tensors} tensors and {n_meta} metadata entries, beyond "
                            f"the limits {MAX_TENSORS} / {MAX_METADATA}: corrupt or truncated")
        metadata: dict[str, Any] = {}
        alignment = DEFAULT_ALIGNMENT
        for _ in range(n_meta):
            key = r.string("metadata key")
            kind = r.scalar("<I")
            if key in metadata:
                raise GGUFError(f"duplicate GGUF metadata key: {key}")
            metadata[key] = v = _value(r, kind, key)
            if key == "general.alignment":
                if isinstance(v, bool) or not isinstance(v, int) or v <= 0 or v & (v - 1):
                    raise GGUFError(f"invalid GGUF alignment {v!r}: must be a positive power of two")
                alignment = v
        infos: list[tuple[str, tuple[int, ...], int, int]] = []
        seen: set[str] = set()
        for _ in range(n_tensors):
            name = r.string("tensor name")
            if name in seen:
                raise GGUFError(f"duplicate GGUF tensor name: {name}")
            if len(name) >= MAX_NAME:
                raise GGUFError(f"tensor name {name[:32]!r}... is {len(name)} bytes; the limit is {MAX_NAME - 1}")
            seen.add(name)
            n_dims = r.scalar("<I")
            if n_dims > MAX_DIMS:
                raise GGUFError(f"GGUF tensor {name!r} has {n_dims} dimensions; at most {MAX_DIMS}")
            dims = tuple(r.scalar("<Q") for _ in range(n_dims))
            if any(d == 0 for d in dims):
                raise GGUFError(f"GGUF tensor {name!r} has a zero-sized dimension: {dims}")
            infos.append((name, dims, r.scalar("<I"), r.scalar("<Q")))
        pos = r.pos
        data_offset = pos + (-pos) % alignment if n_tensors else pos
        if data_offset > size:
            raise GGUFError(f"GGUF tensor data starts at {data_offset}, beyond the {size}-byte file")
        tensors: dict[str, GGUFTensor] = {}
        for name, dims, ggml_type, rel in infos:
            if rel % alignment:
                raise GGUFError(f"unaligned GGUF tensor offset: {name} starts at {rel}, not a multiple of "
                                f"the {alignment}-byte alignment")
            nbytes = tensor_bytes(dims, ggml_type, name)
            if rel > size - data_offset:
                raise GGUFError(f"GGUF tensor {name} offset {rel} lies beyond the file")
            start = data_offset + rel
            if nbytes > size - start:
                raise GGUFError(f"GGUF tensor {name} needs {nbytes} bytes at {start} but the file ends at {size}")
            tensors[name] = GGUFTensor(name, dims, ggml_type, start, nbytes)
        prev_end, prev_name = data_offset, ""
        for t in sorted(tensors.values(), key=lambda t: (t.offset, t.offset + t.nbytes)):
            if t.offset < prev_end:
                raise GGUFError(f"GGUF tensor payload overlaps another tensor: {prev_name}, {t.name}")
            prev_end, prev_name = t.offset + t.nbytes, t.name
    return GGUFFile(path, version, alignment, data_offset, metadata, tensors)


def spec_from_metadata(meta: dict[str, Any], tensors: dict[str, GGUFTensor]):
    """The decoder's model description (DenseSpec or MoESpec) from the file's keys."""
    from .synthetic import DenseSpec, MoESpec

    arch = str(meta.get("general.architecture", ""))
    if arch not in ("llama", "qwen3", "qwen3moe"):
        raise GGUFError(f"unsupported GGUF architecture: {arch or 'unknown'}")

    def n(suffix: str, default=None):
        return meta.get(f"{arch}.{suffix}", default)

    hidden, layers = int(n("embedding_length", 0) or 0), int(n("block_count", 0) or 0)
    heads = int(n("attention.head_count", 0) or 0)
    kv_raw = n("attention.head_count_kv")
    kv = heads if kv_raw is None else int(kv_raw)
    ffn = int(n("feed_forward_length", 0) or 0)
    hd_raw = n("attention.key_length")
    head_dim = int(hidden // heads if hd_raw is None and heads else hd_raw or 0)
    emb = tensors.get("token_embd.weight")
    if emb is None or len(emb.dims) != 2:
        raise GGUFError("GGUF has no 2-D token_embd.weight")
    vocab = int(emb.dims[1])
    missing = [k for k, v in {"embedding_length": hidden, "block_count": layers, "attention.head_count": heads,
                              "attention.head_count_kv": kv, "feed_forward_length": ffn}.items() if v <= 0]
    if missing:
        raise GGUFError("GGUF is missing required metadata: " + ", ".join(f"{arch}.{k}" for k in missing))
    if kv > heads or heads % kv:
        raise GGUFError(f"attention head count {heads} must be divisible by KV head count {kv}")
    if head_dim != 128:
        raise GGUFError(f"head_dim {head_dim}: the decode kernels take 128-value heads")
    eps_raw, theta_raw = n("attention.layer_norm_rms_epsilon"), n("rope.freq_base")
    tied_raw = n("tied_word_embeddings")
    tied = ("output.weight" not in tensors) if tied_raw is None else bool(tied_raw)
    common = dict(architecture=arch, hidden_size=hidden, num_hidden_layers=layers, num_attention_heads=heads,
                  num_key_value_heads=kv, head_dim=head_dim, intermediate_size=ffn, vocab_size=vocab,
                  tied_embeddings=tied, context_length=int(n("context_length", 0) or 0))
    if arch == "qwen3moe":
        experts, per_tok = int(n("expert_count", 0) or 0), int(n("expert_used_count", 0) or 0)
        moe_ffn = int(n("expert_feed_forward_length", 0) or 0)
        if min(experts, per_tok, moe_ffn) <= 0:
            raise GGUFError("GGUF is missing Qwen3-MoE expert metadata (expert_count, expert_used_count, "
                            "expert_feed_forward_length)")
        norm_topk = n("expert_weights_norm")
        return MoESpec(**common, moe_intermediate_size=moe_ffn, num_experts=experts, num_experts_per_tok=per_tok,
                       norm_topk_prob=True if norm_topk is None else bool(norm_topk),
                       rms_norm_eps=float(1e-6 if eps_raw is None else eps_raw),
                       rope_theta=float(1_000_000.0 if theta_raw is None else theta_raw), qk_norm=True)
    qk_raw = n("attention.qk_norm")
    default_eps, default_theta = (1e-5, 500_000.0) if arch == "llama" else (1e-6, 1_000_000.0)
    return DenseSpec(**common, rms_norm_eps=float(default_eps if eps_raw is None else eps_raw),
                     rope_theta=float(default_theta if theta_raw is None else theta_raw),
                     qk_norm=(arch == "qwen3") if qk_raw is None else bool(qk_raw))


def load(path: str | Path, device="cuda", max_ctx: int = 512):
    """A batch-1 greedy decoder (pyrite_b200.model.MixedDecoder) with the
    file's weights in HBM; the file is mapped, read once and closed."""
    from .model import MixedDecoder

    f = read(path)
    try:
        spec = spec_from_metadata(f.metadata, f.tensors)
        tensors = {name: (t.dims, t.ggml_type, f.payload(name)) for name, t in f.tensors.items()}
        dec = MixedDecoder(spec, tensors, device=device, max_ctx=max_ctx)
        del tensors
    finally:
        f.close()
    return dec
