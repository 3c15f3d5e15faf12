"""GGUF -> HBM loader (pyrite_b200.gguf).

Inputs are real GGUF files, byte-identical to what the reference's own fixture
builder writes for the tiny golden checkpoints: tests/gguf_writer.py restates
that builder, and its output must hash to the digests
tests/golden/make_gguf_digests.py recorded from the reference builder.  The
loader must parse them (metadata, tensor table, alignment), derive the model
the reference derives (pyrite/dense.py:103-186, pyrite/qwen3_moe.py:148-254),
reject the malformed files the reference rejects (pyrite/adapters/gguf.py:
209-326, tests/test_gguf_errors.py), and -- on a GPU -- decode the goldens'
greedy ids from the file alone.
"""
from __future__ import annotations

import hashlib
import json
import struct
from pathlib import Path

import pytest

from tests.gguf_writer import gguf_bytes

GOLDEN = Path(__file__).resolve().parent / "golden"
DIGESTS = json.loads((GOLDEN / "gguf_digests.json").read_text())
CASES = ["llama_tiny", "moe_tiny", "c1_small"]


def _build(case: str) -> tuple[dict, bytes]:
    from tests.golden.make_gguf_digests import spec_and_tensors
    golden = json.loads((GOLDEN / DIGESTS[case]["golden"]).read_text())
    spec, meta, tensors = spec_and_tensors(golden)
    return golden, gguf_bytes(spec.architecture, meta, tensors)


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    d = tmp_path_factory.mktemp("gguf")
    out = {}
    for case in CASES:
        golden, data = _build(case)
        p = d / f"{case}.gguf"
        p.write_bytes(data)
        out[case] = (golden, p, data)
    return out


@pytest.mark.parametrize("case", CASES)
def test_files_are_the_reference_builders_bytes(files, case):
    _, _, data = files[case]
    assert len(data) == DIGESTS[case]["bytes"]
    assert hashlib.sha256(data).hexdigest() == DIGESTS[case]["sha256"]


@pytest.mark.parametrize("case", CASES)
def test_read_parses_the_table_and_derives_the_model(files, case):
    from pyrite_b200 import gguf
    from pyrite_b200.ggml_types import spec as ggml_spec
    golden, path, data = files[case]
    f = gguf.read(path)
    try:
        assert f.version == 3 and f.alignment == 32 and f.data_offset % 32 == 0
        s = golden["spec"]
        assert f.metadata["general.architecture"] == s["architecture"]
        prev = f.data_offset
        for t in sorted(f.tensors.values(), key=lambda t: t.offset):
            assert t.offset % 32 == 0 and t.offset >= prev
            g = ggml_spec(t.ggml_type)
            rows = 1
            for d in t.dims[1:]:
                rows *= d
            assert t.nbytes == t.dims[0] // g.block_size * g.bytes_per_block * rows
            assert len(f.payload(t.name)) == t.nbytes
            prev = t.offset + t.nbytes
        spec = gguf.spec_from_metadata(f.metadata, f.tensors)
        for k in ("hidden_size", "num_hidden_layers", "num_attention_heads", "num_key_value_heads", "head_dim",
                  "intermediate_size", "vocab_size", "tied_embeddings", "qk_norm"):
            assert getattr(spec, k) == s[k], k
        assert spec.rope_theta == pytest.approx(s["rope_theta"]) and spec.rms_norm_eps == pytest.approx(s["rms_norm_eps"])
        if s["architecture"] == "qwen3moe":
            for k in ("num_experts", "num_experts_per_tok", "moe_intermediate_size", "norm_topk_prob"):
                assert getattr(spec, k) == s[k], k
    finally:
        f.close()


def _header(version=3, n_tensors=0, n_meta=0) -> bytes:
    return b"GGUF" + struct.pack("<IQQ", version, n_tensors, n_meta)


def _kv_string(key: str, value: str) -> bytes:
    k, v = key.encode(), value.encode()
    return struct.pack("<Q", len(k)) + k + struct.pack("<I", 8) + struct.pack("<Q", len(v)) + v


def _tensor_info(name: str, dims, ggml_type: int, offset: int) -> bytes:
    n = name.encode()
    return (struct.pack("<Q", len(n)) + n + struct.pack("<I", len(dims)) +
            b"".join(struct.pack("<Q", d) for d in dims) + struct.pack("<IQ", ggml_type, offset))


def _one_tensor_file(dims=(32, 2), ggml_type=0, offset=0, payload_bytes=None, version=3, extra_meta=b"", n_meta=0):
    info = _tensor_info("t", dims, ggml_type, offset)
    prefix = _header(version, 1, n_meta) + extra_meta + info
    prefix += b"\0" * ((-len(prefix)) % 32)
    body = b"\0" * (payload_bytes if payload_bytes is not None else 4 * dims[0] * dims[1] + offset)
    return prefix + body


BAD = {
    "bad magic": lambda: b"GGUX" + _one_tensor_file()[4:],
    "version 1": lambda: _one_tensor_file(version=1),
    "version 4": lambda: _one_tensor_file(version=4),
    "unaligned offset": lambda: _one_tensor_file(offset=4, payload_bytes=300),
    "truncated payload": lambda: _one_tensor_file(payload_bytes=100),
    "zero dimension": lambda: _one_tensor_file(dims=(32, 0)),
    "five dimensions": lambda: _one_tensor_file(dims=(32, 1, 1, 1, 1)),
    "row not whole blocks": lambda: _one_tensor_file(dims=(40, 2), ggml_type=8, payload_bytes=512),
    "unknown type": lambda: _one_tensor_file(ggml_type=99),
    "alignment not a power of two": lambda: _one_tensor_file(
        extra_meta=struct.pack("<Q", 17) + b"general.alignment" + struct.pack("<II", 4, 24), n_meta=1),
    "duplicate key": lambda: _one_tensor_file(extra_meta=_kv_string("a", "x") + _kv_string("a", "y"), n_meta=2),
    "truncated header": lambda: _header(3, 5, 0),
    "huge counts": lambda: _header(3, 10 ** 8, 0),
}


@pytest.mark.parametrize("what", sorted(BAD))
def test_rejects_malformed_files_like_the_reference(tmp_path, what):
    from pyrite_b200 import gguf
    p = tmp_path / "bad.gguf"
    p.write_bytes(BAD[what]())
    with pytest.raises(gguf.GGUFError):
        gguf.read(p).close()


def test_rejects_overlapping_and_duplicate_tensors(tmp_path):
    from pyrite_b200 import gguf
    for infos in ([("a", (32, 1), 0, 0), ("b", (32, 1), 0, 64)], [("a", (32, 1), 0, 0), ("a", (32, 1), 0, 128)]):
        prefix = _header(3, len(infos), 0) + b"".join(_tensor_info(*i) for i in infos)
        prefix += b"\0" * ((-len(prefix)) % 32)
        p = tmp_path / "bad.gguf"
        p.write_bytes(prefix + b"\0" * 512)
        if infos[0][0] == infos[1][0]:
            with pytest.raises(gguf.GGUFError, match="duplicate"):
                gguf.read(p).close()
        else:  # 128 bytes of F32 at 0 and at 64 overlap
            with pytest.raises(gguf.GGUFError, match="overlap"):
                gguf.read(p).close()


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_loaded_checkpoint_decodes_the_reference_greedy_ids(cuda_device, files, case):
    """The decoder built from the file alone (no seeds, no synthetic specs)
    reproduces the reference executor's greedy continuation and logits."""
    import torch

    from pyrite_b200 import gguf
    from pyrite_b200.kernels import cuda as K
    from tests.test_gpu_decode import LOGIT_TOL
    golden, path, _ = files[case]
    dec = gguf.load(path, device=cuda_device, max_ctx=512)
    prompt, want = golden["prompt"], golden["generated"]
    got = dec.generate(prompt, len(want))
    assert K.status() == 0
    assert got[len(prompt):] == want
    dec.reset(prompt)
    worst = 0.0
    for top in golden["top_logits"][: len(prompt) + len(want) - 1]:
        dec.run_steps(1)
        logits = dec.logits.double().cpu()
        ids = [i for i, _ in top]
        worst = max(worst, float((logits[ids] - torch.tensor([v for _, v in top], dtype=torch.float64)).abs().max()))
    assert worst <= LOGIT_TOL
