"""Host quantizers: byte identity with the reference's fixture encoders.

The golden bytes were written by the reference's own encoders
(tests/k_quant.py for Q2_K..Q6_K, scripts/build_vocab_fixture.py for Q8_0 and
Q4_0; see tests/golden/make_golden.py) over smooth, Gaussian N(0,0.02) and
edge-case inputs (all-zero block, constant block, a lone spike).  Q4_1, Q5_0
and Q5_1, which the reference tests encode with the gguf package, are
compared with that package's quantizers byte for byte.  IQ4_NL and
IQ4_XS have no reference encoder; their bytes are checked for validity:
decoded by the oracle they land near the input, and the independent gguf
dequantizer decodes them identically.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from pyrite_b200.quantize import gaussian_weights, quantize, quantize_types

REF_TYPES = [2, 8, 10, 11, 12, 13, 14]


def test_quantizer_table():
    assert set(quantize_types()) == {2, 3, 6, 7, 8, 10, 11, 12, 13, 14, 20, 23}


def _gguf_inputs():
    rng = np.random.default_rng(1)
    return {
        "gauss": rng.normal(0, 0.02, 32 * 2048).astype(np.float32),
        "uniform": rng.uniform(-3, 3, 32 * 512).astype(np.float32),
        "zeros": np.zeros(32 * 4, np.float32),
        "constant": np.full(32 * 4, 0.25, np.float32),
        "ties": np.tile(np.array([1.0, -1.0] * 16, np.float32), 4),
        "huge": rng.normal(0, 3e4, 32 * 64).astype(np.float32),   # the stored min overflows binary16
        "tiny": rng.normal(0, 1e-6, 32 * 64).astype(np.float32),  # subnormal scales
    }


@pytest.mark.filterwarnings("ignore::RuntimeWarning")
@pytest.mark.parametrize("ggml_type,gname", [(3, "Q4_1"), (6, "Q5_0"), (7, "Q5_1")])
def test_bytes_equal_the_gguf_quantizer(ggml_type, gname):
    """Q4_1 / Q5_0 / Q5_1 against the gguf package's quantizers (gguf 0.19.0,
    the reference's test oracle for these formats), byte for byte."""
    quants = pytest.importorskip("gguf.quants")
    qtype = getattr(quants.GGMLQuantizationType, gname)
    for name, x in _gguf_inputs().items():
        want = quants.quantize(x.reshape(1, -1), qtype).tobytes()
        assert quantize(ggml_type, x) == want, f"{gname} on {name} inputs"


@pytest.mark.parametrize("name", ["smooth", "gauss", "edge"])
@pytest.mark.parametrize("ggml_type", REF_TYPES)
def test_bytes_equal_the_reference_encoder(golden_encoders, ggml_type, name):
    values = golden_encoders[f"input_{name}"]
    want = golden_encoders[f"enc_{ggml_type}_{name}"].tobytes()
    assert quantize(ggml_type, values) == want


@pytest.mark.parametrize("ggml_type,gname", [(23, "IQ4_XS"), (20, "IQ4_NL")])
def test_iq4_encoders_write_valid_blocks(ggml_type, gname):
    w = gaussian_weights(16, 1024, seed=3)
    payload = quantize(ggml_type, w)
    dec = O.dequantize_rows(ggml_type, payload, 16, 1024).ravel()
    assert np.sqrt(np.mean((dec - w) ** 2)) < 0.1 * np.std(w)
    quants = pytest.importorskip("gguf.quants")
    ref = quants.dequantize(np.frombuffer(payload, dtype=np.uint8), getattr(quants.GGMLQuantizationType, gname))
    assert np.array_equal(ref.ravel().astype(np.float64), dec)


def test_quantizer_rejects_ragged_input():
    with pytest.raises(ValueError):
        quantize(12, np.zeros(255))
    with pytest.raises(ValueError):
        quantize(8, np.zeros(33))


def test_multithreaded_equals_single_threaded():
    w = gaussian_weights(64, 4096, seed=9)
    for t in (8, 12, 14, 23):
        assert quantize(t, w, threads=1) == quantize(t, w, threads=7)


def test_q4_k_m_mix_rule():
    """Q6_K for attn_v, ffn_down of the even layers and the output; Q4_K else;
    the MoE router stays F32."""
    from pyrite_b200.synthetic import DenseSpec, MoESpec, dense_tensor_type, moe_tensor_type
    c3, c4 = DenseSpec.c3(), MoESpec.c4()
    assert dense_tensor_type(c3, "output.weight") == 14
    assert dense_tensor_type(c3, "blk.3.attn_v.weight") == 14
    assert [dense_tensor_type(c3, f"blk.{i}.ffn_down.weight") for i in range(4)] == [14, 12, 14, 12]
    assert dense_tensor_type(c3, "blk.3.attn_q.weight") == 12
    assert dense_tensor_type(DenseSpec.c1(), "blk.0.attn_v.weight") == 8
    assert moe_tensor_type(c4, "blk.0.ffn_gate_inp.weight") == 0
    assert [moe_tensor_type(c4, f"blk.{i}.ffn_down_exps.weight") for i in range(2)] == [14, 12]
    assert moe_tensor_type(c4, "blk.5.ffn_up_exps.weight") == 12


@pytest.mark.parametrize("ggml_type", [8, 12, 13, 14, 23])
def test_numpy_encoders_equal_the_library_quantizer(ggml_type):
    """oracle/encoders.py (the reference arm's input builder, which must not
    load libpyrite_b200.so) writes the same bytes as pyrite_b200.quantize on
    Gaussian weights and on edge blocks (zeros, tiny, huge, constant, ties)."""
    from oracle import encoders as E
    from pyrite_b200.quantize import gaussian_weights, quantize

    rng = np.random.default_rng(ggml_type)
    edge = np.concatenate([np.zeros(256), rng.normal(0, 1, 256) * 1e-6, rng.normal(0, 1, 512) * 300,
                           np.full(256, 0.5), rng.integers(-3, 4, 256).astype(float) * 0.01])
    for v in (gaussian_weights(16, 4096, 11), edge):
        assert E.quantize(ggml_type, v) == quantize(ggml_type, v)
