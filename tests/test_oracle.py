"""Pin the CPU oracle (oracle/ggml_oracle.c) before trusting it.

* Every decoder against the golden vectors made by the reference's own Python
  decoders (pyrite/tensor_ops.py), bit for bit, NaN patterns included.
* matvec against the reference C kernel's outputs stored with them, bit for bit
  (same accumulation order as pyrite/kernels/native.c:541-553).
* When oracle/_ref holds the reference C library built from source, against it
  directly on fresh payloads.
* Known-answer blocks restated from the reference's tests/test_ggml_decoders.py.
* The independent ``gguf`` dequantizer, where it knows the type (<= 1e-6, as in
  test_ggml_decoders.py:68-85).
"""
from __future__ import annotations

import math
import struct

import numpy as np
import pytest

from oracle import oracle as O
from tests.payloads import random_payload

TYPES = [0, 1, 2, 3, 6, 7, 8, 9, 10, 11, 12, 13, 14, 20, 23, 24, 25, 26, 27, 28, 30]
SHAPES = [(2, 512), (3, 1024)]


def test_oracle_type_table_matches_the_reference_set():
    assert O.type_ids() == TYPES
    assert O.geometry(12) == (256, 144)
    assert O.geometry(8) == (32, 34)
    assert O.geometry(23) == (256, 136)


@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("ggml_type", TYPES)
def test_oracle_decoders_equal_golden(golden_decoders, ggml_type, rows, cols):
    key = f"{ggml_type}_{rows}x{cols}"
    payload = golden_decoders[f"payload_{key}"].tobytes()
    got = O.dequantize_rows(ggml_type, payload, rows, cols).ravel()
    want = golden_decoders[f"decoded_{key}"]
    assert np.array_equal(got.view(np.uint64)[~np.isnan(want)], want.view(np.uint64)[~np.isnan(want)])
    assert np.array_equal(np.isnan(got), np.isnan(want))


@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("ggml_type", TYPES)
def test_oracle_matvec_equals_reference_c_golden(golden_decoders, ggml_type, rows, cols):
    key = f"{ggml_type}_{rows}x{cols}"
    if f"matvec_{key}" not in golden_decoders.files:
        pytest.skip("probe payload decodes to non-finite values (reference test skips it too)")
    payload = golden_decoders[f"payload_{key}"].tobytes()
    got = O.matvec(ggml_type, payload, golden_decoders[f"x_{cols}"], rows, cols)
    assert np.array_equal(got, golden_decoders[f"matvec_{key}"])


@pytest.mark.parametrize("ggml_type", TYPES)
def test_oracle_equals_reference_library_on_fresh_payloads(ggml_type):
    if O.reference_lib() is None:
        pytest.skip("oracle/_ref not built (reference source absent on this machine)")
    rows, cols = 5, 2048
    payload = random_payload(ggml_type, rows, cols, seed=ggml_type + 11)
    x = np.random.default_rng(5).normal(0, 1, cols)
    assert np.array_equal(O.matvec(ggml_type, payload, x, rows, cols),
                          O.reference_matvec(ggml_type, payload, x, rows, cols))
    got = O.dequantize_rows(ggml_type, payload, rows, cols)
    ref = O.reference_dequantize_rows(ggml_type, payload, rows, cols)
    assert np.array_equal(got, ref)


def test_oracle_error_codes_follow_the_reference():
    lib = O.oracle_lib()
    x = np.zeros(32)
    out = np.zeros(1)
    pd = O._PD
    buf = np.zeros(34, dtype=np.uint8)
    call = lambda t, n, r, c: lib.oracle_matvec(t, buf.ctypes.data, n, x.ctypes.data_as(pd),  # noqa: E731
                                               out.ctypes.data_as(pd), r, c)
    assert call(8, 34, 1, 32) == 0
    assert call(99, 34, 1, 32) == -1          # unknown type
    assert call(8, 34, 0, 32) == -2           # zero rows
    assert call(8, 34, 1, 33) == -2           # not block aligned
    assert call(8, 33, 1, 32) == -3           # wrong payload length


# ---- known-answer blocks (reference tests/test_ggml_decoders.py) ----------

def _dq(t, payload, count):
    return O.dequantize_rows(t, payload, 1, count).ravel()


def test_q2_k_layout_matches_the_struct():  # test_ggml_decoders.py:112-123
    scales = bytes([0x21] + [0] * 15)
    qs = bytes([0xE4] * 64)
    payload = scales + qs + struct.pack("<ee", 0.5, 0.25)
    v = _dq(10, payload, 256)
    assert v[0] == pytest.approx(0.5 * 1 * (0xE4 & 3) - 0.25 * 2, abs=1e-6)
    assert v[16] == pytest.approx(0.0, abs=1e-6)


def test_bf16_matches_the_definition():  # :156-161
    words = [0x3F80, 0xBF80, 0x4048, 0x0000, 0x7F7F]
    payload = struct.pack("<5H", *words)
    want = [struct.unpack("<f", struct.pack("<I", w << 16))[0] for w in words]
    assert list(_dq(30, payload, 5)) == want


def test_q8_1_is_d_plus_quantized_values():  # :164-168
    payload = struct.pack("<e", 0.5) + struct.pack("<e", 0.25) + bytes([2] * 32)
    assert list(_dq(9, payload, 32)) == [1.0] * 32


def test_q4_0_uses_low_then_high_nibbles():  # :180-184
    payload = struct.pack("<e", 1.0) + bytes([0x80] * 16)
    assert list(_dq(2, payload, 32)) == [-8.0] * 16 + [0.0] * 16


def test_float_decoders_are_exact():  # :171-177
    values = [0.0, -1.5, 3.25, 1e-5]
    as_f32 = list(struct.unpack("<4f", struct.pack("<4f", *values)))
    assert list(_dq(0, struct.pack("<4f", *values), 4)) == as_f32
    assert list(_dq(28, struct.pack("<4d", *values), 4)) == values
    halves = list(struct.unpack("<4e", struct.pack("<4e", *values)))
    assert list(_dq(1, struct.pack("<4e", *values), 4)) == halves


def test_q3_k_known_block():  # :92-108, packing written out by hand
    codes = [32 + v for v in (-16, -12, -8, -4, 0, 4, 8, 12, 15, -15, 3, -3, 7, -7, 11, -11)]
    levels = [(i * 3) % 8 for i in range(256)]
    d = 0.03125
    scales = bytearray(12)
    for j, code in enumerate(codes):
        if j < 8:
            scales[j] |= code & 15
        else:
            scales[j - 8] |= (code & 15) << 4
        scales[8 + j % 4] |= (code >> 4) << (2 * (j // 4))
    hmask = bytearray(32)
    qs = bytearray(64)
    for v in range(256):
        h, g, l = v // 128, (v % 128) // 32, v % 32
        lvl = levels[v]
        if lvl > 3:
            hmask[l] |= 1 << (4 * h + g)
        qs[32 * h + l] |= (lvl & 3) << (2 * g)
    payload = bytes(hmask) + bytes(qs) + bytes(scales) + struct.pack("<e", d)
    got = _dq(11, payload, 256)
    want = []
    for v in range(256):
        k = (v // 128) * 8 + ((v % 128) // 32) * 2 + (v % 32) // 16
        want.append(d * (codes[k] - 32) * (levels[v] - 4))
    assert np.allclose(got, want, atol=1e-6)


LIBRARY_PARITY = [(0, "F32"), (1, "F16"), (2, "Q4_0"), (3, "Q4_1"), (6, "Q5_0"), (7, "Q5_1"),
                  (8, "Q8_0"), (10, "Q2_K"), (11, "Q3_K"), (12, "Q4_K"), (13, "Q5_K"), (14, "Q6_K"),
                  (30, "BF16")]


@pytest.mark.parametrize("ggml_type,name", LIBRARY_PARITY)
def test_oracle_matches_the_gguf_dequantizer(ggml_type, name):  # :68-85 (relative here)
    quants = pytest.importorskip("gguf.quants")
    qtype = getattr(quants.GGMLQuantizationType, name)
    bs, bpb = O.geometry(ggml_type)
    rng = np.random.default_rng(ggml_type * 7919)
    raw = bytearray(rng.integers(0, 256, 3 * bpb, dtype=np.uint8).tobytes())
    for off in range(0, len(raw) - 1, 2):  # sanitise non-finite fp16 words
        if not math.isfinite(struct.unpack_from("<e", raw, off)[0]):
            struct.pack_into("<e", raw, off, 0.5)
    want = quants.dequantize(np.frombuffer(bytes(raw), dtype=np.uint8), qtype).ravel()
    got = _dq(ggml_type, bytes(raw), 3 * bs)
    # gguf decodes in fp32: compare at 1e-6 relative to the value's magnitude
    assert np.all(np.abs(got - want) <= 1e-6 * np.maximum(1.0, np.abs(got)))
