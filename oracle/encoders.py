"""GGML encoders in numpy -- TEST INFRASTRUCTURE, never on the product path.

numpy restatements of the fixture quantizers the reference's tests and scripts
use, so that the benchmark's reference arm (bench.py --impl reference) can
build its inputs without loading libpyrite_b200.so:

  Q8_0            scripts/build_vocab_fixture.py:54-66 (encode_q8_0)
  Q4_K, Q5_K      tests/k_quant.py:61-157 (encode_q4_k / encode_q5_k, naive
                  min/max scales, _pack_k4_scales at :35-49)
  Q6_K            tests/k_quant.py:160-188 (encode_q6_k)
  IQ4_XS          the package's own encoder (the reference has no IQ4_XS
                  quantizer): a signed sub-block scale mapping the value of
                  largest magnitude onto the book's -127 end, a super-block
                  fp16 d with 6-bit signed sub-scales, nearest book entry.

Arithmetic follows the Python originals: fp64 values, Python round() is
round-half-even (np.rint), int() truncates, struct.pack('<e') rounds a double
to binary16 half-even (numpy's float64 -> float16 cast does the same).  The
bytes equal pyrite_b200.quantize's (tests/test_quantize.py checks this), which
in turn equals the reference encoders' (same test file).
"""
from __future__ import annotations

import numpy as np

F16_MAX = 65504.0
IQ4_BOOK = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], dtype=np.float64)
TYPES = (8, 12, 13, 14, 23)
_GEOMETRY = {8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210), 23: (256, 136)}


def _f16_bits(v: np.ndarray) -> np.ndarray:
    """k_quant._f16_bytes: clamp to the half range, round to binary16; little-endian bytes (n, 2)."""
    h = np.clip(v, -F16_MAX, F16_MAX).astype(np.float16)
    return h.view(np.uint8).reshape(-1, 2)


def _f16(v: np.ndarray) -> np.ndarray:
    """k_quant._f16: the clamped half read back as a double."""
    return np.clip(v, -F16_MAX, F16_MAX).astype(np.float16).astype(np.float64)


def _round_half_away(x: np.ndarray) -> np.ndarray:
    """build_vocab_fixture._round_half_away: int(x + 0.5), mirrored for negatives."""
    return np.where(x >= 0, np.trunc(x + 0.5), -np.trunc(-x + 0.5))


def encode_q8_0(v: np.ndarray) -> np.ndarray:
    """Blocks of 32: fp16 d = amax / 127, int8 codes round-half-away(v / d)."""
    b = v.reshape(-1, 32)
    amax = np.abs(b).max(axis=1)
    d = amax / 127.0
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, 1.0 / np.where(d != 0, d, 1.0), 0.0)
    q = np.clip(_round_half_away(b * inv[:, None]), -127, 127).astype(np.int8).view(np.uint8)
    out = np.empty((b.shape[0], 34), dtype=np.uint8)
    out[:, :2] = _f16_bits(d)
    out[:, 2:] = q
    return out.ravel()


def _pack_k4_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """k_quant._pack_k4_scales for (n, 8) 6-bit scales and mins -> (n, 12) bytes."""
    sc = np.clip(sc, 0, 63).astype(np.uint8)
    mn = np.clip(mn, 0, 63).astype(np.uint8)
    s = np.zeros((sc.shape[0], 12), dtype=np.uint8)
    s[:, 0:4] = sc[:, 0:4]
    s[:, 4:8] = mn[:, 0:4]
    s[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mn[:, 4:8] & 0xF) << 4)
    s[:, 0:4] |= (sc[:, 4:8] >> 4) << 6
    s[:, 4:8] |= (mn[:, 4:8] >> 4) << 6
    return s


def _k_levels(b: np.ndarray, qmax: int):
    """Scales, mins and levels of k_quant.encode_q4_k / encode_q5_k for (n, 256) blocks."""
    g = b.reshape(-1, 8, 32)
    lo, hi = g.min(axis=2), g.max(axis=2)
    spread = hi > lo
    scales_f = np.where(spread, (hi - lo) / float(qmax), 0.0)
    mins_f = np.where(spread, -lo, 0.0)
    max_scale, max_min = scales_f.max(axis=1), mins_f.max(axis=1)
    inv_scale = np.where(max_scale > 0, 63.0 / np.where(max_scale > 0, max_scale, 1.0), 0.0)
    inv_min = np.where(max_min > 0, 63.0 / np.where(max_min > 0, max_min, 1.0), 0.0)
    sc = np.rint(inv_scale[:, None] * scales_f)
    mn = np.rint(inv_min[:, None] * mins_f)
    packed = _pack_k4_scales(sc, mn)
    sc_u, mn_u = np.clip(sc, 0, 63), np.clip(mn, 0, 63)  # what _unpack_k4_scales reads back
    d_bits = _f16_bits(np.where(max_scale > 0, max_scale / 63.0, 0.0))
    m_bits = _f16_bits(np.where(max_min > 0, max_min / 63.0, 0.0))
    d = np.where(max_scale > 0, _f16(max_scale / 63.0), 0.0)
    dmin = np.where(max_min > 0, _f16(max_min / 63.0), 0.0)
    step = d[:, None] * sc_u
    offset = dmin[:, None] * mn_u
    with np.errstate(divide="ignore", invalid="ignore"):
        lv = np.clip(np.rint((g + offset[:, :, None]) / np.where(step != 0, step, 1.0)[:, :, None]), 0, qmax)
    lv = np.where((step != 0)[:, :, None], lv, 0).astype(np.uint8).reshape(-1, 256)
    return d_bits, m_bits, packed, lv


def encode_q4_k(v: np.ndarray) -> np.ndarray:
    b = v.reshape(-1, 256)
    d_bits, m_bits, packed, lv = _k_levels(b, 15)
    out = np.empty((b.shape[0], 144), dtype=np.uint8)
    out[:, 0:2], out[:, 2:4], out[:, 4:16] = d_bits, m_bits, packed
    q = lv.reshape(-1, 4, 2, 32)  # 64-value groups: low nibble = first 32, high = next 32
    out[:, 16:] = (q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(-1, 128)
    return out.ravel()


def encode_q5_k(v: np.ndarray) -> np.ndarray:
    b = v.reshape(-1, 256)
    d_bits, m_bits, packed, lv = _k_levels(b, 31)
    out = np.empty((b.shape[0], 176), dtype=np.uint8)
    out[:, 0:2], out[:, 2:4], out[:, 4:16] = d_bits, m_bits, packed
    q = lv.reshape(-1, 4, 2, 32)
    lo, hi = q[:, :, 0, :], q[:, :, 1, :]
    qh = np.zeros((b.shape[0], 32), dtype=np.uint8)
    for n in range(4):  # bits 2n / 2n+1 of qh[j]: the fifth bit of group n's low / high values
        qh |= ((lo[:, n, :] > 15).astype(np.uint8) << (2 * n)) | ((hi[:, n, :] > 15).astype(np.uint8) << (2 * n + 1))
    out[:, 16:48] = qh
    out[:, 48:] = ((lo & 15) | ((hi & 15) << 4)).reshape(-1, 128)
    return out.ravel()


def encode_q6_k(v: np.ndarray) -> np.ndarray:
    b = v.reshape(-1, 256)
    peak = np.abs(b).max(axis=1)
    d_bits = _f16_bits(peak / (64.0 * 31.0))
    step = _f16(peak / (64.0 * 31.0)) * 64.0
    with np.errstate(divide="ignore", invalid="ignore"):
        lv = np.clip(np.rint(b / np.where(step != 0, step, 1.0)[:, None]) + 32, 0, 63)
    lv = np.where((step != 0)[:, None], lv, 32).astype(np.uint8).reshape(-1, 2, 4, 32)  # [half][quarter][i]
    q1, q2, q3, q4 = lv[:, :, 0], lv[:, :, 1], lv[:, :, 2], lv[:, :, 3]
    out = np.zeros((b.shape[0], 210), dtype=np.uint8)
    ql = np.concatenate([(q1 & 15) | ((q3 & 15) << 4), (q2 & 15) | ((q4 & 15) << 4)], axis=2)  # (n, 2, 64)
    out[:, 0:128] = ql.reshape(-1, 128)
    out[:, 128:192] = ((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6)).reshape(-1, 64)
    out[:, 192:208] = 64
    out[:, 208:210] = d_bits
    out[peak <= 0.0] = 0  # an all-zero block is all-zero bytes
    return out.ravel()


def _nearest_code(t: np.ndarray) -> np.ndarray:
    """Index of the IQ4 book entry nearest to t, the first one on ties."""
    return np.argmin(np.abs(t[..., None] - IQ4_BOOK), axis=-1).astype(np.uint8)


def encode_iq4_xs(v: np.ndarray) -> np.ndarray:
    b = v.reshape(-1, 8, 32)
    n = b.shape[0]
    first = np.argmax(np.abs(b), axis=2)  # first value of largest magnitude
    best = np.take_along_axis(b, first[:, :, None], axis=2)[:, :, 0]
    amax = np.abs(b).max(axis=2)
    sub = best / -127.0
    top = (amax / 127.0).max(axis=1)
    d_bits = _f16_bits(np.where(top > 0, top / 31.0, 0.0))
    d = np.where(top > 0, _f16(top / 31.0), 0.0)
    with np.errstate(divide="ignore", invalid="ignore"):
        ls = np.where(d[:, None] > 0, np.clip(32 + np.rint(sub / np.where(d > 0, d, 1.0)[:, None]), 0, 63), 32)
    ls = ls.astype(np.int64)
    dl = d[:, None] * (ls - 32).astype(np.float64)
    with np.errstate(divide="ignore", invalid="ignore"):
        codes = _nearest_code(b / np.where(dl != 0, dl, 1.0)[:, :, None])
    codes = np.where((dl != 0)[:, :, None], codes, 8).astype(np.uint8)
    out = np.zeros((n, 136), dtype=np.uint8)
    out[:, 0:2] = d_bits
    sh = np.zeros(n, dtype=np.uint16)
    for s in range(8):
        out[:, 4 + s // 2] |= ((ls[:, s] & 15) << (4 * (s & 1))).astype(np.uint8)
        sh |= (((ls[:, s] >> 4) & 3) << (2 * s)).astype(np.uint16)
        out[:, 8 + 16 * s:24 + 16 * s] = codes[:, s, :16] | (codes[:, s, 16:] << 4)
    out[:, 2:4] = sh.astype("<u2").view(np.uint8).reshape(n, 2)
    return out.ravel()


_ENCODERS = {8: encode_q8_0, 12: encode_q4_k, 13: encode_q5_k, 14: encode_q6_k, 23: encode_iq4_xs}


def quantize(type_id: int, values, chunk_values: int = 1 << 22) -> bytes:
    """GGML payload of ``values`` (fp64 view of the input), in chunks of whole blocks."""
    if type_id not in _ENCODERS:
        raise ValueError(f"no numpy encoder for GGML type {type_id}")
    bs, _ = _GEOMETRY[type_id]
    v = np.ascontiguousarray(np.asarray(values).ravel())
    if v.size == 0 or v.size % bs:
        raise ValueError(f"type {type_id} needs a multiple of {bs} values, got {v.size}")
    step = max(bs, chunk_values // bs * bs)
    parts = [_ENCODERS[type_id](v[i:i + step].astype(np.float64)) for i in range(0, v.size, step)]
    return np.concatenate(parts).tobytes()
