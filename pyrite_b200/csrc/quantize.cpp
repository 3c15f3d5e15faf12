// quantize.cpp -- host quantizers that write GGML blocks.
//
// Byte-for-byte restatements of the fixture quantizers the reference tests and
// scripts use, so the B200 inputs equal the reference's inputs:
//   Q8_0, Q4_0    scripts/build_vocab_fixture.py:54-92
//   Q4_1, Q5_0, Q5_1  the gguf package's quantizers (the reference's test oracle)
//   Q2_K..Q6_K    tests/k_quant.py:61-285 (naive min/max scale choice)
// plus IQ4_NL / IQ4_XS encoders of our own (the reference has none): a signed
// per-(sub-)block scale that maps the value of largest magnitude onto the
// book's -127 end, for IQ4_XS a super-block fp16 d with 6-bit signed
// sub-scales, and nearest-code-book rounding.
//
// Arithmetic follows the Python originals exactly: values are doubles, Python
// round() is round-half-even (std::nearbyint), int() truncates toward zero,
// struct.pack("<e") rounds a double to binary16 half-even.  Blocks are
// independent, so rows are split over host threads.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/pyrite_b200.h"

namespace {

// Correctly rounded (half-even) double -> binary16.  |v| beyond the largest
// half saturates to +-inf like the IEEE conversion (callers clamp first where
// the Python originals do).
uint16_t to_half(double v) {
  uint16_t sign = std::signbit(v) ? 0x8000 : 0;
  double a = std::fabs(v);
  if (std::isnan(v)) return 0x7e00;
  if (a == 0.0) return sign;
  int e = 0;
  std::frexp(a, &e);  // a = m * 2^e, m in [0.5, 1)
  int E = e - 1;      // a in [2^E, 2^(E+1))
  if (E < -14) {      // subnormal range: units of 2^-24
    double r = std::nearbyint(std::ldexp(a, 24));
    return (uint16_t)(sign | (uint16_t)r);  // r == 1024 is exactly the smallest normal
  }
  double r = std::nearbyint(std::ldexp(a, 10 - E));  // in [1024, 2048]
  if (r >= 2048.0) { r = 1024.0; ++E; }
  if (E > 15) return (uint16_t)(sign | 0x7c00);
  return (uint16_t)(sign | (uint16_t)((E + 15) << 10) | (uint16_t)((int)r - 1024));
}

double half_to_double(uint16_t h) {
  const int e = (h >> 10) & 31, m = h & 1023;
  double v = e == 0 ? std::ldexp((double)m, -24)
                    : e == 31 ? (m ? NAN : INFINITY) : std::ldexp((double)(m | 1024), e - 25);
  return (h & 0x8000) ? -v : v;
}

constexpr double kF16Max = 65504.0;
// tests/k_quant.py:_f16 / _f16_bytes: clamp to the half range, then round.
uint16_t f16_clamped(double v) { return to_half(std::max(-kF16Max, std::min(kF16Max, v))); }

void put16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)(v & 0xff); p[1] = (uint8_t)(v >> 8); }

long long pyround(double x) { return (long long)std::nearbyint(x); }  // Python round()
long long clampll(long long v, long long lo, long long hi) { return std::max(lo, std::min(hi, v)); }

// ---- Q8_0 (build_vocab_fixture.encode_q8_0) ----
void enc_q8_0(const double* v, uint8_t* o) {
  double amax = 0.0;
  for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(v[i]));
  const double d = amax / 127.0;
  const double inv = d != 0.0 ? 1.0 / d : 0.0;
  put16(o, to_half(d));
  for (int i = 0; i < 32; ++i) {
    const double x = v[i] * inv;
    // C roundf: halves away from zero, computed as int(x + 0.5) in double
    long long q = x >= 0 ? (long long)(x + 0.5) : -(long long)(-x + 0.5);
    o[2 + i] = (uint8_t)(clampll(q, -127, 127) & 0xff);
  }
}

// ---- Q4_0 (build_vocab_fixture.encode_q4_0) ----
void enc_q4_0(const double* v, uint8_t* o) {
  double amax = 0.0, best = 0.0;
  for (int i = 0; i < 32; ++i)
    if (amax < std::fabs(v[i])) { amax = std::fabs(v[i]); best = v[i]; }
  const double d = best / -8.0;
  const double inv = d != 0.0 ? 1.0 / d : 0.0;
  put16(o, to_half(d));
  for (int j = 0; j < 16; ++j) {
    const long long lo = clampll((long long)(v[j] * inv + 8.5), 0, 15);
    const long long hi = clampll((long long)(v[j + 16] * inv + 8.5), 0, 15);
    o[2 + j] = (uint8_t)(lo | (hi << 4));
  }
}

// ---- Q4_1, Q5_0, Q5_1 (the gguf package's numpy quantizers, gguf 0.19.0,
// gguf/quants.py Q4_1 / Q5_0 / Q5_1 quantize_blocks: the test oracle the
// reference uses for these formats) ----
// Those run in float32 on float32 input: every step below is one rounded
// float operation in the same order (no contraction: built with
// -ffp-contract=off), truncation toward zero, then the uint8 clip.
// MIN: offset formats (scale over max - min, stored min); otherwise the value
// of largest magnitude (first on ties) maps to -half.  LEVELS: 15 or 31.
template <bool MIN, int LEVELS>
void enc_legacy(const double* v, uint8_t* o) {
  float x[32];
  for (int i = 0; i < 32; ++i) x[i] = (float)v[i];
  float d, lo = 0.0f, bias;
  if constexpr (MIN) {
    float mx = x[0];
    lo = x[0];
    for (int i = 1; i < 32; ++i) {
      mx = std::max(mx, x[i]);
      lo = std::min(lo, x[i]);
    }
    d = (mx - lo) / (float)LEVELS;
    bias = 0.5f;
  } else {
    int imax = 0;
    for (int i = 1; i < 32; ++i)
      if (std::fabs(x[i]) > std::fabs(x[imax])) imax = i;
    d = x[imax] / -(float)((LEVELS + 1) / 2);
    bias = (float)((LEVELS + 1) / 2) + 0.5f;
  }
  const float id = d == 0.0f ? 0.0f : 1.0f / d;
  uint8_t q[32];
  for (int i = 0; i < 32; ++i) {
    const float t = MIN ? (x[i] - lo) * id + bias : x[i] * id + bias;
    q[i] = (uint8_t)std::min<long long>(LEVELS, (long long)std::trunc(t));
  }
  int at = 2;
  put16(o, to_half((double)d));
  if constexpr (MIN) {
    put16(o + 2, to_half((double)lo));
    at = 4;
  }
  if constexpr (LEVELS == 31) {  // fifth bits, value i -> bit i (little-endian words)
    uint32_t qh = 0;
    for (int i = 0; i < 32; ++i) qh |= (uint32_t)((q[i] >> 4) & 1) << i;
    for (int k = 0; k < 4; ++k) o[at + k] = (uint8_t)(qh >> (8 * k));
    at += 4;
  }
  for (int j = 0; j < 16; ++j) o[at + j] = (uint8_t)((q[j] & 15) | ((q[j + 16] & 15) << 4));
}

// 8 (scale, min) 6-bit pairs -> 12 bytes (k_quant._pack_k4_scales)
void pack_k4(const long long (*pairs)[2], uint8_t* s) {
  std::memset(s, 0, 12);
  for (int j = 0; j < 8; ++j) {
    const int sc = (int)clampll(pairs[j][0], 0, 63), mn = (int)clampll(pairs[j][1], 0, 63);
    if (j < 4) {
      s[j] = (uint8_t)sc;
      s[j + 4] = (uint8_t)mn;
    } else {
      s[j + 4] = (uint8_t)((sc & 0xf) | ((mn & 0xf) << 4));
      s[j - 4] |= (uint8_t)((sc >> 4) << 6);
      s[j] |= (uint8_t)((mn >> 4) << 6);
    }
  }
}
void unpack_k4(const uint8_t* s, int j, int& sc, int& mn) {
  if (j < 4) { sc = s[j] & 63; mn = s[j + 4] & 63; }
  else { sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4); mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
}

// ---- Q4_K / Q5_K (k_quant.encode_q4_k / encode_q5_k) ----
template <int QMAX>  // 15 for Q4_K, 31 for Q5_K
void enc_q45_k(const double* v, uint8_t* o) {
  double scales_f[8], mins_f[8];
  for (int g = 0; g < 8; ++g) {
    double lo = v[32 * g], hi = v[32 * g];
    for (int i = 1; i < 32; ++i) { lo = std::min(lo, v[32 * g + i]); hi = std::max(hi, v[32 * g + i]); }
    if (hi > lo) { scales_f[g] = (hi - lo) / (double)QMAX; mins_f[g] = -lo; }
    else { scales_f[g] = 0.0; mins_f[g] = 0.0; }
  }
  double max_scale = scales_f[0], max_min = mins_f[0];
  for (int g = 1; g < 8; ++g) { max_scale = std::max(max_scale, scales_f[g]); max_min = std::max(max_min, mins_f[g]); }
  const double inv_scale = max_scale > 0 ? 63.0 / max_scale : 0.0;
  const double inv_min = max_min > 0 ? 63.0 / max_min : 0.0;
  long long pairs[8][2];
  for (int g = 0; g < 8; ++g) { pairs[g][0] = pyround(inv_scale * scales_f[g]); pairs[g][1] = pyround(inv_min * mins_f[g]); }
  uint8_t packed[12];
  pack_k4(pairs, packed);
  const uint16_t dbits = max_scale > 0 ? f16_clamped(max_scale / 63.0) : 0;
  const uint16_t mbits = max_min > 0 ? f16_clamped(max_min / 63.0) : 0;
  const double d = half_to_double(dbits), dmin = half_to_double(mbits);
  int levels[256] = {0};
  for (int j = 0; j < 8; ++j) {
    int sc, mn;
    unpack_k4(packed, j, sc, mn);
    const double step = d * sc;
    if (step == 0.0) continue;
    const double off = dmin * mn;
    for (int i = 0; i < 32; ++i) levels[32 * j + i] = (int)clampll(pyround((v[32 * j + i] + off) / step), 0, QMAX);
  }
  put16(o, dbits);
  put16(o + 2, mbits);
  std::memcpy(o + 4, packed, 12);
  if (QMAX == 15) {
    uint8_t* qs = o + 16;
    for (int j = 0, k = 0; j < 256; j += 64)
      for (int i = 0; i < 32; ++i) qs[k++] = (uint8_t)(levels[j + i] | (levels[j + i + 32] << 4));
  } else {
    uint8_t* qh = o + 16;
    uint8_t* ql = o + 48;
    std::memset(qh, 0, 32);
    int m1 = 1, m2 = 2, k = 0;
    for (int n = 0; n < 256; n += 64) {
      for (int j = 0; j < 32; ++j) {
        int lo = levels[n + j], hi = levels[n + j + 32];
        if (lo > 15) { lo -= 16; qh[j] |= (uint8_t)m1; }
        if (hi > 15) { hi -= 16; qh[j] |= (uint8_t)m2; }
        ql[k++] = (uint8_t)(lo | (hi << 4));
      }
      m1 <<= 2;
      m2 <<= 2;
    }
  }
}

// ---- Q6_K (k_quant.encode_q6_k) ----
void enc_q6_k(const double* v, uint8_t* o) {
  double peak = 0.0;
  for (int i = 0; i < 256; ++i) peak = std::max(peak, std::fabs(v[i]));
  std::memset(o, 0, 210);
  if (peak <= 0.0) return;
  const uint16_t dbits = f16_clamped(peak / (64.0 * 31.0));
  const double step = half_to_double(dbits) * 64.0;
  int lv[256];
  for (int i = 0; i < 256; ++i)
    // the Python original divides by step (ZeroDivisionError when the half
    // underflows to 0); here such a block encodes as all-zero codes (value 0)
    lv[i] = step != 0.0 ? (int)clampll(pyround(v[i] / step) + 32, 0, 63) : 32;
  uint8_t* ql = o;
  uint8_t* qh = o + 128;
  for (int j = 0; j < 256; j += 128) {
    const int oql = (j / 128) * 64, oqh = (j / 128) * 32;
    for (int i = 0; i < 32; ++i) {
      const int q1 = lv[j + i], q2 = lv[j + i + 32], q3 = lv[j + i + 64], q4 = lv[j + i + 96];
      ql[oql + i] = (uint8_t)((q1 & 0xf) | ((q3 & 0xf) << 4));
      ql[oql + i + 32] = (uint8_t)((q2 & 0xf) | ((q4 & 0xf) << 4));
      qh[oqh + i] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  }
  for (int k = 0; k < 16; ++k) o[192 + k] = 64;
  put16(o + 208, dbits);
}

// ---- Q2_K (k_quant.encode_q2_k) ----
void enc_q2_k(const double* v, uint8_t* o) {
  double lo[16], hi[16], range[16];
  double max_range = 0.0, max_neg = 0.0;
  for (int g = 0; g < 16; ++g) {
    lo[g] = hi[g] = v[16 * g];
    for (int i = 1; i < 16; ++i) { lo[g] = std::min(lo[g], v[16 * g + i]); hi[g] = std::max(hi[g], v[16 * g + i]); }
    range[g] = hi[g] - lo[g];
    max_range = g == 0 ? range[g] : std::max(max_range, range[g]);
    if (lo[g] < 0.0) max_neg = std::max(max_neg, -lo[g]);
  }
  const uint16_t dbits = max_range > 0 ? f16_clamped(max_range / 45.0) : 0;
  const uint16_t mbits = max_neg > 0 ? f16_clamped(max_neg / 15.0) : 0;
  const double d = half_to_double(dbits), dmin = half_to_double(mbits);
  uint8_t* scales = o;
  uint8_t* qs = o + 16;
  std::memset(o, 0, 84);
  for (int g = 0; g < 16; ++g) {
    const int sc = range[g] > 0 ? 15 : 0;
    long long mn = (dmin > 0 && lo[g] < 0.0) ? pyround(-lo[g] / dmin) : 0;
    mn = clampll(mn, 0, 15);
    scales[g] = (uint8_t)((mn << 4) | sc);
    const double step = d * sc, off = dmin * (double)mn;
    const int half = g / 8, shift = 2 * ((g % 8) / 2), base = half * 32 + (g % 2) * 16;
    for (int i = 0; i < 16; ++i) {
      const long long code = step != 0.0 ? clampll(pyround((v[16 * g + i] + off) / step), 0, 3) : 0;
      qs[base + i] |= (uint8_t)(code << shift);
    }
  }
  put16(o + 80, dbits);
  put16(o + 82, mbits);
}

// ---- Q3_K (k_quant.encode_q3_k + pack_q3_k_block) ----
void enc_q3_k(const double* v, uint8_t* o) {
  double lo[16], hi[16], gs[16], peak = 0.0;
  for (int g = 0; g < 16; ++g) {
    lo[g] = hi[g] = v[16 * g];
    for (int i = 1; i < 16; ++i) { lo[g] = std::min(lo[g], v[16 * g + i]); hi[g] = std::max(hi[g], v[16 * g + i]); }
    gs[g] = hi[g] > lo[g] ? (hi[g] - lo[g]) / 7.0 : 0.0;
    peak = g == 0 ? gs[g] : std::max(peak, gs[g]);
  }
  const double d_all = peak > 0 ? half_to_double(f16_clamped(peak / 31.0)) : 0.0;
  int codes[16], levels[256];
  for (int g = 0; g < 16; ++g) {
    codes[g] = d_all > 0 ? (int)clampll(32 + pyround(gs[g] / d_all), 0, 63) : 32;
    for (int i = 0; i < 16; ++i)
      levels[16 * g + i] = hi[g] > lo[g]
                               ? (int)clampll(pyround((v[16 * g + i] - lo[g]) / (hi[g] - lo[g]) * 7.0), 0, 7)
                               : 4;
  }
  std::memset(o, 0, 110);
  uint8_t* hmask = o;
  uint8_t* qs = o + 32;
  uint8_t* sc = o + 96;
  for (int j = 0; j < 16; ++j) {
    const int low = codes[j] & 0xf;
    if (j < 8) sc[j] = (uint8_t)low;
    else sc[j - 8] |= (uint8_t)(low << 4);
    sc[j % 4 + 8] |= (uint8_t)((codes[j] >> 4) << (2 * (j / 4)));
  }
  for (int j = 0; j < 256; ++j)
    if (levels[j] > 3) hmask[j % 32] |= (uint8_t)(1 << (j / 32));
  for (int j = 0; j < 256; j += 128)
    for (int i = 0; i < 32; ++i) {
      auto q = [&](int k) { return levels[k] > 3 ? levels[k] - 4 : levels[k]; };
      qs[j / 4 + i] = (uint8_t)(q(j + i) | (q(j + i + 32) << 2) | (q(j + i + 64) << 4) | (q(j + i + 96) << 6));
    }
  // pack_q3_k_block packs peak / 31 itself (no clamp)
  put16(o + 108, peak > 0 ? to_half(peak / 31.0) : 0);
}

// ---- IQ4_NL / IQ4_XS (own encoders; no reference quantizer exists) ----
const int kBook[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

int nearest_code(double t) {  // index of the book entry nearest to t (first on ties)
  int best = 0;
  double bd = std::fabs(t - kBook[0]);
  for (int k = 1; k < 16; ++k) {
    const double dd = std::fabs(t - kBook[k]);
    if (dd < bd) { bd = dd; best = k; }
  }
  return best;
}

void enc_iq4_nl(const double* v, uint8_t* o) {
  // the value of largest magnitude maps onto the book's -127 end
  double amax = 0.0, best = 0.0;
  for (int i = 0; i < 32; ++i)
    if (std::fabs(v[i]) > amax) { amax = std::fabs(v[i]); best = v[i]; }
  const uint16_t dbits = amax > 0 ? f16_clamped(best / -127.0) : 0;
  const double d = half_to_double(dbits);
  put16(o, dbits);
  for (int i = 0; i < 16; ++i) {
    const int a = d != 0.0 ? nearest_code(v[i] / d) : 8, b = d != 0.0 ? nearest_code(v[16 + i] / d) : 8;
    o[2 + i] = (uint8_t)(a | (b << 4));
  }
}

void enc_iq4_xs(const double* v, uint8_t* o) {
  // signed sub-block scale: the value of largest magnitude maps onto -127
  double sub[8], top = 0.0;
  for (int s = 0; s < 8; ++s) {
    double amax = 0.0, best = 0.0;
    for (int i = 0; i < 32; ++i)
      if (std::fabs(v[32 * s + i]) > amax) { amax = std::fabs(v[32 * s + i]); best = v[32 * s + i]; }
    sub[s] = best / -127.0;
    top = std::max(top, amax / 127.0);
  }
  std::memset(o, 0, 136);
  const uint16_t dbits = top > 0 ? f16_clamped(top / 31.0) : 0;
  const double d = half_to_double(dbits);
  put16(o, dbits);
  uint16_t sh = 0;
  for (int s = 0; s < 8; ++s) {
    const int ls = d > 0 ? (int)clampll(32 + pyround(sub[s] / d), 0, 63) : 32;
    o[4 + s / 2] |= (uint8_t)((ls & 15) << (4 * (s & 1)));
    sh |= (uint16_t)(((ls >> 4) & 3) << (2 * s));
    const double dl = d * (double)(ls - 32);
    for (int i = 0; i < 16; ++i) {
      const int a = dl != 0.0 ? nearest_code(v[32 * s + i] / dl) : 8;
      const int b = dl != 0.0 ? nearest_code(v[32 * s + 16 + i] / dl) : 8;
      o[8 + 16 * s + i] = (uint8_t)(a | (b << 4));
    }
  }
  put16(o + 2, sh);
}

using EncFn = void (*)(const double*, uint8_t*);
struct Enc { int id; int bs; int bpb; EncFn fn; };
const Enc kEncoders[] = {
    {2, 32, 18, enc_q4_0},   {3, 32, 20, enc_legacy<true, 15>}, {6, 32, 22, enc_legacy<false, 31>},
    {7, 32, 24, enc_legacy<true, 31>}, {8, 32, 34, enc_q8_0},  {10, 256, 84, enc_q2_k},   {11, 256, 110, enc_q3_k},
    {12, 256, 144, enc_q45_k<15>}, {13, 256, 176, enc_q45_k<31>}, {14, 256, 210, enc_q6_k},
    {20, 32, 18, enc_iq4_nl}, {23, 256, 136, enc_iq4_xs},
};

}  // namespace

extern "C" int pyrite_quantize(int type_id, const double* src, size_t count, uint8_t* dst, size_t dst_len,
                               int threads) {
  const Enc* e = nullptr;
  for (const Enc& c : kEncoders)
    if (c.id == type_id) e = &c;
  if (!e) return PYRITE_E_TYPE;
  if (count == 0 || count % (size_t)e->bs != 0) return PYRITE_E_SHAPE;
  const size_t nblocks = count / e->bs;
  if (!src || !dst || dst_len != nblocks * (size_t)e->bpb) return PYRITE_E_BUFFER;
  unsigned nt = threads > 0 ? (unsigned)threads : std::max(1u, std::thread::hardware_concurrency());
  nt = (unsigned)std::min<size_t>(nt, std::max<size_t>(1, nblocks / 64));
  auto work = [&](size_t b0, size_t b1) {
    for (size_t b = b0; b < b1; ++b) e->fn(src + b * e->bs, dst + b * e->bpb);
  };
  if (nt <= 1) {
    work(0, nblocks);
  } else {
    std::vector<std::thread> pool;
    for (unsigned t = 0; t < nt; ++t)
      pool.emplace_back(work, nblocks * t / nt, nblocks * (t + 1) / nt);
    for (auto& th : pool) th.join();
  }
  return 0;
}

extern "C" int pyrite_quantize_types(int* ids, size_t capacity) {
  const size_t n = sizeof(kEncoders) / sizeof(kEncoders[0]);
  if (!ids) return (int)n;
  const size_t k = std::min(n, capacity);
  for (size_t i = 0; i < k; ++i) ids[i] = kEncoders[i].id;
  return (int)k;
}
