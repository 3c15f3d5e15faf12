// mv_tile.cu -- batch-1 fused dequantize x matvec for the main GGML formats.
//
// y = W x, the product of the reference's pyrite_matvec
// (pyrite/kernels/native.c:518-555), fp32 out, for every GGML block format:
// Q8_0, Q4_K, Q5_K, Q6_K, IQ4_XS and Q2_K, Q3_K, Q4_0, Q4_1, Q5_0, Q5_1, Q8_1,
// IQ4_NL.  The path is HBM-bound (~2 flop per weight byte); everything here
// serves one goal: stream every weight byte once, at full bandwidth, while
// keeping the per-byte instruction count low.
//
//  * x is prepared once per vector (xprep_kernel): per 32-value block b a
//    scale s_b = max|x|/127 and int8 digits, x ~= s_b (x0 + x1/254 + x2/254^2),
//    plus fp32 sums of x per 16 values.  Codes are multiplied by the digit
//    vectors with dp4a (exact int32 sums); scales and mins are applied once
//    per 16 or 32 values:
//        sum (d*sc*q - m) x = d*sc*(s_b/254)*(254*sum q x0 + sum q x1 [+ sum q x2 / 254]) - m*sum x.
//    The third digit is used only for "wide" blocks (flagged by a negative
//    scale: a few values far below the block's largest, i.e. an outlier
//    channel), where two digits would lose the small values' precision; a
//    CTA adds those terms to its rows after streaming them (wide_pass), and
//    only when x has a wide block, so the streaming loop is the same either way.
//  * A CTA (up to 256 threads) owns whole rows.  Its lanes are split into RS
//    row slots of 16 or a multiple of 32 lanes; lane l of a slot always handles the same units (32-value pieces)
//    of a row, so it loads its x digits once, into registers, for the whole
//    kernel.  Only weights move per row.
//  * Weights are staged through a ring of S shared-memory stages; a stage is
//    RS*M consecutive rows, i.e. one contiguous byte range: 3 stages of up to
//    ~32 KB, or 2 of up to ~48 KB where that doubles the rows per stage,
//    fetched by ONE TMA bulk copy (cp.async.bulk) that completes on the
//    slot's mbarrier.  (Measured on B200: bulk copies below ~4 KB cannot
//    saturate HBM, 16 KB copies stream at ~7 TB/s.)  Lanes then decode their
//    units from shared memory, whatever the block alignment.
//  * Each lane decodes the (scale, min) pairs of its own units, so a unit's
//    header and epilogue are paid once per 64 values (K-quants).
//  * Row sums: a butterfly that reduces M rows at once, then a fixed-order
//    sum of the slot's warps in shared memory (deterministic; any row
//    partition gives bit-identical rows).
//  * With static weights the first stages are requested before waiting for
//    the preceding kernel (programmatic dependent launch), so the weight
//    stream overlaps its tail.  Every mbarrier wait is bounded (2 s); on
//    time-out the kernel sets the device status word and drains its copies.
#include <atomic>

#include "kernels.cuh"
#include "post_ops.cuh"
#include "ptx.cuh"

namespace pyr {
namespace {

using namespace ptx;

__device__ __forceinline__ float half_f(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }
__device__ __forceinline__ uint32_t w4(const uint4& v, int k) { return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w; }

// 32 bytes at a 2-byte aligned shared address, as 8 words (9 aligned loads;
// the extra word lies inside the stage's slack).
__device__ __forceinline__ void lds_32b(uint32_t a, uint32_t (&out)[8]) {
  const uint32_t base = a & ~3u, sh = (a & 3u) * 8;
  uint32_t w[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) w[k] = lds32(base + 4 * k);
#pragma unroll
  for (int k = 0; k < 8; ++k) out[k] = __funnelshift_r(w[k], w[k + 1], sh);
}

}  // namespace

// ---- x preparation ------------------------------------------------------------------
// One warp per 32-value block; lane l owns value l.  Workspace of one column:
// the layout of post_ops.cuh (x0 | x1 | scale | sum16 | x2).
__global__ void __launch_bounds__(256) xprep_kernel(const float* __restrict__ x, long long ldx, int cols, int ncols,
                                                    uint8_t* __restrict__ ws, long long ws_col_bytes) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int nblk = cols / 32;
  const long long gw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long it = gw; it < (long long)nblk * ncols; it += nw) {
    const int c = (int)(it / nblk), b = (int)(it % nblk);
    encode_block(x[c * ldx + 32LL * b + lane], lane, b, cols, ws + c * ws_col_bytes);
  }
}

namespace {

// Q6_K rows of an odd number of super-blocks (a kernel instantiation of its own).
constexpr int kQ6KRealign = 1014;
}  // namespace
template <> struct Geo<1014> { static constexpr int bs = 256, bpb = 210; };
namespace {

struct XView {  // one column of prepared x (global, or this CTA's shared copy)
  const uint8_t* q0;
  const uint8_t* q1;
  const float* scale;  // negative: a wide block (its third digit is used)
  const float* sum16;
  const uint8_t* q2;   // third digits (read by wide_pass only)
};
__device__ __forceinline__ XView xview(const uint8_t* ws, int cols) {
  XView v;
  v.q0 = ws;
  v.q1 = ws + cols;
  v.scale = reinterpret_cast<const float*>(ws + 2LL * cols);
  v.sum16 = v.scale + cols / 32;
  v.q2 = ws + x2_offset(cols);
  return v;
}
constexpr float kInv254 = 1.0f / 254.0f;

struct Dig16 { uint4 a, b; };  // 16 digits of each plane
__device__ __forceinline__ Dig16 dig16(const XView& x, int c) {
  Dig16 d;
  d.a = *reinterpret_cast<const uint4*>(x.q0 + c);
  d.b = *reinterpret_cast<const uint4*>(x.q1 + c);
  return d;
}
// 254 * dot(codes, x0) + dot(codes, x1) over 16 values, exact in int32
__device__ __forceinline__ int dot16(const uint32_t (&c)[4], const Dig16& d) {
  // four independent dp4a chains (two per digit plane) for ILP
  int a0 = __dp4a((int)c[0], (int)d.a.x, 0), a1 = __dp4a((int)c[1], (int)d.a.y, 0);
  int b0 = __dp4a((int)c[0], (int)d.b.x, 0), b1 = __dp4a((int)c[1], (int)d.b.y, 0);
  a0 = __dp4a((int)c[2], (int)d.a.z, a0);
  a1 = __dp4a((int)c[3], (int)d.a.w, a1);
  b0 = __dp4a((int)c[2], (int)d.b.z, b0);
  b1 = __dp4a((int)c[3], (int)d.b.w, b1);
  return (a0 + a1) * 254 + (b0 + b1);
}

// As dot16 with the four code bytes read as unsigned (0..255).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dot16u(const uint32_t (&c)[4], const Dig16& d) {
  int a0 = dp4a_us(c[0], d.a.x, 0), a1 = dp4a_us(c[1], d.a.y, 0);
  int b0 = dp4a_us(c[0], d.b.x, 0), b1 = dp4a_us(c[1], d.b.y, 0);
  a0 = dp4a_us(c[2], d.a.z, a0);
  a1 = dp4a_us(c[3], d.a.w, a1);
  b0 = dp4a_us(c[2], d.b.z, b0);
  b1 = dp4a_us(c[3], d.b.w, b1);
  return (a0 + a1) * 254 + (b0 + b1);
}

// Row sums of M per-lane partials with one butterfly over LANES lanes (32: a
// whole warp; 16: each half of a warp separately): at each level a lane keeps
// half of its rows and trades the other half with its partner, so M rows cost
// log2(LANES) + M - 1 shuffles instead of M log2(LANES).  Returns the full sum
// of row (lane % LANES) / (LANES / M) of the lane's LANES-lane group.
template <int M, int LANES>
__device__ __forceinline__ float reduce_rows(const float (&acc)[M], int lane) {
  constexpr int LEVELS = LANES == 32 ? 5 : 4;
  float v[M];
#pragma unroll
  for (int i = 0; i < M; ++i) v[i] = acc[i];
#pragma unroll
  for (int lvl = 0; lvl < LEVELS; ++lvl) {
    const int stride = (LANES / 2) >> lvl;
    const int n = (M >> lvl) > 1 ? (M >> lvl) : 1;  // rows still held
    if (n > 1) {
      const int half = n / 2;
      const bool up = (lane & stride) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = up ? v[i] : v[half + i];
        const float keep = up ? v[half + i] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, stride);
      }
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], stride);
    }
  }
  return v[0];
}

// ---- per-type unit decoders ------------------------------------------------------
// A unit is 32 (or 64) values of one block.  XU: the x data of one unit (the
// two leading digits and the block scales, as magnitudes), held in registers
// for the whole kernel.  dot(blk, j, XU): the unit's contribution to one row;
// blk is the shared address of the unit's block, j the unit's index inside it.
// The third digits of wide blocks are added after the rows (wide_pass).

// Q4_K / Q5_K (native.c:173-197, 410-437).  Unit j = qs bytes 16j..16j+15:
// low nibbles are values 64p+16h+i (sub-block 2p), high nibbles values
// 64p+32+16h+i (sub-block 2p+1), p = j/2, h = j%2.  16-byte aligned blocks.
// 32-value digit words (8 per plane) starting at column c.
struct Dig32 { uint32_t a[8], b[8]; };
__device__ __forceinline__ void dig32(const XView& x, int c, Dig32& d) {
  const Dig16 lo = dig16(x, c), hi = dig16(x, c + 16);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    d.a[k] = w4(lo.a, k); d.a[4 + k] = w4(hi.a, k);
    d.b[k] = w4(lo.b, k); d.b[4 + k] = w4(hi.b, k);
  }
}
// 254 * dot(codes, x0) + dot(codes, x1) over 32 values (exact int32); U: codes
// read as unsigned bytes (0..255) instead of signed
template <bool U>
__device__ __forceinline__ int dot32(const uint32_t (&c)[8], const Dig32& d) {
  int a0 = 0, a1 = 0, b0 = 0, b1 = 0;
#pragma unroll
  for (int k = 0; k < 8; k += 2) {
    if constexpr (U) {
      a0 = dp4a_us(c[k], d.a[k], a0); a1 = dp4a_us(c[k + 1], d.a[k + 1], a1);
      b0 = dp4a_us(c[k], d.b[k], b0); b1 = dp4a_us(c[k + 1], d.b[k + 1], b1);
    } else {
      a0 = __dp4a((int)c[k], (int)d.a[k], a0); a1 = __dp4a((int)c[k + 1], (int)d.a[k + 1], a1);
      b0 = __dp4a((int)c[k], (int)d.b[k], b0); b1 = __dp4a((int)c[k + 1], (int)d.b[k + 1], b1);
    }
  }
  return (a0 + a1) * 254 + (b0 + b1);
}

// Q4_K / Q5_K (native.c:173-197, 410-437).  A unit is 64 values: pair p of
// sub-blocks = qs bytes 32p..32p+31, whose low nibbles are values 64p+i
// (sub-block 2p) and high nibbles values 64p+32+i (sub-block 2p+1); Q5_K adds
// bits 2p and 2p+1 of qh[i].  The lane decodes its own two (scale, min)
// pairs, so the header, the scales and the epilogue are paid once per 64
// values.  16-byte aligned blocks.
template <int TY> struct UnitK45 {
  static constexpr int UPB = 4, VALS = 64;
  struct XU { Dig32 a, b; float sa, sb, ma, mb; };
  __device__ static void load_x(const XView& x, int unit, XU& u, int, bool& wide) {
    const int ca = 256 * (unit >> 2) + 64 * (unit & 3), cb = ca + 32;
    dig32(x, ca, u.a);
    dig32(x, cb, u.b);
    const float sa = *(x.scale + (ca >> 5)), sb = *(x.scale + (cb >> 5));
    wide |= (sa < 0.f) | (sb < 0.f);
    u.sa = fabsf(sa);
    // Q4_K multiplies the high nibbles in place (16 * code): fold the 1/16 here
    u.sb = fabsf(sb) * (TY == Q4_K ? 0.0625f : 1.0f);
    u.ma = *(x.sum16 + (ca >> 4)) + *(x.sum16 + (ca >> 4) + 1);
    u.mb = *(x.sum16 + (cb >> 4)) + *(x.sum16 + (cb >> 4) + 1);
  }
  __device__ static float dot(uint32_t blk, int p, const XU& u, int) {
    const uint4 hdr = lds128(blk);
    const uint32_t qa = blk + (TY == Q4_K ? 16 : 48) + 32 * p;
    const uint4 q0 = lds128(qa), q1 = lds128(qa + 16);
    uint32_t lo[8], hi[8];
    if constexpr (TY == Q5_K) {
      const uint4 h0 = lds128(blk + 16), h1 = lds128(blk + 32);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t q = k < 4 ? w4(q0, k) : w4(q1, k - 4), qh = k < 4 ? w4(h0, k) : w4(h1, k - 4);
        lo[k] = (q & 0x0F0F0F0Fu) | (((qh >> (2 * p)) & 0x01010101u) << 4);
        hi[k] = ((q >> 4) & 0x0F0F0F0Fu) | (((qh >> (2 * p + 1)) & 0x01010101u) << 4);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t q = k < 4 ? w4(q0, k) : w4(q1, k - 4);
        lo[k] = q & 0x0F0F0F0Fu;
        hi[k] = q & 0xF0F0F0F0u;  // 16 * code, read unsigned
      }
    }
    const int ia = dot32<false>(lo, u.a), ib = dot32<TY == Q4_K>(hi, u.b);
    // (scale, min) pairs 2p and 2p+1 (native.c:52-60): for j < 4 bytes j, j+4;
    // for j >= 4 the low 4 bits in byte j+4 and the top 2 in bytes j-4 / j.
    // All eight of each, four per word, without branches (the four lanes of
    // a super-block take different p); a byte permute picks the lane's pair.
    const uint32_t sc_lo = hdr.y & 0x3F3F3F3Fu, mn_lo = hdr.z & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
    const uint32_t mn_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
    const uint32_t sel = (uint32_t)(34 * p + 16);  // bytes 2p, 2p + 1 of (lo, hi)
    const uint32_t scp = __byte_perm(sc_lo, sc_hi, sel), mnp = __byte_perm(mn_lo, mn_hi, sel);
    const uint32_t sca = scp & 0xffu, scb = (scp >> 8) & 0xffu, mna = mnp & 0xffu, mnb = (mnp >> 8) & 0xffu;
    const float d = half_f(hdr.x & 0xffff), dmin = half_f(hdr.x >> 16);
    return d * ((float)sca * u.sa * (float)ia + (float)scb * u.sb * (float)ib) -
           dmin * ((float)mna * u.ma + (float)mnb * u.mb);
  }
};

// Shifted digit words: x digits of a 32-value run laid out to match 9 weight
// words read from the aligned address below a run that starts `mis` bytes
// (0 or 2) past a 4-byte boundary.  Word k covers run bytes 4k-mis..4k-mis+3;
// positions outside the run get digit 0, so the weight bytes there (whatever
// they are) add nothing.  Built once per lane, so the decoder needs no
// funnel shifts.
__device__ __forceinline__ void shift_digits(const uint32_t (&xw)[8], int mis, uint32_t (&sw)[9]) {
#pragma unroll
  for (int k = 0; k < 9; ++k) {
    const uint32_t prev = k > 0 ? xw[k - 1] : 0u, cur = k < 8 ? xw[k] : 0u;
    sw[k] = mis ? __byte_perm(prev, cur, 0x5432) : cur;
  }
}
__device__ __forceinline__ void words8(const Dig16& lo, const Dig16& hi, bool plane_b, uint32_t (&w)[8]) {
  const uint4 a = plane_b ? lo.b : lo.a, c = plane_b ? hi.b : hi.a;
  w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = c.x; w[5] = c.y; w[6] = c.z; w[7] = c.w;
}

// Q8_0: d | int8 qs[32]  (native.c:330-336); Q8_1: d | s | int8 qs[32]
// (native.c:338-344, s unused by the decode).  One unit per block.  34-byte
// Q8_0 blocks sit 0 or 2 bytes past a word boundary; with the lane's digits
// shifted to match, the 9 aligned words feed dp4a directly.
template <int TY>
struct UnitQ8 {
  static constexpr int UPB = 1, VALS = 32, QS = TY == Q8_1 ? 4 : 2, BPB = Geo<TY>::bpb;
  struct XU { uint32_t a[9], b[9]; float s; };
  __device__ static void load_x(const XView& x, int unit, XU& u, int wmod4, bool& wide) {
    const int mis = (wmod4 + BPB * unit + QS) & 3;  // offset of qs past a word boundary
    const Dig16 lo = dig16(x, 32 * unit), hi = dig16(x, 32 * unit + 16);
    uint32_t w[8];
    words8(lo, hi, false, w);
    shift_digits(w, mis, u.a);
    words8(lo, hi, true, w);
    shift_digits(w, mis, u.b);
    const float s = *(x.scale + unit);
    wide |= s < 0.f;
    u.s = fabsf(s);
  }
  __device__ static float dot(uint32_t blk, int, const XU& u, int) {
    const uint32_t base = (blk + QS) & ~3u;
    int a0 = 0, a1 = 0, b0 = 0, b1 = 0;
#pragma unroll
    for (int k = 0; k < 9; k += 2) {
      const uint32_t q = lds32(base + 4 * k);
      a0 = __dp4a((int)q, (int)u.a[k], a0);
      b0 = __dp4a((int)q, (int)u.b[k], b0);
      if (k + 1 < 9) {
        const uint32_t q1 = lds32(base + 4 * k + 4);
        a1 = __dp4a((int)q1, (int)u.a[k + 1], a1);
        b1 = __dp4a((int)q1, (int)u.b[k + 1], b1);
      }
    }
    const float d = half_f(lds16(blk));
    return d * u.s * (float)((a0 + a1) * 254 + (b0 + b1));
  }
};

// Q6_K: ql[128] | qh[64] | int8 scales[16] | d  (native.c:199-225).  Value
// 128h+32t+l has low 4 bits from ql[64h + 32(t&1) + l] (high nibble when
// t >= 2), two high bits from qh[32h+l] >> 2t and int8 scale 8h + 2t + l/16.
// A unit is 64 values, (h, tt) with t = tt and t = tt+2 ("parts" 0 and 1):
// both parts read the same 32 ql bytes (low / high nibbles) and the same 32
// qh bytes, so each byte is loaded once.  Blocks are 2-byte aligned; the
// lane's digits are shifted to its block's alignment (shift_digits) and split
// at l = 16 where the scale changes, so the 9 aligned words of each field
// feed dp4a directly.
//
// REALIGN: rows of an odd number of super-blocks (row_bytes = 2 mod 4)
// alternate between the two 2-byte alignments; a block whose alignment is not
// the one the lane's digits were shifted for has its words realigned by 16
// bits as they are loaded (one word of look-ahead, or of look-behind with a
// zero first word: digit positions outside the run are zero).
template <bool REALIGN>
struct UnitQ6K {
  static constexpr int UPB = 4, VALS = 64;
  // [part][group g: l<16 -> words 0..4, l>=16 -> words 4..8] x 5 words, per plane;
  // mis: the block alignment (0 or 2) the digits are shifted for
  struct XU { uint32_t a[2][10], b[2][10]; float s[2], m[2][2]; int mis; };
  __device__ static void load_x(const XView& x, int unit, XU& u, int wmod4, bool& wide) {
    const int blk = unit >> 2, j = unit & 3, h = j >> 1, tt = j & 1;
    const int mis = (wmod4 + 210 * blk) & 3;  // 0 or 2 (in row 0)
    u.mis = mis;
    const uint32_t m4g0 = mis ? 0x0000FFFFu : 0u, m4g1 = mis ? 0xFFFF0000u : 0xFFFFFFFFu;
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int c = 256 * blk + 128 * h + 64 * p + 32 * tt;
      const Dig16 lo = dig16(x, c), hi = dig16(x, c + 16);
      uint32_t w[8], sw[9];
#pragma unroll
      for (int plane = 0; plane < 2; ++plane) {
        words8(lo, hi, plane == 1, w);
        shift_digits(w, mis, sw);
        uint32_t* dst = plane ? u.b[p] : u.a[p];
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[k] = sw[k];
        dst[4] = sw[4] & m4g0;
        dst[5] = sw[4] & m4g1;
#pragma unroll
        for (int k = 5; k < 9; ++k) dst[k + 1] = sw[k];
      }
      const float s = *(x.scale + (c >> 5));
      wide |= s < 0.f;
      u.s[p] = fabsf(s);
      u.m[p][0] = *(x.sum16 + (c >> 4));
      u.m[p][1] = *(x.sum16 + (c >> 4) + 1);
    }
  }
  __device__ static float dot(uint32_t blk, int j, const XU& u, int) {
    const int h = j >> 1, tt = j & 1;
    uint32_t aql = (blk + 64 * h + 32 * tt) & ~3u, aqh = (blk + 128 + 32 * h) & ~3u;
    uint32_t sh = 0, pq = 0, ph = 0;  // realignment: shift and the word before word k
    if constexpr (REALIGN) {
      const bool flip = (int)(blk & 3u) != u.mis;
      sh = flip ? 16u : 0u;
      if (flip && u.mis == 2) {  // weights 2 bytes before the digits' positions
        aql -= 4;
        aqh -= 4;
      } else {
        pq = lds32(aql);
        ph = lds32(aqh);
      }
    }
    int acc[2][2][2] = {};  // [part][group][plane]
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      uint32_t ql, s;
      if constexpr (REALIGN) {
        const uint32_t nq = lds32(aql + 4 * k + 4), nh = lds32(aqh + 4 * k + 4);
        ql = __funnelshift_r(pq, nq, sh);
        s = __funnelshift_r(ph, nh, sh) >> (2 * tt);
        pq = nq;
        ph = nh;
      } else {
        ql = lds32(aql + 4 * k);
        s = lds32(aqh + 4 * k) >> (2 * tt);
      }
      const uint32_t c0 = (ql & 0x0F0F0F0Fu) | ((s & 0x03030303u) << 4);
      const uint32_t c1 = ((ql >> 4) & 0x0F0F0F0Fu) | (s & 0x30303030u);
      if (k <= 4) {
        acc[0][0][0] = __dp4a((int)c0, (int)u.a[0][k], acc[0][0][0]);
        acc[0][0][1] = __dp4a((int)c0, (int)u.b[0][k], acc[0][0][1]);
        acc[1][0][0] = __dp4a((int)c1, (int)u.a[1][k], acc[1][0][0]);
        acc[1][0][1] = __dp4a((int)c1, (int)u.b[1][k], acc[1][0][1]);
      }
      if (k >= 4) {
        acc[0][1][0] = __dp4a((int)c0, (int)u.a[0][k + 1], acc[0][1][0]);
        acc[0][1][1] = __dp4a((int)c0, (int)u.b[0][k + 1], acc[0][1][1]);
        acc[1][1][0] = __dp4a((int)c1, (int)u.a[1][k + 1], acc[1][1][0]);
        acc[1][1][1] = __dp4a((int)c1, (int)u.b[1][k + 1], acc[1][1][1]);
      }
    }
    const uint32_t sc01 = lds16(blk + 192 + 8 * h + 2 * tt), sc23 = lds16(blk + 196 + 8 * h + 2 * tt);
    float r = 0.f;
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        const int sc = (int)(int8_t)(((p ? sc23 : sc01) >> (8 * g)) & 0xff);
        // codes are 0..63 and value = d * sc * (code - 32)
        const float q = u.s[p] * (float)(acc[p][g][0] * 254 + acc[p][g][1]) - 32.0f * u.m[p][g];
        r = fmaf((float)sc, q, r);
      }
    return half_f(lds16(blk + 208)) * r;
  }
};

// IQ4_XS: d | scales_h | scales_l[4] | qs[128]  (native.c:364-379).  Unit j
// is sub-block j.  Codes index the non-linear book through two 8-entry byte
// permutes whose results sum to the book value (below); looked-up bytes come out
// in the order [lo0, hi0, lo1, hi1], so the x digits are interleaved the same
// way once, when they are loaded.  8-byte aligned blocks.
struct UnitIQ4XS {
  static constexpr int UPB = 8, VALS = 32;
  struct XU { uint32_t a[8], b[8]; float s; };
  __device__ static void load_x(const XView& x, int unit, XU& u, int, bool& wide) {
    const Dig16 lo = dig16(x, 32 * unit), hi = dig16(x, 32 * unit + 16);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      u.a[2 * k] = __byte_perm(w4(lo.a, k), w4(hi.a, k), 0x5140);
      u.a[2 * k + 1] = __byte_perm(w4(lo.a, k), w4(hi.a, k), 0x7362);
      u.b[2 * k] = __byte_perm(w4(lo.b, k), w4(hi.b, k), 0x5140);
      u.b[2 * k + 1] = __byte_perm(w4(lo.b, k), w4(hi.b, k), 0x7362);
    }
    const float s = *(x.scale + unit);
    wide |= s < 0.f;
    u.s = fabsf(s);
  }
  __device__ static float dot(uint32_t blk, int j, const XU& u, int) {
    const uint2 hdr = lds64(blk);  // d | scales_h | scales_l[4]
    const uint2 q01 = lds64(blk + 8 + 16 * j), q23 = lds64(blk + 16 + 16 * j);
    const uint32_t qw[4] = {q01.x, q01.y, q23.x, q23.y};
    // The book as int8: -127 -104 -83 -65 -49 -35 -22 -10 | 1 13 25 38 53 69 89 113.
    // A code used directly as a prmt selector into the lower half (all
    // negative) gives book[code] for codes 0-7 and -1 (the replicated sign)
    // for codes 8-15; the code with bit 3 flipped, into the upper half plus
    // one (all positive), gives 0 for codes 0-7 and book[code] + 1 for 8-15.
    // The two byte vectors sum to book[code], and dp4a is linear, so each
    // goes to dp4a as it is: two permutes per four codes and no select.
    constexpr uint32_t N0 = 0xBFAD9881u, N1 = 0xF6EADDCFu;  // book[0..7]
    constexpr uint32_t P0 = 0x271A0E02u, P1 = 0x725A4636u;  // book[8..15] + 1
    int a = 0, b = 0, a1 = 0, b1 = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t q = qw[k], f = q ^ 0x88888888u;  // prmt reads a selector's low 16 bits
      const uint32_t n0 = prmt_sx(N0, N1, q), p0 = prmt_sx(P0, P1, f);
      const uint32_t n1 = prmt_sx(N0, N1, q >> 16), p1 = prmt_sx(P0, P1, f >> 16);
      a = __dp4a((int)n0, (int)u.a[2 * k], a);
      b = __dp4a((int)n0, (int)u.b[2 * k], b);
      a1 = __dp4a((int)n1, (int)u.a[2 * k + 1], a1);
      b1 = __dp4a((int)n1, (int)u.b[2 * k + 1], b1);
      a = __dp4a((int)p0, (int)u.a[2 * k], a);
      b = __dp4a((int)p0, (int)u.b[2 * k], b);
      a1 = __dp4a((int)p1, (int)u.a[2 * k + 1], a1);
      b1 = __dp4a((int)p1, (int)u.b[2 * k + 1], b1);
    }
    a += a1;
    b += b1;
    const uint32_t sh = hdr.x >> 16;
    const int ls = ((hdr.y >> (4 * j)) & 15) | (int)(((sh >> (2 * j)) & 3u) << 4);
    return half_f(hdr.x & 0xffff) * (float)(ls - 32) * u.s * (float)(a * 254 + b);
  }
};

// The 32-value blocks with 16 bytes of nibble codes (native.c:281-328, 351-358):
//   Q4_0   d | qs[16]              value d*(q - 8)
//   Q4_1   d | m | qs[16]          value d*q + m
//   Q5_0   d | qh[4] | qs[16]      value d*(q5 - 16), q5 = q | bit i of qh << 4
//   Q5_1   d | m | qh[4] | qs[16]  value d*q5 + m
//   IQ4_NL d | qs[16]              value d*book[q]
// Byte i of qs holds value i (low nibble) and value 16+i (high nibble).  One
// unit per block.  The offsets (-8, -16, m) multiply the exact fp32 sum of the
// block's x, so the digit planes see only d*q.  18- and 22-byte blocks sit 0
// or 2 bytes past a word boundary: the five aligned words around qs are
// funnel-shifted by the block's own misalignment (read from its address).
// IQ4_NL looks its codes up as IQ4_XS does (two sign-replicating byte
// permutes summed through dp4a), with the digits interleaved to match.
template <int TY>
struct UnitLegacy {
  static constexpr int UPB = 1, VALS = 32;
  static constexpr int QS = TY == Q4_1 ? 4 : TY == Q5_0 ? 6 : TY == Q5_1 ? 8 : 2;  // offset of qs
  static constexpr bool A4 = Geo<TY>::bpb % 4 == 0;  // blocks keep the row's word alignment
  static constexpr bool NL = TY == IQ4_NL, Q5 = TY == Q5_0 || TY == Q5_1, MIN = TY == Q4_1 || TY == Q5_1;
  struct XU { uint32_t a[8], b[8]; float s, m; };
  __device__ static void load_x(const XView& x, int unit, XU& u, int, bool& wide) {
    const Dig16 lo = dig16(x, 32 * unit), hi = dig16(x, 32 * unit + 16);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if constexpr (NL) {
        u.a[2 * k] = __byte_perm(w4(lo.a, k), w4(hi.a, k), 0x5140);
        u.a[2 * k + 1] = __byte_perm(w4(lo.a, k), w4(hi.a, k), 0x7362);
        u.b[2 * k] = __byte_perm(w4(lo.b, k), w4(hi.b, k), 0x5140);
        u.b[2 * k + 1] = __byte_perm(w4(lo.b, k), w4(hi.b, k), 0x7362);
      } else {
        u.a[k] = w4(lo.a, k); u.a[4 + k] = w4(hi.a, k);
        u.b[k] = w4(lo.b, k); u.b[4 + k] = w4(hi.b, k);
      }
    }
    const float s = *(x.scale + unit);
    wide |= s < 0.f;
    u.s = fabsf(s);
    u.m = *(x.sum16 + 2 * unit) + *(x.sum16 + 2 * unit + 1);
  }
  // bits 4j..4j+3 of v, one per byte (bit 0 of bytes 0..3)
  __device__ static uint32_t spread4(uint32_t v) { return ((v & 15u) * 0x00204081u) & 0x01010101u; }
  __device__ static float dot(uint32_t blk, int, const XU& u, int) {
    uint32_t q[4];
    if constexpr (A4) {
#pragma unroll
      for (int k = 0; k < 4; ++k) q[k] = lds32(blk + QS + 4 * k);
    } else {
      const uint32_t base = (blk + QS) & ~3u, sh = ((blk + QS) & 3u) * 8u;
      uint32_t w[5];
#pragma unroll
      for (int k = 0; k < 5; ++k) w[k] = lds32(base + 4 * k);
#pragma unroll
      for (int k = 0; k < 4; ++k) q[k] = __funnelshift_r(w[k], w[k + 1], sh);
    }
    int a = 0, b = 0, a1 = 0, b1 = 0;
    if constexpr (NL) {
      constexpr uint32_t N0 = 0xBFAD9881u, N1 = 0xF6EADDCFu;  // book[0..7] (see UnitIQ4XS)
      constexpr uint32_t P0 = 0x271A0E02u, P1 = 0x725A4636u;  // book[8..15] + 1
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t f = q[k] ^ 0x88888888u;
        const uint32_t n0 = prmt_sx(N0, N1, q[k]), p0 = prmt_sx(P0, P1, f);
        const uint32_t n1 = prmt_sx(N0, N1, q[k] >> 16), p1 = prmt_sx(P0, P1, f >> 16);
        a = __dp4a((int)n0, (int)u.a[2 * k], a);
        b = __dp4a((int)n0, (int)u.b[2 * k], b);
        a1 = __dp4a((int)n1, (int)u.a[2 * k + 1], a1);
        b1 = __dp4a((int)n1, (int)u.b[2 * k + 1], b1);
        a = __dp4a((int)p0, (int)u.a[2 * k], a);
        b = __dp4a((int)p0, (int)u.b[2 * k], b);
        a1 = __dp4a((int)p1, (int)u.a[2 * k + 1], a1);
        b1 = __dp4a((int)p1, (int)u.b[2 * k + 1], b1);
      }
    } else {
      uint32_t qh = 0;
      if constexpr (Q5) {  // qh sits just before qs (2-byte aligned for Q5_0)
        const uint32_t ha = blk + QS - 4, hb = ha & ~3u;
        qh = (ha & 3u) ? __funnelshift_r(lds32(hb), lds32(hb + 4), (ha & 3u) * 8u) : lds32(hb);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t lo = q[k] & 0x0F0F0F0Fu, hi = (q[k] >> 4) & 0x0F0F0F0Fu;
        if constexpr (Q5) {
          lo |= spread4(qh >> (4 * k)) << 4;
          hi |= spread4(qh >> (16 + 4 * k)) << 4;
        }
        a = __dp4a((int)lo, (int)u.a[k], a);
        b = __dp4a((int)lo, (int)u.b[k], b);
        a1 = __dp4a((int)hi, (int)u.a[4 + k], a1);
        b1 = __dp4a((int)hi, (int)u.b[4 + k], b1);
      }
    }
    const float d = half_f(lds16(blk));
    const float t = u.s * (float)((a + a1) * 254 + (b + b1));
    if constexpr (MIN) return d * t + half_f(lds16(blk + 2)) * u.m;
    else if constexpr (TY == Q4_0) return d * (t - 8.0f * u.m);
    else if constexpr (TY == Q5_0) return d * (t - 16.0f * u.m);
    else return d * t;
  }
};

// Sum over one 16-value sub-block: 254 * dot(codes, x0) + dot(codes, x1), the
// four code words c against digit words k0..k0+3 of one 32-value run.
__device__ __forceinline__ int dot16w(const uint32_t (&c)[8], int k0, const Dig32& d) {
  int a0 = __dp4a((int)c[k0], (int)d.a[k0], 0), a1 = __dp4a((int)c[k0 + 1], (int)d.a[k0 + 1], 0);
  int b0 = __dp4a((int)c[k0], (int)d.b[k0], 0), b1 = __dp4a((int)c[k0 + 1], (int)d.b[k0 + 1], 0);
  a0 = __dp4a((int)c[k0 + 2], (int)d.a[k0 + 2], a0);
  a1 = __dp4a((int)c[k0 + 3], (int)d.a[k0 + 3], a1);
  b0 = __dp4a((int)c[k0 + 2], (int)d.b[k0 + 2], b0);
  b1 = __dp4a((int)c[k0 + 3], (int)d.b[k0 + 3], b1);
  return (a0 + a1) * 254 + (b0 + b1);
}

// Q2_K: scales[16] | qs[64] | d | dmin  (native.c:381-408) and Q3_K: hmask[32]
// | qs[64] | scales[12] | d  (native.c:129-171).  Value 128h+32g+l takes the
// 2-bit code (qs[32h+l] >> 2g) & 3; Q3_K adds bit 4h+g of hmask[l] as bit 2
// and subtracts 4.  A unit is 64 values (h, p), g = 2p and 2p+1: both read the
// same 32 qs (and hmask) bytes, at shifts 4p and 4p+2, so each byte is loaded
// once, and the unit's four 16-value sub-blocks have their scales in four
// consecutive bytes.  The offsets (Q2_K: dmin*m; Q3_K: -4) multiply the exact
// fp32 sums of x.  Q2_K blocks (84 bytes) keep the row's word alignment; Q3_K
// blocks (110 bytes) sit 0 or 2 bytes past a word boundary and their words are
// funnel-shifted by that misalignment, read from the block's address.
template <int TY>
struct UnitK23 {
  static constexpr int UPB = 4, VALS = 64;
  struct XU { Dig32 lo, hi; float slo, shi; float m[4]; };
  __device__ static void load_x(const XView& x, int unit, XU& u, int, bool& wide) {
    const int ca = 256 * (unit >> 2) + 64 * (unit & 3), cb = ca + 32;
    dig32(x, ca, u.lo);
    dig32(x, cb, u.hi);
    const float sa = *(x.scale + (ca >> 5)), sb = *(x.scale + (cb >> 5));
    wide |= (sa < 0.f) | (sb < 0.f);
    u.slo = fabsf(sa);
    u.shi = fabsf(sb);
#pragma unroll
    for (int i = 0; i < 4; ++i) u.m[i] = *(x.sum16 + (ca >> 4) + i);
  }
  __device__ static float dot(uint32_t blk, int j, const XU& u, int) {
    const int h = j >> 1, p = j & 1;
    uint32_t q[8], c0[8], c1[8];
    if constexpr (TY == Q2_K) {
#pragma unroll
      for (int k = 0; k < 8; ++k) q[k] = lds32(blk + 16 + 32 * h + 4 * k);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        c0[k] = (q[k] >> (4 * p)) & 0x03030303u;
        c1[k] = (q[k] >> (4 * p + 2)) & 0x03030303u;
      }
      const uint32_t sc = lds32(blk + 8 * h + 4 * p);  // scale | min << 4, one byte per sub-block
      const uint32_t dd = lds32(blk + 80);             // d | dmin
      const float r = u.slo * ((float)(sc & 15u) * (float)dot16w(c0, 0, u.lo) +
                               (float)((sc >> 8) & 15u) * (float)dot16w(c0, 4, u.lo)) +
                      u.shi * ((float)((sc >> 16) & 15u) * (float)dot16w(c1, 0, u.hi) +
                               (float)((sc >> 24) & 15u) * (float)dot16w(c1, 4, u.hi));
      const float mins = (float)((sc >> 4) & 15u) * u.m[0] + (float)((sc >> 12) & 15u) * u.m[1] +
                         (float)((sc >> 20) & 15u) * u.m[2] + (float)(sc >> 28) * u.m[3];
      return half_f(dd & 0xffffu) * r - half_f(dd >> 16) * mins;
    } else {
      const uint32_t sh = (blk & 3u) * 8u;  // 0 or 16: every field keeps the block's misalignment
      const uint32_t qb = (blk + 32 + 32 * h) & ~3u, hb = blk & ~3u, sb = (blk + 96) & ~3u;
      uint32_t hm[8];
      uint32_t wq = lds32(qb), wh = lds32(hb);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t nq = lds32(qb + 4 * k + 4), nh = lds32(hb + 4 * k + 4);
        q[k] = __funnelshift_r(wq, nq, sh);
        hm[k] = __funnelshift_r(wh, nh, sh);
        wq = nq;
        wh = nh;
      }
      const int hs = 4 * h + 2 * p;  // hmask bit of g = 2p (g = 2p+1: the next bit)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        c0[k] = ((q[k] >> (4 * p)) & 0x03030303u) | (((hm[k] >> hs) & 0x01010101u) << 2);
        c1[k] = ((q[k] >> (4 * p + 2)) & 0x03030303u) | (((hm[k] >> (hs + 1)) & 0x01010101u) << 2);
      }
      // the unit's scales k = 8h+4p .. 8h+4p+3: low 4 bits from bytes 4p..4p+3
      // (low nibbles for h = 0, high for h = 1), high 2 bits from bytes 8..11
      // at shift 2(2h+p); 6-bit values biased by 32
      const uint32_t s0 = lds32(sb), s1 = lds32(sb + 4), s2 = lds32(sb + 8), s3 = lds32(sb + 12);
      const uint32_t lw = p ? __funnelshift_r(s1, s2, sh) : __funnelshift_r(s0, s1, sh);
      const uint32_t hw = __funnelshift_r(s2, s3, sh);
      const uint32_t sc = ((lw >> (4 * h)) & 0x0F0F0F0Fu) | (((hw >> (2 * (2 * h + p))) & 0x03030303u) << 4);
      const float f0 = (float)((int)(sc & 63u) - 32), f1 = (float)((int)((sc >> 8) & 63u) - 32);
      const float f2 = (float)((int)((sc >> 16) & 63u) - 32), f3 = (float)((int)(sc >> 24) - 32);
      const float r = u.slo * (f0 * (float)dot16w(c0, 0, u.lo) + f1 * (float)dot16w(c0, 4, u.lo)) +
                      u.shi * (f2 * (float)dot16w(c1, 0, u.hi) + f3 * (float)dot16w(c1, 4, u.hi));
      const float offs = f0 * u.m[0] + f1 * u.m[1] + f2 * u.m[2] + f3 * u.m[3];
      return half_f(lds16(blk + 108)) * (r - 4.0f * offs);
    }
  }
};

template <int TY> struct UnitOf;
template <> struct UnitOf<Q4_K> { using T = UnitK45<Q4_K>; };
template <> struct UnitOf<Q5_K> { using T = UnitK45<Q5_K>; };
template <> struct UnitOf<Q8_0> { using T = UnitQ8<Q8_0>; };
template <> struct UnitOf<Q8_1> { using T = UnitQ8<Q8_1>; };
template <> struct UnitOf<Q4_0> { using T = UnitLegacy<Q4_0>; };
template <> struct UnitOf<Q4_1> { using T = UnitLegacy<Q4_1>; };
template <> struct UnitOf<Q5_0> { using T = UnitLegacy<Q5_0>; };
template <> struct UnitOf<Q5_1> { using T = UnitLegacy<Q5_1>; };
template <> struct UnitOf<IQ4_NL> { using T = UnitLegacy<IQ4_NL>; };
template <> struct UnitOf<Q2_K> { using T = UnitK23<Q2_K>; };
template <> struct UnitOf<Q3_K> { using T = UnitK23<Q3_K>; };
template <> struct UnitOf<Q6_K> { using T = UnitQ6K<false>; };
template <> struct UnitOf<kQ6KRealign> { using T = UnitQ6K<true>; };
template <> struct UnitOf<IQ4_XS> { using T = UnitIQ4XS; };

// a tile CTA has up to kThreads threads (rs row slots of lps lanes, tile plan);
// a slot's row partials come from its warps, or from its half warp when a
// slot has 16 lanes (kMaxParts partials per row block)
constexpr int kThreads = 256, kWarps = 8, kMaxParts = 16, kMaxRowsPerStage = 64, kMaxStages = 3;
constexpr size_t kMaxTileSmem = 150 * 1024;  // dynamic shared memory a tile CTA may take

// The last CTA to finish (a ticket counter, no waiting) runs one operation on
// the complete output vector y (n = rows values).  Every CTA publishes its
// rows before taking its ticket (__threadfence), so the last one sees them
// all; it reads them through L2 and leaves the counter at zero.
__device__ void run_post(const PostArgs& p, const float* y, int n, float best_v, int best_i) {
  __shared__ double shm[32];
  __shared__ float bv[32];
  __shared__ int bi[32];
  __shared__ int last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  if (p.op == kPostArgmax) {  // this CTA's best row -> its partial slot
    warp_best(best_v, best_i);
    if (lane == 0) {
      bv[warp] = best_v;
      bi[warp] = best_i;
    }
    __syncthreads();
    if (warp == 0) {
      best_v = lane < nw ? bv[lane] : -FLT_MAX;
      best_i = lane < nw ? bi[lane] : 0x7fffffff;
      warp_best(best_v, best_i);
      if (lane == 0) {
        p.pv[blockIdx.x] = best_v;
        p.pi[blockIdx.x] = best_i;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    last = atomicAdd(p.ticket, 1u) == gridDim.x - 1 ? 1 : 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (p.op == kPostRmsnormEncode) {
    block_rmsnorm_encode(y, p.w, n, p.eps, p.out, p.ws, shm);
  } else if (p.op == kPostSiluMulEncode) {
    warps_silu_mul_encode(y, n / 2, p.out, p.ws, warp, nw);
  } else if (p.op == kPostArgmax) {
    float v = -FLT_MAX;
    int idx = 0x7fffffff;
    for (int c = tid; c < (int)gridDim.x; c += (int)blockDim.x) better(v, idx, __ldcg(p.pv + c), __ldcg(p.pi + c));
    warp_best(v, idx);
    if (lane == 0) {
      bv[warp] = v;
      bi[warp] = idx;
    }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < nw; ++w) better(v, idx, bv[w], bi[w]);
      const int q = *p.pos;
      if (q + 1 < p.max_ctx && q + 1 >= p.prompt_len) p.tokens[q + 1] = idx;
      *p.pos = q + 1;
    }
  }
  if (tid == 0) *p.ticket = 0u;
}

struct TileArgs {
  const uint8_t* w;
  size_t row_bytes;
  int rows, cols;
  const uint8_t* ws;  // prepared x
  float* y;
  int rs, lps;      // rs row slots of lps lanes (16 or a multiple of 32); the CTA has rs * lps threads
  int m;            // rows per slot per stage
  int stage_bytes;  // shared bytes per stage (rs*m rows + alignment slack)
  int slots;        // stages in the ring (2 or 3)
  int static_weights;
  int accumulate;   // y += W x (a residual stream) instead of y = W x
  PostArgs post;    // operation run on the whole y by the last CTA to finish
  // routed experts (experts != nullptr): w is a stack of matrices
  // expert_bytes apart, n_sel / n_ids groups of n_experts; the CTAs form n_sel
  // equal groups, group j multiplies matrix experts[j % n_ids] of stack group
  // j / n_ids (the id read on the device) by prepared x number j % n_ids (ws +
  // (j % n_ids) * ws_stride) into y + j * y_stride.
  const int* experts;
  int n_experts, n_sel, n_ids;
  long long expert_bytes, ws_stride, y_stride;
  int x_div;  // id index i takes prepared x number i / x_div
  // x prologue (xmode != 0): every CTA encodes its own copy of x into shared
  // memory from fp32 input instead of reading a prepared workspace --
  // 1: x = xsrc * xnorm / rms(xsrc) (fp64 statistics), 2: x = silu(xsrc[0:cols])
  // * xsrc[cols:2 cols]; CTA 0 also writes the fp32 x to xout when non-null
  int xmode;
  const float* xsrc;
  const float* xnorm;
  double xeps;
  float* xout;
  int xenc_off;  // byte offset of the shared copy in the dynamic shared memory
};

// CTAs per SM each format's register budget allows (launch bounds).
// CTAs per SM the register budget is sized for (65,536 / (256 * this)): Q6_K,
// Q4_K and every lane holding two or more units need more than 80 registers,
// and their stages (32 KB for the 4096 x 14336 shapes) fit two CTAs per SM
// anyway (Q4_K: -3% on 4096 x 14336 with 128 registers, no change elsewhere).
template <int TY, int UL> constexpr int tile_min_blocks() {
  return (TY == Q6_K || TY == kQ6KRealign || TY == Q4_K || TY == Q2_K || TY == Q3_K || UL >= 2) ? 2 : 3;
}

// The part of 32 weights (unit u of block b) that the streaming loop multiplies
// by the encoded x: d*sc*q, without the offsets it applies to the exact fp32
// sums of x (Q4_K / Q5_K: dmin*m, native.c:173-197 and 410-437; Q6_K: the
// -32 of d*sc*(q - 32), native.c:199-225; Q4_0 / Q5_0: the -8 / -16, Q4_1 /
// Q5_1: m, native.c:281-328; Q2_K: dmin*m, native.c:381-408; Q3_K: the -4 of
// d*sc*(q - 4), native.c:129-171).  Q8_0, Q8_1, IQ4_NL and IQ4_XS have no offset.
template <int TY>
__device__ __forceinline__ void code_part(const uint8_t* b, int u, float (&v)[32]) {
  if constexpr (TY == Q2_K) {
    const float d = half_val<float>(ld_u16(b + 80));
    const int h = u >> 2, g = u & 3;
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const int sc = b[8 * h + 2 * g + (l >> 4)] & 15;
      v[l] = d * (float)sc * (float)((b[16 + 32 * h + l] >> (2 * g)) & 3);
    }
  } else if constexpr (TY == Q3_K) {
    const float d = half_val<float>(ld_u16(b + 108));
    const int h = u >> 2, g = u & 3;
    float dl[2];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int k = 8 * h + 2 * g + s;
      const int low = (k < 8) ? (b[96 + k] & 15) : (b[96 + k - 8] >> 4);
      const int high = (b[104 + (k & 3)] >> (2 * (k >> 2))) & 3;
      dl[s] = d * (float)((low | (high << 4)) - 32);
    }
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const int q = ((b[32 + 32 * h + l] >> (2 * g)) & 3) | (((b[l] >> (4 * h + g)) & 1) << 2);
      v[l] = dl[l >> 4] * (float)q;
    }
  } else if constexpr (TY == Q4_0 || TY == Q4_1 || TY == Q5_0 || TY == Q5_1) {
    constexpr int QS = UnitLegacy<TY>::QS;
    const float d = half_val<float>(ld_u16(b));
    const uint32_t qh = (TY == Q5_0 || TY == Q5_1) ? ld_u32(b + QS - 4) : 0u;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int lo = (b[QS + i] & 15) | (int)(((qh >> i) & 1u) << 4);
      const int hi = (b[QS + i] >> 4) | (int)(((qh >> (16 + i)) & 1u) << 4);
      v[i] = d * (float)lo;
      v[16 + i] = d * (float)hi;
    }
  } else if constexpr (TY == Q4_K || TY == Q5_K) {
    int sc, mn;
    k4_scale_min(b + 4, u, sc, mn);
    const float d1 = half_val<float>(ld_u16(b)) * (float)sc;
    const uint8_t* qs = b + (TY == Q4_K ? 16 : 48) + 32 * (u >> 1);
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      int q = (u & 1) ? (qs[l] >> 4) : (qs[l] & 15);
      if constexpr (TY == Q5_K) q += ((b[16 + l] >> u) & 1) ? 16 : 0;
      v[l] = d1 * (float)q;
    }
  } else if constexpr (TY == Q6_K) {
    const float d = half_val<float>(ld_u16(b + 208));
    const int h = u >> 2, t = u & 3;
#pragma unroll
    for (int l = 0; l < 32; ++l) {
      const unsigned lq = b[64 * h + 32 * (t & 1) + l];
      const int low = (t >= 2) ? (int)(lq >> 4) : (int)(lq & 15);
      const int high = (b[128 + 32 * h + l] >> (2 * t)) & 3;
      v[l] = d * (float)(int8_t)b[192 + 8 * h + 2 * t + (l >> 4)] * (float)(low | (high << 4));
    }
  } else {
    decode_unit<TY, float>(b, u, v);
  }
}

// The third digits of the wide blocks of x (negative scales), for the rows a
// CTA owns (stages cta, cta + ncta, ... of rps rows).  Warp 0 lists the wide
// blocks in increasing order in `list` (shared memory: list[0] = count, then
// the block indices).  Then each row takes a group of G lanes (G: the next
// power of two >= the count n, at most 32; a warp serves 32 / G rows at
// once): lane g of a group takes listed blocks g, g + G, ... (one block per
// lane when n <= 32), decodes the d*sc*q part of its 32 weights (code_part,
// fp32) and dots it with the block's third digits; a butterfly over the group
// sums the lanes, and the sum is added to y.  The result does not depend on
// G: a 32-lane butterfly whose lanes past n hold +0 differs from the G-lane
// one only in turning a -0 into +0, which the "+ 0" before the butterfly
// does for G < 32.  (One warp per row left all but n lanes idle: with 683
// rows per CTA this pass cost as much as the streaming loop.)  Runs after
// the rows are final, only when x has a wide block, so the streaming loop
// keeps its registers and instruction mix.
template <int TY>
__device__ __forceinline__ void wide_pass(const uint8_t* wb, size_t row_bytes, int cols, const float* scale,
                                          const uint8_t* q2, float* yb, int cta, int ncta, int rps, int rows, int my,
                                          int* list) {
  constexpr int DT = TY == kQ6KRealign ? (int)Q6_K : TY;  // the format the realigning kernel reads
  constexpr int BS = Geo<DT>::bs, BPB = Geo<DT>::bpb, UPB = BS / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, nblk = cols / 32;
  if (warp == 0) {
    int n = 0;
    for (int b0 = 0; b0 < nblk; b0 += 32) {
      const int b = b0 + lane;
      const bool w = b < nblk && (__float_as_uint(scale[b]) >> 31);
      const unsigned m = __ballot_sync(0xffffffffu, w);
      if (w) list[1 + n + __popc(m & ((1u << lane) - 1u))] = b;
      n += __popc(m);
    }
    if (lane == 0) list[0] = n;
  }
  __syncthreads();
  const int n = list[0];
  int G = 1;
  while (G < n && G < 32) G *= 2;
  const int per_warp = 32 / G, g = lane & (G - 1);  // rows per warp pass; this lane's place in its group
  const int total = my * rps;
  for (int base = warp * per_warp; base < total; base += nw * per_warp) {  // warp-uniform trip count
    const int idx = base + lane / G;
    const int row = idx < total ? (cta + (idx / rps) * ncta) * rps + idx % rps : rows;
    const bool on = row < rows;
    float part = 0.f;
    if (on) {
      const uint8_t* rp = wb + (size_t)row * row_bytes;
      for (int j = g; j < n; j += G) {
        const int b = list[1 + j];
        float w[32];
        code_part<DT>(rp + (size_t)(b / UPB) * BPB, b % UPB, w);
        const int8_t* d2 = reinterpret_cast<const int8_t*>(q2 + 32 * b);
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) t = fmaf(w[i], (float)d2[i], t);
        part = fmaf(-scale[b], t, part);  // a negative scale: its magnitude is s_b / 254
      }
    }
    if (G < 32) part = part + 0.0f;  // -0 -> +0, as the lanes past n of a 32-lane sum do
    for (int o = G / 2; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (on && g == 0) yb[row] += part * kInv254;
  }
}

// HALF: 16-lane row slots, two per warp (rows of at most 16 units; one unit
// per lane), a separate instantiation so the common kernels keep their
// registers.
template <int TY, int UL, int M, bool HALF>
__global__ void __launch_bounds__(kThreads, tile_min_blocks<TY, UL>()) mv_tile_kernel(TileArgs a, int* status) {
  using U = typename UnitOf<TY>::T;
  constexpr int BPB = Geo<TY>::bpb;
  const int S = a.slots;
  extern __shared__ __align__(128) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem + (size_t)S * a.stage_bytes);  // [2][kMaxParts][M]
  uint64_t* bars = reinterpret_cast<uint64_t*>(red + 2 * kMaxParts * M);      // [S] full barriers
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lps = a.lps, slot = tid / lps, ls = tid - slot * lps;
  const int rows_per_stage = M * a.rs;
  const int nstages = (a.rows + rows_per_stage - 1) / rows_per_stage;
  const int units = a.cols / U::VALS;
  // routed experts: CTA group `sel` takes stacked matrix a.experts[sel]
  int cta = blockIdx.x, ncta = gridDim.x, sel = 0;
  if (a.experts) {
    ncta = gridDim.x / a.n_sel;
    sel = blockIdx.x / ncta;
    cta = blockIdx.x - sel * ncta;
  }
  const uint8_t* wb = a.w;  // this CTA's matrix (an expert's: set once its id is readable)
  const uint32_t ring = smem_addr(smem);
  const size_t stage_stride = (size_t)rows_per_stage * a.row_bytes;

  auto stage_rows = [&](int st) { return min(rows_per_stage, a.rows - st * rows_per_stage); };
  // the CTA's k-th stage -> ring slot `rs_i` (= k % S, known to the caller
  // without a division), one bulk copy of its contiguous bytes
  auto issue = [&](int k, int rs_i) {  // thread 0
    const int st = cta + k * ncta;
    if (st >= nstages) return;
    const uintptr_t src = (uintptr_t)wb + (uintptr_t)st * stage_stride;
    const uintptr_t al = src & ~(uintptr_t)15;
    const uint32_t len = (uint32_t)(((src - al) + (uintptr_t)stage_rows(st) * a.row_bytes + 15) & ~(uintptr_t)15);
    const uint32_t bar = smem_addr(&bars[rs_i]);
    mbar_expect_tx(bar, len);
    bulk_g2s(ring + (uint32_t)(rs_i * a.stage_bytes), reinterpret_cast<const void*>(al), len, bar);
  };

  const int my = cta < nstages ? (nstages - 1 - cta) / ncta + 1 : 0;
  if (tid == 0) {
    for (int k = 0; k < S; ++k) mbar_init(smem_addr(&bars[k]), 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Weights are read-only: with static weights the first stages stream while
  // the preceding kernel drains; x and y are touched only after pdl_wait().
  const bool early = a.static_weights && !a.experts;
  if (early && tid == 0)
    for (int k = 0; k < min(my, S - 1); ++k) issue(k, k);
  pdl_wait();
  pdl_launch_dependents();
  if (a.experts) {  // written by the routing kernel this one waited for
    const int idn = sel % a.n_ids;
    int eid = a.experts[idn];
    if (eid == -1) return;  // selected, but held by another GPU: nothing issued yet
    if (eid < 0 || eid >= a.n_experts) {  // never read outside the stack
      if (tid == 0) atomicOr(status, (int)kStatusBadExpert);
      eid = 0;
    }
    eid += (sel / a.n_ids) * a.n_experts;
    wb = a.w + (size_t)eid * (size_t)a.expert_bytes;
  }
  const int wmod4 = (int)((uintptr_t)wb & 3);
  float* const yb = a.y + (size_t)sel * (size_t)a.y_stride;
  if (!early && tid == 0)
    for (int k = 0; k < min(my, S - 1); ++k) issue(k, k);

  const uint8_t* xws = a.ws + (size_t)(a.experts ? (sel % a.n_ids) / a.x_div : 0) * (size_t)a.ws_stride;
  if (a.xmode) {  // this CTA's own encoding of x (the input was written by the preceding kernel)
    __shared__ double xshm[32];
    uint8_t* enc = smem + a.xenc_off;
    float* xo = blockIdx.x == 0 ? a.xout : nullptr;
    if (a.xmode == 1) cta_rmsnorm_encode(a.xsrc, a.xnorm, a.cols, a.xeps, xo, enc, xshm);
    else cta_silu_mul_encode(a.xsrc, a.cols, xo, enc);
    __syncthreads();
    xws = enc;
  }
  // this lane's units (inactive ones point at block 0 and are masked out, so
  // every lane runs the same instructions -- the K-quant decode shuffles)
  int uoff[UL], uj[UL];
  float uon[UL];
#pragma unroll
  for (int k = 0; k < UL; ++k) {
    const int u = ls + k * lps;
    uon[k] = u < units ? 1.f : 0.f;
    uoff[k] = u < units ? (u / U::UPB) * BPB : 0;
    uj[k] = u < units ? u % U::UPB : 0;
  }
  typename U::XU xu[UL];  // this lane's x, for the whole kernel
  const XView xv = xview(xws, a.cols);
  bool lane_wide = false;  // a unit of this lane touches a wide block (every unit is some lane's)
#pragma unroll
  for (int k = 0; k < UL; ++k) U::load_x(xv, ls + k * lps < units ? ls + k * lps : 0, xu[k], wmod4, lane_wide);

  float best_v = -FLT_MAX;  // POST_ARGMAX: this thread's best finalized row
  int best_i = 0x7fffffff;
  auto finalize = [&](int k) {  // fixed-order sum of the slot's partials (its warps, or its half warp)
    const int st = cta + k * ncta;
    if (tid < stage_rows(st)) {
      const int s_slot = tid / M, i = tid % M, parts = HALF ? 1 : lps >> 5;
      const float* r = red + (size_t)(k & 1) * kMaxParts * M;
      float v = 0.f;
      for (int w = 0; w < parts; ++w) v += r[(s_slot * parts + w) * M + i];
      float* yp = yb + (size_t)st * rows_per_stage + tid;
      v = a.accumulate ? *yp + v : v;
      *yp = v;
      better(best_v, best_i, v, st * rows_per_stage + tid);
    }
  };

  int k = 0;
  __shared__ int gave_up;
  if (tid == 0) gave_up = 0;
  __syncthreads();
  int ring_i = 0;         // ring slot of stage k (k % S) ...
  uint32_t ring_ph = 0u;  // ... and the phase parity of its barrier ((k / S) & 1)
  for (; k < my; ++k) {
    // stage k landed; the barrier also retires iteration k-1, whose slot the
    // refill below reuses.  A thread whose bounded wait gives up raises the
    // shared flag before the barrier, so every thread leaves the loop at the
    // same iteration.
    if (!mbar_wait_bounded(smem_addr(&bars[ring_i]), ring_ph)) gave_up = 1;
    __syncthreads();
    if (gave_up) {
      if (tid == 0) atomicOr(status, (int)kStatusWaitTimeout);
      break;
    }
    // refill stage k-1's slot (every warp finished it before the barrier) first,
    // then finalize stage k-1's rows from the reduction buffer
    if (tid == 0 && k + S - 1 < my) {
      fence_proxy_async();  // generic reads of the slot precede its async refill
      issue(k + S - 1, ring_i == 0 ? S - 1 : ring_i - 1);
    }
    if (k > 0) finalize(k - 1);
    const int st = cta + k * ncta;
    const int nr = stage_rows(st);
    const uint32_t base = ring + (uint32_t)(ring_i * a.stage_bytes) +
                          (uint32_t)(((uintptr_t)wb + (uintptr_t)st * stage_stride) & 15) +
                          (uint32_t)(slot * M) * (uint32_t)a.row_bytes;
    float acc[M];
#pragma unroll
    for (int i = 0; i < M; ++i) {
      // rows past the matrix end decode stale shared bytes and are dropped
      const float on = slot * M + i < nr ? 1.f : 0.f;
      const uint32_t rowa = base + (uint32_t)i * (uint32_t)a.row_bytes;
      float v = 0.f;
#pragma unroll
      for (int kk = 0; kk < UL; ++kk) v += uon[kk] * U::dot(rowa + (uint32_t)uoff[kk], uj[kk], xu[kk], lane);
      acc[i] = on * v;
    }
    float* r = red + (size_t)(k & 1) * kMaxParts * M;
    if constexpr (!HALF) {  // partial of warp `warp` (part `warp` of slot warp / (lps / 32))
      const float v = reduce_rows<M, 32>(acc, lane);
      if ((lane & (32 / M - 1)) == 0) r[warp * M + lane / (32 / M)] = v;
    } else {  // two 16-lane slots per warp: the partial of slot 2 warp + lane / 16
      const float v = reduce_rows<M, 16>(acc, lane);
      if ((lane & (16 / M - 1)) == 0) r[(2 * warp + (lane >> 4)) * M + (lane & 15) / (16 / M)] = v;
    }
    if (++ring_i == S) {
      ring_i = 0;
      ring_ph ^= 1u;
    }
  }
  __syncthreads();
  if (k == my && my > 0) finalize(my - 1);
  if (k < my && tid == 0) {
    // a copy timed out: wait (bounded) for every copy still in flight
    for (int t = k; t < min(my, k + S - 1); ++t) (void)mbar_wait_bounded(smem_addr(&bars[t % S]), (uint32_t)(t / S) & 1u);
  }
  // x holds a wide block (a negative scale): its third digits are added now
  if (__syncthreads_or(lane_wide) && k == my) {
    // add them to this CTA's rows, then take the argmax post op's candidate
    // again from the corrected rows (the barrier above ordered finalize's writes)
    // (the list of wide blocks goes to the stage ring: every copy has landed and been read)
    // (x's encoding is located again from the arguments, so no pointer to it
    // stays live through the streaming loop)
    const uint8_t* xe = a.xmode ? smem + a.xenc_off
                                : a.ws + (size_t)(a.experts ? (sel % a.n_ids) / a.x_div : 0) * (size_t)a.ws_stride;
    wide_pass<TY>(wb, a.row_bytes, a.cols, reinterpret_cast<const float*>(xe + 2LL * a.cols), xe + x2_offset(a.cols),
                  yb, cta, ncta, rows_per_stage, a.rows, my, reinterpret_cast<int*>(smem));
    __syncthreads();
    if (a.post.op == kPostArgmax) {
      best_v = -FLT_MAX;
      best_i = 0x7fffffff;
      for (int kk = 0; kk < my; ++kk) {
        const int st = cta + kk * ncta;
        if (tid < stage_rows(st)) better(best_v, best_i, yb[(size_t)st * rows_per_stage + tid], st * rows_per_stage + tid);
      }
    }
  }
  if (a.post.op != kPostNone) run_post(a.post, a.y, a.rows, best_v, best_i);
}

struct TilePlan { int rs, lps, m, stage_bytes, slots, ul; size_t smem; int xenc_off; };

TilePlan plan_tile(size_t row_bytes, int rows, int cols, int vals, size_t xenc_bytes) {
  TilePlan p{};
  const int units = cols / vals;
  // a row's units over lps lanes, ul units per lane; lps is the smallest
  // multiple of 32 that holds them (or 16), so no warp of a slot is idle and at most
  // 31 lanes are (14336 columns: 224 or 448 units -> 224 lanes, 7 warps);
  // rs slots of rows side by side fill up to kThreads threads
  // Rows of at most 16 units (64-value units: 1024 columns and less, e.g. the
  // 768-column MoE expert down products) take 16-lane slots, two per warp.
  p.ul = (units + kThreads - 1) / kThreads;
  p.lps = units <= 16 ? 16 : 32 * (((units + p.ul - 1) / p.ul + 31) / 32);
  p.rs = kThreads / p.lps;
  const int rs = p.rs;
  // rows per slot per stage (1, 2, 4 or 8): stages of up to 32 KB amortise the
  // per-stage barrier, copy issue and row reduction; 3 slots keep 2 in flight.
  // Where 48 KB doubles the rows of a stage and the matrix still has a full
  // wave of such stages, 2 slots of the larger stage (the same bytes in
  // flight per SM, half the per-stage work per byte; measured 5-11% faster on
  // the rows x 4096 shapes, and slower where the stage stays the same size).
  // A matrix too small for a full wave of stages keeps 20 KB stages, so more
  // CTAs share it.
  // M is capped by the rows a stage may hold and by the instantiated (UL, M):
  // up to 8 for one unit per lane, 4 for two, 2 for more
  const size_t per = (size_t)rs * row_bytes;
  int max_m = p.ul == 1 ? 8 : p.ul == 2 ? 4 : 2;
  if (rs * max_m > kMaxRowsPerStage) max_m = kMaxRowsPerStage / rs;
  auto m_for = [&](size_t cap) {
    const int m = per * 8 <= cap ? 8 : per * 4 <= cap ? 4 : per * 2 <= cap ? 2 : 1;
    return m < max_m ? m : max_m;
  };
  const long long wave = 148LL * 3;
  p.slots = 3;
  p.m = m_for(32 * 1024);
  const int m48 = m_for(48 * 1024);
  if (m48 > p.m && (long long)rows / ((long long)rs * m48) >= wave) {
    p.m = m48;
    p.slots = 2;
  } else if ((long long)rows / ((long long)rs * p.m) < wave) {
    p.m = m_for(20 * 1024);
  }
  for (;;) {
    const size_t sb = ((size_t)rs * p.m * row_bytes + 16 + 32 + 127) & ~(size_t)127;
    p.stage_bytes = (int)sb;
    p.smem = (size_t)p.slots * sb + 2 * kMaxParts * p.m * sizeof(float) + (size_t)kMaxStages * 8;
    if (xenc_bytes) {
      p.xenc_off = (int)((p.smem + 255) & ~(size_t)255);
      p.smem = (size_t)p.xenc_off + xenc_bytes;
    }
    // a prologue's copy of x shares the CTA's shared memory: smaller stages
    if (p.smem <= kMaxTileSmem || p.m == 1) return p;
    p.m /= 2;
    p.slots = 3;
  }
}

template <int TY, int UL, int M, bool HALF>
int launch_tile_t(const TileArgs& ta, size_t smem, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return -4;
  // First-call caches per device, safe under concurrent callers: both values
  // are idempotent, so two threads racing on a first call only repeat the query.
  static std::atomic<int> sms[64];
  static std::atomic<bool> smem_set[64];
  int nsm = sms[dev].load(std::memory_order_relaxed);
  if (!nsm) {
    if (cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || nsm <= 0)
      return -100 - (int)cudaGetLastError();
    sms[dev].store(nsm, std::memory_order_relaxed);
  }
  constexpr int kMaxSmem = (int)kMaxTileSmem;
  if (!smem_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(mv_tile_kernel<TY, UL, M, HALF>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) !=
        cudaSuccess)
      return -100 - (int)cudaGetLastError();
    smem_set[dev].store(true, std::memory_order_release);
  }
  if (smem > (size_t)kMaxSmem) return 1;
  const int rows_per_stage = M * ta.rs;
  const int nstages = (ta.rows + rows_per_stage - 1) / rows_per_stage;
  int per_sm = (int)((227 * 1024) / (smem + 1024));
  const int minb = tile_min_blocks<TY, UL>();
  if (per_sm > minb) per_sm = minb;
  if (per_sm < 1) per_sm = 1;
  int grid = nsm * per_sm;
  if (ta.experts) {  // n_sel equal CTA groups
    int cpe = grid / ta.n_sel;
    if (cpe > nstages) cpe = nstages;
    if (cpe < 1) cpe = 1;
    grid = cpe * ta.n_sel;
  } else if (grid > nstages) {
    grid = nstages;
  }
  return launch_pdl(mv_tile_kernel<TY, UL, M, HALF>, dim3(grid), dim3(ta.rs * ta.lps), smem, stream, ta,
                    device_status_word());
}

template <int TY>
int launch_tile_type(const TileArgs& ta, int ul, size_t smem, cudaStream_t stream) {
#define PYR_UM(UL_, M_) \
  if (ul == UL_ && ta.m == M_) return launch_tile_t<TY, UL_, M_, false>(ta, smem, stream);
  if (ta.lps == 16) {  // 16-lane slots: one unit per lane, at most 4 rows per slot (16 slots)
    if (ul != 1) return 1;
    if (ta.m == 1) return launch_tile_t<TY, 1, 1, true>(ta, smem, stream);
    if (ta.m == 2) return launch_tile_t<TY, 1, 2, true>(ta, smem, stream);
    if (ta.m == 4) return launch_tile_t<TY, 1, 4, true>(ta, smem, stream);
    return 1;
  }
  PYR_UM(1, 1) PYR_UM(1, 2) PYR_UM(1, 4) PYR_UM(1, 8) PYR_UM(2, 1) PYR_UM(2, 2) PYR_UM(2, 4)
  // three or four units per lane: only 32-value units reach them (rows of at
  // most 32768 columns are at most 512 64-value units, two per lane)
  if constexpr (UnitOf<TY>::T::VALS == 32) {
    PYR_UM(3, 1) PYR_UM(3, 2) PYR_UM(4, 1) PYR_UM(4, 2)
  }
#undef PYR_UM
  return 1;
}

}  // namespace

int lane_max_grid() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return -1;
  return sms * 3;  // tile_min_blocks <= 3 CTAs per SM
}

size_t lane_workspace_bytes(int cols) { return (size_t)encoded_bytes(cols); }

bool lane_supported(int type_id, const uint8_t* w, size_t row_bytes, int cols) {
  if (cols % 256 != 0 || cols / 32 > 4 * kThreads) return false;
  const uintptr_t base = (uintptr_t)w;
  switch (type_id) {
    case Q4_K: case Q5_K: return (base & 15) == 0 && (row_bytes & 15) == 0;
    // the shifted-digit decoders need 2-byte aligned blocks; Q8_0 rows keep the
    // word alignment, Q6_K rows may alternate (a realigning instantiation)
    case Q8_0: case Q8_1: return (base & 1) == 0 && (row_bytes & 3) == 0;
    case Q6_K: return (base & 1) == 0;
    case IQ4_XS: return (base & 7) == 0;
    // 32-value blocks: rows of a multiple of 256 columns are 16-byte multiples;
    // 18 / 22-byte blocks need 2-byte, 20 / 24-byte blocks 4-byte alignment
    case Q4_0: case Q5_0: case IQ4_NL: return (base & 1) == 0;
    case Q4_1: case Q5_1: return (base & 3) == 0;
    // 84-byte Q2_K blocks keep word alignment; 110-byte Q3_K blocks need 2 bytes
    case Q2_K: return (base & 3) == 0;
    case Q3_K: return (base & 1) == 0;
    default: return false;
  }
}

int launch_xprep(const float* x, long long ldx, int cols, int ncols, uint8_t* ws, long long ws_col_bytes,
                 cudaStream_t stream) {
  const long long blocks = (long long)(cols / 32) * ncols;
  int grid = (int)((blocks + 7) / 8);
  if (grid > 148 * 8) grid = 148 * 8;
  if (grid < 1) grid = 1;
  return launch_pdl(xprep_kernel, dim3(grid), dim3(256), 0, stream, x, ldx, cols, ncols, ws, ws_col_bytes);
}

int launch_mv_lane(int type_id, const uint8_t* w, size_t row_bytes, int rows, int cols, const uint8_t* ws,
                   float* y, bool static_weights, cudaStream_t stream, bool accumulate, const PostArgs* post,
                   const ExpertArgs* ex, const XPrologue* xp) {
  const int vals = (type_id == Q6_K || type_id == Q4_K || type_id == Q5_K || type_id == Q2_K || type_id == Q3_K) ? 64 : 32;
  const size_t xenc = xp ? ((lane_workspace_bytes(cols) + 255) & ~(size_t)255) : 0;
  const TilePlan p = plan_tile(row_bytes, rows, cols, vals, xenc);
  TileArgs ta{w, row_bytes, rows, cols, ws, y, p.rs, p.lps, p.m, p.stage_bytes, p.slots, static_weights ? 1 : 0,
              accumulate ? 1 : 0, post ? *post : PostArgs{}, nullptr, 0, 0, 0, 0, 0, 0, 1,
              xp ? xp->mode : 0, xp ? xp->src : nullptr, xp ? xp->norm : nullptr, xp ? xp->eps : 0.0,
              xp ? xp->out : nullptr, p.xenc_off};
  if (ex) {
    ta.experts = ex->ids;
    ta.n_experts = ex->n_experts;
    ta.n_sel = ex->n_sel;
    ta.n_ids = ex->n_ids > 0 ? ex->n_ids : ex->n_sel;
    ta.x_div = ex->x_div > 0 ? ex->x_div : 1;
    ta.expert_bytes = ex->expert_bytes;
    ta.ws_stride = ex->ws_stride;
    ta.y_stride = ex->y_stride;
    ta.static_weights = 0;
  }
  switch (type_id) {
    case Q4_K: return launch_tile_type<Q4_K>(ta, p.ul, p.smem, stream);
    case Q5_K: return launch_tile_type<Q5_K>(ta, p.ul, p.smem, stream);
    case Q8_0: return launch_tile_type<Q8_0>(ta, p.ul, p.smem, stream);
    case Q6_K:
      return (row_bytes & 3) ? launch_tile_type<kQ6KRealign>(ta, p.ul, p.smem, stream)
                             : launch_tile_type<Q6_K>(ta, p.ul, p.smem, stream);
    case IQ4_XS: return launch_tile_type<IQ4_XS>(ta, p.ul, p.smem, stream);
    case Q8_1: return launch_tile_type<Q8_1>(ta, p.ul, p.smem, stream);
    case Q4_0: return launch_tile_type<Q4_0>(ta, p.ul, p.smem, stream);
    case Q4_1: return launch_tile_type<Q4_1>(ta, p.ul, p.smem, stream);
    case Q5_0: return launch_tile_type<Q5_0>(ta, p.ul, p.smem, stream);
    case Q5_1: return launch_tile_type<Q5_1>(ta, p.ul, p.smem, stream);
    case IQ4_NL: return launch_tile_type<IQ4_NL>(ta, p.ul, p.smem, stream);
    case Q2_K: return launch_tile_type<Q2_K>(ta, p.ul, p.smem, stream);
    case Q3_K: return launch_tile_type<Q3_K>(ta, p.ul, p.smem, stream);
    default: return 1;
  }
}

}  // namespace pyr
