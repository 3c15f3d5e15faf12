// mm_tc.cu -- several columns at once: the fused dequantize x matrix product
// on the 5th-generation tensor cores (tcgen05, fp32 accumulators in TMEM).
//
// Y[n, r] = sum_k W[r, k] X[n, k] for ncols = 2..64 columns per pass (the
// reference computes each column with pyrite_matvec, pyrite/kernels/native.c:
// 518-555; batched prefill and multi-sequence decode call it per token).  With
// several columns the product is a real contraction, so it runs on the tensor
// pipe: weights are decoded to bf16 in shared memory and multiplied there.
//
// Precision (the north-star bar is 1e-4 of sum |w x| per row): each fp32
// value v (a decoded weight, or an activation) is split into two bf16 parts,
// v = hi + lo + e with |e| <= 2^-18 |v|, and
//     W X = (Whi + Wlo) (Xhi + Xlo)
// with all four bf16 products accumulated in fp32 (the split remainders stay
// below ~8e-6 of |w x| per term).  Two MMAs per 16 values of K: each weight
// plane times B = [Xhi; Xlo] (2 NP columns); the epilogue adds the halves.
//
// Layout of one CTA (288 threads): a tile of 128 weight rows (the MMA M) x
// NP columns (N, a multiple of 16; padded with zero columns) over a range of
// K.  K advances in stages of 64 values: one 128-byte row of bf16 per matrix
// row, in the 128-byte swizzle layout the MMA reads (8-row atoms of 1 KB,
// 16-byte chunk c of row r stored at chunk c ^ (r % 8)).
//   * warps 0-15 (producers, two groups of 8 warps on alternate stages): raw
//     weight bytes of 256 values per row (a super-block) stream into a ring
//     of shared buffers by 16-byte cp.async, several chunks ahead; each
//     thread then decodes 32 values of one row per stage (exact fp32 values),
//     splits them and writes Whi / Wlo.  The group's first thread also
//     requests the stage's activation tile (Xhi | Xlo, pre-swizzled in global
//     memory by xprep_tc_kernel) with one bulk copy;
//   * the MMA warp owns the TMEM accumulator; one elected lane issues the 8
//     MMAs of each stage (4 K-steps of 16 x 2 weight planes) and commits them
//     to the stage's "empty" barrier, which frees it for the producers;
//   * epilogue: the producer warps read the accumulator (warp w: TMEM lanes
//     32 (w%4), 8 columns at a time).  When K is split over a cluster of CTAs, the
//     partial tiles meet in distributed shared memory and each CTA sums a
//     slice of rows in fixed rank order (deterministic, no atomics).
// Every mbarrier wait is bounded (2 s); on a time-out the kernel records it
// in the device status word, stops waiting, and still drains its copies and
// MMAs before releasing TMEM.
#include <atomic>

#include <cuda_bf16.h>

#include "kernels.cuh"
#include "ptx.cuh"

namespace pyr {
namespace {

using namespace ptx;

constexpr int kTcGroup = 256;                  // one producer group: 8 warps, 2 threads per row
constexpr int kTcProducers = 2 * kTcGroup;     // warps 0-15: two groups on alternate stages
constexpr int kTcMmaWarp = kTcProducers / 32;  // warp 16: TMEM owner and MMA issuer
constexpr int kTcThreads = kTcProducers + 32;
constexpr int kBM = 128;                       // weight rows per tile = MMA M
constexpr int kKC = 64;                        // K values per stage
constexpr int kSC = 256;                       // K values per raw chunk
constexpr uint32_t kAPlane = kBM * 128;        // one bf16 A plane of a stage: 16 KB

struct TcArgs {
  const uint8_t* w;
  size_t row_bytes;
  int rows, cols;
  const uint8_t* xb;  // this column group's pre-swizzled activation planes
  float* y;
  long long ldy;
  int ncols;       // columns of this group (<= NP)
  int chunks;      // raw chunks (256 values) per K split
  int raw_stride;  // bytes per row in a raw buffer (multiple of 16)
  int raw_bufs;    // raw chunk buffers (2..4): chunks in flight ahead of the decoders
  int stages;      // MMA stages in the ring
  int accumulate;  // y += W X instead of y = W X
};

__device__ __forceinline__ uint32_t bf16x2_bits(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // a in the low half
  return *reinterpret_cast<const uint32_t*>(&h);
}
// hi / lo bf16 pairs of (a, b): a = hi_a + lo_a + O(2^-18 a)
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = bf16x2_bits(a, b);
  const float ha = __uint_as_float(hi << 16), hb = __uint_as_float(hi & 0xFFFF0000u);
  lo = bf16x2_bits(a - ha, b - hb);
}

// ---- packed fp32 pairs (sm_100 f32x2 arithmetic) ---------------------------------
typedef unsigned long long u64;
__device__ __forceinline__ u64 pk2(float a, float b) {
  u64 r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(u64 r, float& a, float& b) { asm("mov.b64 {%0,%1}, %2;" : "=f"(a), "=f"(b) : "l"(r)); }
__device__ __forceinline__ u64 add2(u64 a, u64 b) {
  u64 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ u64 sub2(u64 a, u64 b) {
  u64 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ u64 fma2(u64 a, u64 b, u64 c) {
  u64 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float half_f(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }
__device__ __forceinline__ uint32_t w4(const uint4& v, int k) { return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w; }
// 32 bytes at a 2-byte aligned shared address as 8 words (9 aligned loads)
__device__ __forceinline__ void lds_32b(uint32_t a, uint32_t (&out)[8]) {
  const uint32_t base = a & ~3u, sh = (a & 3u) * 8;
  uint32_t w[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) w[k] = lds32(base + 4 * k);
#pragma unroll
  for (int k = 0; k < 8; ++k) out[k] = __funnelshift_r(w[k], w[k + 1], sh);
}

// The 32 values of one unit as unsigned code bytes (word k = values 4k..4k+3):
// value l = (code_l - bias) * s[l / 16] + t[l / 16].  Every format's value is
// an exact or singly rounded fp32 in this form, equal to its exact decoder's.
struct Codes32 {
  uint32_t w[8];
  float s0, s1, t0, t1, bias;
};

// Fast producers: the codes of unit j (values 32j..32j+31) of the 256-value
// chunk at shared address `c` (the data start, whatever its alignment, within
// the rules of tc_fast_ok).  Layouts restate pyrite/kernels/native.c:129-437.
template <int TY> struct TcCodes;
template <int TY> struct TcCodesK45 {  // Q4_K / Q5_K, 16-byte aligned super-block
  __device__ static void get(uint32_t c, int j, Codes32& o) {
    const uint4 hdr = lds128(c);
    const int p = j >> 1, hi = j & 1;
    uint32_t sc, mn;
    if (j < 4) {
      sc = (hdr.y >> (8 * j)) & 63;
      mn = (hdr.z >> (8 * j)) & 63;
    } else {  // native.c:52-60: low 4 bits in bytes 8..11, top 2 in bytes 0..7
      const int k = 8 * (j - 4);
      sc = ((hdr.w >> k) & 15) | (((hdr.y >> k) >> 6 & 3) << 4);
      mn = ((hdr.w >> k) >> 4 & 15) | (((hdr.z >> k) >> 6 & 3) << 4);
    }
    const float d = half_f(hdr.x & 0xffff), dmin = half_f(hdr.x >> 16);
    o.s0 = o.s1 = d * (float)sc;
    o.t0 = o.t1 = -(dmin * (float)mn);
    o.bias = 0.f;
    const uint32_t qa = c + (TY == Q4_K ? 16 : 48) + 32 * p;
    const uint4 q0 = lds128(qa), q1 = lds128(qa + 16);
    uint4 h0 = make_uint4(0, 0, 0, 0), h1 = h0;
    if constexpr (TY == Q5_K) {
      h0 = lds128(c + 16);
      h1 = lds128(c + 32);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t q = k < 4 ? w4(q0, k) : w4(q1, k - 4);
      uint32_t code = (hi ? q >> 4 : q) & 0x0F0F0F0Fu;
      if constexpr (TY == Q5_K) {
        const uint32_t qh = k < 4 ? w4(h0, k) : w4(h1, k - 4);
        code |= ((qh >> j) & 0x01010101u) << 4;
      }
      o.w[k] = code;
    }
  }
};
template <> struct TcCodes<Q4_K> : TcCodesK45<Q4_K> {};
template <> struct TcCodes<Q5_K> : TcCodesK45<Q5_K> {};
template <> struct TcCodes<Q6_K> {  // 2-byte aligned super-block
  __device__ static void get(uint32_t c, int j, Codes32& o) {
    const int hh = j >> 2, t = j & 3;
    uint32_t ql[8], qh[8];
    lds_32b(c + 64 * hh + 32 * (t & 1), ql);
    lds_32b(c + 128 + 32 * hh, qh);
    const uint32_t sc = lds16(c + 192 + 8 * hh + 2 * t);
    const float d = half_f(lds16(c + 208));
    o.s0 = d * (float)(int)(int8_t)(sc & 0xff);
    o.s1 = d * (float)(int)(int8_t)(sc >> 8);
    o.t0 = o.t1 = 0.f;
    o.bias = 32.f;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      o.w[k] = ((ql[k] >> (t >= 2 ? 4 : 0)) & 0x0F0F0F0Fu) | (((qh[k] >> (2 * t)) & 0x03030303u) << 4);
  }
};
template <> struct TcCodes<Q8_0> {  // 2-byte aligned blocks of 34 bytes
  __device__ static void get(uint32_t c, int j, Codes32& o) {
    const uint32_t b = c + 34 * j;
    uint32_t q[8];
    lds_32b(b + 2, q);
    o.s0 = o.s1 = half_f(lds16(b));
    o.t0 = o.t1 = 0.f;
    o.bias = 128.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) o.w[k] = q[k] ^ 0x80808080u;  // int8 -> code + 128
  }
};
template <> struct TcCodes<IQ4_XS> {  // 8-byte aligned super-block
  __device__ static void get(uint32_t c, int j, Codes32& o) {
    const uint2 hdr = lds64(c);  // d | scales_h | scales_l[4]
    const uint2 qa = lds64(c + 8 + 16 * j), qb = lds64(c + 16 + 16 * j);
    const uint32_t qw[4] = {qa.x, qa.y, qb.x, qb.y};
    const uint32_t sh = hdr.x >> 16;
    const int ls = (int)((hdr.y >> (4 * j)) & 15) | (int)(((sh >> (2 * j)) & 3u) << 4);
    o.s0 = o.s1 = half_f(hdr.x & 0xffff) * (float)(ls - 32);
    o.t0 = o.t1 = 0.f;
    o.bias = 128.f;
    // the book as int8: -127 -104 -83 -65 -49 -35 -22 -10 | 1 13 25 38 53 69 89 113
    const uint32_t T0 = 0xBFAD9881u, T1 = 0xF6EADDCFu, T2 = 0x26190D01u, T3 = 0x71594535u;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      // values 4k..4k+3: low nibbles of bytes 4k..4k+3 (k < 4), else high nibbles
      const uint32_t nl = (k < 4 ? qw[k] : qw[k - 4] >> 4) & 0x0F0F0F0Fu;
      const uint32_t n = __byte_perm(nl | (nl >> 4), 0, 0x0020);  // nibble i = code of byte i
      const uint32_t sel = n & 0x7777u;
      const uint32_t v = __byte_perm(__byte_perm(T0, T1, sel), __byte_perm(T2, T3, sel), 0x3210u | ((n & 0x8888u) >> 1));
      o.w[k] = v ^ 0x80808080u;
    }
  }
};

// Alignment the fast producers need of the payload base (rows of these types
// are whole 256-value chunks, so every row keeps the base alignment modulo it).
bool tc_fast_ok(int type_id, const uint8_t* w) {
  const uintptr_t b = (uintptr_t)w;
  switch (type_id) {
    case Q4_K: case Q5_K: return (b & 15) == 0;
    case IQ4_XS: return (b & 7) == 0;
    case Q8_0: case Q6_K: return (b & 1) == 0;
    default: return false;
  }
}

// Byte offset of (row r, 16-byte chunk c) in a 128-byte-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Write a unit's 32 values (natural K order, 16-byte chunks 4h..4h+3 of row r
// of the stage) as the Whi and Wlo planes.
__device__ __forceinline__ void emit_codes(const Codes32& cd, uint32_t a_hi, int r, int h) {
  const float nb = -(8388608.0f + cd.bias);  // (2^23 + code) - (2^23 + bias) = code - bias, exact
  const u64 off2 = pk2(nb, nb);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const u64 sv = c < 2 ? pk2(cd.s0, cd.s0) : pk2(cd.s1, cd.s1);
    const u64 tv = c < 2 ? pk2(cd.t0, cd.t0) : pk2(cd.t1, cd.t1);
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t cw = cd.w[2 * c + (e >> 1)];
      const uint32_t b0 = 2u * (uint32_t)(e & 1);
      const float f0 = __uint_as_float(__byte_perm(cw, 0x4B000000u, 0x7440u + b0));
      const float f1 = __uint_as_float(__byte_perm(cw, 0x4B000000u, 0x7441u + b0));
      const u64 v = fma2(add2(pk2(f0, f1), off2), sv, tv);
      float v0, v1;
      upk2(v, v0, v1);
      hw[e] = bf16x2_bits(v0, v1);
      const float l0 = v0 - __uint_as_float(hw[e] << 16), l1 = v1 - __uint_as_float(hw[e] & 0xFFFF0000u);
      lw[e] = bf16x2_bits(l0, l1);
    }
    const uint32_t off = sw128_off(r, 4 * h + c);
    sts128(a_hi + off, hw[0], hw[1], hw[2], hw[3]);
    sts128(a_hi + kAPlane + off, lw[0], lw[1], lw[2], lw[3]);
  }
}
__device__ __forceinline__ void emit_values(const float (&v)[32], uint32_t a_hi, int r, int h) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) split2(v[8 * c + 2 * e], v[8 * c + 2 * e + 1], hw[e], lw[e]);
    const uint32_t off = sw128_off(r, 4 * h + c);
    sts128(a_hi + off, hw[0], hw[1], hw[2], hw[3]);
    sts128(a_hi + kAPlane + off, lw[0], lw[1], lw[2], lw[3]);
  }
}

template <int TY, int NP, bool FAST>
__global__ void __launch_bounds__(kTcThreads, 1) mm_tc_kernel(TcArgs a, int* status) {
  constexpr int BS = Geo<TY>::bs, BPB = Geo<TY>::bpb, UPB = BS / 32;
  constexpr uint32_t kBPlane = NP * 128;
  constexpr uint32_t kStage = 2 * kAPlane + 2 * kBPlane;
  // one MMA multiplies a weight plane by both activation planes at once: B is
  // the 2 NP rows [Xhi; Xlo], D columns [0, NP) collect W Xhi, [NP, 2 NP) W Xlo
  constexpr uint32_t kIdesc = idesc_bf16_f32(kBM, 2 * NP);
  constexpr uint32_t kTmemCols = 2 * NP < 32 ? 32 : 2 * NP;
  constexpr uint32_t kSeg = (uint32_t)(kSC / BS * BPB);  // raw bytes of one chunk of a row
  constexpr int kSub = kSC / kKC;                        // stages per raw chunk (4)

  extern __shared__ uint8_t smem_raw[];
  const uint32_t base0 = smem_addr(smem_raw);
  const uint32_t sbase = (base0 + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (sbase - base0);
  const int S = a.stages;
  const uint32_t raw_bytes = (uint32_t)kBM * (uint32_t)a.raw_stride;
  const uint32_t raw_off = (uint32_t)S * kStage;
  const int R = a.raw_bufs;
  const uint32_t bar_off = raw_off + (uint32_t)R * raw_bytes;
  const uint32_t bars = sbase + bar_off;  // afull[S] | xfull[S] | empty[S] | accf
  const uint32_t accf = bars + 24u * (uint32_t)S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + bar_off + 24u * (uint32_t)S + 8u);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t ks = cluster_nctarank(), rank = cluster_ctarank();
  const int m0 = (int)(blockIdx.x / ks) * kBM;
  const int nsc_total = a.cols / kSC;
  const int sc0 = (int)rank * a.chunks;
  const int nsc = min(a.chunks, nsc_total - sc0);  // >= 1 (host guarantees)
  const int nst = nsc * kSub;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(bars + 8u * s, kTcGroup);      // A planes written (one producer group)
      mbar_init(bars + 8u * (S + s), 1);       // X planes landed
      mbar_init(bars + 8u * (2 * S + s), 1);   // MMAs done reading
    }
    mbar_init(accf, 1);
    fence_mbar_init();
    *abort_flag = 0;
  }
  if (warp == kTcMmaWarp) {
    tmem_alloc(smem_addr(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_wait();
  pdl_launch_dependents();

  // a bounded wait that gives up at once after any earlier time-out
  auto wait = [&](uint32_t bar, uint32_t parity) {
    if (*abort_flag) return;
    if (!mbar_wait_bounded(bar, parity)) {
      *abort_flag = 1;
      atomicOr(status, (int)kStatusWaitTimeout);
    }
  };

  if (warp < kTcMmaWarp) {
    // ---------------- producers: two groups take alternate stages ----------------
    const int grp = tid / kTcGroup, gt = tid % kTcGroup;
    const int r = gt >> 1, h = gt & 1;
    const int row = m0 + r;
    const uint32_t raw_base = sbase + raw_off;
    const int n16max = a.raw_stride >> 4;
    // raw chunk sc of every row of the tile -> raw[buf]: thread t copies the
    // 16-byte pieces t%4, t%4+4, ... of row t/4
    const int crow = tid >> 2, cq0 = tid & 3;
    auto issue_raw = [&](int sc, int buf) {
      const int grow = m0 + crow;
      if (grow < a.rows) {
        const uintptr_t src = (uintptr_t)a.w + (uintptr_t)grow * a.row_bytes + (uintptr_t)(sc0 + sc) * kSeg;
        const uintptr_t al = src & ~(uintptr_t)15;
        const int n16 = (int)(((src - al) + kSeg + 15) >> 4);
        const uint32_t dst = raw_base + (uint32_t)buf * raw_bytes + (uint32_t)(crow * a.raw_stride);
        for (int q = cq0; q < n16 && q < n16max; q += 4)
          cp_async16(dst + 16u * (uint32_t)q, reinterpret_cast<const void*>(al + 16u * (uintptr_t)q));
      }
      cp_async_commit();
    };
    // chunks 0 .. R-2 in flight before the first decode; one commit group per
    // chunk (empty past the end), so chunk sc is complete once at most R-1
    // groups are pending
    for (int c = 0; c < R - 1; ++c) {
      if (c < nsc) issue_raw(c, c);
      else cp_async_commit();
    }
    // this group's stages g = grp, grp + 2, ... (g = 4 sc + sub): ring slot
    // s = g % S and pass kround = g / S, advanced incrementally (S >= 2)
    int s = grp, kround = 0;
    int buf = 0;  // sc % R
    for (int sc = 0; sc < nsc; ++sc) {
      if (sc > 0) named_bar_sync(1, kTcProducers);  // everyone is done with chunk sc-1's buffer
      const int ahead = sc + R - 1, abuf = buf == 0 ? R - 1 : buf - 1;  // (sc + R - 1) % R
      if (ahead < nsc) issue_raw(ahead, abuf);
      else cp_async_commit();
      if (R == 4) cp_async_wait<3>();
      else if (R == 3) cp_async_wait<2>();
      else cp_async_wait<1>();
      named_bar_sync(1, kTcProducers);  // chunk sc is in raw[buf] for every thread
      const uintptr_t src = (uintptr_t)a.w + (uintptr_t)row * a.row_bytes + (uintptr_t)(sc0 + sc) * kSeg;
      const uint32_t rp = raw_base + (uint32_t)buf * raw_bytes + (uint32_t)(r * a.raw_stride) + (uint32_t)(src & 15);
      if (++buf == R) buf = 0;
#pragma unroll 1
      for (int sub = grp; sub < kSub; sub += 2) {
        // stage g = 4 sc + sub reuses slot s for the kround-th time: wait until
        // the MMAs of its previous use are done reading it
        if (kround > 0) wait(bars + 8u * (2 * S + s), (uint32_t)(kround - 1) & 1u);
        const uint32_t st = sbase + (uint32_t)s * kStage;
        if (gt == 0) {
          const uint32_t xbar = bars + 8u * (S + s);
          mbar_expect_tx(xbar, 2 * kBPlane);
          bulk_g2s(st + 2 * kAPlane, a.xb + (size_t)((sc0 + sc) * kSub + sub) * (2 * kBPlane), 2 * kBPlane, xbar);
        }
        const int unit = sub * 2 + h;  // 32-value unit of the chunk
        if constexpr (FAST) {
          Codes32 cd;
          if (row < a.rows) {
            TcCodes<TY>::get(rp, unit, cd);
          } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) cd.w[k] = 0u;
            cd.s0 = cd.s1 = cd.t0 = cd.t1 = cd.bias = 0.f;
          }
          emit_codes(cd, st, r, h);
        } else {
          float v[32];
          if (row < a.rows) {
            const uint8_t* rb = smem + (rp - sbase);
            decode_unit<TY, float>(rb + (unit / UPB) * BPB, unit % UPB, v);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.f;
          }
          emit_values(v, st, r, h);
        }
        fence_proxy_async();
        mbar_arrive(bars + 8u * s);
        s += 2;  // next stage of this group: g + 2
        if (s >= S) {
          s -= S;
          ++kround;
        }
      }
    }
    cp_async_wait<0>();
  } else {
    // ---------------- MMA issue: the whole warp walks the stages (uniform
    // descriptors), one elected lane issues ----------------
    int s = 0;
    uint32_t par = 0;
    for (int g = 0; g < nst; ++g) {
      wait(bars + 8u * s, par);
      wait(bars + 8u * (S + s), par);
      tc_fence_after();
      const uint32_t st = sbase + (uint32_t)s * kStage;
      if (elect_one()) {
#pragma unroll
        for (int k = 0; k < kKC / 16; ++k) {
          const uint64_t ahi = desc_sw128(st + 32 * k), alo = desc_sw128(st + kAPlane + 32 * k);
          const uint64_t b = desc_sw128(st + 2 * kAPlane + 32 * k);
          tc_mma_bf16(tmem, ahi, b, kIdesc, (g | k) != 0 ? 1u : 0u);
          tc_mma_bf16(tmem, alo, b, kIdesc, 1u);
        }
        tc_commit(bars + 8u * (2 * S + s));
      }
      __syncwarp();
      if (++s == S) {
        s = 0;
        par ^= 1u;
      }
    }
    if (elect_one()) tc_commit(accf);
  }
  __syncwarp();

  // ---------------- epilogue ----------------
  // The accumulator is complete once accf fires (waited on even after a
  // time-out: the MMAs already issued must finish before TMEM is freed).
  if (warp < kTcMmaWarp) {
    if (!mbar_wait_bounded(accf, 0)) atomicOr(status, (int)kStatusWaitTimeout);
    tc_fence_after();
    const uint32_t part = sbase;  // [NP][kBM] fp32 partial tile, over stage 0 (its MMAs are done)
    // work item: (TMEM lane quarter q = warp % 4, 8 columns c0); warp w takes items w, w + 16, ...
    for (int item = warp; item < 4 * (NP / 8); item += kTcMmaWarp) {
      const int q = item & 3, c0 = (item >> 2) * 8;
      const int rl = 32 * q + lane, row = m0 + rl;
      float v[8], vl[8];
      tmem_ld8(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
      tmem_ld8(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(NP + c0), vl);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] += vl[e];
      if (ks == 1) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int n = c0 + e;
          if (n < a.ncols && row < a.rows) {
            float* yp = a.y + (size_t)n * a.ldy + row;
            *yp = a.accumulate ? *yp + v[e] : v[e];
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) sts32f(part + 4u * (uint32_t)((c0 + e) * kBM + rl), v[e]);
      }
    }
  }
  if (ks > 1) {
    cluster_sync();  // every partial tile is in its CTA's shared memory
    const int per = kBM / (int)ks;  // rows this CTA sums
    for (int i = tid; i < per * a.ncols; i += kTcThreads) {
      const int n = i / per, rl = (int)rank * per + (i - n * per);
      const uint32_t addr = sbase + 4u * (uint32_t)(n * kBM + rl);
      float sum = 0.f;
      for (uint32_t src = 0; src < ks; ++src) sum += ld_cluster_f32(addr, src);
      const int row = m0 + rl;
      if (row < a.rows) {
        float* yp = a.y + (size_t)n * a.ldy + row;
        *yp = a.accumulate ? *yp + sum : sum;
      }
    }
    cluster_sync();  // no CTA leaves while another reads its shared memory
  }
  // drain: every activation copy has landed (they all have unless a wait gave up)
  if (tid == 0 && *abort_flag) {
    for (int g = max(0, nst - S); g < nst; ++g)
      (void)mbar_wait_bounded(bars + 8u * (S + g % S), (uint32_t)(g / S) & 1u);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kTcMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- activation planes ----------------------------------------------------------------
// X (ncols x cols fp32, row stride ldx) -> per column group of 64 (NP rows,
// zero padded) and per 64-value K stage: [Xhi | Xlo], each NP rows x 128 bytes
// in the 128-byte swizzle layout, so one bulk copy lands a stage's B operand.
__global__ void __launch_bounds__(256) xprep_tc_kernel(const float* __restrict__ x, long long ldx, int cols,
                                                       int ncols, int np, int ngroups, uint8_t* __restrict__ ws) {
  pdl_wait();
  pdl_launch_dependents();
  const int k8s = cols / 8, nkc = cols / kKC;
  const long long total = (long long)ngroups * np * k8s;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int k8 = (int)(i % k8s);
    const long long gn = i / k8s;
    const int n = (int)(gn % np), g = (int)(gn / np);
    const int col = g * 64 + n;
    float v[8];
    if (col < ncols && n < 64) {
      const float* xp = x + (long long)col * ldx + 8LL * k8;
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = xp[e];
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
    }
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) split2(v[2 * e], v[2 * e + 1], hw[e], lw[e]);
    const int kc = k8 >> 3, c = k8 & 7;
    uint8_t* dst = ws + ((size_t)g * nkc + kc) * (2 * (size_t)np * 128) + sw128_off(n, c);
    *reinterpret_cast<uint4*>(dst) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(dst + (size_t)np * 128) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
}

constexpr size_t kTcSmemMax = 227 * 1024;

int np_for(int ncols) { return ncols <= 16 ? 16 : ncols <= 32 ? 32 : 64; }

template <int TY, int NP, bool FAST>
int launch_tc_t(const TcArgs& ta, int ks, size_t smem, cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -4;
  static std::atomic<bool> smem_set[64];  // idempotent: concurrent first calls only repeat it
  if (!smem_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(mm_tc_kernel<TY, NP, FAST>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmemMax) !=
        cudaSuccess)
      return -100 - (int)cudaGetLastError();
    smem_set[dev].store(true, std::memory_order_release);
  }
  const int m_tiles = (ta.rows + kBM - 1) / kBM;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(m_tiles * ks));
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;  // K split: one cluster per row tile
  attr[1].val.clusterDim.x = (unsigned)ks;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = ks > 1 ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, mm_tc_kernel<TY, NP, FAST>, ta, device_status_word());
  return e == cudaSuccess ? 0 : -100 - (int)e;
}

template <int TY>
int launch_tc_type(const TcArgs& ta, int np, int ks, size_t smem, bool fast, cudaStream_t stream) {
  switch (np * 2 + (fast ? 1 : 0)) {
    case 32: return launch_tc_t<TY, 16, false>(ta, ks, smem, stream);
    case 33: return launch_tc_t<TY, 16, true>(ta, ks, smem, stream);
    case 64: return launch_tc_t<TY, 32, false>(ta, ks, smem, stream);
    case 65: return launch_tc_t<TY, 32, true>(ta, ks, smem, stream);
    case 128: return launch_tc_t<TY, 64, false>(ta, ks, smem, stream);
    case 129: return launch_tc_t<TY, 64, true>(ta, ks, smem, stream);
    default: return 1;
  }
}

}  // namespace

bool tc_supported(int type_id, int cols, int ncols) {
  if (ncols < 2 || cols % kSC != 0) return false;
  switch (type_id) {
    case Q8_0: case Q4_K: case Q5_K: case Q6_K: case IQ4_XS:
      return true;
    default:
      return false;
  }
}

size_t tc_workspace_bytes(int cols, int ncols) {
  const int np = ncols > 64 ? 64 : np_for(ncols);
  const size_t groups = (size_t)(ncols + 63) / 64;
  return groups * (size_t)(cols / kKC) * 2 * (size_t)np * 128;
}

int launch_mm_tc(int type_id, const uint8_t* w, size_t row_bytes, int rows, int cols, const float* x, long long ldx,
                 float* y, long long ldy, int ncols, uint8_t* ws, bool accumulate, cudaStream_t stream) {
  const TypeGeo* t = find_type(type_id);
  if (!t || t->bs < 32) return 1;
  const int np = ncols > 64 ? 64 : np_for(ncols);
  const int ngroups = (ncols + 63) / 64;
  {
    const long long items = (long long)ngroups * np * (cols / 8);
    int grid = (int)((items + 255) / 256);
    if (grid > 148 * 8) grid = 148 * 8;
    const int rc = launch_pdl(xprep_tc_kernel, dim3(grid), dim3(256), 0, stream, x, ldx, cols, ncols, np, ngroups, ws);
    if (rc) return rc;
  }
  // K split over a cluster of ks CTAs: pick the split with the least modelled
  // time, waves x (stages per CTA + ~4 stages of fill and epilogue).
  const int m_tiles = (rows + kBM - 1) / kBM, nsc = cols / kSC;
  int best_ks = 1, best_chunks = nsc;
  long long best_cost = -1;
  for (int ks = 1; ks <= 8; ks *= 2) {
    if (ks > nsc) break;
    const int chunks = (nsc + ks - 1) / ks;
    const int eff_ks = (nsc + chunks - 1) / chunks;
    if (eff_ks != ks) continue;
    const long long waves = ((long long)m_tiles * ks + 147) / 148;
    const long long cost = waves * (4LL * chunks + 4);
    if (best_cost < 0 || cost < best_cost) best_cost = cost, best_ks = ks, best_chunks = chunks;
  }
  const int seg = kSC / t->bs * t->bpb;
  const int raw_stride = ((seg + 30) / 16) * 16;
  // shared memory: as many raw chunks in flight as fit (up to 4), then MMA
  // stages (2..3)
  const size_t stage = 2 * (size_t)kAPlane + 2 * (size_t)np * 128;
  int raw_bufs = 4, stages = 0;
  for (; raw_bufs >= 2; --raw_bufs) {
    const size_t fixed = 1024 /* alignment */ + (size_t)raw_bufs * kBM * raw_stride + 512 /* barriers, slot */;
    stages = fixed < kTcSmemMax ? (int)((kTcSmemMax - fixed) / stage) : 0;
    if (stages >= 2) break;
  }
  if (raw_bufs < 2 || stages < 2) return 1;
  if (stages > 3) stages = 3;
  const size_t smem = 1024 + (size_t)raw_bufs * kBM * raw_stride + 512 + (size_t)stages * stage;
  const size_t group_bytes = (size_t)(cols / kKC) * 2 * (size_t)np * 128;
  for (int g = 0; g < ngroups; ++g) {
    const int ncg = ncols - 64 * g < 64 ? ncols - 64 * g : 64;
    TcArgs ta{w, row_bytes, rows, cols, ws + (size_t)g * group_bytes, y + (size_t)g * 64 * ldy, ldy, ncg,
              best_chunks, raw_stride, raw_bufs, stages, accumulate ? 1 : 0};
    const bool fast = tc_fast_ok(type_id, w);
    int rc;
    switch (type_id) {
      case Q8_0: rc = launch_tc_type<Q8_0>(ta, np, best_ks, smem, fast, stream); break;
      case Q4_K: rc = launch_tc_type<Q4_K>(ta, np, best_ks, smem, fast, stream); break;
      case Q5_K: rc = launch_tc_type<Q5_K>(ta, np, best_ks, smem, fast, stream); break;
      case Q6_K: rc = launch_tc_type<Q6_K>(ta, np, best_ks, smem, fast, stream); break;
      case IQ4_XS: rc = launch_tc_type<IQ4_XS>(ta, np, best_ks, smem, fast, stream); break;
      default: rc = 1;
    }
    if (rc) return rc;
  }
  return 0;
}

}  // namespace pyr
