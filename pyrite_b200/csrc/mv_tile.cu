// mv_tile.cu -- batch-1 fused dequantize x matvec for the main GGML formats.
//
// y = W x, the product of the reference's pyrite_matvec
// (pyrite/kernels/native.c:518-555), fp32 out, for Q8_0, Q4_K, Q5_K, Q6_K and
// IQ4_XS.  The path is HBM-bound (~2 flop per weight byte); everything here
// serves one goal: stream every weight byte once, at full bandwidth, while
// keeping the per-byte instruction count low.
//
//  * x is prepared once per vector (xprep_kernel): per 32-value block b a
//    scale s_b = max|x|/127 and two int8 digits, x ~= s_b (x0 + x1/254)
//    (|error| <= s_b/508 = 1.6e-5 max|x_b|), plus fp32 sums of x per 16
//    values.  Codes are multiplied by both digit vectors with dp4a (exact
//    int32 sums); scales and mins are applied once per 16 or 32 values:
//        sum (d*sc*q - m) x = d*sc*(s_b/254)*(254*sum q x0 + sum q x1) - m*sum x.
//  * A CTA (256 threads) owns whole rows.  Its lanes are split into RS row
//    slots; lane l of a slot always handles the same units (32-value pieces)
//    of a row, so it loads its x digits once, into registers, for the whole
//    kernel.  Only weights move per row.
//  * Weights are staged through a ring of S shared-memory stages with
//    cp.async (16 bytes per thread per copy, fully coalesced, L1 bypassed); a
//    stage is RS*m consecutive rows, i.e. one contiguous byte range.  Lanes
//    then decode their units from shared memory, whatever the block alignment.
//  * Row sums: warp shuffle, then a fixed-order sum of the slot's warps in
//    shared memory (deterministic; any row partition gives identical rows).
//  * With static weights each CTA first asks the TMA unit to prefetch its
//    first stages into L2 (cp.async.bulk.prefetch.L2) before waiting for the
//    preceding kernel (programmatic dependent launch).
#include "kernels.cuh"

namespace pyr {
namespace {

// ---- shared / global access helpers -----------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
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
// One warp per 32-value block; lane l owns value l.  Workspace of one column
// (cols values): xq0[cols] int8 | xq1[cols] int8 | xscale[cols/32] fp32
// (s_b / 254) | xsum16[cols/16] fp32.
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
    const float v = x[c * ldx + 32LL * b + lane];
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = amax / 127.0f;
    int d0 = 0, d1 = 0;
    if (s > 0.0f) {
      const float t = v / s;
      d0 = max(-127, min(127, (int)rintf(t)));
      d1 = max(-127, min(127, (int)rintf((t - (float)d0) * 254.0f)));
    }
    float s16 = v;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
    uint8_t* w = ws + c * ws_col_bytes;
    w[32LL * b + lane] = (uint8_t)(int8_t)d0;
    w[(long long)cols + 32LL * b + lane] = (uint8_t)(int8_t)d1;
    float* xscale = reinterpret_cast<float*>(w + 2LL * cols);
    float* xsum16 = xscale + nblk;
    if (lane == 0) xscale[b] = s / 254.0f;
    if ((lane & 15) == 0) xsum16[2 * b + (lane >> 4)] = s16;
  }
}

namespace {

struct XView {  // one column of prepared x (global)
  const uint8_t* q0;
  const uint8_t* q1;
  const float* scale;
  const float* sum16;
};
__device__ __forceinline__ XView xview(const uint8_t* ws, int cols) {
  XView v;
  v.q0 = ws;
  v.q1 = ws + cols;
  v.scale = reinterpret_cast<const float*>(ws + 2LL * cols);
  v.sum16 = v.scale + cols / 32;
  return v;
}

struct Dig16 { uint4 a, b; };  // 16 digits of each plane
__device__ __forceinline__ Dig16 dig16(const XView& x, int c) {
  Dig16 d;
  d.a = __ldg(reinterpret_cast<const uint4*>(x.q0 + c));
  d.b = __ldg(reinterpret_cast<const uint4*>(x.q1 + c));
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

// ---- per-type unit decoders ------------------------------------------------------
// A unit is 32 values of one block.  XU: the x data of one unit, held in
// registers for the whole kernel.  dot(blk, j, XU): the unit's contribution
// to one row; blk is the shared address of the unit's block, j the unit's
// index inside it.

// Q4_K / Q5_K (native.c:173-197, 410-437).  Unit j = qs bytes 16j..16j+15:
// low nibbles are values 64p+16h+i (sub-block 2p), high nibbles values
// 64p+32+16h+i (sub-block 2p+1), p = j/2, h = j%2.  16-byte aligned blocks.
template <int TY> struct UnitK45 {
  static constexpr int UPB = 8;
  struct XU { Dig16 a, b; float sa, sb, ma, mb; };
  __device__ static void load_x(const XView& x, int unit, XU& u) {
    const int j = unit & 7, p = j >> 1, h = j & 1;
    const int ca = 256 * (unit >> 3) + 64 * p + 16 * h, cb = ca + 32;
    u.a = dig16(x, ca);
    u.b = dig16(x, cb);
    u.sa = __ldg(x.scale + (ca >> 5));
    u.sb = __ldg(x.scale + (cb >> 5));
    u.ma = __ldg(x.sum16 + (ca >> 4));
    u.mb = __ldg(x.sum16 + (cb >> 4));
  }
  __device__ static float dot(uint32_t blk, int j, const XU& u) {
    const int p = j >> 1, h = j & 1;
    const uint4 hdr = lds128(blk);
    const uint4 qv = lds128(blk + (TY == Q4_K ? 16 : 48) + 16 * j);
    uint32_t lo[4], hi[4];
    if constexpr (TY == Q5_K) {
      const uint4 hv = lds128(blk + 16 + 16 * h);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t q = w4(qv, k), qh = w4(hv, k);
        lo[k] = (q & 0x0F0F0F0Fu) | (((qh >> (2 * p)) & 0x01010101u) << 4);
        hi[k] = ((q >> 4) & 0x0F0F0F0Fu) | (((qh >> (2 * p + 1)) & 0x01010101u) << 4);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        lo[k] = w4(qv, k) & 0x0F0F0F0Fu;
        hi[k] = (w4(qv, k) >> 4) & 0x0F0F0F0Fu;
      }
    }
    const int ia = dot16(lo, u.a), ib = dot16(hi, u.b);
    // 6-bit (scale, min) pairs 2p and 2p+1 (native.c:52-60)
    const int sh = 8 * ((2 * p) & 3);
    int sca, mna, scb, mnb;
    if (p < 2) {
      sca = (hdr.y >> sh) & 63;        mna = (hdr.z >> sh) & 63;
      scb = (hdr.y >> (sh + 8)) & 63;  mnb = (hdr.z >> (sh + 8)) & 63;
    } else {
      const uint32_t ca = (hdr.w >> sh) & 0xff, cb = (hdr.w >> (sh + 8)) & 0xff;
      sca = (ca & 15) | (((hdr.y >> (sh + 6)) & 3) << 4);
      mna = (ca >> 4) | (((hdr.z >> (sh + 6)) & 3) << 4);
      scb = (cb & 15) | (((hdr.y >> (sh + 14)) & 3) << 4);
      mnb = (cb >> 4) | (((hdr.z >> (sh + 14)) & 3) << 4);
    }
    const float d = half_f(hdr.x & 0xffff), dmin = half_f(hdr.x >> 16);
    return d * ((float)sca * u.sa * (float)ia + (float)scb * u.sb * (float)ib) -
           dmin * ((float)mna * u.ma + (float)mnb * u.mb);
  }
};

// Q8_0: d | int8 qs[32]  (native.c:330-336).  One unit per block; blocks are
// 2-byte aligned.
struct UnitQ80 {
  static constexpr int UPB = 1;
  struct XU { Dig16 a, b; float s; };
  __device__ static void load_x(const XView& x, int unit, XU& u) {
    u.a = dig16(x, 32 * unit);
    u.b = dig16(x, 32 * unit + 16);
    u.s = __ldg(x.scale + unit);
  }
  __device__ static float dot(uint32_t blk, int, const XU& u) {
    uint32_t q[8];
    lds_32b(blk + 2, q);
    const float d = half_f(lds16(blk));
    const uint32_t c0[4] = {q[0], q[1], q[2], q[3]}, c1[4] = {q[4], q[5], q[6], q[7]};
    return d * u.s * (float)(dot16(c0, u.a) + dot16(c1, u.b));
  }
};

// Q6_K: ql[128] | qh[64] | int8 scales[16] | d  (native.c:199-225).  Unit
// j = (h = j/4, t = j%4) is values 128h+32t+l: low 4 bits from
// ql[64h + 32(t&1) + l] (high nibble when t >= 2), two high bits from
// qh[32h+l] >> 2t, int8 scale 8h + 2t + l/16.  Blocks are 2-byte aligned.
struct UnitQ6K {
  static constexpr int UPB = 8;
  struct XU { Dig16 a, b; float s, m0, m1; };
  __device__ static void load_x(const XView& x, int unit, XU& u) {
    u.a = dig16(x, 32 * unit);
    u.b = dig16(x, 32 * unit + 16);
    u.s = __ldg(x.scale + unit);
    u.m0 = __ldg(x.sum16 + 2 * unit);
    u.m1 = __ldg(x.sum16 + 2 * unit + 1);
  }
  __device__ static float dot(uint32_t blk, int j, const XU& u) {
    const int h = j >> 2, t = j & 3;
    uint32_t ql[8], qh[8];
    lds_32b(blk + 64 * h + 32 * (t & 1), ql);
    lds_32b(blk + 128 + 32 * h, qh);
    const uint32_t sc2 = lds16(blk + 192 + 8 * h + 2 * t);
    const float d = half_f(lds16(blk + 208));
    const int lsh = (t >= 2) ? 4 : 0;
    uint32_t c0[4], c1[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      c0[k] = ((ql[k] >> lsh) & 0x0F0F0F0Fu) | (((qh[k] >> (2 * t)) & 0x03030303u) << 4);
      c1[k] = ((ql[k + 4] >> lsh) & 0x0F0F0F0Fu) | (((qh[k + 4] >> (2 * t)) & 0x03030303u) << 4);
    }
    // codes are 0..63, value = d * sc * (code - 32)
    const float qa = u.s * (float)dot16(c0, u.a) - 32.0f * u.m0;
    const float qb = u.s * (float)dot16(c1, u.b) - 32.0f * u.m1;
    return d * ((float)(int8_t)(sc2 & 0xff) * qa + (float)(int8_t)(sc2 >> 8) * qb);
  }
};

// IQ4_XS: d | scales_h | scales_l[4] | qs[128]  (native.c:364-379).  Unit j
// is sub-block j.  Codes index the non-linear book through a 16-entry byte
// table (two 8-entry permutes and a select on bit 3); looked-up bytes come out
// in the order [lo0, hi0, lo1, hi1], so the x digits are interleaved the same
// way once, when they are loaded.  8-byte aligned blocks.
struct UnitIQ4XS {
  static constexpr int UPB = 8;
  struct XU { uint32_t a[8], b[8]; float s; };
  __device__ static void load_x(const XView& x, int unit, XU& u) {
    const Dig16 lo = dig16(x, 32 * unit), hi = dig16(x, 32 * unit + 16);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      u.a[2 * k] = __byte_perm(w4(lo.a, k), w4(hi.a, k), 0x5140);
      u.a[2 * k + 1] = __byte_perm(w4(lo.a, k), w4(hi.a, k), 0x7362);
      u.b[2 * k] = __byte_perm(w4(lo.b, k), w4(hi.b, k), 0x5140);
      u.b[2 * k + 1] = __byte_perm(w4(lo.b, k), w4(hi.b, k), 0x7362);
    }
    u.s = __ldg(x.scale + unit);
  }
  __device__ static float dot(uint32_t blk, int j, const XU& u) {
    const uint2 hdr = lds64(blk);  // d | scales_h | scales_l[4]
    const uint2 q01 = lds64(blk + 8 + 16 * j), q23 = lds64(blk + 16 + 16 * j);
    const uint32_t qw[4] = {q01.x, q01.y, q23.x, q23.y};
    // the book as int8: -127 -104 -83 -65 -49 -35 -22 -10 | 1 13 25 38 53 69 89 113
    const uint32_t T0 = 0xBFAD9881u, T1 = 0xF6EADDCFu, T2 = 0x26190D01u, T3 = 0x71594535u;
    int a = 0, b = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint32_t n = (qw[k] >> (16 * half)) & 0xffffu;
        const uint32_t sel = n & 0x7777u;
        const uint32_t v = __byte_perm(__byte_perm(T0, T1, sel), __byte_perm(T2, T3, sel),
                                       0x3210u | ((n & 0x8888u) >> 1));
        a = __dp4a((int)v, (int)u.a[2 * k + half], a);
        b = __dp4a((int)v, (int)u.b[2 * k + half], b);
      }
    }
    const uint32_t sh = hdr.x >> 16;
    const int ls = ((hdr.y >> (4 * j)) & 15) | (int)(((sh >> (2 * j)) & 3u) << 4);
    return half_f(hdr.x & 0xffff) * (float)(ls - 32) * u.s * (float)(a * 254 + b);
  }
};

template <int TY> struct UnitOf;
template <> struct UnitOf<Q4_K> { using T = UnitK45<Q4_K>; };
template <> struct UnitOf<Q5_K> { using T = UnitK45<Q5_K>; };
template <> struct UnitOf<Q8_0> { using T = UnitQ80; };
template <> struct UnitOf<Q6_K> { using T = UnitQ6K; };
template <> struct UnitOf<IQ4_XS> { using T = UnitIQ4XS; };

constexpr int kThreads = 256, kWarps = 8, kMaxRowsPerStage = 16;

struct TileArgs {
  const uint8_t* w;
  size_t row_bytes;
  int rows, cols;
  const uint8_t* ws;  // prepared x
  float* y;
  int rs;           // row slots (lanes per slot = 256 / rs, a multiple of 32)
  int m;            // rows per slot per stage
  int stages;       // ring depth S
  int stage_bytes;  // shared bytes per stage (rs*m rows + alignment slack)
  int static_weights;
};

template <int TY, int UL, int M>
__global__ void __launch_bounds__(kThreads, 3) mv_tile_kernel(TileArgs a) {
  using U = typename UnitOf<TY>::T;
  constexpr int BPB = Geo<TY>::bpb;
  extern __shared__ __align__(128) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem + (size_t)a.stages * a.stage_bytes);  // [2][kWarps][M]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lps = kThreads / a.rs, slot = tid / lps, ls = tid % lps;
  const int rows_per_stage = a.rs * M;
  const int nstages = (a.rows + rows_per_stage - 1) / rows_per_stage;
  const int units = a.cols / 32;
  const uint32_t ring = smem_addr(smem);
  const size_t stage_stride = (size_t)rows_per_stage * a.row_bytes;  // bytes between stages
  const int S = a.stages;

  // per-thread constants: this lane's units, their offsets inside a row
  int uoff[UL], uj[UL];
  bool uon[UL];
#pragma unroll
  for (int k = 0; k < UL; ++k) {
    const int u = ls + k * lps;
    uon[k] = u < units;
    uoff[k] = (u / U::UPB) * BPB;
    uj[k] = u % U::UPB;
  }

  auto stage_rows = [&](int st) { return min(rows_per_stage, a.rows - st * rows_per_stage); };
  // the CTA's k-th stage -> ring slot k % S: one contiguous byte range
  auto issue = [&](int k) {
    const int st = blockIdx.x + k * gridDim.x;
    if (st < nstages) {
      const uintptr_t src = (uintptr_t)a.w + (uintptr_t)st * stage_stride;
      const uintptr_t al = src & ~(uintptr_t)15;
      const uint32_t len = (uint32_t)(((src - al) + (uintptr_t)stage_rows(st) * a.row_bytes + 15) & ~(uintptr_t)15);
      const uint32_t dst = ring + (uint32_t)((k % S) * a.stage_bytes);
      for (uint32_t c = (uint32_t)tid * 16; c < len; c += kThreads * 16)
        cp_async16(dst + c, reinterpret_cast<const void*>(al + c));
    }
    cp_async_commit();  // one group per k, empty or not, keeps the wait count uniform
  };

  const int my = blockIdx.x < nstages ? (nstages - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  if (a.static_weights && tid < min(my, S)) {
    // pull the first stages into L2 while the preceding kernel drains
    const int st = blockIdx.x + tid * gridDim.x;
    const uintptr_t src = (uintptr_t)a.w + (uintptr_t)st * stage_stride;
    const uintptr_t s0 = (src + 15) & ~(uintptr_t)15;
    const uintptr_t e0 = (src + (uintptr_t)stage_rows(st) * a.row_bytes) & ~(uintptr_t)15;
    if (e0 > s0) prefetch_l2(reinterpret_cast<const void*>(s0), (uint32_t)(e0 - s0));
  }
  pdl_wait();  // x (prepared by the preceding kernel) and y are ordered after it
  pdl_launch_dependents();

  typename U::XU xu[UL];  // this lane's x, for the whole kernel
  const XView xv = xview(a.ws, a.cols);
#pragma unroll
  for (int k = 0; k < UL; ++k)
    if (uon[k]) U::load_x(xv, ls + k * lps, xu[k]);

  for (int k = 0; k < S - 1; ++k) issue(k);

  auto finalize = [&](int k) {  // fixed-order sum of the slot warps' partials
    const int st = blockIdx.x + k * gridDim.x;
    if (tid < stage_rows(st)) {
      const int s_slot = tid / M, i = tid % M, wps = lps / 32;
      const float* r = red + (size_t)(k & 1) * kWarps * M;
      float v = 0.f;
      for (int w = 0; w < wps; ++w) v += r[(s_slot * wps + w) * M + i];
      a.y[(size_t)st * rows_per_stage + tid] = v;
    }
  };

  for (int k = 0; k < my; ++k) {
    // stage k landed (own copies), then visible to all (barrier); the barrier
    // also retires iteration k-1, whose slot the refill below reuses
    if (S >= 4) cp_async_wait<2>(); else cp_async_wait<1>();
    __syncthreads();
    if (k > 0) finalize(k - 1);
    issue(k + S - 1);
    const int st = blockIdx.x + k * gridDim.x;
    const int nr = stage_rows(st);
    const uint32_t base = ring + (uint32_t)((k % S) * a.stage_bytes) +
                          (uint32_t)(((uintptr_t)a.w + (uintptr_t)st * stage_stride) & 15) +
                          (uint32_t)(slot * M) * (uint32_t)a.row_bytes;
    float acc[M];
#pragma unroll
    for (int i = 0; i < M; ++i) {
      acc[i] = 0.f;
      if (slot * M + i < nr) {
        const uint32_t rowa = base + (uint32_t)i * (uint32_t)a.row_bytes;
#pragma unroll
        for (int kk = 0; kk < UL; ++kk)
          if (uon[kk]) acc[i] += U::dot(rowa + (uint32_t)uoff[kk], uj[kk], xu[kk]);
      }
    }
    float* r = red + (size_t)(k & 1) * kWarps * M;
#pragma unroll
    for (int i = 0; i < M; ++i) {
      float v = acc[i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) r[warp * M + i] = v;
    }
  }
  __syncthreads();
  if (my > 0) finalize(my - 1);
  cp_async_wait<0>();  // no copy may still target this CTA's shared memory
}

struct TilePlan { int rs, m, stages, stage_bytes, ul; size_t smem; };

TilePlan plan_tile(size_t row_bytes, int cols) {
  TilePlan p{};
  const int units = cols / 32;
  int pow2 = 32;
  while (pow2 < units && pow2 < kThreads) pow2 *= 2;
  p.rs = kThreads / pow2;  // row slots: 1..8, each 32..256 lanes
  const int lps = kThreads / p.rs;
  p.ul = (units + lps - 1) / lps;
  // rows per slot per stage (1, 2 or 4): about 8-12 KB per stage
  const size_t per = (size_t)p.rs * row_bytes;
  p.m = per * 4 <= 12 * 1024 ? 4 : per * 2 <= 12 * 1024 ? 2 : 1;
  const size_t sb = ((size_t)p.rs * p.m * row_bytes + 16 + 32 + 127) & ~(size_t)127;
  p.stage_bytes = (int)sb;
  p.stages = sb <= 16 * 1024 ? 4 : 3;
  p.smem = (size_t)p.stages * sb + 2 * kWarps * p.m * sizeof(float);
  return p;
}

template <int TY, int UL, int M>
int launch_tile_t(const TileArgs& ta, size_t smem, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return -4;
  static int sms[64] = {};
  static bool smem_set[64] = {};
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  constexpr int kMaxSmem = 72 * 1024;
  if (!smem_set[dev]) {
    if (cudaFuncSetAttribute(mv_tile_kernel<TY, UL, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) !=
        cudaSuccess)
      return -100 - (int)cudaGetLastError();
    smem_set[dev] = true;
  }
  if (smem > (size_t)kMaxSmem) return 1;
  const int rows_per_stage = ta.rs * M;
  const int nstages = (ta.rows + rows_per_stage - 1) / rows_per_stage;
  int per_sm = (int)((227 * 1024) / (smem + 1024));
  if (per_sm > 3) per_sm = 3;
  if (per_sm < 1) per_sm = 1;
  int grid = sms[dev] * per_sm;
  if (grid > nstages) grid = nstages;
  return launch_pdl(mv_tile_kernel<TY, UL, M>, dim3(grid), dim3(kThreads), smem, stream, ta);
}

template <int TY>
int launch_tile_type(const TileArgs& ta, int ul, size_t smem, cudaStream_t stream) {
#define PYR_UM(UL_, M_) \
  if (ul == UL_ && ta.m == M_) return launch_tile_t<TY, UL_, M_>(ta, smem, stream);
  PYR_UM(1, 1) PYR_UM(1, 2) PYR_UM(1, 4) PYR_UM(2, 1) PYR_UM(2, 2) PYR_UM(2, 4)
  PYR_UM(3, 1) PYR_UM(3, 2) PYR_UM(4, 1) PYR_UM(4, 2)
#undef PYR_UM
  return 1;
}

}  // namespace

size_t lane_workspace_bytes(int cols) { return (size_t)cols * 2 + (size_t)(cols / 32) * 4 + (size_t)(cols / 16) * 4; }

bool lane_supported(int type_id, const uint8_t* w, size_t row_bytes, int cols) {
  if (cols % 256 != 0 || cols / 32 > 4 * kThreads) return false;
  const uintptr_t base = (uintptr_t)w;
  switch (type_id) {
    case Q4_K: case Q5_K: return (base & 15) == 0 && (row_bytes & 15) == 0;
    case Q8_0: case Q6_K: return (base & 1) == 0;
    case IQ4_XS: return (base & 7) == 0;
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
                   float* y, bool static_weights, cudaStream_t stream) {
  const TilePlan p = plan_tile(row_bytes, cols);
  TileArgs ta{w, row_bytes, rows, cols, ws, y, p.rs, p.m, p.stages, p.stage_bytes, static_weights ? 1 : 0};
  switch (type_id) {
    case Q4_K: return launch_tile_type<Q4_K>(ta, p.ul, p.smem, stream);
    case Q5_K: return launch_tile_type<Q5_K>(ta, p.ul, p.smem, stream);
    case Q8_0: return launch_tile_type<Q8_0>(ta, p.ul, p.smem, stream);
    case Q6_K: return launch_tile_type<Q6_K>(ta, p.ul, p.smem, stream);
    case IQ4_XS: return launch_tile_type<IQ4_XS>(ta, p.ul, p.smem, stream);
    default: return 1;
  }
}

}  // namespace pyr
