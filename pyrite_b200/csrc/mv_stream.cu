// mv_stream.cu -- batch-1 fused dequantize x matvec, weights streamed by TMA.
//
// The product y = W x of the reference's pyrite_matvec
// (pyrite/kernels/native.c:518-555), in fp32 with fp32 accumulation.
//
// Design (B200):
//   * Each warp owns groups of R consecutive rows and runs its own ring of S
//     shared-memory slots.  Lane 0 fills a slot with R bulk copies
//     (cp.async.bulk global->shared, one per row segment of CB blocks) that
//     complete on the slot's mbarrier; the warp decodes the slot from shared
//     memory while the next S-1 slots are in flight.  Row segments are
//     contiguous in HBM, so every byte is read exactly once, in whole 16-byte
//     sectors.
//   * A slot holds CB blocks per row: exactly 32 "units" of 32 values, so
//     lane l always decodes unit l of the chunk for all R rows and loads its x
//     values once per chunk (x reuse across rows keeps L1 traffic low).
//   * Decoding is type specific (FastUnit<TY>): codes are widened four at a
//     time with byte permutes into the mantissa of a float whose exponent
//     encodes 128 (value 128 + code), so one PRMT + one FFMA handles a value;
//     the constant 128 * sum(x) is removed once per unit, and the per-sub-block
//     scale / min are applied once per unit:  sum((d*sc*q - m) x) =
//     d*sc*sum(q x) - m*sum(x).
//   * Work is dealt to warps CTA-major so every SM gets the same share; the
//     grid is two CTAs per SM.  Programmatic dependent launch lets the next
//     kernel's weight prefetch overlap this kernel's tail.
//   * Every mbarrier wait is bounded (2 s of globaltimer); on time-out the
//     kernel sets a status bit, waits (bounded) for its own copies and returns.
#include "kernels.cuh"

namespace pyr {
namespace {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far above any legal copy latency

// Bounded wait on an mbarrier phase; warp-uniform result.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity) {
  bool ok = mbar_try_wait(bar, parity);
  if (!__all_sync(0xffffffffu, ok)) {
    const uint64_t t0 = globaltimer_ns();
    while (!ok) {
      ok = mbar_try_wait(bar, parity);
      if (!ok && globaltimer_ns() - t0 > kWaitLimitNs) break;
    }
    // The phase is monotonic: if any lane saw it complete, it is complete.
    ok = __any_sync(0xffffffffu, ok);
  }
  return ok;
}

__device__ __forceinline__ float half_f(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

// 4 bytes holding codes 0..127 -> float(128 + code) for byte b.
__device__ __forceinline__ float code_f(uint32_t codes, int b) {
  return __uint_as_float(__byte_perm(codes, 0x4300u, 0x5044u | ((uint32_t)b << 8)));
}
// 4 bytes holding u = int8 ^ 0x80 -> float(int8) for byte b.
__device__ __forceinline__ float s8x_f(uint32_t u, int b) {
  return __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440u | (uint32_t)b)) - 8388736.0f;
}

// 32 bit-aligned words covering n bytes from an arbitrary shared address.
template <int NW>
__device__ __forceinline__ void load_words(const uint8_t* p, uint32_t (&out)[NW]) {
  const uintptr_t a = (uintptr_t)p;
  const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
  const uint32_t sh = (uint32_t)(a & 3) * 8;
  uint32_t w[NW + 1];
#pragma unroll
  for (int k = 0; k <= NW; ++k) w[k] = base[k];
#pragma unroll
  for (int k = 0; k < NW; ++k) out[k] = __funnelshift_r(w[k], w[k + 1], sh);
}

__device__ __forceinline__ void ldg_x(const float* p, float* dst, int n4) {
#pragma unroll
  for (int k = 0; k < n4; ++k) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(p) + k);
    dst[4 * k] = t.x; dst[4 * k + 1] = t.y; dst[4 * k + 2] = t.z; dst[4 * k + 3] = t.w;
  }
}

// ---- per-type unit decoders --------------------------------------------------
// load_x(xb, j, X): gather the x values unit j of a block (whose first column is
// xb) multiplies, in the order dot() consumes them.  dot(blk, j, X): the unit's
// contribution to one row, blk pointing at the block in shared memory.

// Fallback: exact per-value decode from shared memory (any block format).
template <int TY> struct FastUnit {
  struct X { float v[32]; };
  __device__ static void load_x(const float* xb, int j, X& x) { ldg_x(xb + 32 * j, x.v, 8); }
  __device__ static float dot(const uint8_t* blk, int j, const X& x) {
    float v[32];
    decode_unit<TY, float>(blk, j, v);
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i += 2) { s0 = fmaf(v[i], x.v[i], s0); s1 = fmaf(v[i + 1], x.v[i + 1], s1); }
    return s0 + s1;
  }
};

// Q8_0: d | int8 qs[32]  (pyrite/kernels/native.c:330-336).  34-byte blocks
// are only 2-byte aligned, so qs is read as funnel-shifted aligned words.
template <> struct FastUnit<Q8_0> {
  struct X { float v[32]; };
  __device__ static void load_x(const float* xb, int, X& x) { ldg_x(xb, x.v, 8); }
  __device__ static float dot(const uint8_t* blk, int, const X& x) {
    uint32_t q[8];
    load_words<8>(blk + 2, q);
    const float d = half_f(ld_u16(blk));
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t u = q[k] ^ 0x80808080u;
      s0 = fmaf(s8x_f(u, 0), x.v[4 * k + 0], s0);
      s1 = fmaf(s8x_f(u, 1), x.v[4 * k + 1], s1);
      s0 = fmaf(s8x_f(u, 2), x.v[4 * k + 2], s0);
      s1 = fmaf(s8x_f(u, 3), x.v[4 * k + 3], s1);
    }
    return d * (s0 + s1);
  }
};

// K-quant 6-bit (scale, min) pair j from the 12 scale bytes held in three
// registers s0 = bytes 0..3, s1 = 4..7, s2 = 8..11 (native.c:52-60).
__device__ __forceinline__ void k4_pair(uint32_t s0, uint32_t s1, uint32_t s2, int j, int& sc, int& mn) {
  const int k = (j & 3) * 8;
  const uint32_t a = (s0 >> k) & 0xff, b = (s1 >> k) & 0xff, c = (s2 >> k) & 0xff;
  if (j < 4) {
    sc = (int)(a & 63);
    mn = (int)(b & 63);
  } else {
    sc = (int)((c & 15) | ((a >> 6) << 4));
    mn = (int)((c >> 4) | ((b >> 6) << 4));
  }
}

// Q4_K / Q5_K: d | dmin | scales[12] | (Q5_K: qh[32]) | qs[128]
// (native.c:173-197, 410-437).  Unit j = (p = j/2, h = j%2) takes qs bytes
// 32p+16h .. +15: their low nibbles are values 64p+16h+i (sub-block 2p), their
// high nibbles values 64p+32+16h+i (sub-block 2p+1).  Needs 16-byte aligned
// blocks (the host only routes aligned payloads here).
template <int TY> struct KQuant45 {
  struct X { float v[32]; float sa, sb; };
  __device__ static void load_x(const float* xb, int j, X& x) {
    const int p = j >> 1, h = j & 1;
    ldg_x(xb + 64 * p + 16 * h, x.v, 4);
    ldg_x(xb + 64 * p + 32 + 16 * h, x.v + 16, 4);
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) { a += x.v[i]; b += x.v[16 + i]; }
    x.sa = a; x.sb = b;
  }
  __device__ static float dot(const uint8_t* blk, int j, const X& x) {
    const int p = j >> 1, h = j & 1;
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const uint4 qv = *reinterpret_cast<const uint4*>(blk + (TY == Q4_K ? 16 : 48) + 32 * p + 16 * h);
    uint4 hv = make_uint4(0, 0, 0, 0);
    if constexpr (TY == Q5_K) hv = *reinterpret_cast<const uint4*>(blk + 16 + 16 * h);
    const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
    const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
    float sa0 = 0.f, sa1 = 0.f, sb0 = 0.f, sb1 = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t lo = qw[k] & 0x0F0F0F0Fu, hi = (qw[k] >> 4) & 0x0F0F0F0Fu;
      if constexpr (TY == Q5_K) {
        lo |= ((hw[k] >> (2 * p)) & 0x01010101u) << 4;
        hi |= ((hw[k] >> (2 * p + 1)) & 0x01010101u) << 4;
      }
      sa0 = fmaf(code_f(lo, 0), x.v[4 * k + 0], sa0);
      sa1 = fmaf(code_f(lo, 1), x.v[4 * k + 1], sa1);
      sa0 = fmaf(code_f(lo, 2), x.v[4 * k + 2], sa0);
      sa1 = fmaf(code_f(lo, 3), x.v[4 * k + 3], sa1);
      sb0 = fmaf(code_f(hi, 0), x.v[16 + 4 * k + 0], sb0);
      sb1 = fmaf(code_f(hi, 1), x.v[16 + 4 * k + 1], sb1);
      sb0 = fmaf(code_f(hi, 2), x.v[16 + 4 * k + 2], sb0);
      sb1 = fmaf(code_f(hi, 3), x.v[16 + 4 * k + 3], sb1);
    }
    const float qa = (sa0 + sa1) - 128.f * x.sa;  // sum(q x), run A
    const float qb = (sb0 + sb1) - 128.f * x.sb;  // sum(q x), run B
    int sca, mna, scb, mnb;
    k4_pair(hdr.y, hdr.z, hdr.w, 2 * p, sca, mna);
    k4_pair(hdr.y, hdr.z, hdr.w, 2 * p + 1, scb, mnb);
    const float d = half_f(hdr.x & 0xffff), dmin = half_f(hdr.x >> 16);
    return (d * (float)sca) * qa - (dmin * (float)mna) * x.sa + (d * (float)scb) * qb -
           (dmin * (float)mnb) * x.sb;
  }
};
template <> struct FastUnit<Q4_K> : KQuant45<Q4_K> {};
template <> struct FastUnit<Q5_K> : KQuant45<Q5_K> {};

// Q6_K: ql[128] | qh[64] | int8 scales[16] | d  (native.c:199-225).  Unit
// j = (h = j/4, t = j%4) is values 128h+32t+l: low 4 bits from
// ql[64h + 32(t&1) + l] (high nibble when t >= 2), two high bits from
// qh[32h+l] >> 2t, scale 8h + 2t + l/16.  Blocks are 2-byte aligned only.
template <> struct FastUnit<Q6_K> {
  struct X { float v[32]; float s0, s1; };
  __device__ static void load_x(const float* xb, int j, X& x) {
    ldg_x(xb + 32 * j, x.v, 8);
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) { a += x.v[i]; b += x.v[16 + i]; }
    x.s0 = a; x.s1 = b;
  }
  __device__ static float dot(const uint8_t* blk, int j, const X& x) {
    const int h = j >> 2, t = j & 3;
    uint32_t ql[8], qh[8];
    load_words<8>(blk + 64 * h + 32 * (t & 1), ql);
    load_words<8>(blk + 128 + 32 * h, qh);
    const int lsh = (t >= 2) ? 4 : 0;
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t c = ((ql[k] >> lsh) & 0x0F0F0F0Fu) | (((qh[k] >> (2 * t)) & 0x03030303u) << 4);
      if (k < 4) {
        a0 = fmaf(code_f(c, 0), x.v[4 * k + 0], a0);
        a1 = fmaf(code_f(c, 1), x.v[4 * k + 1], a1);
        a0 = fmaf(code_f(c, 2), x.v[4 * k + 2], a0);
        a1 = fmaf(code_f(c, 3), x.v[4 * k + 3], a1);
      } else {
        b0 = fmaf(code_f(c, 0), x.v[4 * k + 0], b0);
        b1 = fmaf(code_f(c, 1), x.v[4 * k + 1], b1);
        b0 = fmaf(code_f(c, 2), x.v[4 * k + 2], b0);
        b1 = fmaf(code_f(c, 3), x.v[4 * k + 3], b1);
      }
    }
    // value = d * sc * (code - 32);  sum(code x) = acc - 128 sum(x)
    const float qa = (a0 + a1) - 160.f * x.s0;
    const float qb = (b0 + b1) - 160.f * x.s1;
    const int sca = (int8_t)blk[192 + 8 * h + 2 * t], scb = (int8_t)blk[192 + 8 * h + 2 * t + 1];
    const float d = half_f(ld_u16(blk + 208));
    return (d * (float)sca) * qa + (d * (float)scb) * qb;
  }
};

// IQ4_XS: d | scales_h | scales_l[4] | qs[128]  (native.c:364-379).  Unit j is
// sub-block j; 4-bit codes index the non-linear book through a 16-entry byte
// table (two 8-entry permutes and a select on bit 3).  The table stores
// book + 128 so the bytes feed the int8 widening directly.
template <> struct FastUnit<IQ4_XS> {
  struct X { float v[32]; };
  // Selector order within a qs word: [lo0, hi0, lo1, hi1 | lo2, hi2, lo3, hi3],
  // lo = value 4k+i, hi = value 16+4k+i.
  __device__ static void load_x(const float* xb, int j, X& x) {
    float t[32];
    ldg_x(xb + 32 * j, t, 8);
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        x.v[8 * k + 2 * i] = t[4 * k + i];
        x.v[8 * k + 2 * i + 1] = t[16 + 4 * k + i];
      }
  }
  __device__ static float dot(const uint8_t* blk, int j, const X& x) {
    uint32_t q[4];
    load_words<4>(blk + 8 + 16 * j, q);
    const uint32_t U0 = 0x3F2D1801u, U1 = 0x766A5D4Fu, U2 = 0xA6998D81u, U3 = 0xF1D9C5B5u;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint32_t n = (q[k] >> (16 * half)) & 0xffffu;
        const uint32_t sel = n & 0x7777u;
        const uint32_t lo = __byte_perm(U0, U1, sel), hi = __byte_perm(U2, U3, sel);
        const uint32_t u = __byte_perm(lo, hi, 0x3210u | ((n & 0x8888u) >> 1));
        const float* xv = x.v + 8 * k + 4 * half;
        s0 = fmaf(s8x_f(u, 0), xv[0], s0);
        s1 = fmaf(s8x_f(u, 1), xv[1], s1);
        s0 = fmaf(s8x_f(u, 2), xv[2], s0);
        s1 = fmaf(s8x_f(u, 3), xv[3], s1);
      }
    }
    const unsigned sh = ld_u16(blk + 2);
    const int ls = ((blk[4 + j / 2] >> (4 * (j & 1))) & 15) | (int)(((sh >> (2 * j)) & 3u) << 4);
    return (half_f(ld_u16(blk)) * (float)(ls - 32)) * (s0 + s1);
  }
};

// ---- kernel configuration ----------------------------------------------------
// CB blocks per row per slot = exactly 32 units of 32 values; R rows per warp
// group; S slots per warp; W warps per CTA.  Shared memory per CTA stays
// near or under 110 KB so two CTAs fit an SM.
template <int TY> struct StreamCfg {
  static constexpr int CB = Geo<TY>::bs == 256 ? 4 : 32;
  static constexpr int R = Geo<TY>::bpb * CB > 800 ? 2 : 4;
  static constexpr int S = 4;
  static constexpr int W = 8;
  static constexpr int SEG = (CB * Geo<TY>::bpb + 32 + 15) / 16 * 16;  // + alignment slack
  static constexpr int SLOT = R * SEG;
  static constexpr int SMEM = W * S * SLOT + W * S * 8;
};

template <int TY>
__global__ void __launch_bounds__(StreamCfg<TY>::W * 32, 2)
mv_stream_kernel(MatvecArgs<float> a, int* status, int early_prefetch) {
  using C = StreamCfg<TY>;
  using U = FastUnit<TY>;
  constexpr int BS = Geo<TY>::bs, BPB = Geo<TY>::bpb, UPB = BS / 32;
  constexpr int R = C::R, CB = C::CB, S = C::S, W = C::W, SEG = C::SEG, SLOT = C::SLOT;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem + warp * (S * SLOT);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + W * S * SLOT) + warp * S;

  const int nb = a.cols / BS;
  const int nchunks = (nb + CB - 1) / CB;
  const int ngroups = (a.rows + R - 1) / R;
  const int gstride = gridDim.x * W;
  const int g0 = blockIdx.x + gridDim.x * warp;  // CTA-major deal: SMs share work evenly
  const int my_groups = g0 < ngroups ? (ngroups - 1 - g0) / gstride + 1 : 0;
  const int total = my_groups * nchunks;

  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(smem_u32(&bars[s]), 1);
    fence_mbar_init();
  }
  __syncwarp();

  auto row_src = [&](int r, int blk0) -> const uint8_t* {
    return a.w + (size_t)r * a.row_bytes + (size_t)blk0 * BPB;
  };
  auto issue = [&](int s) {  // lane 0 only
    const int gi = s / nchunks, ch = s - gi * nchunks;
    const int r0 = (g0 + gi * gstride) * R;
    const int blk0 = ch * CB, nblk = min(CB, nb - blk0);
    const uint32_t slot = smem_u32(ring + (s % S) * SLOT);
    const uint32_t bar = smem_u32(&bars[s % S]);
    uint32_t tx = 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r0 + r < a.rows) {
        const uintptr_t src = (uintptr_t)row_src(r0 + r, blk0);
        tx += (uint32_t)(((src & 15) + (uintptr_t)nblk * BPB + 15) & ~(uintptr_t)15);
      }
    }
    mbar_expect_tx(bar, tx);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r0 + r < a.rows) {
        const uintptr_t src = (uintptr_t)row_src(r0 + r, blk0);
        const uintptr_t al = src & ~(uintptr_t)15;
        const uint32_t len = (uint32_t)(((src - al) + (uintptr_t)nblk * BPB + 15) & ~(uintptr_t)15);
        bulk_g2s(slot + r * SEG, reinterpret_cast<const void*>(al), len, bar);
      }
    }
  };

  // With static weights the first slots stream while the previous kernel
  // drains; x and y (which it may produce or read) are touched only after
  // pdl_wait().
  if (early_prefetch && lane == 0)
    for (int s = 0; s < min(S, total); ++s) issue(s);
  pdl_wait();
  pdl_launch_dependents();
  if (!early_prefetch && lane == 0)
    for (int s = 0; s < min(S, total); ++s) issue(s);

  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;

  int s = 0;
  bool ok = true;
  for (; s < total; ++s) {
    if (!warp_wait(smem_u32(&bars[s % S]), (uint32_t)(s / S) & 1u)) { ok = false; break; }
    const int gi = s / nchunks, ch = s - gi * nchunks;
    const int r0 = (g0 + gi * gstride) * R;
    const int blk0 = ch * CB, nblk = min(CB, nb - blk0);
    const uint8_t* slot = ring + (s % S) * SLOT;
    if (lane < nblk * UPB) {
      const int b = lane / UPB, j = lane % UPB;
      typename U::X xr;
      U::load_x(a.x + (size_t)(blk0 + b) * BS, j, xr);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (r0 + r < a.rows) {
          const uint8_t* blk = slot + r * SEG + ((uintptr_t)row_src(r0 + r, blk0) & 15) + b * BPB;
          acc[r] += U::dot(blk, j, xr);
        }
      }
    }
    if (ch == nchunks - 1) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float v = acc[r];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && r0 + r < a.rows) a.y[r0 + r] = v;
        acc[r] = 0.f;
      }
    }
    __syncwarp();
    if (lane == 0 && s + S < total) {
      fence_proxy_async();  // generic-proxy reads of this slot precede the async refill
      issue(s + S);
    }
  }
  if (!ok) {
    if (lane == 0) atomicOr(status, (int)kStatusWaitTimeout);
    // Drain every copy this warp still has in flight before the CTA exits.
    const int issued = min(total, s + S);
    for (int t = s; t < issued; ++t) (void)warp_wait(smem_u32(&bars[t % S]), (uint32_t)(t / S) & 1u);
  }
}

template <int TY>
int launch_stream_t(const MatvecArgs<float>& a, bool early, cudaStream_t stream) {
  using C = StreamCfg<TY>;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  static bool configured[64] = {};  // the attribute is set once per device
  if (dev < 0 || dev >= 64) return -4;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(mv_stream_kernel<TY>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return -100 - (int)cudaGetLastError();
    configured[dev] = true;
  }
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int ngroups = (a.rows + C::R - 1) / C::R;
  int grid = 2 * sms;
  const int need = (ngroups + C::W - 1) / C::W;
  if (need < grid) grid = need < 1 ? 1 : need;
  return launch_pdl(mv_stream_kernel<TY>, dim3(grid), dim3(C::W * 32), (size_t)C::SMEM, stream, a,
                    device_status_word(), early ? 1 : 0);
}

}  // namespace

int launch_mv_stream(int type_id, const MatvecArgs<float>& a, bool early, cudaStream_t stream) {
  const TypeGeo* g = find_type(type_id);
  if (!g || g->bs == 1) return 1;
  // x is read as float4: its base must be 16-byte aligned.
  if (((uintptr_t)a.x & 15) != 0) return 1;
  const bool w16 = ((uintptr_t)a.w & 15) == 0 && (a.row_bytes & 15) == 0;
  switch (type_id) {
    case Q4_K: return w16 ? launch_stream_t<Q4_K>(a, early, stream) : 1;
    case Q5_K: return w16 ? launch_stream_t<Q5_K>(a, early, stream) : 1;
#define PYR_CASE(TY) case TY: return launch_stream_t<TY>(a, early, stream);
    PYR_CASE(Q4_0) PYR_CASE(Q4_1) PYR_CASE(Q5_0) PYR_CASE(Q5_1) PYR_CASE(Q8_0) PYR_CASE(Q8_1)
    PYR_CASE(Q2_K) PYR_CASE(Q3_K) PYR_CASE(Q6_K) PYR_CASE(IQ4_NL) PYR_CASE(IQ4_XS)
#undef PYR_CASE
    default: return 1;
  }
}

}  // namespace pyr
