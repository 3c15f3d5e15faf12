// post_ops.cuh -- the small vector operations between the projections of a
// decode step, as block-level device functions.  decode.cu launches them as
// kernels of their own; the batch-1 matvec runs them in its last CTA to
// finish (a "post op"), which saves a launch and its latency per operation.
#pragma once
#include <cfloat>
#include <cstdint>

namespace pyr {

// Encoded activation (the batch-1 kernels' prepared x), per column of `cols`
// values (cols % 32 == 0):
//   x0[cols] int8 | x1[cols] int8 | scale[cols/32] fp32 | sum16[cols/16] fp32 | x2[cols] int8
// For a 32-value block of largest magnitude amax, t = v * 127 / amax and
//   v ~ (amax / 127) * (x0 + x1 / 254 + x2 / 254^2),
// x0 = rint(t), x1 = rint((t - x0) * 254), x2 = rint(((t - x0) * 254 - x1) * 254)
// (no clamps: |t| rounds to at most 127 and each remainder is at most 1/2).
// scale[b] = amax / 127 / 254, stored NEGATIVE for a "wide" block: one in which
// at most 8 of the 32 values lie within a factor 32 of amax, i.e. one or a few
// outliers (an outlier channel) over values far smaller.  Two digits bound
// each value's error by amax / 64516, which is large next to those smaller
// values; the kernels add the third digit for wide blocks, bringing the bound
// to amax / 16.4e6.  Gaussian, Laplace and SiLU(gate) * up activations are
// almost never wide (0 to ~4% of blocks), so the common path pays nothing.
__host__ __device__ constexpr long long x2_offset(long long cols) { return 2 * cols + cols / 8 + cols / 4; }
__host__ __device__ constexpr long long encoded_bytes(long long cols) { return x2_offset(cols) + cols; }
constexpr int kWideMaxBig = 8;      // a block is wide when at most this many values are "big":
constexpr float kBigRatio = 32.0f;  // within this factor of the block's largest magnitude

__device__ __forceinline__ float digit_ratio(float amax) { return amax > 0.0f ? 127.0f / amax : 0.0f; }
// Every step rounded on its own (no fused multiply-add), so every encoder
// writes the same digits for the same value whatever the compiler contracts.
__device__ __forceinline__ void three_digits(float v, float r, int& d0, int& d1, int& d2) {
  const float t = __fmul_rn(v, r);
  d0 = __float2int_rn(t);
  const float u = __fmul_rn(__fsub_rn(t, (float)d0), 254.0f);
  d1 = __float2int_rn(u);
  d2 = __float2int_rn(__fmul_rn(__fsub_rn(u, (float)d1), 254.0f));
}
__device__ __forceinline__ bool is_big(float v, float amax) { return fabsf(v) * kBigRatio >= amax; }
__device__ __forceinline__ bool wide_block(int n_big, float amax) { return amax > 0.0f && n_big <= kWideMaxBig; }

// Encode 32 values (lane l holds value l of block b) into the layout above.
__device__ __forceinline__ void encode_block(float v, int lane, int b, int cols, uint8_t* ws) {
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = amax / 127.0f;
  const bool wide = wide_block(__popc(__ballot_sync(0xffffffffu, is_big(v, amax))), amax);
  int d0, d1, d2;
  three_digits(v, digit_ratio(amax), d0, d1, d2);
  float s16 = v;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
  ws[32 * b + lane] = (uint8_t)(int8_t)d0;
  ws[cols + 32 * b + lane] = (uint8_t)(int8_t)d1;
  ws[x2_offset(cols) + 32 * b + lane] = (uint8_t)(int8_t)d2;
  float* scale = reinterpret_cast<float*>(ws + 2 * cols);
  float* sum16 = scale + cols / 32;
  if (lane == 0) scale[b] = wide ? -(s / 254.0f) : s / 254.0f;
  if ((lane & 15) == 0) sum16[2 * b + (lane >> 4)] = s16;
}

template <typename T>
__device__ __forceinline__ T block_sum(T v, T* shm) {  // blockDim.x multiple of 32, <= 1024
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) shm[warp] = v;
  __syncthreads();
  T t = lane < nw ? shm[lane] : T(0);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

// out = x * w / sqrt(mean(x^2) + eps), statistics in fp64 (executor.py:621-624),
// then encoded; one CTA, any multiple of 32 threads.  out may be NULL.  x is
// read through L2 (it may have just been written by other CTAs).
__device__ __forceinline__ void block_rmsnorm_encode(const float* x, const float* w, int n, double eps, float* out,
                                                     uint8_t* ws, double* shm) {
  double ss = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const double xi = (double)__ldcg(x + i);
    ss += xi * xi;
  }
  const double total = block_sum(ss, shm);
  const double inv = 1.0 / sqrt(total / (double)(n > 0 ? n : 1) + eps);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int b = warp; b < n / 32; b += nw) {
    const int i = 32 * b + lane;
    const float v = (float)((double)__ldcg(x + i) * inv * (double)w[i]);
    if (out) out[i] = v;
    encode_block(v, lane, b, n, ws);
  }
}

// act = silu(gate) * up for gu = [gate (f) | up (f)] (silu(x) = x / (1 + exp(-x)),
// 0 for x <= -60 as the reference, tensor_ops.py:509-510), then encoded.
// Warps take 32-value blocks b = first, first + stride, ...
__device__ __forceinline__ void warps_silu_mul_encode(const float* gu, int f, float* act, uint8_t* ws, int first,
                                                      int stride) {
  const int lane = threadIdx.x & 31;
  for (int b = first; b < f / 32; b += stride) {
    const int i = 32 * b + lane;
    const float g = __ldcg(gu + i), u = __ldcg(gu + f + i);
    const float sg = g > -60.0f ? g / (1.0f + expf(-g)) : 0.0f;
    const float v = sg * u;
    if (act) act[i] = v;
    encode_block(v, lane, b, f, ws);
  }
}

// ---- the same encodings for a matvec CTA's prologue -------------------------
// Every CTA of a matvec that computes its own x' encodes the whole vector, so
// the work is laid out for latency: thread t takes the 16-value groups
// g = t, t + blockDim.x, ... as four float4 loads; a 32-value block is the
// group pair (2b, 2b + 1), held by adjacent lanes.  Per value the arithmetic is
// encode_block's, and the 16-value sums add in the order of its shuffle tree
// (offsets 8, 4, 2, 1), so the bytes equal those of the kernels above for the
// same input values.

// Encode group g (values v): both lanes of a pair call this together (the
// amax exchange is a shuffle), `on` equal for the pair.
__device__ __forceinline__ void encode_group(const float (&v)[16], int g, int cols, bool on, uint8_t* enc,
                                             float* out) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  const float s = amax / 127.0f, r = digit_ratio(amax);
  int nbig = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) nbig += is_big(v[i], amax) ? 1 : 0;
  nbig += __shfl_xor_sync(0xffffffffu, nbig, 1);
  uint32_t p0[4], p1[4], p2[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    p0[q] = 0u;
    p1[q] = 0u;
    p2[q] = 0u;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int d0, d1, d2;
      three_digits(v[4 * q + j], r, d0, d1, d2);
      p0[q] |= ((uint32_t)d0 & 0xffu) << (8 * j);
      p1[q] |= ((uint32_t)d1 & 0xffu) << (8 * j);
      p2[q] |= ((uint32_t)d2 & 0xffu) << (8 * j);
    }
  }
  float a8[8], a4[4];
#pragma unroll
  for (int i = 0; i < 8; ++i) a8[i] = v[i] + v[i + 8];
#pragma unroll
  for (int i = 0; i < 4; ++i) a4[i] = a8[i] + a8[i + 4];
  const float s16 = (a4[0] + a4[2]) + (a4[1] + a4[3]);
  if (!on) return;
  *reinterpret_cast<uint4*>(enc + 16 * g) = make_uint4(p0[0], p0[1], p0[2], p0[3]);
  *reinterpret_cast<uint4*>(enc + cols + 16 * g) = make_uint4(p1[0], p1[1], p1[2], p1[3]);
  *reinterpret_cast<uint4*>(enc + x2_offset(cols) + 16 * g) = make_uint4(p2[0], p2[1], p2[2], p2[3]);
  float* scale = reinterpret_cast<float*>(enc + 2 * cols);
  if ((g & 1) == 0) scale[g >> 1] = wide_block(nbig, amax) ? -(s / 254.0f) : s / 254.0f;
  scale[cols / 32 + g] = s16;
  if (out) {
    float4* o = reinterpret_cast<float4*>(out + 16 * g);
#pragma unroll
    for (int q = 0; q < 4; ++q) o[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  }
}

__device__ __forceinline__ void load16(const float* p, float (&v)[16]) {  // through L2: p may be fresh
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 t = __ldcg(q + i);
    v[4 * i] = t.x;
    v[4 * i + 1] = t.y;
    v[4 * i + 2] = t.z;
    v[4 * i + 3] = t.w;
  }
}

// block_rmsnorm_encode for a CTA prologue (x, w 16-byte aligned, n % 128 == 0:
// the x2 plane's 16-byte stores need x2_offset(n) % 16 == 0).
// Each thread's first group of x and w stays in registers, so for n up to
// 16 * blockDim.x the statistics and the encoding cost one round trip to L2.
// 1 / sqrt(mean(x^2) + eps) of n values (x 16-byte aligned, n % 16 == 0) for
// the whole CTA, in a fixed order (every CTA that calls it gets the same
// bits); x0 returns the thread's first 16-value group (zeros past the end).
__device__ __forceinline__ double cta_rms_inv(const float* x, int n, double eps, double* shm, float4 (&x0)[4]) {
  const int G = n / 16, nt = blockDim.x, tid = threadIdx.x;
  double ss = 0.0;
#pragma unroll
  for (int q = 0; q < 4; ++q) x0[q] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (tid < G) {
#pragma unroll
    for (int q = 0; q < 4; ++q) x0[q] = __ldcg(reinterpret_cast<const float4*>(x + 16 * tid) + q);
  }
#pragma unroll
  for (int q = 0; q < 4; ++q)
    ss += (double)x0[q].x * x0[q].x + (double)x0[q].y * x0[q].y + (double)x0[q].z * x0[q].z +
          (double)x0[q].w * x0[q].w;
  for (int g = tid + nt; g < G; g += nt) {
    float v[16];
    load16(x + 16 * g, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) ss += (double)v[i] * (double)v[i];
  }
  const double total = block_sum(ss, shm);
  return 1.0 / sqrt(total / (double)(n > 0 ? n : 1) + eps);
}

__device__ __forceinline__ void cta_rmsnorm_encode(const float* x, const float* w, int n, double eps, float* out,
                                                   uint8_t* enc, double* shm) {
  const int G = n / 16, nt = blockDim.x, tid = threadIdx.x;
  float4 x0[4], w0[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) w0[q] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (tid < G) {
#pragma unroll
    for (int q = 0; q < 4; ++q) w0[q] = __ldg(reinterpret_cast<const float4*>(w + 16 * tid) + q);
  }
  const double inv = cta_rms_inv(x, n, eps, shm, x0);
  for (int g0 = 0; g0 < G; g0 += nt) {  // same trip count in every thread
    const int g = g0 + tid;
    const bool on = g < G;
    float v[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float4 xv = x0[q], wv = w0[q];
      if (g0 > 0 && on) {
        xv = __ldcg(reinterpret_cast<const float4*>(x + 16 * g) + q);
        wv = __ldg(reinterpret_cast<const float4*>(w + 16 * g) + q);
      }
      v[4 * q] = (float)((double)xv.x * inv * (double)wv.x);
      v[4 * q + 1] = (float)((double)xv.y * inv * (double)wv.y);
      v[4 * q + 2] = (float)((double)xv.z * inv * (double)wv.z);
      v[4 * q + 3] = (float)((double)xv.w * inv * (double)wv.w);
    }
    encode_group(v, g, n, on, enc, out);
  }
}

// warps_silu_mul_encode for a CTA prologue (gu 16-byte aligned, f % 128 == 0).
__device__ __forceinline__ void cta_silu_mul_encode(const float* gu, int f, float* out, uint8_t* enc) {
  const int G = f / 16, nt = blockDim.x;
  for (int g0 = 0; g0 < G; g0 += nt) {
    const int g = g0 + threadIdx.x;
    const bool on = g < G;
    float v[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float4 gv = make_float4(0.f, 0.f, 0.f, 0.f), uv = gv;
      if (on) {
        gv = __ldcg(reinterpret_cast<const float4*>(gu + 16 * g) + q);
        uv = __ldcg(reinterpret_cast<const float4*>(gu + f + 16 * g) + q);
      }
      const float ga[4] = {gv.x, gv.y, gv.z, gv.w}, ua[4] = {uv.x, uv.y, uv.z, uv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float sg = ga[j] > -60.0f ? ga[j] / (1.0f + expf(-ga[j])) : 0.0f;
        v[4 * q + j] = sg * ua[j];
      }
    }
    encode_group(v, g, f, on, enc, out);
  }
}

// Greedy order: larger value first, then the lower index (sampler.py:12-15).
__device__ __forceinline__ void better(float& v, int& i, float ov, int oi) {
  if (ov > v || (ov == v && oi < i)) {
    v = ov;
    i = oi;
  }
}
__device__ __forceinline__ void warp_best(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) better(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
}

}  // namespace pyr
