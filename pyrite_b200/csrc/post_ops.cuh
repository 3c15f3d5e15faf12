// post_ops.cuh -- the small vector operations between the projections of a
// decode step, as block-level device functions.  decode.cu launches them as
// kernels of their own; the batch-1 matvec runs them in its last CTA to
// finish (a "post op"), which saves a launch and its latency per operation.
#pragma once
#include <cfloat>
#include <cstdint>

namespace pyr {

// Encode 32 values (lane l holds value l of block b) into the prepared-x
// layout of mv_tile.cu: digits x0, x1, scale s/254, and the two 16-value sums.
__device__ __forceinline__ void encode_block(float v, int lane, int b, int cols, uint8_t* ws) {
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
  ws[32 * b + lane] = (uint8_t)(int8_t)d0;
  ws[cols + 32 * b + lane] = (uint8_t)(int8_t)d1;
  float* scale = reinterpret_cast<float*>(ws + 2 * cols);
  float* sum16 = scale + cols / 32;
  if (lane == 0) scale[b] = s / 254.0f;
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
    act[i] = v;
    encode_block(v, lane, b, f, ws);
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
