// decode.cu -- the glue of one batch-1 decode step, device resident.
//
// The reference's executor runs these between its matvecs in Python fp64
// (pyrite/executor.py:621-755, pyrite/dense.py:473-513, pyrite/tensor_ops.py:
// 502-521, pyrite/sampler.py:12-15).  Here each is one small kernel; the token
// id and the position live in device memory, so a whole step can be captured
// in one CUDA graph and replayed token after token with no host round trip.
//
//   embed_kernel          hidden = token_embd[tokens[pos]]          (executor.py:647-652)
//   rmsnorm_encode_kernel out = x / rms(x) * w, re-encoded for the next matvec
//                                                                   (executor.py:621-624)
//   qk_rope_kv_kernel     per-head RMSNorm of q, k, NEOX RoPE at pos, k/v appended
//                         to the fp32 KV cache                      (executor.py:700-731)
//   attention_kernel      GQA softmax attention over positions 0..pos (executor.py:733-755)
//   silu_mul_encode_kernel act = silu(gate) * up, re-encoded       (dense.py:491-494)
//   argmax_*              greedy next token (first index of the max), tokens[pos+1],
//                         pos += 1                                  (sampler.py:12-15)
//
// Norms, RoPE and the per-head math are done in fp64 like the reference; the
// residual stream, q, k, v and logits are fp32.
#include <cfloat>

#include "kernels.cuh"
#include "../../include/pyrite_b200.h"

namespace pyr {
namespace {

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

template <int TY>
__global__ void __launch_bounds__(256) embed_kernel(const uint8_t* __restrict__ table, size_t row_bytes, int rows,
                                                    int cols, const int* __restrict__ tokens,
                                                    const int* __restrict__ pos, float* __restrict__ out) {
  pdl_wait();
  const int row = tokens[*pos];
  if (row < 0 || row >= rows) return;  // ids are validated on the host; never read outside the table
  const uint8_t* r = table + (size_t)row * row_bytes;
  constexpr int BS = Geo<TY>::bs, BPB = Geo<TY>::bpb;
  if constexpr (BS == 1) {
    for (int c = threadIdx.x; c < cols; c += blockDim.x) out[c] = scalar_val<TY, float>(r + (size_t)c * BPB);
  } else {
    for (int u = threadIdx.x; u < cols / 32; u += blockDim.x) {
      float v[32];
      decode_unit<TY, float>(r + (size_t)(u / (BS / 32)) * BPB, u % (BS / 32), v);
#pragma unroll
      for (int i = 0; i < 32; ++i) out[32 * u + i] = v[i];
    }
  }
  pdl_launch_dependents();
}

// out = x * inv * w with inv = 1/sqrt(mean(x^2) + eps) in fp64, then encoded.
__global__ void __launch_bounds__(1024) rmsnorm_encode_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                              int n, double eps, float* __restrict__ out,
                                                              uint8_t* __restrict__ ws) {
  __shared__ double shm[32];
  pdl_wait();
  double ss = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss += (double)x[i] * (double)x[i];
  const double total = block_sum(ss, shm);
  const double inv = 1.0 / sqrt(total / (double)(n > 0 ? n : 1) + eps);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int b = warp; b < n / 32; b += nw) {
    const int i = 32 * b + lane;
    const float v = (float)((double)x[i] * inv * (double)w[i]);
    if (out) out[i] = v;
    encode_block(v, lane, b, n, ws);
  }
  pdl_launch_dependents();
}

// One warp per head (q heads, then k heads, then v heads); head_dim 128, lane
// l holds elements l, l+32, l+64, l+96, so each NEOX pair (i, i+64) is in one
// lane.  q/k: optional RMSNorm with the head norm weight, then RoPE with the
// (cos, sin) table row of this position; v: copied.
__global__ void __launch_bounds__(256) qk_rope_kv_kernel(const float* __restrict__ qkv, const float* __restrict__ qnw,
                                                         const float* __restrict__ knw, int nq, int nkv, double eps,
                                                         const int* __restrict__ pos_ptr,
                                                         const double2* __restrict__ rope, int max_ctx,
                                                         float* __restrict__ qout, float* __restrict__ kcache,
                                                         float* __restrict__ vcache) {
  pdl_wait();
  constexpr int HD = 128;
  const int lane = threadIdx.x & 31;
  const int head = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int pos = *pos_ptr;
  if (head >= nq + 2 * nkv || pos < 0 || pos >= max_ctx) return;
  const float* src = qkv + (size_t)head * HD;
  double v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = (double)src[lane + 32 * k];
  const int kv_dim = nkv * HD;
  if (head >= nq + nkv) {  // v head: append as is
    float* dst = vcache + (size_t)pos * kv_dim + (size_t)(head - nq - nkv) * HD;
#pragma unroll
    for (int k = 0; k < 4; ++k) dst[lane + 32 * k] = (float)v[k];
    return;
  }
  const float* nw = head < nq ? qnw : knw;
  if (nw) {
    double ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const double inv = 1.0 / sqrt(ss / HD + eps);
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = v[k] * inv * (double)nw[lane + 32 * k];
  }
  // NEOX rotation of pairs (i, i + 64): (lane, lane+64) and (lane+32, lane+96)
  const double2 cs0 = rope[(size_t)pos * (HD / 2) + lane], cs1 = rope[(size_t)pos * (HD / 2) + lane + 32];
  const double r0 = v[0] * cs0.x - v[2] * cs0.y, r2 = v[0] * cs0.y + v[2] * cs0.x;
  const double r1 = v[1] * cs1.x - v[3] * cs1.y, r3 = v[1] * cs1.y + v[3] * cs1.x;
  float* dst = head < nq ? qout + (size_t)head * HD : kcache + (size_t)pos * kv_dim + (size_t)(head - nq) * HD;
  dst[lane] = (float)r0;
  dst[lane + 32] = (float)r1;
  dst[lane + 64] = (float)r2;
  dst[lane + 96] = (float)r3;
}

// One CTA per q head; scores for positions 0..pos (one warp per position at a
// time), softmax, then the value mix (thread i <- dim i).  fp32.
__global__ void __launch_bounds__(256) attention_kernel(const float* __restrict__ q, const float* __restrict__ kcache,
                                                        const float* __restrict__ vcache, const int* __restrict__ pos_ptr,
                                                        int nq, int nkv, float scale, int max_ctx,
                                                        float* __restrict__ out) {
  constexpr int HD = 128;
  extern __shared__ float sh[];  // [max_ctx] scores
  __shared__ float red[32];
  pdl_wait();
  const int h = blockIdx.x, kvh = h / (nq / nkv), kv_dim = nkv * HD;
  const int T = min(*pos_ptr + 1, max_ctx);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const float4 qv = reinterpret_cast<const float4*>(q + (size_t)h * HD)[lane];
  for (int t = warp; t < T; t += nw) {
    const float4 kk = reinterpret_cast<const float4*>(kcache + (size_t)t * kv_dim + (size_t)kvh * HD)[lane];
    float d = qv.x * kk.x + qv.y * kk.y + qv.z * kk.z + qv.w * kk.w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    if (lane == 0) sh[t] = d * scale;
  }
  __syncthreads();
  float m = -FLT_MAX;
  for (int t = threadIdx.x; t < T; t += blockDim.x) m = fmaxf(m, sh[t]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
  for (int w = 1; w < nw; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  float s = 0.f;
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const float e = expf(sh[t] - m);
    sh[t] = e;
    s += e;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  float total = 0.f;
  for (int w = 0; w < nw; ++w) total += red[w];
  const float invt = 1.0f / total;
  for (int i = threadIdx.x; i < HD; i += blockDim.x) {
    float acc = 0.f;
    for (int t = 0; t < T; ++t) acc += sh[t] * vcache[(size_t)t * kv_dim + (size_t)kvh * HD + i];
    out[(size_t)h * HD + i] = acc * invt;
  }
  pdl_launch_dependents();
}

// act = silu(gate) * up (silu(x) = x / (1 + exp(-x)), 0 for x <= -60 as the
// reference), written as fp32 and re-encoded for the down projection.
__global__ void __launch_bounds__(1024) silu_mul_encode_kernel(const float* __restrict__ gu, int f,
                                                               float* __restrict__ act, uint8_t* __restrict__ ws) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
  for (int b = gw; b < f / 32; b += nw) {
    const int i = 32 * b + lane;
    const float g = gu[i], u = gu[f + i];
    const float sg = g > -60.0f ? g / (1.0f + expf(-g)) : 0.0f;
    const float v = sg * u;
    act[i] = v;
    encode_block(v, lane, b, f, ws);
  }
  pdl_launch_dependents();
}

// Greedy sampling: per-CTA (max, first index), then one CTA picks the global
// one, stores it at tokens[pos+1] (unless that position is still prompt) and
// advances pos.
__device__ __forceinline__ void better(float& v, int& i, float ov, int oi) {
  if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
}

__global__ void __launch_bounds__(1024) argmax_partial_kernel(const float* __restrict__ x, int n,
                                                              float* __restrict__ pv, int* __restrict__ pi) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_wait();
  float v = -FLT_MAX;
  int idx = 0x7fffffff;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) better(v, idx, x[i], i);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) better(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { sv[warp] = v; si[warp] = idx; }
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? sv[lane] : -FLT_MAX;
    idx = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) better(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
    if (lane == 0) { pv[blockIdx.x] = v; pi[blockIdx.x] = idx; }
  }
  pdl_launch_dependents();
}

__global__ void __launch_bounds__(32) argmax_final_kernel(const float* __restrict__ pv, const int* __restrict__ pi,
                                                          int parts, int* __restrict__ tokens, int* __restrict__ pos,
                                                          int prompt_len, int max_ctx) {
  pdl_wait();
  float v = -FLT_MAX;
  int idx = 0x7fffffff;
  for (int k = threadIdx.x; k < parts; k += 32) better(v, idx, pv[k], pi[k]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) better(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
  if (threadIdx.x == 0) {
    const int p = *pos;
    if (p + 1 < max_ctx && p + 1 >= prompt_len) tokens[p + 1] = idx;
    *pos = p + 1;
  }
  pdl_launch_dependents();
}

int rc(int e) { return e > 0 ? PYRITE_E_CUDA : e; }

}  // namespace
}  // namespace pyr

using namespace pyr;

extern "C" {

int pyrite_cuda_embed(int type_id, const void* table, size_t rows, size_t cols, const int* tokens, const int* pos,
                      float* out, void* stream) {
  const TypeGeo* t = find_type(type_id);
  if (!t) return PYRITE_E_TYPE;
  if (!table || !tokens || !pos || !out || rows == 0 || cols == 0 || cols % (size_t)t->bs) return PYRITE_E_SHAPE;
  const size_t rb = cols / t->bs * t->bpb;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (type_id) {
#define PYR_CASE(TY)                                                                                          \
  case TY:                                                                                                    \
    return rc(launch_pdl(embed_kernel<TY>, dim3(1), dim3(256), 0, s, static_cast<const uint8_t*>(table), rb, \
                         (int)rows, (int)cols, tokens, pos, out));
    PYR_FOR_EACH_TYPE(PYR_CASE)
#undef PYR_CASE
    default:
      return PYRITE_E_TYPE;
  }
}

int pyrite_cuda_rmsnorm_encode(const float* x, const float* weight, size_t n, double eps, float* out, void* workspace,
                               size_t workspace_len, void* stream) {
  if (!x || !weight || !workspace || n == 0 || n % 32 || n > (1u << 20)) return PYRITE_E_SHAPE;
  if (workspace_len < pyrite_cuda_workspace_size(0, n, 1) || ((uintptr_t)workspace & 255)) return PYRITE_E_BUFFER;
  return rc(launch_pdl(rmsnorm_encode_kernel, dim3(1), dim3(1024), 0, static_cast<cudaStream_t>(stream), x, weight,
                       (int)n, eps, out, static_cast<uint8_t*>(workspace)));
}

int pyrite_cuda_qk_rope_kv(const float* qkv, const float* q_norm, const float* k_norm, int n_heads, int n_kv_heads,
                           int head_dim, double eps, const int* pos, const void* rope_table, int max_ctx, float* q_out,
                           float* k_cache, float* v_cache, void* stream) {
  if (head_dim != 128 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || !qkv || !pos || !rope_table ||
      !q_out || !k_cache || !v_cache || max_ctx <= 0)
    return PYRITE_E_SHAPE;
  const int warps = n_heads + 2 * n_kv_heads;
  return rc(launch_pdl(qk_rope_kv_kernel, dim3((warps + 7) / 8), dim3(256), 0, static_cast<cudaStream_t>(stream), qkv,
                       q_norm, k_norm, n_heads, n_kv_heads, eps, pos, static_cast<const double2*>(rope_table), max_ctx,
                       q_out, k_cache, v_cache));
}

int pyrite_cuda_attention(const float* q, const float* k_cache, const float* v_cache, const int* pos, int n_heads,
                          int n_kv_heads, int head_dim, int max_ctx, float* out, void* stream) {
  if (head_dim != 128 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || max_ctx <= 0 || !q ||
      !k_cache || !v_cache || !pos || !out)
    return PYRITE_E_SHAPE;
  const size_t smem = (size_t)max_ctx * sizeof(float);
  if (smem > 48 * 1024) return PYRITE_E_SHAPE;
  return rc(launch_pdl(attention_kernel, dim3(n_heads), dim3(256), smem, static_cast<cudaStream_t>(stream), q, k_cache,
                       v_cache, pos, n_heads, n_kv_heads, (float)(1.0 / sqrt((double)head_dim)), max_ctx, out));
}

int pyrite_cuda_silu_mul_encode(const float* gate_up, size_t f, float* act, void* workspace, size_t workspace_len,
                                void* stream) {
  if (!gate_up || !act || !workspace || f == 0 || f % 32) return PYRITE_E_SHAPE;
  if (workspace_len < pyrite_cuda_workspace_size(0, f, 1) || ((uintptr_t)workspace & 255)) return PYRITE_E_BUFFER;
  const int blocks = (int)((f / 32 + 31) / 32);
  return rc(launch_pdl(silu_mul_encode_kernel, dim3(blocks), dim3(1024), 0, static_cast<cudaStream_t>(stream),
                       gate_up, (int)f, act, static_cast<uint8_t*>(workspace)));
}

int pyrite_cuda_argmax_step(const float* logits, size_t n, void* scratch, size_t scratch_len, int* tokens, int* pos,
                            int prompt_len, int max_ctx, void* stream) {
  constexpr int kParts = 148;
  if (!logits || n == 0 || n > 0x7fffffffu || !scratch || !tokens || !pos) return PYRITE_E_SHAPE;
  if (scratch_len < kParts * 8) return PYRITE_E_BUFFER;
  float* pv = static_cast<float*>(scratch);
  int* pi = reinterpret_cast<int*>(pv + kParts);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int e = launch_pdl(argmax_partial_kernel, dim3(kParts), dim3(1024), 0, s, logits, (int)n, pv, pi);
  if (e) return rc(e);
  return rc(launch_pdl(argmax_final_kernel, dim3(1), dim3(32), 0, s, (const float*)pv, (const int*)pi, kParts, tokens,
                       pos, prompt_len, max_ctx));
}

}  // extern "C"
