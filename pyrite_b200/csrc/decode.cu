// decode.cu -- the glue of one batch-1 decode step, device resident.
//
// The reference's executor runs these between its matvecs in Python fp64
// (pyrite/executor.py:621-755, pyrite/dense.py:473-513, pyrite/tensor_ops.py:
// 502-521, pyrite/sampler.py:12-15).  Here each is one small kernel; the token
// id and the position live in device memory, so a whole step can be captured
// in one CUDA graph and replayed token after token with no host round trip.
// The RMSNorm, SwiGLU and argmax bodies (post_ops.cuh) also run fused into the
// last CTA of the preceding matvec (mv_tile.cu "post ops").
//
//   embed_kernel          hidden = token_embd[tokens[pos]]          (executor.py:647-652)
//   rmsnorm_encode_kernel out = x / rms(x) * w, re-encoded for the next matvec
//                                                                   (executor.py:621-624)
//   qk_rope_kv_kernel     per-head RMSNorm of q, k, NEOX RoPE at pos, k/v appended
//                         to the fp32 KV cache                      (executor.py:700-731)
//   attention_kernel      GQA softmax attention over positions 0..pos (executor.py:733-755)
//   attention_step_kernel the two above in one launch, one CTA per q head, plus the
//                         encoding of the output for the output projection
//   silu_mul_encode_kernel act = silu(gate) * up, re-encoded       (dense.py:491-494)
//   argmax_*              greedy next token (first index of the max), tokens[pos+1],
//                         pos += 1                                  (sampler.py:12-15)
//
// Norms, RoPE and the per-head math are done in fp64 like the reference; the
// residual stream, q, k, v and logits are fp32.
#include <cfloat>

#include "kernels.cuh"
#include "post_ops.cuh"
#include "../../include/pyrite_b200.h"

namespace pyr {
namespace {

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

// Row j of out (ld values apart) = table row ids[j * ids_stride + *pos] (the
// embedding lookup of several positions or sequences; pos may be NULL: 0; one
// CTA per row).
template <int TY>
__global__ void __launch_bounds__(256) embed_rows_kernel(const uint8_t* __restrict__ table, size_t row_bytes, int rows,
                                                         int cols, const int* __restrict__ ids, long long ids_stride,
                                                         const int* __restrict__ pos, float* __restrict__ out,
                                                         long long ld) {
  pdl_wait();
  const int row = ids[(size_t)blockIdx.x * ids_stride + (pos ? *pos : 0)];
  float* o = out + (size_t)blockIdx.x * ld;
  if (row >= 0 && row < rows) {  // ids are validated on the host; never read outside the table
    const uint8_t* r = table + (size_t)row * row_bytes;
    constexpr int BS = Geo<TY>::bs, BPB = Geo<TY>::bpb;
    if constexpr (BS == 1) {
      for (int c = threadIdx.x; c < cols; c += blockDim.x) o[c] = scalar_val<TY, float>(r + (size_t)c * BPB);
    } else {
      for (int u = threadIdx.x; u < cols / 32; u += blockDim.x) {
        float v[32];
        decode_unit<TY, float>(r + (size_t)(u / (BS / 32)) * BPB, u % (BS / 32), v);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[32 * u + i] = v[i];
      }
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
  block_rmsnorm_encode(x, w, n, eps, out, ws, shm);
  pdl_launch_dependents();
}

// Per-head RMSNorm (norm weight nw, may be NULL) and NEOX RoPE of one
// 128-value head by one warp: lane l holds elements l, l+32, l+64, l+96, so
// each rotated pair (i, i+64) is in one lane.  fp64 like the reference
// (executor.py:626-644, 700-731); rope_row = the (cos, sin) pairs of this
// position; rope = false copies the head (v).
__device__ __forceinline__ void head_norm_rope(const float* src, const float* nw, double eps, const double2* rope_row,
                                               bool rope, float* dst, int lane) {
  constexpr int HD = 128;
  double v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = (double)src[lane + 32 * k];
  if (!rope) {
#pragma unroll
    for (int k = 0; k < 4; ++k) dst[lane + 32 * k] = (float)v[k];
    return;
  }
  if (nw) {
    double ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const double inv = 1.0 / sqrt(ss / HD + eps);
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = v[k] * inv * (double)nw[lane + 32 * k];
  }
  const double2 cs0 = rope_row[lane], cs1 = rope_row[lane + 32];
  const double r0 = v[0] * cs0.x - v[2] * cs0.y, r2 = v[0] * cs0.y + v[2] * cs0.x;
  const double r1 = v[1] * cs1.x - v[3] * cs1.y, r3 = v[1] * cs1.y + v[3] * cs1.x;
  dst[lane] = (float)r0;
  dst[lane + 32] = (float)r1;
  dst[lane + 64] = (float)r2;
  dst[lane + 96] = (float)r3;
}

// One warp per head (q heads, then k heads, then v heads): q to qout, k and v
// appended to the caches at row pos.
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
  const int kv_dim = nkv * HD;
  const double2* rr = rope + (size_t)pos * (HD / 2);
  const float* src = qkv + (size_t)head * HD;
  if (head < nq) head_norm_rope(src, qnw, eps, rr, true, qout + (size_t)head * HD, lane);
  else if (head < nq + nkv)
    head_norm_rope(src, knw, eps, rr, true, kcache + (size_t)pos * kv_dim + (size_t)(head - nq) * HD, lane);
  else head_norm_rope(src, nullptr, eps, rr, false, vcache + (size_t)pos * kv_dim + (size_t)(head - nq - nkv) * HD, lane);
}

// Softmax attention of one q head (qh, 128 values, any address space) over
// cache rows 0..T-1 of kv head kvh (executor.py:733-755), one CTA of 256
// threads: one warp per position for the scores (kept in shared memory),
// max-subtracted softmax, then thread i < 128 mixes dimension i.  Returns the
// output value of dimension threadIdx.x (threads < 128).
__device__ __forceinline__ float attend_head(const float* qh, const float* __restrict__ kcache,
                                             const float* __restrict__ vcache, int kvh, int kv_dim, int T,
                                             float scale, float* sh, float* red) {
  constexpr int HD = 128;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const float4 qv = reinterpret_cast<const float4*>(qh)[lane];
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
  float acc = 0.f;
  if (threadIdx.x < HD)
    for (int t = 0; t < T; ++t) acc += sh[t] * vcache[(size_t)t * kv_dim + (size_t)kvh * HD + threadIdx.x];
  return acc * invt;
}

// One CTA per q head (256 threads).
__global__ void __launch_bounds__(256) attention_kernel(const float* __restrict__ q, const float* __restrict__ kcache,
                                                        const float* __restrict__ vcache, const int* __restrict__ pos_ptr,
                                                        int nq, int nkv, float scale, int max_ctx,
                                                        float* __restrict__ out) {
  constexpr int HD = 128;
  extern __shared__ float sh[];  // [max_ctx] scores
  __shared__ float red[32];
  pdl_wait();
  const int h = blockIdx.x, kvh = h / (nq / nkv);
  const int T = min(*pos_ptr + 1, max_ctx);
  const float o = attend_head(q + (size_t)h * HD, kcache, vcache, kvh, nkv * HD, T, scale, sh, red);
  if (threadIdx.x < HD) out[(size_t)h * HD + threadIdx.x] = o;
  pdl_launch_dependents();
}

// The fused step of one q head, its context split over CTAs (positions
// [c L, (c+1) L) in CTA c, L = ceil(max_ctx / nsplit)): every CTA with work
// normalises and rotates q; the CTA holding position pos also normalises and
// rotates its kv head's k and appends k and v at row pos (the CTAs of one GQA
// group write identical values).  Each CTA leaves (max score m_c, sum of
// exp(s - m_c), sum of exp(s - m_c) v) for its positions; the last CTA of the
// head to finish (a ticket, no waiting) merges them in chunk order, writes the
// head's output and encodes it for the output projection.  Within a CTA the 8
// warps take every 8th position, four at a time, so a long context keeps many
// loads in flight.
constexpr int kAttnPart = 132;    // floats per partial: m, s, 2 pad, o[128]

__global__ void __launch_bounds__(256) attention_step_kernel(
    const float* __restrict__ qkv, const float* __restrict__ qnw, const float* __restrict__ knw, int nq, int nkv,
    double eps, const int* __restrict__ pos_ptr, const double2* __restrict__ rope, int max_ctx, int chunk,
    float* __restrict__ kcache, float* __restrict__ vcache, float scale, float* __restrict__ out,
    uint8_t* __restrict__ ws, unsigned* __restrict__ tickets, float* __restrict__ parts) {
  constexpr int HD = 128;
  extern __shared__ float sh[];  // [chunk] scores
  __shared__ __align__(16) float qs[HD];
  __shared__ __align__(16) float acc[8][HD];
  __shared__ float red[32];
  __shared__ int last;
  pdl_wait();
  const int c = blockIdx.x, h = blockIdx.y, nsplit = gridDim.x;
  const int kvh = h / (nq / nkv), kv_dim = nkv * HD;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pos = *pos_ptr;
  const bool valid = pos >= 0 && pos < max_ctx;
  const int T = valid ? pos + 1 : 0;
  const int t0 = c * chunk, t1 = min(t0 + chunk, T), n = t1 - t0;
  float* part = parts + ((size_t)h * nsplit + c) * kAttnPart;
  if (n > 0) {
    const double2* rr = rope + (size_t)pos * (HD / 2);
    if (warp == 0) head_norm_rope(qkv + (size_t)h * HD, qnw, eps, rr, true, qs, lane);
    if (t1 == T) {  // this chunk holds the new position
      if (warp == 1)
        head_norm_rope(qkv + (size_t)(nq + kvh) * HD, knw, eps, rr, true,
                       kcache + (size_t)pos * kv_dim + (size_t)kvh * HD, lane);
      else if (warp == 2)
        head_norm_rope(qkv + (size_t)(nq + nkv + kvh) * HD, nullptr, eps, rr, false,
                       vcache + (size_t)pos * kv_dim + (size_t)kvh * HD, lane);
    }
    __syncthreads();
    // scores of this chunk: warp w takes positions t0 + w, t0 + w + 8, ... four at a time
    const float4 qv = reinterpret_cast<const float4*>(qs)[lane];
    for (int i = warp; i < n; i += 32) {
      float d[4];
      float4 kk[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = t0 + min(i + 8 * u, n - 1);
        kk[u] = reinterpret_cast<const float4*>(kcache + (size_t)t * kv_dim + (size_t)kvh * HD)[lane];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        d[u] = qv.x * kk[u].x + qv.y * kk[u].y + qv.z * kk[u].z + qv.w * kk[u].w;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d[u] += __shfl_xor_sync(0xffffffffu, d[u], o);
      }
      if (lane == 0) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (i + 8 * u < n) sh[i + 8 * u] = d[u] * scale;
      }
    }
    __syncthreads();
    float m = -FLT_MAX;
    for (int i = tid; i < n; i += blockDim.x) m = fmaxf(m, sh[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
    __syncthreads();
    float ssum = 0.f;
    for (int i = tid; i < n; i += blockDim.x) {
      const float e = expf(sh[i] - m);
      sh[i] = e;
      ssum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
    if (lane == 0) red[8 + warp] = ssum;
    __syncthreads();
    // value mix: warp w sums positions w, w + 8, ...; lane holds dims 4 lane .. 4 lane + 3
    float4 o4 = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = warp; i < n; i += 32) {
      float4 vv[4];
      float pw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = min(i + 8 * u, n - 1);
        vv[u] = reinterpret_cast<const float4*>(vcache + (size_t)(t0 + j) * kv_dim + (size_t)kvh * HD)[lane];
        pw[u] = i + 8 * u < n ? sh[j] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        o4.x += pw[u] * vv[u].x;
        o4.y += pw[u] * vv[u].y;
        o4.z += pw[u] * vv[u].z;
        o4.w += pw[u] * vv[u].w;
      }
    }
    reinterpret_cast<float4*>(acc[warp])[lane] = o4;
    __syncthreads();
    if (tid < HD) {
      float o = 0.f;
      for (int w = 0; w < 8; ++w) o += acc[w][tid];
      part[4 + tid] = o;
    }
    if (tid == 0) {
      float st = 0.f;
      for (int w = 0; w < 8; ++w) st += red[8 + w];
      part[0] = m;
      part[1] = st;
    }
  } else if (tid == 0) {
    part[0] = -FLT_MAX;
    part[1] = 0.f;
  }
  // the last CTA of this head merges the chunks
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    last = atomicAdd(tickets + h, 1u) == (unsigned)nsplit - 1 ? 1 : 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float* hp = parts + (size_t)h * nsplit * kAttnPart;
  float M = -FLT_MAX;
  for (int k = 0; k < nsplit; ++k) M = fmaxf(M, __ldcg(hp + (size_t)k * kAttnPart));
  if (tid < HD && T > 0) {
    float S = 0.f, O = 0.f;
    for (int k = 0; k < nsplit; ++k) {
      const float* pk = hp + (size_t)k * kAttnPart;
      const float sk = __ldcg(pk + 1);
      if (sk == 0.f) continue;
      const float f = expf(__ldcg(pk) - M);
      S += sk * f;
      O += __ldcg(pk + 4 + tid) * f;
    }
    const float o = O / S;
    out[(size_t)h * HD + tid] = o;
    encode_block(o, lane, h * (HD / 32) + warp, nq * HD, ws);
  }
  if (tid == 0) tickets[h] = 0u;
  pdl_launch_dependents();
}

// act = silu(gate) * up, written as fp32 and re-encoded for the down projection.
__global__ void __launch_bounds__(1024) silu_mul_encode_kernel(const float* __restrict__ gu, int f,
                                                               float* __restrict__ act, uint8_t* __restrict__ ws) {
  pdl_wait();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
  warps_silu_mul_encode(gu, f, act, ws, gw, nw);
  pdl_launch_dependents();
}

// Greedy sampling: per-CTA (max, first index), then one CTA picks the global
// one, stores it at tokens[pos+1] (unless that position is still prompt) and
// advances pos.
__global__ void __launch_bounds__(1024) argmax_partial_kernel(const float* __restrict__ x, int n,
                                                              float* __restrict__ pv, int* __restrict__ pi) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_wait();
  float v = -FLT_MAX;
  int idx = 0x7fffffff;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) better(v, idx, x[i], i);
  warp_best(v, idx);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { sv[warp] = v; si[warp] = idx; }
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? sv[lane] : -FLT_MAX;
    idx = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
    warp_best(v, idx);
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
  warp_best(v, idx);
  if (threadIdx.x == 0) {
    const int p = *pos;
    if (p + 1 < max_ctx && p + 1 >= prompt_len) tokens[p + 1] = idx;
    *pos = p + 1;
  }
  pdl_launch_dependents();
}

// ---- a block of prompt positions at once (batched prefill) ---------------------
// The same operations as above for `count` consecutive positions, each
// position's vectors a row of a row-major [count x n] array (the layout of the
// multi-column products: column j of the tensor-core product is row j here).

// Position of row j: first + *pos (pos may be NULL) + j * step -- consecutive
// positions of one sequence (prefill: step 1) or one position shared by
// several sequences (multi-sequence decode: step 0, each with its own cache
// cache_stride floats apart).  Rows outside [0, max_ctx) are skipped.
struct RowPos {
  int first;
  const int* pos;
  int step;
  long long cache_stride;
  int max_ctx;
  __device__ __forceinline__ int at(int j) const { return first + (pos ? *pos : 0) + j * step; }
};

// out[j] = x[j] * w / sqrt(mean(x[j]^2) + eps), fp64 statistics like
// rmsnorm_encode_kernel (executor.py:621-624); one CTA per row.
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const float* __restrict__ x, long long ldx,
                                                           const float* __restrict__ w, int n, double eps,
                                                           float* __restrict__ out, long long ldo) {
  __shared__ double shm[32];
  pdl_wait();
  const float* xr = x + (size_t)blockIdx.x * ldx;
  double ss = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss += (double)xr[i] * (double)xr[i];
  const double inv = 1.0 / sqrt(block_sum(ss, shm) / (double)(n > 0 ? n : 1) + eps);
  float* o = out + (size_t)blockIdx.x * ldo;
  for (int i = threadIdx.x; i < n; i += blockDim.x) o[i] = (float)((double)xr[i] * inv * (double)w[i]);
  pdl_launch_dependents();
}

// qk_rope_kv_kernel for row j of qkv (blockIdx.y = j) at position rp.at(j): q
// (normed, rotated) to row j of qout, k and v to row rp.at(j) of row j's
// caches (rp.cache_stride floats apart; 0: one cache).
__global__ void __launch_bounds__(256) qk_rope_kv_rows_kernel(const float* __restrict__ qkv, long long ldqkv,
                                                              const float* __restrict__ qnw,
                                                              const float* __restrict__ knw, int nq, int nkv,
                                                              double eps, RowPos rp, const double2* __restrict__ rope,
                                                              float* __restrict__ qout, long long ldq,
                                                              float* __restrict__ kcache_base,
                                                              float* __restrict__ vcache_base) {
  pdl_wait();
  constexpr int HD = 128;
  const int lane = threadIdx.x & 31;
  const int head = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int j = blockIdx.y, pos = rp.at(j);
  float* kcache = kcache_base + (size_t)j * rp.cache_stride;
  float* vcache = vcache_base + (size_t)j * rp.cache_stride;
  if (head < nq + 2 * nkv && pos >= 0 && pos < rp.max_ctx) {
    const int kv_dim = nkv * HD;
    const double2* rr = rope + (size_t)pos * (HD / 2);
    const float* src = qkv + (size_t)j * ldqkv + (size_t)head * HD;
    if (head < nq) head_norm_rope(src, qnw, eps, rr, true, qout + (size_t)j * ldq + (size_t)head * HD, lane);
    else if (head < nq + nkv)
      head_norm_rope(src, knw, eps, rr, true, kcache + (size_t)pos * kv_dim + (size_t)(head - nq) * HD, lane);
    else
      head_norm_rope(src, nullptr, eps, rr, false, vcache + (size_t)pos * kv_dim + (size_t)(head - nq - nkv) * HD,
                     lane);
  }
  pdl_launch_dependents();
}

// Causal GQA attention for queries at positions first + j (j < count, rows of
// q) over cache rows 0..first + j (executor.py:733-755, one new token after
// the other): one CTA per (q head, 16 queries), keys in tiles of 32 staged in
// shared memory, online max-subtracted softmax in fp32.  Thread t owns query
// t / 16 of the tile: scores of keys 2 (t % 16) and 2 (t % 16) + 1, output
// dimensions 8 (t % 16) .. 8 (t % 16) + 7.
constexpr int kAttnQB = 16, kAttnKT = 32, kAttnKStride = 129;  // padded K rows: no bank conflicts
__global__ void __launch_bounds__(256) attention_rows_kernel(const float* __restrict__ q, long long ldq,
                                                             const float* __restrict__ kcache_base,
                                                             const float* __restrict__ vcache_base, RowPos rp,
                                                             int count, int nq, int nkv, float* __restrict__ out,
                                                             long long ldo) {
  constexpr int HD = 128;
  __shared__ float qs[kAttnQB][HD];
  __shared__ float ks[kAttnKT * kAttnKStride];
  __shared__ __align__(16) float vs[kAttnKT][HD];
  __shared__ float ps[kAttnQB][kAttnKT];
  pdl_wait();
  // A CTA's 16 query slots: 16 consecutive positions of one sequence and one
  // head (rp.step 1: blockIdx = (head, block of rows)), or up to 16 query
  // heads of one KV head at the one position of one sequence (rp.step 0, each
  // row its own cache: blockIdx = (KV head x head block, row)); either way the
  // slots share every K/V tile the CTA loads.  A query's arithmetic does not
  // depend on its slot.
  const int group = nq / nkv, nhb = (group + kAttnQB - 1) / kAttnQB;
  const bool heads = rp.step == 0;
  const int tid = threadIdx.x, kv_dim = nkv * HD;
  const int j0 = heads ? blockIdx.y : blockIdx.y * kAttnQB;
  const int kvh = heads ? blockIdx.x / nhb : blockIdx.x / group;
  const int h0 = heads ? kvh * group + (blockIdx.x % nhb) * kAttnQB : blockIdx.x;  // slot 0's head
  const float* kcache = kcache_base + (size_t)j0 * rp.cache_stride;
  const float* vcache = vcache_base + (size_t)j0 * rp.cache_stride;
  const int qi = tid >> 4, sub = tid & 15;
  const int nqb = heads ? min(kAttnQB, kvh * group + group - h0) : min(kAttnQB, count - j0);
  for (int e = tid; e < kAttnQB * HD; e += blockDim.x) {
    const int i = e / HD, d = e % HD;
    const size_t src = heads ? (size_t)j0 * ldq + (size_t)(h0 + i) * HD : (size_t)(j0 + i) * ldq + (size_t)h0 * HD;
    qs[i][d] = i < nqb ? q[src + d] : 0.f;
  }
  const int qrow = heads ? j0 : j0 + min(qi, nqb - 1);  // this thread's query row
  const int qpos = rp.at(qrow);                         // and its position
  const bool qon = qi < nqb && qpos >= 0 && qpos < rp.max_ctx;
  // keys 0 .. kend - 1 are needed by some query (positions grow with the row)
  const int kend = min(rp.at(heads ? j0 : j0 + nqb - 1) + 1, rp.max_ctx);
  const float scale = (float)(1.0 / sqrt((double)HD));
  float m = -FLT_MAX, l = 0.f, o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int t0 = 0; t0 < kend; t0 += kAttnKT) {
    __syncthreads();  // the previous tile is consumed (and q is staged)
    for (int e = tid; e < kAttnKT * (HD / 4); e += blockDim.x) {
      const int k = e / (HD / 4), d4 = e % (HD / 4), t = t0 + k;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (t < kend) {
        kv = reinterpret_cast<const float4*>(kcache + (size_t)t * kv_dim + (size_t)kvh * HD)[d4];
        vv = reinterpret_cast<const float4*>(vcache + (size_t)t * kv_dim + (size_t)kvh * HD)[d4];
      }
      float* kr = ks + k * kAttnKStride + 4 * d4;
      kr[0] = kv.x; kr[1] = kv.y; kr[2] = kv.z; kr[3] = kv.w;
      reinterpret_cast<float4*>(vs[k])[d4] = vv;
    }
    __syncthreads();
    float sc[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int k = 2 * sub + u;
      const float* kr = ks + k * kAttnKStride;
      float d = 0.f;
#pragma unroll 8
      for (int e = 0; e < HD; ++e) d = fmaf(qs[qi][e], kr[e], d);
      sc[u] = (qon && t0 + k <= qpos) ? d * scale : -FLT_MAX;
    }
    float tm = fmaxf(sc[0], sc[1]);
#pragma unroll
    for (int o2 = 8; o2 > 0; o2 >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, o2));
    const float mn = fmaxf(m, tm);
    const float alpha = m == -FLT_MAX ? 0.f : expf(m - mn);
    float p0 = sc[0] == -FLT_MAX ? 0.f : expf(sc[0] - mn), p1 = sc[1] == -FLT_MAX ? 0.f : expf(sc[1] - mn);
    ps[qi][2 * sub] = p0;
    ps[qi][2 * sub + 1] = p1;
    float ps_sum = p0 + p1;
#pragma unroll
    for (int o2 = 8; o2 > 0; o2 >>= 1) ps_sum += __shfl_xor_sync(0xffffffffu, ps_sum, o2);
    l = l * alpha + ps_sum;
    m = mn;
    __syncthreads();
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] *= alpha;
    for (int k = 0; k < kAttnKT; ++k) {
      const float pk = ps[qi][k];
      const float4 a = reinterpret_cast<const float4*>(vs[k])[2 * sub], b = reinterpret_cast<const float4*>(vs[k])[2 * sub + 1];
      o[0] = fmaf(pk, a.x, o[0]); o[1] = fmaf(pk, a.y, o[1]); o[2] = fmaf(pk, a.z, o[2]); o[3] = fmaf(pk, a.w, o[3]);
      o[4] = fmaf(pk, b.x, o[4]); o[5] = fmaf(pk, b.y, o[5]); o[6] = fmaf(pk, b.z, o[6]); o[7] = fmaf(pk, b.w, o[7]);
    }
  }
  if (qon) {
    float* orow = out + (size_t)(heads ? j0 : j0 + qi) * ldo + (size_t)(heads ? h0 + qi : h0) * HD + 8 * sub;
    const float inv = 1.f / l;
#pragma unroll
    for (int e = 0; e < 8; ++e) orow[e] = o[e] * inv;
  }
  pdl_launch_dependents();
}

// act[j][i] = silu(gate) * up for row j = [gate (f) | up (f)] (dense.py:491-494).
__global__ void __launch_bounds__(256) silu_mul_rows_kernel(const float* __restrict__ gu, long long ldgu, int f,
                                                            float* __restrict__ act, long long lda) {
  pdl_wait();
  const float* g = gu + (size_t)blockIdx.y * ldgu;
  float* a = act + (size_t)blockIdx.y * lda;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < f; i += gridDim.x * blockDim.x) {
    const float x = g[i];
    a[i] = (x > -60.0f ? x / (1.0f + expf(-x)) : 0.0f) * g[f + i];
  }
  pdl_launch_dependents();
}

// Greedy token of row j of a [count x n] logits array (one sequence per row):
// the first index of the row's largest logit to tokens[j * tok_stride + *pos +
// 1] unless that position still holds the prompt (sampler.py:12-15); *pos is
// not advanced here (pyrite_cuda_advance_pos, once for all rows).
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float* __restrict__ x, long long ld, int n,
                                                           int* __restrict__ tokens, long long tok_stride,
                                                           const int* __restrict__ pos, int prompt_len, int max_ctx) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_wait();
  const float* r = x + (size_t)blockIdx.x * ld;
  float v = -FLT_MAX;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x) better(v, idx, r[i], i);
  warp_best(v, idx);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { sv[warp] = v; si[warp] = idx; }
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? sv[lane] : -FLT_MAX;
    idx = lane < (int)(blockDim.x >> 5) ? si[lane] : 0x7fffffff;
    warp_best(v, idx);
    const int p = *pos;
    if (lane == 0 && p + 1 < max_ctx && p + 1 >= prompt_len) tokens[(size_t)blockIdx.x * tok_stride + p + 1] = idx;
  }
  pdl_launch_dependents();
}

__global__ void advance_pos_kernel(int* pos) {
  pdl_wait();
  if (threadIdx.x == 0) *pos += 1;
  pdl_launch_dependents();
}

// One (value, index) pair from the partials of argmax_partial_kernel: this
// GPU's best logit of its vocabulary slice and its global id (base + index).
__global__ void __launch_bounds__(32) argmax_pair_kernel(const float* __restrict__ pv, const int* __restrict__ pi,
                                                         int parts, long long base, float* __restrict__ pair) {
  pdl_wait();
  float v = -FLT_MAX;
  int idx = 0x7fffffff;
  for (int k = threadIdx.x; k < parts; k += 32) better(v, idx, pv[k], pi[k]);
  warp_best(v, idx);
  if (threadIdx.x == 0) {
    pair[0] = v;
    reinterpret_cast<int*>(pair)[1] = (int)(base + idx);
  }
  pdl_launch_dependents();
}

// The greedy token from every GPU's pair (larger value first, then the lower
// id: sampler.py:12-15 over the whole vocabulary), written like argmax_final.
__global__ void __launch_bounds__(32) argmax_pick_kernel(const float* __restrict__ pairs, int n_pairs,
                                                         int* __restrict__ tokens, int* __restrict__ pos, int prompt_len,
                                                         int max_ctx) {
  pdl_wait();
  float v = -FLT_MAX;
  int idx = 0x7fffffff;
  for (int k = threadIdx.x; k < n_pairs; k += 32)
    better(v, idx, pairs[2 * k], reinterpret_cast<const int*>(pairs)[2 * k + 1]);
  warp_best(v, idx);
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

size_t pyrite_cuda_attention_scratch_size(int n_heads, int max_ctx) {
  if (n_heads <= 0 || max_ctx <= 0) return 0;
  const int nsplit = (max_ctx + 63) / 64 < 32 ? (max_ctx + 63) / 64 : 32;
  return 256 + (size_t)n_heads * nsplit * kAttnPart * sizeof(float) + ((size_t)n_heads * 4 + 255) / 256 * 256;
}

int pyrite_cuda_attention_step(const float* qkv, const float* q_norm, const float* k_norm, int n_heads, int n_kv_heads,
                               int head_dim, double eps, const int* pos, const void* rope_table, int max_ctx,
                               float* k_cache, float* v_cache, float* out, void* workspace, size_t workspace_len,
                               void* scratch, size_t scratch_len, void* stream) {
  if (head_dim != 128 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || !qkv || !pos || !rope_table ||
      !k_cache || !v_cache || !out || !workspace || max_ctx <= 0)
    return PYRITE_E_SHAPE;
  // context split: up to 32 CTAs per head, at least 64 positions each
  const int nsplit = (max_ctx + 63) / 64 < 32 ? (max_ctx + 63) / 64 : 32;
  const int chunk = (max_ctx + nsplit - 1) / nsplit;
  const size_t smem = (size_t)chunk * sizeof(float);
  if (smem > 32 * 1024) return PYRITE_E_SHAPE;
  const size_t n = (size_t)n_heads * head_dim;
  if (workspace_len < pyrite_cuda_workspace_size(0, n, 1) || ((uintptr_t)workspace & 255)) return PYRITE_E_BUFFER;
  if (!scratch || scratch_len < pyrite_cuda_attention_scratch_size(n_heads, max_ctx) || ((uintptr_t)scratch & 15))
    return PYRITE_E_BUFFER;
  unsigned* tickets = static_cast<unsigned*>(scratch);
  float* parts = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + ((size_t)n_heads * 4 + 255) / 256 * 256);
  return rc(launch_pdl(attention_step_kernel, dim3(nsplit, n_heads), dim3(256), smem, static_cast<cudaStream_t>(stream),
                       qkv, q_norm, k_norm, n_heads, n_kv_heads, eps, pos, static_cast<const double2*>(rope_table),
                       max_ctx, chunk, k_cache, v_cache, (float)(1.0 / sqrt((double)head_dim)), out,
                       static_cast<uint8_t*>(workspace), tickets, parts));
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

int pyrite_cuda_embed_rows(int type_id, const void* table, size_t rows, size_t cols, const int* ids,
                           long long ids_stride, const int* pos, size_t count, float* out, long long ldo,
                           void* stream) {
  const TypeGeo* t = find_type(type_id);
  if (!t) return PYRITE_E_TYPE;
  if (!table || !ids || !out || rows == 0 || cols == 0 || cols % (size_t)t->bs || count == 0 || count > 65535 ||
      ldo < (long long)cols || ids_stride < 0)
    return PYRITE_E_SHAPE;
  const size_t rb = cols / t->bs * t->bpb;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (type_id) {
#define PYR_CASE(TY)                                                                                            \
  case TY:                                                                                                      \
    return rc(launch_pdl(embed_rows_kernel<TY>, dim3((unsigned)count), dim3(256), 0, s,                         \
                         static_cast<const uint8_t*>(table), rb, (int)rows, (int)cols, ids, ids_stride, pos, out, \
                         ldo));
    PYR_FOR_EACH_TYPE(PYR_CASE)
#undef PYR_CASE
    default:
      return PYRITE_E_TYPE;
  }
}

int pyrite_cuda_rmsnorm_rows(const float* x, long long ldx, const float* weight, size_t n, size_t count, double eps,
                             float* out, long long ldo, void* stream) {
  if (!x || !weight || !out || n == 0 || n > (1u << 20) || count == 0 || count > 65535 || ldx < (long long)n ||
      ldo < (long long)n)
    return PYRITE_E_SHAPE;
  return rc(launch_pdl(rmsnorm_rows_kernel, dim3((unsigned)count), dim3(256), 0, static_cast<cudaStream_t>(stream), x,
                       ldx, weight, (int)n, eps, out, ldo));
}

namespace {
// Host checks of the row positions: with a device position only the kernel
// can check (it skips rows outside the cache); without one, all of them here.
bool rows_in_cache(int first, const int* pos, int step, int count, int max_ctx) {
  if (count <= 0 || count > 65535 || max_ctx <= 0 || (step != 0 && step != 1)) return false;
  if (pos) return true;
  return first >= 0 && (long long)first + (long long)(count - 1) * step < max_ctx;
}
}  // namespace

int pyrite_cuda_qk_rope_kv_rows(const float* qkv, long long ldqkv, const float* q_norm, const float* k_norm,
                                int n_heads, int n_kv_heads, int head_dim, double eps, int first, const int* pos,
                                int pos_step, long long cache_stride, int count, const void* rope_table, int max_ctx,
                                float* q_out, long long ldq, float* k_cache, float* v_cache, void* stream) {
  if (head_dim != 128 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || !qkv || !rope_table || !q_out ||
      !k_cache || !v_cache || !rows_in_cache(first, pos, pos_step, count, max_ctx) || cache_stride < 0 ||
      (pos_step == 0 && count > 1 && cache_stride < (long long)max_ctx * n_kv_heads * 128) ||
      ldqkv < (long long)(n_heads + 2 * n_kv_heads) * 128 || ldq < (long long)n_heads * 128)
    return PYRITE_E_SHAPE;
  const int heads = n_heads + 2 * n_kv_heads;
  RowPos rp{first, pos, pos_step, cache_stride, max_ctx};
  return rc(launch_pdl(qk_rope_kv_rows_kernel, dim3((unsigned)((heads + 7) / 8), (unsigned)count), dim3(256), 0,
                       static_cast<cudaStream_t>(stream), qkv, ldqkv, q_norm, k_norm, n_heads, n_kv_heads, eps, rp,
                       static_cast<const double2*>(rope_table), q_out, ldq, k_cache, v_cache));
}

int pyrite_cuda_attention_rows(const float* q, long long ldq, const float* k_cache, const float* v_cache,
                               long long cache_stride, int first, const int* pos, int pos_step, int count, int n_heads,
                               int n_kv_heads, int head_dim, int max_ctx, float* out, long long ldo, void* stream) {
  if (head_dim != 128 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || !q || !k_cache || !v_cache ||
      !out || !rows_in_cache(first, pos, pos_step, count, max_ctx) || cache_stride < 0 ||
      (pos_step == 0 && count > 1 && cache_stride < (long long)max_ctx * n_kv_heads * 128) ||
      ldq < (long long)n_heads * 128 || ldo < (long long)n_heads * 128 ||
      (((uintptr_t)k_cache | (uintptr_t)v_cache) & 15) || (cache_stride & 3))
    return PYRITE_E_SHAPE;
  // pos_step 1: (head, block of 16 rows); pos_step 0: (KV head x block of 16
  // of its query heads, row)
  const int group = n_heads / n_kv_heads, nhb = (group + kAttnQB - 1) / kAttnQB;
  const dim3 grid = pos_step ? dim3((unsigned)n_heads, (unsigned)((count + kAttnQB - 1) / kAttnQB))
                             : dim3((unsigned)(n_kv_heads * nhb), (unsigned)count);
  RowPos rp{first, pos, pos_step, cache_stride, max_ctx};
  return rc(launch_pdl(attention_rows_kernel, grid, dim3(256), 0,
                       static_cast<cudaStream_t>(stream), q, ldq, k_cache, v_cache, rp, count, n_heads, n_kv_heads,
                       out, ldo));
}

int pyrite_cuda_argmax_rows(const float* logits, long long ld, size_t n, size_t count, int* tokens,
                            long long tok_stride, const int* pos, int prompt_len, int max_ctx, void* stream) {
  if (!logits || !tokens || !pos || n == 0 || n > 0x7fffffffu || count == 0 || count > 65535 || ld < (long long)n ||
      tok_stride < max_ctx)
    return PYRITE_E_SHAPE;
  return rc(launch_pdl(argmax_rows_kernel, dim3((unsigned)count), dim3(1024), 0, static_cast<cudaStream_t>(stream),
                       logits, ld, (int)n, tokens, tok_stride, pos, prompt_len, max_ctx));
}

int pyrite_cuda_advance_pos(int* pos, void* stream) {
  if (!pos) return PYRITE_E_BUFFER;
  return rc(launch_pdl(advance_pos_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), pos));
}

int pyrite_cuda_silu_mul_rows(const float* gate_up, long long ldgu, size_t f, size_t count, float* act, long long lda,
                              void* stream) {
  if (!gate_up || !act || f == 0 || f > (1u << 24) || count == 0 || count > 65535 || ldgu < 2 * (long long)f ||
      lda < (long long)f)
    return PYRITE_E_SHAPE;
  const unsigned bx = (unsigned)((f + 1023) / 1024);
  return rc(launch_pdl(silu_mul_rows_kernel, dim3(bx, (unsigned)count), dim3(256), 0,
                       static_cast<cudaStream_t>(stream), gate_up, ldgu, (int)f, act, lda));
}

int pyrite_cuda_argmax_local(const float* logits, size_t n, long long index_base, void* scratch, size_t scratch_len,
                             void* pair, void* stream) {
  constexpr int kParts = 148;
  if (!logits || n == 0 || n > 0x7fffffffu || index_base < 0 || index_base + (long long)n > 0x7fffffffLL || !pair)
    return PYRITE_E_SHAPE;
  if (!scratch || scratch_len < kParts * 8 || ((uintptr_t)pair & 7)) return PYRITE_E_BUFFER;
  float* pv = static_cast<float*>(scratch);
  int* pi = reinterpret_cast<int*>(pv + kParts);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int e = launch_pdl(argmax_partial_kernel, dim3(kParts), dim3(1024), 0, s, logits, (int)n, pv, pi);
  if (e) return rc(e);
  return rc(launch_pdl(argmax_pair_kernel, dim3(1), dim3(32), 0, s, (const float*)pv, (const int*)pi, kParts,
                       index_base, static_cast<float*>(pair)));
}

int pyrite_cuda_argmax_pick(const void* pairs, size_t n_pairs, int* tokens, int* pos, int prompt_len, int max_ctx,
                            void* stream) {
  if (!pairs || n_pairs == 0 || n_pairs > 4096 || ((uintptr_t)pairs & 7) || !tokens || !pos) return PYRITE_E_BUFFER;
  return rc(launch_pdl(argmax_pick_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream),
                       static_cast<const float*>(pairs), (int)n_pairs, tokens, pos, prompt_len, max_ctx));
}

}  // extern "C"
