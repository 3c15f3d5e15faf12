// moe.cu -- the routed-expert feed-forward of a Qwen3-MoE decode step
// (pyrite/executor.py:672-683 _expert, :757-793 _moe), device resident.
//
//   moe_route_kernel        softmax over the router logits (fp64), the top-k
//                           experts in (-p, e) order, their weights
//                           (renormalised when norm_topk_prob, then scaled)
//   pyrite_cuda_matvec_experts
//                           the batch-1 matvec over the k selected slices of a
//                           stacked expert tensor in one launch; the expert ids
//                           are read on the device, so the whole step stays in
//                           one CUDA graph (qwen3_moe.py:364-398: expert e of a
//                           stacked (cols, rows, E) tensor is the contiguous
//                           byte range e * rows * row_bytes)
//   moe_silu_mul_encode_kernel
//                           act_j = silu(gate_j) * up_j for every selected
//                           expert j, each encoded for the down projection
//   moe_combine_kernel      hidden += sum_j w_j * down_j, summed in rank order
#include <cfloat>

#include "kernels.cuh"
#include "post_ops.cuh"
#include "../../include/pyrite_b200.h"

namespace pyr {
namespace {

struct RouteArgs {
  int n, k, norm;
  double scale;
  int shards, index;
  int* ids;
  float* weights;
  int* global_ids;
};

// The routing of one token by the first warp of a CTA (the other threads
// return at once; no block barrier inside): n <= 4096 router logits (read
// through L2: other CTAs may just have written them), k <= 32.  Lane l takes
// experts l, l + 32, ...; maxima, sums and the k argmax rounds are warp
// butterflies (the same bits on every lane).  Experts sharded by id over
// `shards` GPUs: this one (shard `index`) holds experts e % shards == index
// at local slot e / shards; a selected expert it does not hold gets id -1
// and weight 0 (the expert matvecs skip it).  (The block-wide form took two
// block barriers per argmax round: ~17 us per layer for the configs[3]
// router, cold.)
__device__ void route_block(const float* __restrict__ logits, const RouteArgs& a) {
  __shared__ double p[4096];
  const int tid = threadIdx.x, lane = tid & 31;
  if (tid >= 32) return;
  const int n = a.n, k = a.k;
  // softmax in fp64 (tensor_ops.py:513-521): exp(v - max) / sum
  double m = -DBL_MAX;
  for (int e = lane; e < n; e += 32) m = fmax(m, (double)__ldcg(logits + e));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
  double s = 0.0;
  for (int e = lane; e < n; e += 32) {
    const double x = exp((double)__ldcg(logits + e) - m);
    p[e] = x;
    s += x;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  for (int e = lane; e < n; e += 32) p[e] /= s;
  // k rounds of (max p, lowest e); a chosen expert drops out with p = -1.
  // Round r's choice stays in lane r (cp, ci).
  double cp = 0.0;
  int ci = 0;
  for (int r = 0; r < k; ++r) {
    int bi = 0x7fffffff;
    double bp = -2.0;
    for (int e = lane; e < n; e += 32)
      if (p[e] > bp || (p[e] == bp && e < bi)) {
        bp = p[e];
        bi = e;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {  // compare in fp64, lowest index on ties
      const double op = __shfl_xor_sync(0xffffffffu, bp, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (op > bp || (op == bp && oi < bi)) {
        bp = op;
        bi = oi;
      }
    }
    if (lane == r) {
      cp = bp;
      ci = bi;
    }
    if (lane == (bi & 31)) p[bi] = -1.0;  // the lane that owns expert bi
    __syncwarp();
  }
  double tot = 0.0;  // in round order, as the weights are renormalised
  for (int r = 0; r < k; ++r) tot += __shfl_sync(0xffffffffu, cp, r);
  if (lane < k) {
    double w = cp;
    if (a.norm && tot > 0.0) w = w / tot;
    if (a.scale != 1.0) w = w * a.scale;
    const bool mine = ci % a.shards == a.index;
    a.ids[lane] = mine ? ci / a.shards : -1;
    a.weights[lane] = mine ? (float)w : 0.0f;
    if (a.global_ids) a.global_ids[lane] = ci;
  }
}

__global__ void __launch_bounds__(32) moe_route_kernel(const float* __restrict__ logits, RouteArgs a) {
  pdl_wait();
  route_block(logits, a);
  pdl_launch_dependents();
}

// The F32 router product of several sequences: logits[b][e] = sum_c W[e][c] x[b][c]
// accumulated in fp64 and rounded to fp32 once, as the one-sequence routing
// launch computes it (one CTA per (expert, sequence)).
__global__ void __launch_bounds__(256) moe_router_rows_kernel(const float* __restrict__ W, int h,
                                                              const float* __restrict__ x, long long ldx,
                                                              float* __restrict__ logits, long long ld) {
  __shared__ double dshm[32];
  pdl_wait();
  const int e = blockIdx.x, b = blockIdx.y;
  const float* rf = W + (size_t)e * (size_t)h;
  const float* xb = x + (size_t)b * ldx;
  double acc = 0.0;
  for (int c = threadIdx.x; c < h; c += blockDim.x) acc += (double)__ldg(rf + c) * (double)xb[c];
  const double total = block_sum(acc, dshm);
  if (threadIdx.x == 0) logits[(size_t)b * ld + e] = (float)total;
  pdl_launch_dependents();
}

// moe_route_kernel for row blockIdx.x of a [count x n] logits array: its top_k
// experts and weights to row blockIdx.x of ids / weights (top_k apart).
__global__ void __launch_bounds__(32) moe_route_rows_kernel(const float* __restrict__ logits, long long ld,
                                                             RouteArgs a) {
  pdl_wait();
  RouteArgs r = a;
  r.ids += (size_t)blockIdx.x * a.k;
  r.weights += (size_t)blockIdx.x * a.k;
  if (r.global_ids) r.global_ids += (size_t)blockIdx.x * a.k;
  route_block(logits + (size_t)blockIdx.x * ld, r);
  pdl_launch_dependents();
}

// The F32 router matvec and the routing in one launch.  CTA r computes logit
// r: every thread a strided share of the row in fp64 (the reference's native
// products accumulate in fp64), one fixed-order block sum, rounded to fp32
// once -- one round trip to memory per CTA instead of a warp walking the row.
// The last CTA to finish (a ticket, no CTA waits) routes.  W: E rows of h F32
// values; float4 loads when W and x are 16-byte aligned and h % 4 == 0.
struct RouterNorm {  // x is the residual: RMSNorm it first (nw != nullptr)
  const float* nw;
  double eps;
  float* out;    // the normalised x (fp32), written by CTA 0
  uint8_t* ws;   // and its encoding for the expert products
};

__global__ void __launch_bounds__(256) moe_router_route_kernel(const float* __restrict__ W, int h,
                                                               const float* __restrict__ x,
                                                               float* __restrict__ logits, unsigned* ticket,
                                                               RouteArgs a, RouterNorm nm) {
  __shared__ double dshm[32];
  __shared__ int last;
  pdl_wait();
  const int r = blockIdx.x, tid = threadIdx.x;
  const float* rf = W + (size_t)r * (size_t)h;
  double acc = 0.0;
  if (nm.nw) {  // every CTA computes the same statistics; the row takes the normalised values
    float4 x0[4];
    const double inv = cta_rms_inv(x, h, nm.eps, dshm, x0);
    for (int g = tid; g < h / 16; g += blockDim.x) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 xv = g == tid ? x0[q] : __ldcg(reinterpret_cast<const float4*>(x + 16 * g) + q);
        const float4 wv = __ldg(reinterpret_cast<const float4*>(nm.nw + 16 * g) + q);
        const float4 rv = __ldg(reinterpret_cast<const float4*>(rf + 16 * g) + q);
        acc += (double)rv.x * (double)(float)((double)xv.x * inv * (double)wv.x);
        acc += (double)rv.y * (double)(float)((double)xv.y * inv * (double)wv.y);
        acc += (double)rv.z * (double)(float)((double)xv.z * inv * (double)wv.z);
        acc += (double)rv.w * (double)(float)((double)xv.w * inv * (double)wv.w);
      }
    }
    if (r == 0) cta_rmsnorm_encode(x, nm.nw, h, nm.eps, nm.out, nm.ws, dshm);
  } else if ((((uintptr_t)rf | (uintptr_t)x) & 15) == 0 && (h & 3) == 0) {
    for (int c = 4 * tid; c < h; c += 4 * (int)blockDim.x) {
      const float4 w4 = __ldg(reinterpret_cast<const float4*>(rf + c));
      const float4 x4 = __ldcg(reinterpret_cast<const float4*>(x + c));
      acc += (double)w4.x * (double)x4.x;
      acc += (double)w4.y * (double)x4.y;
      acc += (double)w4.z * (double)x4.z;
      acc += (double)w4.w * (double)x4.w;
    }
  } else {
    for (int c = tid; c < h; c += blockDim.x) acc += (double)__ldg(rf + c) * (double)__ldcg(x + c);
  }
  const double total = block_sum(acc, dshm);
  if (tid == 0) {
    logits[r] = (float)total;
    __threadfence();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1 ? 1 : 0;
  }
  __syncthreads();
  if (last) {
    __threadfence();
    route_block(logits, a);
    if (tid == 0) *ticket = 0u;
  }
  pdl_launch_dependents();
}

// act_j = silu(gate_j) * up_j for j < n_sel (gate and up: n_sel x ff), encoded
// at ws + j * ws_stride.  One warp per 32-value block.
__global__ void __launch_bounds__(256) moe_silu_mul_encode_kernel(const float* __restrict__ gate,
                                                                  const float* __restrict__ up, int ff, int n_sel,
                                                                  float* __restrict__ act, uint8_t* __restrict__ ws,
                                                                  long long ws_stride) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
  const int per = ff / 32;
  for (int t = gw; t < per * n_sel; t += nw) {
    const int j = t / per, b = t - j * per;
    const int i = 32 * b + lane;
    const float g = gate[(size_t)j * ff + i], u = up[(size_t)j * ff + i];
    const float sg = g > -60.0f ? g / (1.0f + expf(-g)) : 0.0f;
    const float v = sg * u;
    act[(size_t)j * ff + i] = v;
    encode_block(v, lane, b, ff, ws + (size_t)j * (size_t)ws_stride);
  }
  pdl_launch_dependents();
}

// Row b of hidden (ldh apart) += sum_{j < k} w[b k + j] * out[b k + j], j
// ascending (executor.py:786-792) for each sequence b = blockIdx.y.
__global__ void __launch_bounds__(256) moe_combine_rows_kernel(const float* __restrict__ out,
                                                               const float* __restrict__ w, int k, int h,
                                                               float* __restrict__ hidden, long long ldh) {
  pdl_wait();
  const int b = blockIdx.y;
  const float* ob = out + (size_t)b * k * h;
  const float* wb = w + (size_t)b * k;
  float* hb = hidden + (size_t)b * ldh;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < h; i += gridDim.x * blockDim.x) {
    float acc = hb[i];
    for (int j = 0; j < k; ++j) acc += wb[j] * ob[(size_t)j * h + i];
    hb[i] = acc;
  }
  pdl_launch_dependents();
}

// hidden[i] += sum_{j < n_sel} w_j * out[j][i], j ascending (executor.py:786-792).
__global__ void __launch_bounds__(256) moe_combine_kernel(const float* __restrict__ out, const float* __restrict__ w,
                                                          int n_sel, int h, float* __restrict__ hidden) {
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < h; i += gridDim.x * blockDim.x) {
    float r = 0.f;
    for (int j = 0; j < n_sel; ++j) {
      const float wj = w[j];
      if (wj != 0.0f) r += wj * out[(size_t)j * h + i];
    }
    hidden[i] += r;
  }
  pdl_launch_dependents();
}

int rc(int e) { return e > 0 ? PYRITE_E_CUDA : e; }

}  // namespace
}  // namespace pyr

using namespace pyr;

extern "C" {

int pyrite_cuda_moe_route(const float* router_logits, int n_experts, int top_k, int norm_topk_prob, double scale,
                          int shard_count, int shard_index, int* expert_ids, float* expert_weights, int* global_ids,
                          void* stream) {
  if (!router_logits || !expert_ids || !expert_weights || n_experts <= 0 || n_experts > 4096 || top_k <= 0 ||
      top_k > 32 || top_k > n_experts || !(scale > 0.0) || shard_count <= 0 || shard_index < 0 ||
      shard_index >= shard_count)
    return PYRITE_E_SHAPE;
  RouteArgs a{n_experts, top_k, norm_topk_prob ? 1 : 0, scale, shard_count, shard_index, expert_ids, expert_weights,
              global_ids};
  return rc(launch_pdl(moe_route_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), router_logits, a));
}

int pyrite_cuda_moe_router_rows(int router_type, const void* router, size_t router_len, size_t hidden,
                                const float* x, long long ldx, size_t count, float* router_logits, long long ld,
                                int n_experts, void* stream) {
  if (router_type != 0) return PYRITE_E_TYPE;  // F32 routers, as the reference keeps them
  if (!router || !x || !router_logits || n_experts <= 0 || n_experts > 65535 || hidden == 0 ||
      hidden > 0x7fffffffu || count == 0 || count > 65535 || ldx < (long long)hidden || ld < n_experts)
    return PYRITE_E_SHAPE;
  if (router_len != (size_t)n_experts * hidden * 4 || ((uintptr_t)router & 3)) return PYRITE_E_BUFFER;
  return rc(launch_pdl(moe_router_rows_kernel, dim3((unsigned)n_experts, (unsigned)count), dim3(256), 0,
                       static_cast<cudaStream_t>(stream), static_cast<const float*>(router), (int)hidden, x, ldx,
                       router_logits, ld));
}

int pyrite_cuda_moe_route_rows(const float* router_logits, long long ld, size_t count, int n_experts, int top_k,
                               int norm_topk_prob, double scale, int* expert_ids, float* expert_weights,
                               void* stream) {
  if (!router_logits || !expert_ids || !expert_weights || n_experts <= 0 || n_experts > 4096 || top_k <= 0 ||
      top_k > 32 || top_k > n_experts || !(scale > 0.0) || count == 0 || count > 65535 || ld < n_experts)
    return PYRITE_E_SHAPE;
  RouteArgs a{n_experts, top_k, norm_topk_prob ? 1 : 0, scale, 1, 0, expert_ids, expert_weights, nullptr};
  return rc(launch_pdl(moe_route_rows_kernel, dim3((unsigned)count), dim3(32), 0, static_cast<cudaStream_t>(stream),
                       router_logits, ld, a));
}

int pyrite_cuda_moe_combine_rows(const float* expert_out, const float* expert_weights, size_t top_k, size_t h,
                                 size_t count, float* hidden, long long ldh, void* stream) {
  if (!expert_out || !expert_weights || !hidden || top_k == 0 || top_k > 64 || h == 0 || h > 0x7fffffffu ||
      count == 0 || count > 65535 || ldh < (long long)h)
    return PYRITE_E_SHAPE;
  int gx = (int)((h + 255) / 256);
  if (gx > 64) gx = 64;
  return rc(launch_pdl(moe_combine_rows_kernel, dim3(gx, (unsigned)count), dim3(256), 0,
                       static_cast<cudaStream_t>(stream), expert_out, expert_weights, (int)top_k, (int)h, hidden, ldh));
}

int pyrite_cuda_moe_router_route(int router_type, const void* router, size_t router_len, size_t hidden,
                                 const float* x, float* router_logits, int n_experts, int top_k, int norm_topk_prob,
                                 double scale, int shard_count, int shard_index, int* expert_ids,
                                 float* expert_weights, int* global_ids, unsigned* ticket, void* stream) {
  return pyrite_cuda_moe_norm_router_route(router_type, router, router_len, hidden, x, nullptr, 0.0, nullptr, nullptr,
                                           0, router_logits, n_experts, top_k, norm_topk_prob, scale, shard_count,
                                           shard_index, expert_ids, expert_weights, global_ids, ticket, stream);
}

int pyrite_cuda_moe_norm_router_route(int router_type, const void* router, size_t router_len, size_t hidden,
                                      const float* x, const float* norm_weight, double eps, float* normed,
                                      void* workspace, size_t workspace_len, float* router_logits, int n_experts,
                                      int top_k, int norm_topk_prob, double scale, int shard_count, int shard_index,
                                      int* expert_ids, float* expert_weights, int* global_ids, unsigned* ticket,
                                      void* stream) {
  if (router_type != 0) return PYRITE_E_TYPE;  // F32 routers (the reference keeps them unquantized)
  if (!router || !x || !router_logits || !ticket || !expert_ids || !expert_weights || n_experts <= 0 ||
      n_experts > 4096 || top_k <= 0 || top_k > 32 || top_k > n_experts || !(scale > 0.0) || shard_count <= 0 ||
      shard_index < 0 || shard_index >= shard_count || hidden == 0 || hidden > 0x7fffffffu)
    return PYRITE_E_SHAPE;
  if (router_len != (size_t)n_experts * hidden * 4 || ((uintptr_t)router & 3)) return PYRITE_E_BUFFER;
  RouterNorm nm{norm_weight, eps, normed, static_cast<uint8_t*>(workspace)};
  if (norm_weight) {  // the norm prologue reads whole float4 groups; the encoding needs the workspace
    if (!normed || !workspace || hidden % 32 || ((uintptr_t)router & 15) ||
        (((uintptr_t)x | (uintptr_t)norm_weight | (uintptr_t)normed) & 15) || ((uintptr_t)workspace & 255) ||
        workspace_len < pyrite_cuda_workspace_size(0, hidden, 1))
      return PYRITE_E_BUFFER;
  }
  RouteArgs a{n_experts, top_k, norm_topk_prob ? 1 : 0, scale, shard_count, shard_index, expert_ids, expert_weights,
              global_ids};
  return rc(launch_pdl(moe_router_route_kernel, dim3(n_experts), dim3(256), 0, static_cast<cudaStream_t>(stream),
                       static_cast<const float*>(router), (int)hidden, x, router_logits, ticket, a, nm));
}

int pyrite_cuda_matvec_experts(int type_id, const void* stacked, size_t stacked_len, size_t n_experts,
                               const int* expert_ids, size_t n_sel, const float* x, size_t x_stride,
                               const void* workspace, size_t workspace_len, size_t ws_stride, float* y,
                               size_t y_stride, size_t rows, size_t cols, unsigned flags, void* stream) {
  return pyrite_cuda_matvec_expert_groups(type_id, stacked, stacked_len, n_experts, 1, expert_ids, n_sel, x, x_stride,
                                          workspace, workspace_len, ws_stride, y, y_stride, rows, cols, flags, stream);
}

namespace {
// pyrite_cuda_matvec_expert_groups; id index i takes activation i / x_div.
int expert_groups(int type_id, const void* stacked, size_t stacked_len, size_t n_experts, size_t n_groups,
                  const int* expert_ids, size_t n_ids, size_t x_div, const float* x, size_t x_stride,
                  const void* workspace, size_t workspace_len, size_t ws_stride, float* y, size_t y_stride,
                  size_t rows, size_t cols, unsigned flags, void* stream);
}  // namespace

int pyrite_cuda_matvec_expert_groups(int type_id, const void* stacked, size_t stacked_len, size_t n_experts,
                                     size_t n_groups, const int* expert_ids, size_t n_ids, const float* x,
                                     size_t x_stride, const void* workspace, size_t workspace_len, size_t ws_stride,
                                     float* y, size_t y_stride, size_t rows, size_t cols, unsigned flags,
                                     void* stream) {
  return expert_groups(type_id, stacked, stacked_len, n_experts, n_groups, expert_ids, n_ids, 1, x, x_stride,
                       workspace, workspace_len, ws_stride, y, y_stride, rows, cols, flags, stream);
}

int pyrite_cuda_matvec_expert_rows(int type_id, const void* stacked, size_t stacked_len, size_t n_experts,
                                   size_t n_groups, const int* expert_ids, size_t count, size_t top_k, const float* x,
                                   size_t x_stride, const void* workspace, size_t workspace_len, size_t ws_stride,
                                   float* y, size_t y_stride, size_t rows, size_t cols, unsigned flags,
                                   void* stream) {
  if (count == 0 || top_k == 0 || top_k > 64 || count > 65535) return PYRITE_E_BUFFER;
  return expert_groups(type_id, stacked, stacked_len, n_experts, n_groups, expert_ids, count * top_k, top_k, x,
                       x_stride, workspace, workspace_len, ws_stride, y, y_stride, rows, cols, flags, stream);
}

}  // extern "C"

namespace {
int expert_groups(int type_id, const void* stacked, size_t stacked_len, size_t n_experts, size_t n_groups,
                  const int* expert_ids, size_t n_ids, size_t x_div, const float* x, size_t x_stride,
                  const void* workspace, size_t workspace_len, size_t ws_stride, float* y, size_t y_stride,
                  size_t rows, size_t cols, unsigned flags, void* stream) {
  if (n_groups == 0 || n_groups > 8 || x_div == 0) return PYRITE_E_BUFFER;
  const size_t n_sel = n_ids * n_groups;
  const TypeGeo* t = find_type(type_id);
  if (!t) return PYRITE_E_TYPE;
  if (rows == 0 || cols == 0 || cols % (size_t)t->bs || rows > 0x7fffffffu || cols > 0x7fffffffu)
    return PYRITE_E_SHAPE;
  const size_t rb = cols / t->bs * t->bpb;
  const size_t expert_bytes = rb * rows;
  if (!stacked || !expert_ids || !x || !y || !workspace || n_experts == 0 || n_experts > 0x7fffffffu || n_ids == 0 ||
      n_sel > 1024 || stacked_len != expert_bytes * n_experts * n_groups)
    return PYRITE_E_BUFFER;
  if (y_stride < rows) return PYRITE_E_BUFFER;
  const size_t per = pyrite_cuda_workspace_size(0, cols, 1);
  const size_t n_x = (n_ids - 1) / x_div + 1;  // activations (and their encodings) read
  if (((uintptr_t)workspace & 255) || (ws_stride && (ws_stride < per || ws_stride % 256)) ||
      workspace_len < (ws_stride ? ws_stride * (n_x - 1) + per : per))
    return PYRITE_E_BUFFER;
  const uint8_t* w = static_cast<const uint8_t*>(stacked);
  ExpertArgs ex{expert_ids, (int)n_experts, (int)n_sel, (long long)expert_bytes, (long long)ws_stride,
                (long long)y_stride, (int)n_ids, (int)x_div};
  const bool acc = (flags & PYRITE_F_ACCUMULATE) != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int r;
  // every expert keeps the stack's alignment when expert_bytes is a multiple
  // of 16, so the batch-1 kernel's rule on the base covers them all
  if (expert_bytes % 16 == 0 && lane_supported(type_id, w, rb, (int)cols)) {
    r = launch_mv_lane(type_id, w, rb, (int)rows, (int)cols, static_cast<const uint8_t*>(workspace), y, false, s, acc,
                       nullptr, &ex);
  } else {  // the generic kernel on the fp32 activations
    MatvecArgs<float> a{w, rb, (int)rows, (int)cols, x, (long long)cols, y, (long long)rows};
    r = launch_mv_generic<float, 1>(type_id, a, s, acc, &ex, (long long)x_stride);
  }
  return r > 0 ? PYRITE_E_CUDA : r;
}
}  // namespace

extern "C" {

int pyrite_cuda_moe_silu_mul_encode(const float* gate, const float* up, size_t ff, size_t n_sel, float* act,
                                    void* workspace, size_t workspace_len, void* stream) {
  if (!gate || !up || !act || !workspace || ff == 0 || ff % 32 || ff > 0x7fffffffu || n_sel == 0 || n_sel > 1024)
    return PYRITE_E_SHAPE;
  const size_t per = pyrite_cuda_workspace_size(0, ff, 1);
  if (((uintptr_t)workspace & 255) || workspace_len < per * n_sel) return PYRITE_E_BUFFER;
  const long long blocks = (long long)(ff / 32) * (long long)n_sel;
  int grid = (int)((blocks + 7) / 8);
  if (grid > 148 * 8) grid = 148 * 8;
  return rc(launch_pdl(moe_silu_mul_encode_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), gate,
                       up, (int)ff, (int)n_sel, act, static_cast<uint8_t*>(workspace), (long long)per));
}

int pyrite_cuda_moe_combine(const float* expert_out, const float* expert_weights, size_t n_sel, size_t h,
                            float* hidden, void* stream) {
  if (!expert_out || !expert_weights || !hidden || n_sel == 0 || n_sel > 64 || h == 0 || h > 0x7fffffffu)
    return PYRITE_E_SHAPE;
  int grid = (int)((h + 255) / 256);
  if (grid > 148 * 4) grid = 148 * 4;
  return rc(launch_pdl(moe_combine_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), expert_out,
                       expert_weights, (int)n_sel, (int)h, hidden));
}

}  // extern "C"
