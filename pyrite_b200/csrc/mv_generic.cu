// mv_generic.cu -- portable kernels for every decodable GGML type.
//
// These serve three roles:
//   * the fp64 path behind the reference-compatible host entry points
//     (pyrite_matvec / pyrite_dequantize_rows take fp64 host buffers,
//     pyrite/kernels/native.c:518-576), which must agree with the reference to
//     ~1e-11, so they decode and accumulate in double;
//   * the fp32 path for multi-column products (ncols > 1) and for payloads
//     whose base address is not 16-byte aligned;
//   * the fp32 dequantize kernel (embedding row lookups).
// One warp computes one output row; lane l walks the 32-value units
// l, l+32, ... of the row, so neighbouring lanes read neighbouring bytes.
#include "kernels.cuh"

namespace pyr {

// Routed experts (ex.ids != nullptr): blockIdx.y = j picks stacked matrix
// ids[j] (expert_bytes apart), x + j * x_stride and y + j * y_stride.
struct GenericExperts {  // as ExpertArgs: slice j = expert ids[j % n_ids] of group j / n_ids
  const int* ids = nullptr;
  int n_experts = 0, n_ids = 1, x_div = 1;
  long long expert_bytes = 0, x_stride = 0, y_stride = 0;
};

template <int TY, typename T, int NC>
__global__ void __launch_bounds__(256)
mv_generic_kernel(const uint8_t* __restrict__ w, size_t row_bytes, int rows, int cols,
                  const T* __restrict__ x, long long ldx, T* __restrict__ y, long long ldy, int accumulate,
                  GenericExperts ex, int* status) {
  constexpr int BS = Geo<TY>::bs, BPB = Geo<TY>::bpb;
  if (ex.ids) {
    pdl_wait();  // the ids come from the preceding kernel
    const int j = blockIdx.y, idn = j % ex.n_ids;
    int e = ex.ids[idn];
    if (e == -1) return;  // held by another GPU
    if (e < 0 || e >= ex.n_experts) {  // never read outside the stack
      if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(status, (int)kStatusBadExpert);
      e = 0;
    }
    e += (j / ex.n_ids) * ex.n_experts;
    w += (size_t)e * (size_t)ex.expert_bytes;
    x += (size_t)(idn / ex.x_div) * (size_t)ex.x_stride;
    y += (size_t)j * (size_t)ex.y_stride;
  }
  const int lane = threadIdx.x & 31;
  const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  pdl_wait();
  for (long long r = warp; r < rows; r += nwarps) {
    const uint8_t* row = w + (size_t)r * row_bytes;
    T acc[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) acc[c] = T(0);
    if constexpr (TY == F32) {
      if (((uintptr_t)row & 3) == 0) {  // whole-word loads (a router, a norm-sized matrix)
        const float* rf = reinterpret_cast<const float*>(row);
#pragma unroll 4
        for (int col = lane; col < cols; col += 32) {
          const T v = (T)rf[col];
#pragma unroll
          for (int c = 0; c < NC; ++c) acc[c] += v * x[c * ldx + col];
        }
      } else {
        for (int col = lane; col < cols; col += 32) {
          const T v = scalar_val<TY, T>(row + (size_t)col * BPB);
#pragma unroll
          for (int c = 0; c < NC; ++c) acc[c] += v * x[c * ldx + col];
        }
      }
    } else if constexpr (BS == 1) {
      for (int col = lane; col < cols; col += 32) {
        const T v = scalar_val<TY, T>(row + (size_t)col * BPB);
#pragma unroll
        for (int c = 0; c < NC; ++c) acc[c] += v * x[c * ldx + col];
      }
    } else {
      constexpr int UPB = BS / 32;
      const int units = cols / 32;
      for (int u = lane; u < units; u += 32) {
        T v[32];
        decode_unit<TY, T>(row + (size_t)(u / UPB) * BPB, u % UPB, v);
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const T* xc = x + c * ldx + (size_t)u * 32;
          T s = T(0);
#pragma unroll
          for (int i = 0; i < 32; ++i) s += v[i] * xc[i];
          acc[c] += s;
        }
      }
    }
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      T s = acc[c];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) y[c * ldy + r] = accumulate ? y[c * ldy + r] + s : s;
    }
  }
}

template <int TY, typename T>
__global__ void __launch_bounds__(256)
dq_generic_kernel(const uint8_t* __restrict__ w, size_t row_bytes, int rows, int cols,
                  T* __restrict__ out, long long ldo) {
  constexpr int BS = Geo<TY>::bs, BPB = Geo<TY>::bpb;
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long nthreads = (long long)gridDim.x * blockDim.x;
  pdl_wait();
  if constexpr (BS == 1) {
    const long long total = (long long)rows * cols;
    for (long long i = tid; i < total; i += nthreads) {
      const long long r = i / cols, c = i % cols;
      out[r * ldo + c] = scalar_val<TY, T>(w + (size_t)r * row_bytes + (size_t)c * BPB);
    }
  } else {
    constexpr int UPB = BS / 32;
    const int units = cols / 32;
    const long long total = (long long)rows * units;
    for (long long i = tid; i < total; i += nthreads) {
      const long long r = i / units;
      const int u = (int)(i % units);
      T v[32];
      decode_unit<TY, T>(w + (size_t)r * row_bytes + (size_t)(u / UPB) * BPB, u % UPB, v);
      T* o = out + r * ldo + (size_t)u * 32;
#pragma unroll
      for (int k = 0; k < 32; ++k) o[k] = v[k];
    }
  }
}

namespace {
int grid_for(long long work_items, int per_block) {
  long long g = (work_items + per_block - 1) / per_block;
  const long long cap = 148LL * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}
}  // namespace

template <typename T, int NC>
int launch_mv_generic(int type_id, const MatvecArgs<T>& a, cudaStream_t stream, bool accumulate,
                      const ExpertArgs* experts, long long x_stride) {
  GenericExperts ex;
  int n_sel = 1;
  if (experts) {
    ex.ids = experts->ids;
    ex.n_experts = experts->n_experts;
    ex.n_ids = experts->n_ids > 0 ? experts->n_ids : experts->n_sel;
    ex.x_div = experts->x_div > 0 ? experts->x_div : 1;
    ex.expert_bytes = experts->expert_bytes;
    ex.x_stride = x_stride;
    ex.y_stride = experts->y_stride;
    n_sel = experts->n_sel;
  }
  int grid = grid_for((long long)a.rows * 32, 256);
  if (experts && grid * n_sel > 148 * 16) grid = (148 * 16 + n_sel - 1) / n_sel;
  switch (type_id) {
#define PYR_CASE(TY)                                                                                       \
  case TY:                                                                                                 \
    return launch_pdl(mv_generic_kernel<TY, T, NC>, dim3(grid, n_sel), dim3(256), 0, stream, a.w,         \
                      a.row_bytes, a.rows, a.cols, a.x, a.ldx, a.y, a.ldy, accumulate ? 1 : 0, ex,          \
                      device_status_word());
    PYR_FOR_EACH_TYPE(PYR_CASE)
#undef PYR_CASE
    default:
      return -1;
  }
}

template <typename T>
int launch_dq_generic(int type_id, const uint8_t* w, size_t row_bytes, int rows, int cols, T* out,
                      long long ldo, cudaStream_t stream) {
  const TypeGeo* g = find_type(type_id);
  if (!g) return -1;
  const long long items = g->bs == 1 ? (long long)rows * cols : (long long)rows * (cols / 32);
  const int grid = grid_for(items, 256);
  switch (type_id) {
#define PYR_CASE(TY)                                                                         \
  case TY:                                                                                   \
    return launch_pdl(dq_generic_kernel<TY, T>, dim3(grid), dim3(256), 0, stream, w, row_bytes, \
                      rows, cols, out, ldo);
    PYR_FOR_EACH_TYPE(PYR_CASE)
#undef PYR_CASE
    default:
      return -1;
  }
}

template int launch_mv_generic<double, 1>(int, const MatvecArgs<double>&, cudaStream_t, bool, const ExpertArgs*,
                                          long long);
template int launch_mv_generic<float, 1>(int, const MatvecArgs<float>&, cudaStream_t, bool, const ExpertArgs*,
                                         long long);
template int launch_mv_generic<float, 2>(int, const MatvecArgs<float>&, cudaStream_t, bool, const ExpertArgs*,
                                         long long);
template int launch_mv_generic<float, 4>(int, const MatvecArgs<float>&, cudaStream_t, bool, const ExpertArgs*,
                                         long long);
template int launch_mv_generic<float, 8>(int, const MatvecArgs<float>&, cudaStream_t, bool, const ExpertArgs*,
                                         long long);
template int launch_dq_generic<double>(int, const uint8_t*, size_t, int, int, double*, long long, cudaStream_t);
template int launch_dq_generic<float>(int, const uint8_t*, size_t, int, int, float*, long long, cudaStream_t);

}  // namespace pyr
