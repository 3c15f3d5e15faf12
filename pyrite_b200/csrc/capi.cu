// capi.cu -- the C ABI of libpyrite_b200.so.
//
// Two families of entry points (declared in include/pyrite_b200.h):
//   * pyrite_native_types / pyrite_matvec / pyrite_dequantize_rows: the exact
//     symbols, signatures and return codes of the reference's C kernel
//     library (pyrite/kernels/native.c:484-576), so the reference's ctypes
//     shim can load this library unchanged.  Buffers are host memory and fp64;
//     the work runs on the current CUDA device in fp64.
//   * pyrite_cuda_*: the device-resident path.  Weights, x and y live in device
//     memory; fp32 activations; the call enqueues on the caller's stream and
//     returns without synchronising.
#include <atomic>
#include <cstring>
#include <mutex>

#include "kernels.cuh"
#include "../../include/pyrite_b200.h"

namespace pyr {

__device__ int g_status_word;

int* device_status_word() {
  // one lookup per device; concurrent first calls look up the same address
  static std::atomic<int*> addr[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  int* a = addr[dev].load(std::memory_order_acquire);
  if (!a) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
    a = static_cast<int*>(p);
    addr[dev].store(a, std::memory_order_release);
  }
  return a;
}

namespace {

// Same validation and codes as the reference's matrix_geometry
// (pyrite/kernels/native.c:496-516): -1 unknown type, -2 bad shape/overflow.
int geometry(int type_id, size_t rows, size_t cols, size_t* row_bytes, const TypeGeo** out) {
  const TypeGeo* t = find_type(type_id);
  if (!t) return PYRITE_E_TYPE;
  if (rows == 0 || cols == 0 || cols % (size_t)t->bs != 0 || cols / t->bs > SIZE_MAX / t->bpb)
    return PYRITE_E_SHAPE;
  *row_bytes = cols / t->bs * t->bpb;
  if (*row_bytes > SIZE_MAX / rows) return PYRITE_E_SHAPE;
  // Kernels index rows and columns with 32-bit ints.
  if (rows > 0x7fffffffu || cols > 0x7fffffffu) return PYRITE_E_SHAPE;
  if (out) *out = t;
  return 0;
}

int cuda_code(cudaError_t e) { return e == cudaSuccess ? 0 : PYRITE_E_CUDA; }

// Library-owned staging for the host-buffer entry points: a compute stream, a
// copy stream, a ring of events and one growable device buffer per device,
// serialised by a mutex.  Nothing is kept between calls except this reusable
// scratch.
constexpr int kStageEvents = 8;
struct HostStage {
  std::mutex mu;
  cudaStream_t stream = nullptr;  // kernels and the result copy
  cudaStream_t copy = nullptr;    // host-to-device copies of the payload
  cudaEvent_t ev[kStageEvents] = {};
  void* buf = nullptr;
  size_t cap = 0;
};
HostStage g_stage[64];

int stage_reserve(HostStage& st, size_t bytes) {
  if (!st.stream && cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking) != cudaSuccess)
    return PYRITE_E_CUDA;
  if (!st.copy) {
    if (cudaStreamCreateWithFlags(&st.copy, cudaStreamNonBlocking) != cudaSuccess) return PYRITE_E_CUDA;
    for (cudaEvent_t& e : st.ev)
      if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return PYRITE_E_CUDA;
  }
  if (bytes <= st.cap) return 0;
  if (st.buf) cudaFree(st.buf);
  st.buf = nullptr;
  st.cap = 0;
  const size_t want = (bytes + 0xFFFFF) & ~(size_t)0xFFFFF;
  if (cudaMalloc(&st.buf, want) != cudaSuccess) {
    cudaGetLastError();
    return PYRITE_E_CUDA;
  }
  st.cap = want;
  return 0;
}

size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

// Prepared-x bytes per column, rounded so every column's planes stay aligned.
size_t ws_col_bytes(int cols) { return align256(lane_workspace_bytes(cols)); }

}  // namespace
}  // namespace pyr

using namespace pyr;

extern "C" {

int pyrite_native_types(int* ids, size_t capacity) {
  if (ids == nullptr) return kNumTypes;
  const size_t n = capacity < (size_t)kNumTypes ? capacity : (size_t)kNumTypes;
  for (size_t i = 0; i < n; ++i) ids[i] = kTypes[i].id;
  return (int)n;
}

int pyrite_type_geometry(int type_id, size_t* block_size, size_t* bytes_per_block) {
  const TypeGeo* t = find_type(type_id);
  if (!t) return PYRITE_E_TYPE;
  if (block_size) *block_size = (size_t)t->bs;
  if (bytes_per_block) *bytes_per_block = (size_t)t->bpb;
  return 0;
}

int pyrite_matvec(int type_id, const uint8_t* data, size_t data_len, const double* x, double* out,
                  size_t rows, size_t cols) {
  size_t rb = 0;
  int rc = geometry(type_id, rows, cols, &rb, nullptr);
  if (rc) return rc;
  if (!data || !x || !out || data_len != rb * rows) return PYRITE_E_BUFFER;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return PYRITE_E_CUDA;
  HostStage& st = g_stage[dev];
  std::lock_guard<std::mutex> lock(st.mu);
  const size_t xoff = align256(data_len), yoff = xoff + align256(cols * sizeof(double));
  if ((rc = stage_reserve(st, yoff + rows * sizeof(double)))) return rc;
  uint8_t* dw = static_cast<uint8_t*>(st.buf);
  double* dx = reinterpret_cast<double*>(dw + xoff);
  double* dy = reinterpret_cast<double*>(dw + yoff);
  // The payload crosses PCIe in row chunks of ~8 MB on the copy stream; each
  // chunk's rows are computed on the compute stream as soon as it has landed,
  // so the products overlap the copies of the chunks after them.  Rows are
  // independent, so the results are the same bits as one launch over all rows.
  // (An event of the ring is recorded again only after the compute stream's
  // wait on its previous recording was enqueued, which is all a wait needs.)
  // On an error, copies already queued may still read the caller's buffers:
  // both streams are drained before returning, so nothing touches them after.
  auto fail = [&](int code) {
    cudaStreamSynchronize(st.copy);
    cudaStreamSynchronize(st.stream);
    cudaGetLastError();
    return code;
  };
  if ((rc = cuda_code(cudaMemcpyAsync(dx, x, cols * sizeof(double), cudaMemcpyHostToDevice, st.copy))))
    return fail(rc);
  const size_t chunk_rows = rb >= ((size_t)8 << 20) ? 1 : ((size_t)8 << 20) / rb;
  int k = 0;
  for (size_t r0 = 0; r0 < rows; r0 += chunk_rows, k = (k + 1) % kStageEvents) {
    const size_t n = rows - r0 < chunk_rows ? rows - r0 : chunk_rows;
    if ((rc = cuda_code(cudaMemcpyAsync(dw + r0 * rb, data + r0 * rb, n * rb, cudaMemcpyHostToDevice, st.copy))))
      return fail(rc);
    if ((rc = cuda_code(cudaEventRecord(st.ev[k], st.copy)))) return fail(rc);
    if ((rc = cuda_code(cudaStreamWaitEvent(st.stream, st.ev[k], 0)))) return fail(rc);
    MatvecArgs<double> a{dw + r0 * rb, rb, (int)n, (int)cols, dx, 0, dy + r0, 0};
    if ((rc = launch_mv_generic<double, 1>(type_id, a, st.stream))) return fail(rc > 0 ? PYRITE_E_CUDA : rc);
  }
  if ((rc = cuda_code(cudaMemcpyAsync(out, dy, rows * sizeof(double), cudaMemcpyDeviceToHost, st.stream))))
    return fail(rc);
  return cuda_code(cudaStreamSynchronize(st.stream));
}

int pyrite_dequantize_rows(int type_id, const uint8_t* data, size_t data_len, double* out, size_t rows,
                           size_t cols) {
  size_t rb = 0;
  int rc = geometry(type_id, rows, cols, &rb, nullptr);
  if (rc) return rc;
  if (!data || !out || data_len != rb * rows || cols > SIZE_MAX / rows) return PYRITE_E_BUFFER;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return PYRITE_E_CUDA;
  HostStage& st = g_stage[dev];
  std::lock_guard<std::mutex> lock(st.mu);
  const size_t ooff = align256(data_len);
  if ((rc = stage_reserve(st, ooff + rows * cols * sizeof(double)))) return rc;
  uint8_t* dw = static_cast<uint8_t*>(st.buf);
  double* dout = reinterpret_cast<double*>(dw + ooff);
  // as in pyrite_matvec: drain the stream before an error return
  auto fail = [&](int code) {
    cudaStreamSynchronize(st.stream);
    cudaGetLastError();
    return code;
  };
  if ((rc = cuda_code(cudaMemcpyAsync(dw, data, data_len, cudaMemcpyHostToDevice, st.stream)))) return fail(rc);
  if ((rc = launch_dq_generic<double>(type_id, dw, rb, (int)rows, (int)cols, dout, (long long)cols, st.stream)))
    return fail(rc > 0 ? PYRITE_E_CUDA : rc);
  if ((rc = cuda_code(cudaMemcpyAsync(out, dout, rows * cols * sizeof(double), cudaMemcpyDeviceToHost,
                                      st.stream))))
    return fail(rc);
  return cuda_code(cudaStreamSynchronize(st.stream));
}

size_t pyrite_cuda_workspace_size(int type_id, size_t cols, size_t ncols) {
  if (cols == 0 || ncols == 0 || cols > 0x7fffffffu || ncols > 0x7fffffffu) return 0;
  size_t need = ncols * ws_col_bytes((int)cols);
  if (tc_supported(type_id, (int)cols, (int)ncols)) {
    const size_t tc = align256(tc_workspace_bytes((int)cols, (int)ncols));
    if (tc > need) need = tc;
  }
  return need;
}

int pyrite_cuda_matvec(int type_id, const void* weights, size_t weights_len, const float* x, long long ldx,
                       float* y, long long ldy, size_t rows, size_t cols, size_t ncols, unsigned flags,
                       void* workspace, size_t workspace_len, void* stream) {
  size_t rb = 0;
  int rc = geometry(type_id, rows, cols, &rb, nullptr);
  if (rc) return rc;
  if (!weights || !x || !y || weights_len != rb * rows || ncols == 0) return PYRITE_E_BUFFER;
  if (ncols > 1 && (ldx < (long long)cols || ldy < (long long)rows)) return PYRITE_E_BUFFER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* w = static_cast<const uint8_t*>(weights);
  const bool acc = (flags & PYRITE_F_ACCUMULATE) != 0;
  if (ncols == 1 && lane_supported(type_id, w, rb, (int)cols)) {
    const size_t need = ws_col_bytes((int)cols);
    if (!workspace || workspace_len < need || ((uintptr_t)workspace & 255) != 0) return PYRITE_E_BUFFER;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    if ((rc = launch_xprep(x, ldx, (int)cols, 1, ws, (long long)need, s))) return rc > 0 ? PYRITE_E_CUDA : rc;
    rc = launch_mv_lane(type_id, w, rb, (int)rows, (int)cols, ws, y, (flags & PYRITE_F_STATIC_WEIGHTS) != 0, s, acc);
    return rc > 0 ? PYRITE_E_CUDA : rc;
  }
  // Several columns of the main formats: the tensor-core product.
  if (ncols > 1 && ncols <= 0x7fffffffu && tc_supported(type_id, (int)cols, (int)ncols)) {
    const size_t need = tc_workspace_bytes((int)cols, (int)ncols);
    if (!workspace || workspace_len < need || ((uintptr_t)workspace & 255) != 0) return PYRITE_E_BUFFER;
    rc = launch_mm_tc(type_id, w, rb, (int)rows, (int)cols, x, ldx, y, ldy, (int)ncols,
                      static_cast<uint8_t*>(workspace), acc, s);
    return rc > 0 ? PYRITE_E_CUDA : rc;
  }
  // Other types, unaligned payloads and several columns: the generic kernels,
  // as many 8-, 4-, 2- and 1-column passes as needed.
  size_t c = 0;
  while (c < ncols) {
    const size_t left = ncols - c;
    MatvecArgs<float> a{w, rb, (int)rows, (int)cols, x + c * ldx, ldx, y + c * ldy, ldy};
    if (left >= 8) { rc = launch_mv_generic<float, 8>(type_id, a, s, acc); c += 8; }
    else if (left >= 4) { rc = launch_mv_generic<float, 4>(type_id, a, s, acc); c += 4; }
    else if (left >= 2) { rc = launch_mv_generic<float, 2>(type_id, a, s, acc); c += 2; }
    else { rc = launch_mv_generic<float, 1>(type_id, a, s, acc); c += 1; }
    if (rc) return rc > 0 ? PYRITE_E_CUDA : rc;
  }
  return 0;
}

int pyrite_cuda_prepare_x(const float* x, long long ldx, size_t cols, size_t ncols, void* workspace,
                          size_t workspace_len, void* stream) {
  if (!x || !workspace || cols == 0 || ncols == 0 || cols > 0x7fffffffu || cols % 32 != 0) return PYRITE_E_BUFFER;
  if (ncols > 1 && ldx < (long long)cols) return PYRITE_E_BUFFER;
  const size_t per = ws_col_bytes((int)cols);
  if (workspace_len < per * ncols || ((uintptr_t)workspace & 255) != 0) return PYRITE_E_BUFFER;
  const int rc = launch_xprep(x, ncols > 1 ? ldx : (long long)cols, (int)cols, (int)ncols,
                              static_cast<uint8_t*>(workspace), (long long)per, static_cast<cudaStream_t>(stream));
  return rc > 0 ? PYRITE_E_CUDA : rc;
}

int pyrite_cuda_matvec_prepared(int type_id, const void* weights, size_t weights_len, const float* x,
                                const void* workspace, size_t workspace_len, float* y, size_t rows, size_t cols,
                                unsigned flags, void* stream) {
  size_t rb = 0;
  int rc = geometry(type_id, rows, cols, &rb, nullptr);
  if (rc) return rc;
  if (!weights || !x || !y || weights_len != rb * rows) return PYRITE_E_BUFFER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* w = static_cast<const uint8_t*>(weights);
  if (lane_supported(type_id, w, rb, (int)cols)) {
    if (!workspace || workspace_len < ws_col_bytes((int)cols) || ((uintptr_t)workspace & 255) != 0)
      return PYRITE_E_BUFFER;
    rc = launch_mv_lane(type_id, w, rb, (int)rows, (int)cols, static_cast<const uint8_t*>(workspace), y,
                        (flags & PYRITE_F_STATIC_WEIGHTS) != 0, s, (flags & PYRITE_F_ACCUMULATE) != 0);
  } else {
    MatvecArgs<float> a{w, rb, (int)rows, (int)cols, x, (long long)cols, y, (long long)rows};
    rc = launch_mv_generic<float, 1>(type_id, a, s, (flags & PYRITE_F_ACCUMULATE) != 0);
  }
  return rc > 0 ? PYRITE_E_CUDA : rc;
}

// Validation and the choice of form shared by pyrite_cuda_matvec_transformed
// and pyrite_cuda_matvec_transformed_form: 1 = prologue, 0 = the operation's
// own kernel then the product, < 0 = error code.
static int transformed_plan(int type_id, const void* weights, size_t weights_len, const float* x, int x_op,
                            const float* norm_weight, const float* x_out, bool have_ws, size_t rows, size_t cols,
                            size_t* row_bytes) {
  size_t rb = 0;
  int rc = geometry(type_id, rows, cols, &rb, nullptr);
  if (rc) return rc;
  if (!weights || !x || weights_len != rb * rows || cols % 32) return PYRITE_E_BUFFER;
  if (x_op != PYRITE_X_RMSNORM && x_op != PYRITE_X_SILU_MUL) return PYRITE_E_BUFFER;
  if (x_op == PYRITE_X_RMSNORM && !norm_weight) return PYRITE_E_BUFFER;
  *row_bytes = rb;
  // the prologue reads and writes the vectors as float4
  const bool vec16 = (((uintptr_t)x | (uintptr_t)norm_weight | (uintptr_t)x_out) & 15) == 0;
  const bool lane = vec16 && lane_supported(type_id, static_cast<const uint8_t*>(weights), rb, (int)cols);
  // Every CTA of the prologue form encodes the whole vector after the
  // preceding kernel finished, one L2 round trip under the weight stream of
  // the whole grid.  Measured on B200: that beats a kernel of its own for an
  // RMSNorm over 4096 values and more (Llama-3-8B: -1 us on Q/K, -2 us on
  // gate/up); shorter norms and SiLU * up (more work per value, ffn-wide
  // vectors) are faster as their own kernel, which is used when the caller
  // gives a workspace.
  if (lane && (!have_ws || (x_op == PYRITE_X_RMSNORM && cols >= 4096))) return 1;
  return have_ws ? 0 : PYRITE_E_BUFFER;
}

int pyrite_cuda_matvec_transformed_form(int type_id, const void* weights, size_t weights_len, const float* x,
                                        int x_op, const float* norm_weight, const float* x_out, size_t rows,
                                        size_t cols) {
  size_t rb = 0;
  return transformed_plan(type_id, weights, weights_len, x, x_op, norm_weight, x_out, x_out != nullptr, rows, cols,
                          &rb);
}

int pyrite_cuda_matvec_transformed(int type_id, const void* weights, size_t weights_len, const float* x, int x_op,
                                   const float* norm_weight, double eps, float* x_out, void* workspace,
                                   size_t workspace_len, float* y, size_t rows, size_t cols, unsigned flags,
                                   void* stream) {
  if (!y) return PYRITE_E_BUFFER;
  const bool have_ws = x_out && workspace && workspace_len >= ws_col_bytes((int)cols) && !((uintptr_t)workspace & 255);
  size_t rb = 0;
  int rc = transformed_plan(type_id, weights, weights_len, x, x_op, norm_weight, x_out, have_ws, rows, cols, &rb);
  if (rc < 0) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* w = static_cast<const uint8_t*>(weights);
  const bool acc = (flags & PYRITE_F_ACCUMULATE) != 0;
  if (rc == 1) {
    XPrologue xp{x_op == PYRITE_X_RMSNORM ? 1 : 2, x, norm_weight, eps, x_out};
    rc = launch_mv_lane(type_id, w, rb, (int)rows, (int)cols, nullptr, y, (flags & PYRITE_F_STATIC_WEIGHTS) != 0, s,
                        acc, nullptr, nullptr, &xp);
    return rc > 0 ? PYRITE_E_CUDA : rc;
  }
  // formats without the batch-1 kernel (or vectors not 16-byte aligned), or
  // sizes where that is faster: the operation's own kernel into the workspace
  // and x_out, then the product
  rc = x_op == PYRITE_X_RMSNORM
           ? pyrite_cuda_rmsnorm_encode(x, norm_weight, cols, eps, x_out, workspace, workspace_len, stream)
           : pyrite_cuda_silu_mul_encode(x, cols, x_out, workspace, workspace_len, stream);
  if (rc) return rc;
  return pyrite_cuda_matvec_prepared(type_id, weights, weights_len, x_out, workspace, workspace_len, y, rows, cols,
                                     flags, stream);
}

size_t pyrite_cuda_post_scratch_size(void) {
  const int g = lane_max_grid();
  return g > 0 ? (size_t)g * 8 : 0;
}

int pyrite_cuda_matvec_prepared_post(int type_id, const void* weights, size_t weights_len, const float* x,
                                     const void* workspace, size_t workspace_len, float* y, size_t rows, size_t cols,
                                     unsigned flags, const pyrite_post_op* post, void* stream) {
  if (!post || post->op == PYRITE_POST_NONE)
    return pyrite_cuda_matvec_prepared(type_id, weights, weights_len, x, workspace, workspace_len, y, rows, cols, flags,
                                       stream);
  size_t rb = 0;
  int rc = geometry(type_id, rows, cols, &rb, nullptr);
  if (rc) return rc;
  if (!weights || !x || !y || weights_len != rb * rows) return PYRITE_E_BUFFER;
  // the post op's own arguments
  PostArgs pa;
  pa.ticket = post->ticket;
  if (!pa.ticket) return PYRITE_E_BUFFER;
  size_t n_out = 0;
  switch (post->op) {
    case PYRITE_POST_RMSNORM_ENCODE:
      n_out = rows;
      if (!post->weight || rows % 32) return PYRITE_E_BUFFER;
      pa.op = kPostRmsnormEncode;
      break;
    case PYRITE_POST_SILU_MUL_ENCODE:
      n_out = rows / 2;
      if (!post->out || rows % 64) return PYRITE_E_BUFFER;
      pa.op = kPostSiluMulEncode;
      break;
    case PYRITE_POST_ARGMAX:
      if (!post->scratch || post->scratch_len < pyrite_cuda_post_scratch_size() || !post->tokens || !post->pos)
        return PYRITE_E_BUFFER;
      pa.op = kPostArgmax;
      break;
    default:
      return PYRITE_E_BUFFER;
  }
  if (n_out && (!post->workspace || post->workspace_len < ws_col_bytes((int)n_out) ||
                ((uintptr_t)post->workspace & 255) != 0))
    return PYRITE_E_BUFFER;
  pa.w = post->weight;
  pa.eps = post->eps;
  pa.out = post->out;
  pa.ws = static_cast<uint8_t*>(post->workspace);
  const int g = lane_max_grid();
  pa.pv = static_cast<float*>(post->scratch);
  pa.pi = post->scratch ? reinterpret_cast<int*>(pa.pv + (g > 0 ? g : 0)) : nullptr;
  pa.tokens = post->tokens;
  pa.pos = post->pos;
  pa.prompt_len = post->prompt_len;
  pa.max_ctx = post->max_ctx;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* w = static_cast<const uint8_t*>(weights);
  if (lane_supported(type_id, w, rb, (int)cols)) {
    if (!workspace || workspace_len < ws_col_bytes((int)cols) || ((uintptr_t)workspace & 255) != 0)
      return PYRITE_E_BUFFER;
    rc = launch_mv_lane(type_id, w, rb, (int)rows, (int)cols, static_cast<const uint8_t*>(workspace), y,
                        (flags & PYRITE_F_STATIC_WEIGHTS) != 0, s, (flags & PYRITE_F_ACCUMULATE) != 0, &pa);
    return rc > 0 ? PYRITE_E_CUDA : rc;
  }
  // formats without the batch-1 kernel: the product, then the operation as its own kernel
  rc = pyrite_cuda_matvec_prepared(type_id, weights, weights_len, x, workspace, workspace_len, y, rows, cols, flags,
                                   stream);
  if (rc) return rc;
  switch (post->op) {
    case PYRITE_POST_RMSNORM_ENCODE:
      return pyrite_cuda_rmsnorm_encode(y, post->weight, rows, post->eps, post->out, post->workspace,
                                        post->workspace_len, stream);
    case PYRITE_POST_SILU_MUL_ENCODE:
      return pyrite_cuda_silu_mul_encode(y, rows / 2, post->out, post->workspace, post->workspace_len, stream);
    default:
      return pyrite_cuda_argmax_step(y, rows, post->scratch, post->scratch_len, post->tokens, post->pos,
                                     post->prompt_len, post->max_ctx, stream);
  }
}

int pyrite_cuda_dequantize_rows(int type_id, const void* weights, size_t weights_len, float* out, size_t rows,
                                size_t cols, void* stream) {
  size_t rb = 0;
  int rc = geometry(type_id, rows, cols, &rb, nullptr);
  if (rc) return rc;
  if (!weights || !out || weights_len != rb * rows) return PYRITE_E_BUFFER;
  rc = launch_dq_generic<float>(type_id, static_cast<const uint8_t*>(weights), rb, (int)rows, (int)cols, out,
                                (long long)cols, static_cast<cudaStream_t>(stream));
  return rc > 0 ? PYRITE_E_CUDA : rc;
}

int pyrite_cuda_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int pyrite_cuda_status(int clear) {
  int* p = device_status_word();
  if (!p) return PYRITE_E_CUDA;
  int v = 0;
  if (cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return PYRITE_E_CUDA;
  if (clear && v) {
    const int zero = 0;
    if (cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return PYRITE_E_CUDA;
  }
  return v;
}

const char* pyrite_error_string(int code) {
  switch (code) {
    case 0: return "ok";
    case PYRITE_E_TYPE: return "unknown or non-decodable GGML type";
    case PYRITE_E_SHAPE: return "invalid or overflowing matrix shape";
    case PYRITE_E_BUFFER: return "null pointer or payload length does not match rows x row_bytes";
    case PYRITE_E_CUDA: return "CUDA runtime error";
    default: return "unknown error";
  }
}

}  // extern "C"
