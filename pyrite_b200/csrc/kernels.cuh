// kernels.cuh -- shared launch helpers, PTX wrappers and kernel entry points.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "ggml_blocks.cuh"

namespace pyr {

// One matrix-vector (or matrix x few-columns) problem on device memory.
// Row r of the matrix starts at w + r * row_bytes; column c of x / y starts at
// x + c * ldx / y + c * ldy.
template <typename T> struct MatvecArgs {
  const uint8_t* w;
  size_t row_bytes;
  int rows;
  int cols;
  const T* x;
  long long ldx;
  T* y;
  long long ldy;
};

// Device-side status word: kernels set bits here instead of trapping, so a
// timed-out wait leaves the context usable and the host can report it.
enum DeviceStatus : int { kStatusOk = 0, kStatusWaitTimeout = 1, kStatusBadExpert = 2 };
int* device_status_word();  // this device's status word (address valid in kernels)

// ---- programmatic dependent launch (PDL) ------------------------------------
// Kernels may start (and prefetch weights) while the previous kernel in the
// stream drains; pdl_wait() orders them after it before touching its outputs.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  return e == cudaSuccess ? 0 : -100 - (int)e;
}

struct ExpertArgs;

// ---- generic kernels (mv_generic.cu) ----------------------------------------
// experts: routed slices (ExpertArgs; x advances x_stride values per slice).
template <typename T, int NC>
int launch_mv_generic(int type_id, const MatvecArgs<T>& a, cudaStream_t stream, bool accumulate = false,
                      const ExpertArgs* experts = nullptr, long long x_stride = 0);
template <typename T>
int launch_dq_generic(int type_id, const uint8_t* w, size_t row_bytes, int rows, int cols, T* out,
                      long long ldo, cudaStream_t stream);

// ---- post ops: run by the last CTA of a batch-1 matvec on its whole output -----
enum PostOp : int { kPostNone = 0, kPostRmsnormEncode = 1, kPostSiluMulEncode = 2, kPostArgmax = 3 };
struct PostArgs {
  int op = kPostNone;
  const float* w = nullptr;  // RMSNorm weight (n values)
  double eps = 0.0;
  float* out = nullptr;      // fp32 result (normed vector / activation)
  uint8_t* ws = nullptr;     // its encoding for the next matvec
  unsigned* ticket = nullptr;  // device counter, zero between launches
  float* pv = nullptr;       // argmax: per-CTA partial values / indices
  int* pi = nullptr;
  int* tokens = nullptr;     // argmax: the chosen id goes to tokens[*pos + 1]
  int* pos = nullptr;
  int prompt_len = 0, max_ctx = 0;
};

// ---- batch-1 dp4a kernels, weights staged by cp.async (mv_tile.cu) -------------
// Bytes of prepared x one column needs (int8 digit planes, scales, sums).
size_t lane_workspace_bytes(int cols);
// True when the type has a lane kernel and the payload alignment suits it.
bool lane_supported(int type_id, const uint8_t* w, size_t row_bytes, int cols);
// x (ncols columns, stride ldx) -> prepared digits at ws + c * ws_col_bytes.
int launch_xprep(const float* x, long long ldx, int cols, int ncols, uint8_t* ws, long long ws_col_bytes,
                 cudaStream_t stream);
// y[0..rows) from the prepared column at ws; static_weights enables the L2
// prefetch of weights before the preceding kernel ends.
// Routed experts for launch_mv_lane: w is a stack of n_experts matrices
// expert_bytes apart; ids[0..n_sel) (device memory, read after the preceding
// kernel) pick the ones to multiply, each by its own prepared x (ws_stride
// bytes apart, 0: one shared x) into y + j * y_stride.
// Selection j (of n_sel) multiplies expert ids[j % n_ids] of group j / n_ids:
// the stack holds n_sel / n_ids groups of n_experts experts each (one group
// per matrix, e.g. gate and up), so one launch covers every group.  x and the
// workspace advance per id (j % n_ids), y per selection.
struct ExpertArgs {
  const int* ids;
  int n_experts, n_sel;
  long long expert_bytes, ws_stride, y_stride;
  int n_ids = 0;  // 0: n_sel (one group)
  int x_div = 1;  // id index i takes activation i / x_div (top-k selections of one sequence share its x)
};
// The activation computed in every CTA's prologue instead of a prepared
// workspace: mode 1 RMSNorm of src with weight norm, mode 2 silu(src[:cols]) *
// src[cols:]; CTA 0 also stores the fp32 activation to out (may be NULL).
struct XPrologue {
  int mode;
  const float* src;
  const float* norm;
  double eps;
  float* out;
};
int launch_mv_lane(int type_id, const uint8_t* w, size_t row_bytes, int rows, int cols, const uint8_t* ws,
                   float* y, bool static_weights, cudaStream_t stream, bool accumulate = false,
                   const PostArgs* post = nullptr, const ExpertArgs* ex = nullptr, const XPrologue* xp = nullptr);
// Largest grid launch_mv_lane uses (argmax partial slots needed).
int lane_max_grid();

// ---- several columns on the tensor cores (mm_tc.cu) ---------------------------
// True when (type, cols, ncols) runs on the tcgen05 path.
bool tc_supported(int type_id, int cols, int ncols);
// Workspace bytes for the split activation planes of ncols columns.
size_t tc_workspace_bytes(int cols, int ncols);
// Y[c*ldy + r] (+)= sum_k W[r,k] X[c*ldx + k]; ws 256-byte aligned, at least
// tc_workspace_bytes(cols, ncols).
int launch_mm_tc(int type_id, const uint8_t* w, size_t row_bytes, int rows, int cols, const float* x, long long ldx,
                 float* y, long long ldy, int ncols, uint8_t* ws, bool accumulate, cudaStream_t stream);

}  // namespace pyr
