// noalloc.cu -- a matvec entry point that never allocates device memory.
//
// pyrite_cuda_matvec needs a device workspace for the re-encoded activation,
// and the caller allocates it.  Some callers cannot: a host runtime that owns
// every byte of GPU memory through its own pool and forbids plugins from
// calling cudaMalloc, code that runs where allocation is not allowed or too
// slow (inside a real-time decode loop, or between a memory-budget check and
// the kernels it admitted), or a foreign-language host (Go, Java, Node) whose
// FFI layer has no device allocator at all.  pyrite_cuda_matvec_noalloc gives
// them the same product with the workspace taken from a fixed array that is
// part of the library image itself.
//
// The array below lives in every GPU's memory from the moment the library's
// module is loaded on that GPU until the process exits.  Its size fixes the
// largest activation this entry point accepts (PYRITE_NOALLOC_MAX_COLS).
#include <mutex>

#include "kernels.cuh"
#include "post_ops.cuh"
#include "../../include/pyrite_b200.h"

namespace pyr {
namespace {

// Encoded-activation bytes for the widest activation the batch-1 kernel takes
// (kNoAllocLaneCols values): three int8 digit planes, one fp32 scale per 32
// values and one fp32 sum per 16 values -- 108 KiB.  Wider activations (up to
// PYRITE_NOALLOC_MAX_COLS) go to the generic kernel, which reads x directly
// and needs no scratch.
constexpr int kNoAllocLaneCols = 32768;
constexpr size_t kNoAllocScratchBytes = (size_t)encoded_bytes(kNoAllocLaneCols);

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// The array's address on each device.  Host code cannot use the symbol name
// itself as a device pointer (on the host it names a host-side stand-in), so
// the address is looked up once per device, with that device current.
std::mutex g_noalloc_mu;
uint8_t* g_noalloc_addr[64] = {};

int scratch_for_current_device(uint8_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PYRITE_E_CUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return PYRITE_E_CUDA;
    }
    g_noalloc_addr[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_noalloc_addr[dev];
  return 0;
}

int noalloc_geometry(int type_id, size_t rows, size_t cols, size_t* row_bytes) {
  const TypeGeo* t = find_type(type_id);
  if (!t) return PYRITE_E_TYPE;
  if (rows == 0 || cols == 0 || cols % (size_t)t->bs != 0 || rows > 0x7fffffffu) return PYRITE_E_SHAPE;
  if (cols > (size_t)PYRITE_NOALLOC_MAX_COLS) return PYRITE_E_SHAPE;  // beyond the fixed scratch
  *row_bytes = cols / t->bs * t->bpb;
  if (*row_bytes > SIZE_MAX / rows) return PYRITE_E_SHAPE;
  return 0;
}

}  // namespace
}  // namespace pyr

using namespace pyr;

extern "C" int pyrite_cuda_matvec_noalloc(int type_id, const void* weights, size_t weights_len, const float* x,
                                          float* y, size_t rows, size_t cols, unsigned flags, void* stream) {
  size_t rb = 0;
  int rc = noalloc_geometry(type_id, rows, cols, &rb);
  if (rc) return rc;
  if (!weights || !x || !y || weights_len != rb * rows) return PYRITE_E_BUFFER;
  uint8_t* scratch = nullptr;
  if ((rc = scratch_for_current_device(&scratch))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* w = static_cast<const uint8_t*>(weights);
  if (cols <= (size_t)kNoAllocLaneCols && lane_supported(type_id, w, rb, (int)cols)) {
    // The encoding kernel writes every byte the product kernel then reads, so
    // nothing in the array has to start at zero; what an earlier call left
    // there is simply overwritten.
    if ((rc = launch_xprep(x, (long long)cols, (int)cols, 1, scratch, (long long)kNoAllocScratchBytes, s)))
      return rc > 0 ? PYRITE_E_CUDA : rc;
    rc = launch_mv_lane(type_id, w, rb, (int)rows, (int)cols, scratch, y, (flags & PYRITE_F_STATIC_WEIGHTS) != 0, s);
  } else {
    MatvecArgs<float> a{w, rb, (int)rows, (int)cols, x, (long long)cols, y, (long long)rows};
    rc = launch_mv_generic<float, 1>(type_id, a, s);
  }
  return rc > 0 ? PYRITE_E_CUDA : rc;
}
