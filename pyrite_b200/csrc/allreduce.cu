// allreduce.cu -- the tensor-parallel decode step's sum across GPUs over
// NVLink peer memory, one kernel per call.
//
// After the attention output and the feed-forward down projection, every GPU
// holds a partial residual update of `n` floats (a few KB); the decode step
// needs their sum on every GPU.  A collective library spends ~10 us of launch
// and protocol latency on such a message.  Here each GPU instead publishes its
// partial in a buffer that all GPUs map (symmetric memory), raises one flag in
// every peer's buffer, waits until every peer's flag for this call is up, and
// reads all partials directly over NVLink, summing them in rank order -- so
// every GPU gets bit-identical sums.
//
// Buffer of each GPU (pyrite_cuda_allreduce_buffer_size bytes, zeroed before
// the first call): 64 flags (uint32, one per source rank) | slot 0 | slot 1,
// each slot n floats rounded up to 256 bytes.  Calls alternate slots, so a
// GPU one call ahead never overwrites a partial a slower peer still reads: it
// cannot get two calls ahead, since call e + 1 waits for every peer's flag
// e + 1, raised only after that peer finished call e.  The call counter lives
// in device memory (`epoch`), so the kernel can be replayed in a CUDA graph.
//
// The buffers are plain device allocations shared by CUDA IPC handles
// (pyrite_cuda_ipc_buffer_*): peer loads and stores over NVLink, no
// multicast object.  Every wait is bounded (5 s of globaltimer): on timeout
// the kernel sets status bit kStatusWaitTimeout and finishes without waiting
// further.
#include <cstdint>
#include <cstring>

#include "kernels.cuh"
#include "ptx.cuh"
#include "../../include/pyrite_b200.h"

namespace pyr {
namespace {

constexpr int kMaxRanks = 64;
constexpr size_t kFlagBytes = 256;

__host__ __device__ inline size_t slot_bytes(size_t n) { return (n * sizeof(float) + 255) & ~(size_t)255; }

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One CTA of 1024 threads: n floats, a few thousand at most in a decode step.
__global__ void __launch_bounds__(1024) allreduce_oneshot_kernel(const float* __restrict__ part,
                                                                 float* __restrict__ inout, int n,
                                                                 const unsigned long long* __restrict__ peers,
                                                                 int world, int rank, unsigned* epoch, int* status) {
  __shared__ int timed_out;
  pdl_wait();
  const int tid = threadIdx.x;
  const unsigned e = *epoch + 1u;
  const size_t sb = slot_bytes((size_t)n);
  const size_t off = kFlagBytes + (size_t)(e & 1u) * sb;
  // 1. this GPU's partial into its own slot (n % 4 == 0: float4 throughout)
  float4* mine = reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(peers[rank]) + off);
  const int n4 = n >> 2;
  for (int i = tid; i < n4; i += blockDim.x) mine[i] = reinterpret_cast<const float4*>(part)[i];
  if (tid == 0) timed_out = 0;
  __syncthreads();
  // 2. publish: raise flag `rank` of every GPU (a system-scope release after
  //    the barrier makes the whole CTA's slot writes visible first)
  if (tid < world) {
    __threadfence_system();
    unsigned* flags = reinterpret_cast<unsigned*>(peers[tid]);
    st_release_sys(flags + rank, e);
  }
  // 3. wait for every source's flag of this call (flags only grow)
  if (tid < world) {
    const unsigned* flags = reinterpret_cast<const unsigned*>(peers[rank]);
    if (ld_acquire_sys(flags + tid) < e) {
      const uint64_t t0 = ptx::globaltimer_ns();
      while (ld_acquire_sys(flags + tid) < e) {
        if (ptx::globaltimer_ns() - t0 > 5000000000ull) {
          timed_out = 1;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (timed_out) {
    if (tid == 0) {
      atomicOr(status, (int)kStatusWaitTimeout);
      *epoch = e;
    }
    return;
  }
  // 4. every partial over NVLink, summed in rank order (the same bits on every
  //    GPU); the loads of up to 8 ranks are issued before the adds, so a
  //    thread waits for one NVLink round trip per 8 ranks, not one per rank
  for (int i = tid; i < n4; i += blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r0 = 0; r0 < world; r0 += 8) {
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (r0 + j < world)
          v[j] = __ldcv(reinterpret_cast<const float4*>(reinterpret_cast<const uint8_t*>(peers[r0 + j]) + off) + i);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (r0 + j < world) {
          acc.x += v[j].x;
          acc.y += v[j].y;
          acc.z += v[j].z;
          acc.w += v[j].w;
        }
    }
    float4 io = reinterpret_cast<float4*>(inout)[i];
    io.x += acc.x;
    io.y += acc.y;
    io.z += acc.z;
    io.w += acc.w;
    reinterpret_cast<float4*>(inout)[i] = io;
  }
  __syncthreads();
  if (tid == 0) *epoch = e;
  pdl_launch_dependents();
}

}  // namespace
}  // namespace pyr

using namespace pyr;

extern "C" {

size_t pyrite_cuda_allreduce_buffer_size(size_t n) { return kFlagBytes + 2 * slot_bytes(n); }

int pyrite_cuda_ipc_buffer_create(size_t bytes, void** dev_ptr, void* handle_out) {
  if (!dev_ptr || !handle_out || bytes == 0) return PYRITE_E_BUFFER;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return PYRITE_E_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return PYRITE_E_CUDA;
  }
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  memcpy(handle_out, &h, sizeof(h));
  *dev_ptr = p;
  return 0;
}

int pyrite_cuda_ipc_buffer_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return PYRITE_E_BUFFER;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return PYRITE_E_CUDA;
  *dev_ptr = p;
  return 0;
}

int pyrite_cuda_ipc_buffer_close(void* dev_ptr, int owned) {
  if (!dev_ptr) return PYRITE_E_BUFFER;
  const cudaError_t e = owned ? cudaFree(dev_ptr) : cudaIpcCloseMemHandle(dev_ptr);
  return e == cudaSuccess ? 0 : PYRITE_E_CUDA;
}

int pyrite_cuda_allreduce_sum(const float* part, float* inout, size_t n, const unsigned long long* peer_buffers,
                              size_t buffer_len, int world, int rank, unsigned* epoch, void* stream) {
  if (!part || !inout || !peer_buffers || !epoch || n == 0 || n % 4 || n > (1u << 20) || world < 1 ||
      world > kMaxRanks || rank < 0 || rank >= world || (((uintptr_t)part | (uintptr_t)inout) & 15))
    return PYRITE_E_BUFFER;
  // every rank's buffer must hold the flags and both slots of n values
  if (buffer_len < pyrite_cuda_allreduce_buffer_size(n)) return PYRITE_E_BUFFER;
  const int r = launch_pdl(allreduce_oneshot_kernel, dim3(1), dim3(1024), 0, static_cast<cudaStream_t>(stream), part,
                           inout, (int)n, peer_buffers, world, rank, epoch, device_status_word());
  return r > 0 ? PYRITE_E_CUDA : r;
}

}  // extern "C"
