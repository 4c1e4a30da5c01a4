// Shared device/host helpers for the Kshipra B200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/kshipra_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "kshipra_b200 kernels target sm_100a only"
#endif

namespace ksh {

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  Every kernel of the forward is launched with
// the programmatic-stream-serialization attribute; the kernel may run
// prologue work that touches only constant data (weights) before
// grid_dep_wait(), which returns once the previous grid in the stream has
// completed and its writes are visible.  No kernel writes global memory
// before grid_dep_wait().
// ---------------------------------------------------------------------------
__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// L2 prefetch of a global range (bulk, no shared memory involved).  Size must
// be a multiple of 16 and the address 16-byte aligned.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Prefetch [base, base+bytes) to L2 cooperatively over the threads of a CTA,
// in pieces of at most `piece` bytes.  Only the 16-byte aligned interior is
// prefetched; the ragged edges are left to the demand loads.
__device__ __forceinline__ void prefetch_range_l2(const void* base, size_t bytes, int tid,
                                                  int nthreads) {
  uintptr_t b = reinterpret_cast<uintptr_t>(base);
  uintptr_t lo = (b + 15) & ~uintptr_t(15);
  uintptr_t hi = (b + bytes) & ~uintptr_t(15);
  if (hi <= lo) return;
  const uintptr_t piece = 8192;
  for (uintptr_t p = lo + uintptr_t(tid) * piece; p < hi; p += uintptr_t(nthreads) * piece) {
    uintptr_t n = hi - p < piece ? hi - p : piece;
    prefetch_l2_bulk(reinterpret_cast<const void*>(p), static_cast<uint32_t>(n));
  }
}

// ---------------------------------------------------------------------------
// Reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Raise a bit in the caller's device status word.
__device__ __forceinline__ void raise_flag(int32_t* flags, int32_t bit) {
  if (flags) atomicOr(flags, bit);
}

// ---------------------------------------------------------------------------
// Host-side launch helper
// ---------------------------------------------------------------------------
bool pdl_enabled();
bool prefetch_enabled();
// Records e for ksh_last_cuda_error() and returns KSH_ERR_CUDA.
int record_cuda_error(cudaError_t e);
// Every successful kernel launch of the library (ksh_kernel_launches).
void count_launch();

template <typename... KArgs, typename... Args>
inline int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                  cudaStream_t stream, Args... args) {
  if (grid.x == 0 || grid.y == 0 || grid.z == 0) return KSH_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return record_cuda_error(e);
  count_launch();
  return KSH_OK;
}

int num_sms();
int set_smem_optin(const void* kernel, size_t bytes);
// CTAs of `kernel` resident per SM at this block size / dynamic smem (cached).
int resident_ctas(const void* kernel, int threads, size_t smem);
// CTAs of `kernel` resident on the GPU at once when launched in clusters of
// `cluster` CTAs (cluster placement can leave SMs unusable; cached).  The
// kernel's shared-memory opt-in must be set first.
int64_t cluster_slots(const void* kernel, int threads, size_t smem, int cluster);

}  // namespace ksh

#define KSH_CHECK_ARG(cond)            \
  do {                                 \
    if (!(cond)) return KSH_ERR_SHAPE; \
  } while (0)
