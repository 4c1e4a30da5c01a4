// lm_head + greedy argmax for callers that cannot allocate device memory.
//
// ksh_lm_head_argmax needs a caller-provided workspace for its per-CTA
// (max, index) partials and the completion counter of its last-CTA
// reduction.  Some callers have no way to provide one: an FFI binding that
// only receives device pointers from a host runtime whose allocator it cannot
// reach, or a latency-critical loop that must not call cudaMalloc (which can
// synchronize the whole device).  This entry point runs the same kernel with
// its scratch in a fixed file-scope device array instead:
//
// * kScratchBytes (256 KiB) per GPU that loads the library, held until the
//   process exits; it covers m <= 16 rows at any vocabulary the GEMV grid
//   supports (the partials need grid * m * 8 bytes, grid <= 8 CTAs per SM);
// * the first call on each device looks up the array's device address with
//   cudaGetSymbolAddress (with that device current); make that first call
//   before any stream capture;
// * every call shares the array: the counter is cleared at the start of each
//   call, and two calls that overlap on the GPU (different streams, or
//   concurrent host threads) race on it;
// * nothing here calls cudaMalloc, cudaFree or an allocating library routine.

#include <mutex>

#include "linear.cuh"

namespace ksh {
int64_t gemv_argmax_grid(int64_t n);

namespace {

constexpr int64_t kScratchBytes = 256 * 1024;
constexpr int64_t kHeader = 256;          // completion counter lives in the first 4 bytes
constexpr int kMaxDevices = 64;
constexpr int64_t kMaxRows = 16;

static __device__ __align__(256) unsigned char g_lm_scratch[kScratchBytes];

void* scratch_address(int* status) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *status = KSH_ERR_CUDA;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_lm_scratch);
    if (e != cudaSuccess || !p) {
      *status = record_cuda_error(e == cudaSuccess ? cudaErrorInvalidSymbol : e);
      return nullptr;
    }
    addr[dev] = p;
  }
  *status = KSH_OK;
  return addr[dev];
}

}  // namespace
}  // namespace ksh

using namespace ksh;

extern "C" int64_t ksh_lm_head_argmax_noalloc_max_bytes(void) { return kScratchBytes; }

extern "C" int ksh_lm_head_argmax_noalloc(const float* x, int64_t m, int64_t hidden,
                                          const float* norm_w, float norm_eps, const float* w,
                                          int64_t vocab, float* logits, int64_t* tokens,
                                          void* stream) {
  KSH_CHECK_ARG(m >= 0 && hidden > 0 && vocab > 0 && vocab <= INT32_MAX && x && w && tokens);
  if (m == 0) return KSH_OK;
  // The fused GEMV + argmax kernel wants float4 weight rows.
  if (hidden % 4 != 0 || (reinterpret_cast<uintptr_t>(w) & 15) != 0) return KSH_ERR_UNSUPPORTED;
  // Row counts and vocabularies whose partials do not fit the fixed scratch.
  if (m > kMaxRows) return KSH_ERR_TOO_LARGE;
  const int64_t grid = gemv_argmax_grid(vocab);
  if (kHeader + grid * m * 8 > kScratchBytes) return KSH_ERR_TOO_LARGE;
  int st = KSH_OK;
  char* ws = static_cast<char*>(scratch_address(&st));
  if (st != KSH_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The counter must start at zero; a completed call leaves it at zero, but
  // clear it anyway so a call never depends on the previous one.
  const cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) return record_cuda_error(e);
  LinArgs a = {};
  a.x = x;
  a.m = m;
  a.k = hidden;
  a.kp = hidden;
  a.w = w;
  a.y = logits;
  a.n = vocab;
  a.norm_w = norm_w;
  a.norm_eps = norm_eps;
  a.counter = reinterpret_cast<uint32_t*>(ws);
  a.part_val = reinterpret_cast<float*>(ws + kHeader);
  a.part_idx = reinterpret_cast<int32_t*>(ws + kHeader + grid * m * 4);
  a.argmax_out = tokens;
  return launch_gemv(WK_F32, EPI_STORE, a, s);
}
