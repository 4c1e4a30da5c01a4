// C ABI of the linear layers: shape checks and path selection.
//
//   m <= 16 and 16-byte aligned rows  -> vectorised GEMV (gemv.cu)
//   17 <= m <= 64, quantized weights  -> swap-AB tcgen05 kernel (qgemm_mid.cu)
//   m  > 16, tensor-core friendly     -> tcgen05 GEMM (qgemm_tc.cu)
//   anything else                     -> generic CUDA-core GEMM (gemm_simt.cu)

#include <float.h>

#include <algorithm>

#include "linear.cuh"

namespace ksh {
int64_t gemv_argmax_grid(int64_t n);
int launch_gemm_tc(int wk, int epi, const LinArgs& a, void* ws, int64_t ws_bytes,
                   cudaStream_t stream, bool* taken);
int64_t gemm_tc_workspace_size(int64_t m, int64_t k, int64_t n);

namespace {

constexpr int kGemvMaxM = 16;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool gemv_ok(int wk, const LinArgs& a) {
  if (a.m > kGemvMaxM) return false;
  if (!aligned16(a.w)) return false;
  switch (wk) {
    case WK_F32: return a.k % 4 == 0;
    case WK_I8: return a.k % 16 == 0;
    case WK_I4: return a.g % 32 == 0 && a.kp % 32 == 0;
  }
  return false;
}

int run_linear(int wk, int epi, LinArgs& a, void* ws, int64_t ws_bytes, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (gemv_i4_dp4a_eligible(wk, epi, a)) return launch_gemv_i4_dp4a(epi, a, s);
  if (a.m <= kGemvMaxM && gemv_tc_eligible(wk, epi, a)) return launch_gemv_tc(wk, epi, a, s);
  if (gemv_ok(wk, a)) return launch_gemv(wk, epi, a, s);
  if (a.m > kGemvMaxM && gemm_mid_eligible(wk, epi, a, ws, ws_bytes)) return launch_gemm_mid(wk, epi, a, ws, s);
  if (a.m > kGemvMaxM) {
    bool taken = false;
    int st = launch_gemm_tc(wk, epi, a, ws, ws_bytes, s, &taken);
    if (taken) return st;
  }
  return launch_gemm_simt(wk, epi, a, s);
}

LinArgs base(const float* x, int64_t m, int64_t k, int64_t kp, const void* w,
             const uint16_t* scales, int64_t g, float* y, int64_t n) {
  LinArgs a = {};
  a.x = x;
  a.m = m;
  a.k = k;
  a.kp = kp;
  a.w = w;
  a.scales = reinterpret_cast<const __half*>(scales);
  a.g = g;
  a.y = y;
  a.n = n;
  return a;
}

void set_norm(LinArgs& a, const float* norm_w, float eps) {
  a.norm_w = norm_w;
  a.norm_eps = eps;
}

}  // namespace
}  // namespace ksh

using namespace ksh;

extern "C" int64_t ksh_linear_workspace_size(int64_t m, int64_t k, int64_t n) {
  return gemm_tc_workspace_size(m, k, n);
}

extern "C" int ksh_qlinear_w8(const float* x, int64_t m, int64_t k, const float* norm_w, float norm_eps, const int8_t* payload,
                              const uint16_t* scales, const float* bias,
                              const float* residual, float* y, int64_t n, void* workspace,
                              int64_t workspace_bytes, void* stream) {
  KSH_CHECK_ARG(m >= 0 && k > 0 && n > 0 && x && payload && scales && y);
  if (m == 0) return KSH_OK;
  LinArgs a = base(x, m, k, k, payload, scales, 0, y, n);
  set_norm(a, norm_w, norm_eps);
  a.bias = bias;
  a.residual = residual;
  return run_linear(WK_I8, EPI_STORE, a, workspace, workspace_bytes, stream);
}

extern "C" int ksh_qlinear_w4(const float* x, int64_t m, int64_t k, const float* norm_w, float norm_eps, const uint8_t* payload,
                              const uint16_t* scales, int64_t group_size, int64_t k_padded,
                              const float* bias, const float* residual, float* y, int64_t n,
                              void* workspace, int64_t workspace_bytes, void* stream) {
  KSH_CHECK_ARG(m >= 0 && k > 0 && n > 0 && x && payload && scales && y);
  KSH_CHECK_ARG(group_size > 0 && group_size % 2 == 0 && k_padded % group_size == 0 &&
                k_padded >= k && k_padded - k < group_size);
  if (m == 0) return KSH_OK;
  LinArgs a = base(x, m, k, k_padded, payload, scales, group_size, y, n);
  set_norm(a, norm_w, norm_eps);
  a.bias = bias;
  a.residual = residual;
  return run_linear(WK_I4, EPI_STORE, a, workspace, workspace_bytes, stream);
}

extern "C" int ksh_linear_f32(const float* x, int64_t m, int64_t k, const float* norm_w, float norm_eps, const float* w,
                              const float* bias, const float* residual, float* y, int64_t n,
                              void* workspace, int64_t workspace_bytes, void* stream) {
  KSH_CHECK_ARG(m >= 0 && k > 0 && n > 0 && x && w && y);
  if (m == 0) return KSH_OK;
  LinArgs a = base(x, m, k, k, w, nullptr, 0, y, n);
  set_norm(a, norm_w, norm_eps);
  a.bias = bias;
  a.residual = residual;
  return run_linear(WK_F32, EPI_STORE, a, workspace, workspace_bytes, stream);
}

extern "C" int ksh_qlinear_swiglu_w8(const float* x, int64_t m, int64_t k, const float* norm_w, float norm_eps,
                                     const int8_t* payload, const uint16_t* scales, float* h,
                                     int64_t inter, void* workspace, int64_t workspace_bytes,
                                     void* stream) {
  KSH_CHECK_ARG(m >= 0 && k > 0 && inter > 0 && x && payload && scales && h);
  if (m == 0) return KSH_OK;
  LinArgs a = base(x, m, k, k, payload, scales, 0, h, 2 * inter);
  set_norm(a, norm_w, norm_eps);
  a.inter = inter;
  return run_linear(WK_I8, EPI_SWIGLU, a, workspace, workspace_bytes, stream);
}

extern "C" int ksh_qlinear_swiglu_w4(const float* x, int64_t m, int64_t k, const float* norm_w, float norm_eps,
                                     const uint8_t* payload, const uint16_t* scales,
                                     int64_t group_size, int64_t k_padded, float* h,
                                     int64_t inter, void* workspace, int64_t workspace_bytes,
                                     void* stream) {
  KSH_CHECK_ARG(m >= 0 && k > 0 && inter > 0 && x && payload && scales && h);
  KSH_CHECK_ARG(group_size > 0 && group_size % 2 == 0 && k_padded % group_size == 0 &&
                k_padded >= k && k_padded - k < group_size);
  if (m == 0) return KSH_OK;
  LinArgs a = base(x, m, k, k_padded, payload, scales, group_size, h, 2 * inter);
  set_norm(a, norm_w, norm_eps);
  a.inter = inter;
  return run_linear(WK_I4, EPI_SWIGLU, a, workspace, workspace_bytes, stream);
}

extern "C" int ksh_linear_swiglu_f32(const float* x, int64_t m, int64_t k, const float* norm_w, float norm_eps, const float* w,
                                     float* h, int64_t inter, void* workspace,
                                     int64_t workspace_bytes, void* stream) {
  KSH_CHECK_ARG(m >= 0 && k > 0 && inter > 0 && x && w && h);
  if (m == 0) return KSH_OK;
  LinArgs a = base(x, m, k, k, w, nullptr, 0, h, 2 * inter);
  set_norm(a, norm_w, norm_eps);
  a.inter = inter;
  return run_linear(WK_F32, EPI_SWIGLU, a, workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------------------
// lm_head + argmax
// ---------------------------------------------------------------------------

namespace ksh {
namespace {
constexpr int64_t kLmHeadHeader = 256;  // counter lives in the first 4 bytes

__global__ void __launch_bounds__(256)
argmax_rows_kernel(const float* __restrict__ logits, int64_t vocab, int64_t* out) {
  grid_dep_wait();
  grid_dep_launch();
  const float* row = logits + static_cast<int64_t>(blockIdx.x) * vocab;
  float bv = -FLT_MAX;
  int64_t bi = INT64_MAX;
  for (int64_t i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float v = row[i];
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
  __shared__ float sv[256];
  __shared__ int64_t si[256];
  sv[threadIdx.x] = bv;
  si[threadIdx.x] = bi;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) {
      const float ov = sv[threadIdx.x + s];
      const int64_t oi = si[threadIdx.x + s];
      if (ov > sv[threadIdx.x] || (ov == sv[threadIdx.x] && oi < si[threadIdx.x])) {
        sv[threadIdx.x] = ov;
        si[threadIdx.x] = oi;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) out[blockIdx.x] = si[0];
}
}  // namespace
}  // namespace ksh

// Rows above which the batch lm_head (one pass over the weight per 64 rows)
// replaces the GEMV (one pass per 16 rows).
constexpr int64_t kLmGemvMaxRows = 16;

extern "C" int64_t ksh_lm_head_workspace_size(int64_t m, int64_t vocab) {
  const int64_t mm = std::min<int64_t>(std::max<int64_t>(m, 1), kLmGemvMaxRows);
  const int64_t gemv = kLmHeadHeader + gemv_argmax_grid(vocab) * mm * 8;
  return m > kLmGemvMaxRows ? std::max(gemv, lm_gemm_workspace_size(m, vocab)) : gemv;
}

extern "C" int ksh_argmax_rows(const float* logits, int64_t m, int64_t vocab, int64_t* out,
                               void* stream) {
  KSH_CHECK_ARG(m >= 0 && vocab > 0 && logits && out && m <= INT32_MAX);
  if (m == 0) return KSH_OK;
  return launch(argmax_rows_kernel, dim3(static_cast<unsigned>(m)), dim3(256), 0,
                static_cast<cudaStream_t>(stream), logits, vocab, out);
}

extern "C" int ksh_lm_head_argmax(const float* x, int64_t m, int64_t hidden,
                                  const float* norm_w, float norm_eps, const float* w,
                                  int64_t vocab, float* logits, int64_t* tokens,
                                  void* workspace, int64_t workspace_bytes, void* stream) {
  KSH_CHECK_ARG(m >= 0 && hidden > 0 && vocab > 0 && vocab <= INT32_MAX && x && w);
  KSH_CHECK_ARG(logits || tokens);
  if (m == 0) return KSH_OK;
  LinArgs a = base(x, m, hidden, hidden, w, nullptr, 0, logits, vocab);
  set_norm(a, norm_w, norm_eps);
  if (m > kLmGemvMaxRows && workspace &&
      lm_gemm_ok(std::min<int64_t>(m, 64), hidden, vocab, x, norm_w, w)) {
    // batch rows: 64 per launch, the weight read once per launch
    const int64_t need = ksh_lm_head_workspace_size(m, vocab);
    if (workspace_bytes < need) return KSH_ERR_WORKSPACE;
    if (!aligned16(workspace)) return KSH_ERR_ALIGN;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int64_t r0 = 0; r0 < m; r0 += 64) {
      const int64_t rows = std::min<int64_t>(64, m - r0);
      const int st = launch_lm_gemm(x + r0 * hidden, rows, hidden, norm_w, norm_eps, w, vocab,
                                    logits ? logits + r0 * vocab : nullptr,
                                    tokens ? tokens + r0 : nullptr, static_cast<char*>(workspace), s);
      if (st != KSH_OK) return st;
    }
    return KSH_OK;
  }
  if (tokens && gemv_ok(WK_F32, a)) {
    const int64_t need = ksh_lm_head_workspace_size(m, vocab);
    if (!workspace || workspace_bytes < need) return KSH_ERR_WORKSPACE;
    if (!aligned16(workspace)) return KSH_ERR_ALIGN;
    char* ws = static_cast<char*>(workspace);
    const int64_t grid = gemv_argmax_grid(vocab);
    a.counter = reinterpret_cast<uint32_t*>(ws);
    // The completion counter must start at zero whatever the workspace held.
    const cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(uint32_t),
                                          static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return record_cuda_error(e);
    a.part_val = reinterpret_cast<float*>(ws + kLmHeadHeader);
    a.part_idx = reinterpret_cast<int32_t*>(ws + kLmHeadHeader + grid * m * 4);
    a.argmax_out = tokens;
    return launch_gemv(WK_F32, EPI_STORE, a, static_cast<cudaStream_t>(stream));
  }
  // General path: materialise logits, then a row argmax.
  if (!logits) return KSH_ERR_WORKSPACE;
  int st = run_linear(WK_F32, EPI_STORE, a, nullptr, 0, stream);
  if (st != KSH_OK || !tokens) return st;
  return ksh_argmax_rows(logits, m, vocab, tokens, stream);
}

extern "C" int ksh_set_gemv_dp4a(int enabled) { return set_gemv_dp4a_mode(enabled); }
extern "C" int ksh_set_gemm_mid(int enabled) { return set_gemm_mid_mode(enabled); }
extern "C" int64_t ksh_set_gemm_predeq(int64_t min_rows) { return set_gemm_predeq_min(min_rows); }
