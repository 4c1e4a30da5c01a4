// Argument block and weight kinds shared by the linear-layer kernels.
#pragma once

#include "common.cuh"

namespace ksh {

enum WeightKind : int { WK_F32 = 0, WK_I8 = 1, WK_I4 = 2 };
enum Epilogue : int { EPI_STORE = 0, EPI_SWIGLU = 1 };

struct LinArgs {
  const float* x;        // [m, k] fp32, row stride k
  int64_t m;
  int64_t k;             // logical in_features
  int64_t kp;            // padded in_features (INT4: multiple of g; else = k)
  const void* w;         // f32 [n, k] | int8 [n, k] | uint8 [n, kp/2]
  const __half* scales;  // INT8 [n] | INT4 [n, kp/g] | nullptr
  int64_t g;             // INT4 group size
  const float* bias;     // [n] or nullptr
  const float* residual; // [m, n] or nullptr (may alias y)
  const float* norm_w;   // [k]: RMSNorm of x folded into the load, or nullptr
  float norm_eps;
  float* y;              // STORE: [m, n]; SWIGLU: [m, inter]
  int64_t n;             // rows of W (SWIGLU: 2 * inter)
  int64_t inter;         // SWIGLU only
  // fused argmax (lm_head): per-CTA partials then last-CTA reduce
  float* part_val;       // [gridDim.x, m]
  int32_t* part_idx;     // [gridDim.x, m]
  uint32_t* counter;     // single counter, zero on entry, reset by the last CTA
  int64_t* argmax_out;   // [m]
};

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

// Exact integer -> float for packed weights without the int-to-float
// conversion unit (a quarter-rate pipe that caps a decode GEMV well below HBM
// speed): an offset-binary byte u (0..255) is moved into the low mantissa
// bits of 2^23 with one byte permute, giving the float 2^23 + u exactly, and
// one float add removes 2^23 and the offset.
//
// INT8: bias the word once (w ^ 0x80808080: u = q + 128), then dq_i8(wb, b)
// is q of byte b.
__device__ __forceinline__ uint32_t bias_i8(uint32_t w) { return w ^ 0x80808080u; }
__device__ __forceinline__ float dq_i8(uint32_t wb, int b) {
  return __int_as_float(static_cast<int>(__byte_perm(wb, 0x4B000000u, 0x7540u | b))) -
         8388736.0f;   // 2^23 + 128
}
// INT4 (low nibble = even element): split a word into the low and high
// nibbles of each byte, biased (u = q + 8); nibble t of the word is byte t/2
// of lo (t even) or hi (t odd).
__device__ __forceinline__ uint32_t nib_lo(uint32_t w) { return (w & 0x0F0F0F0Fu) ^ 0x08080808u; }
__device__ __forceinline__ uint32_t nib_hi(uint32_t w) {
  return ((w >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
}
__device__ __forceinline__ float dq_i4(uint32_t nb, int b) {
  return __int_as_float(static_cast<int>(__byte_perm(nb, 0x4B000000u, 0x7540u | b))) -
         8388616.0f;   // 2^23 + 8
}

int launch_gemv(int wk, int epi, const LinArgs& a, cudaStream_t stream);
// Register-resident decode GEMV for small matrices; false if not applicable.
bool launch_gemv_resident(int wk, int epi, const LinArgs& a, cudaStream_t stream, int* status);
// Tensor-core decode path (M <= 16, quantized weights, qgemv_tc.cu).
bool gemv_tc_eligible(int wk, int epi, const LinArgs& a);
int launch_gemv_tc(int wk, int epi, const LinArgs& a, cudaStream_t stream);
int set_gemv_tc_mode(int mode);
// Force the streaming GEMV (tests compare both paths); returns the previous value.
int set_gemv_resident_enabled(int on);
bool gemv_resident_enabled();
int launch_gemm_simt(int wk, int epi, const LinArgs& a, cudaStream_t stream);
// Rows from which the prefill GEMM widens the weight to fp16 once per call (0: never).
int64_t set_gemm_predeq_min(int64_t rows);
// One-row INT4 linear with dp4a integer dot products (gemv_i4_dp4a.cu).
bool gemv_i4_dp4a_eligible(int wk, int epi, const LinArgs& a);
int launch_gemv_i4_dp4a(int epi, const LinArgs& a, cudaStream_t stream);
int set_gemv_dp4a_mode(int mode);
// Batched decode linears, 17..64 rows, swap-AB on tcgen05 (qgemm_mid.cu).
bool gemm_mid_eligible(int wk, int epi, const LinArgs& a, const void* ws, int64_t ws_bytes);
int launch_gemm_mid(int wk, int epi, const LinArgs& a, void* ws, cudaStream_t stream);
int set_gemm_mid_mode(int mode);
// lm_head for 17..64 rows per launch (lm_head_gemm.cu): fused RMSNorm, fp32
// GEMM reading the weight once, optional logits, optional greedy argmax.
bool lm_gemm_ok(int64_t m, int64_t k, int64_t vocab, const float* x, const float* norm_w,
                const float* w);
int64_t lm_gemm_workspace_size(int64_t m, int64_t vocab);
int launch_lm_gemm(const float* x, int64_t m, int64_t k, const float* norm_w, float eps,
                   const float* w, int64_t vocab, float* logits, int64_t* tokens, char* ws,
                   cudaStream_t stream);

}  // namespace ksh
