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

int launch_gemv(int wk, int epi, const LinArgs& a, cudaStream_t stream);
// Register-resident decode GEMV for small matrices; false if not applicable.
bool launch_gemv_resident(int wk, int epi, const LinArgs& a, cudaStream_t stream, int* status);
// Force the streaming GEMV (tests compare both paths); returns the previous value.
int set_gemv_resident_enabled(int on);
bool gemv_resident_enabled();
int launch_gemm_simt(int wk, int epi, const LinArgs& a, cudaStream_t stream);

}  // namespace ksh
