// K1 / K2: weight-only INT8 per-channel and INT4 per-group packing.
//
// Byte-exact restatement of the reference quantizers
// (engine/quantization.py:196-223 and :238-318):
//   s   = fp16_rne(max(fp32(absmax) / qmax, fp32(1e-8)))
//   q   = clamp(round_half_even(w / fp32(s)), qmin, qmax), NaN -> 0
// with a true IEEE division (__fdiv_rn), not a reciprocal multiply: the
// reference divides by the fp16-rounded scale widened to fp32.  When the fp16
// scale underflows to 0, w / 0 is +-inf (clamped to the range end) and 0 / 0
// is NaN, which the reference's float->int8 conversion turns into 0.
//
// One CTA per output row; the row is read twice (absmax, then quantize), both
// passes coalesced.  Packing runs once at load time.

#include "common.cuh"

namespace ksh {
namespace {

constexpr int kPackThreads = 256;

__device__ __forceinline__ int quant_one(float w, float s, float qmin, float qmax) {
  float v = __fdiv_rn(w, s);
  if (isnan(v)) return 0;
  float r = rintf(v);
  r = r < qmin ? qmin : (r > qmax ? qmax : r);
  return static_cast<int>(r);
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  if (wid == 0) {
    float t = lane < (blockDim.x >> 5) ? red[lane] : 0.0f;
    t = warp_max(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

__global__ void __launch_bounds__(kPackThreads)
pack_int8_kernel(const float* __restrict__ w, int64_t n, int64_t k,
                 int8_t* __restrict__ payload, __half* __restrict__ scales,
                 int32_t* flags) {
  __shared__ float red[32];
  grid_dep_wait();
  const int64_t row = blockIdx.x;
  if (row >= n) return;
  const float* wr = w + row * k;
  float amax = 0.0f;
  bool bad = false;
  for (int64_t j = threadIdx.x; j < k; j += blockDim.x) {
    float v = wr[j];
    bad |= !isfinite(v);
    amax = fmaxf(amax, fabsf(v));
  }
  if (bad) raise_flag(flags, KSH_FLAG_NONFINITE);
  amax = block_max(amax, red);
  const float s32 = fmaxf(__fdiv_rn(amax, 127.0f), 1e-8f);
  const __half s16 = __float2half_rn(s32);
  const float sq = __half2float(s16);
  if (threadIdx.x == 0) scales[row] = s16;
  int8_t* pr = payload + row * k;
  for (int64_t j = threadIdx.x; j < k; j += blockDim.x)
    pr[j] = static_cast<int8_t>(quant_one(wr[j], sq, -127.0f, 127.0f));
  grid_dep_launch();
}

// One CTA per row; warp w handles groups w, w + nwarps, ...  Lane i handles
// the element pairs (2i, 2i+1), (2i+64, 2i+65), ... of the group so each
// pair lands in one packed byte.
__global__ void __launch_bounds__(kPackThreads)
pack_int4_kernel(const float* __restrict__ w, int64_t n, int64_t k, int64_t g,
                 int64_t kp, uint8_t* __restrict__ payload, __half* __restrict__ scales,
                 int32_t* flags) {
  grid_dep_wait();
  const int64_t row = blockIdx.x;
  if (row >= n) return;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const float* wr = w + row * k;
  const int64_t ngroups = kp / g;
  uint8_t* pr = payload + row * (kp / 2);
  bool bad = false;
  for (int64_t grp = wid; grp < ngroups; grp += nw) {
    const int64_t base = grp * g;
    float amax = 0.0f;
    for (int64_t j = lane; j < g; j += 32) {
      const int64_t kk = base + j;
      float v = kk < k ? wr[kk] : 0.0f;
      bad |= !isfinite(v);
      amax = fmaxf(amax, fabsf(v));
    }
    amax = warp_max(amax);
    const float s32 = fmaxf(__fdiv_rn(amax, 7.0f), 1e-8f);
    const __half s16 = __float2half_rn(s32);
    const float sq = __half2float(s16);
    if (lane == 0) scales[row * ngroups + grp] = s16;
    for (int64_t j = 2 * lane; j < g; j += 64) {
      const int64_t k0 = base + j, k1 = k0 + 1;
      const float v0 = k0 < k ? wr[k0] : 0.0f;
      const float v1 = k1 < k ? wr[k1] : 0.0f;
      const int q0 = quant_one(v0, sq, -8.0f, 7.0f);
      const int q1 = quant_one(v1, sq, -8.0f, 7.0f);
      pr[k0 >> 1] = static_cast<uint8_t>((q0 & 0xF) | ((q1 & 0xF) << 4));
    }
  }
  if (bad) raise_flag(flags, KSH_FLAG_NONFINITE);
  grid_dep_launch();
}

}  // namespace
}  // namespace ksh

using namespace ksh;

extern "C" int ksh_pack_int8(const float* w, int64_t n, int64_t k, int8_t* payload,
                             uint16_t* scales, int32_t* flags, void* stream) {
  KSH_CHECK_ARG(n > 0 && k > 0 && n <= INT32_MAX);
  KSH_CHECK_ARG(w && payload && scales);
  return launch(pack_int8_kernel, dim3(static_cast<unsigned>(n)), dim3(kPackThreads), 0,
                static_cast<cudaStream_t>(stream), w, n, k, payload,
                reinterpret_cast<__half*>(scales), flags);
}

extern "C" int ksh_pack_int4(const float* w, int64_t n, int64_t k, int64_t group_size,
                             uint8_t* payload, uint16_t* scales, int32_t* flags,
                             void* stream) {
  KSH_CHECK_ARG(n > 0 && k > 0 && n <= INT32_MAX);
  KSH_CHECK_ARG(group_size > 0 && group_size % 2 == 0);
  KSH_CHECK_ARG(w && payload && scales);
  const int64_t kp = (k + group_size - 1) / group_size * group_size;
  return launch(pack_int4_kernel, dim3(static_cast<unsigned>(n)), dim3(kPackThreads), 0,
                static_cast<cudaStream_t>(stream), w, n, k, group_size, kp, payload,
                reinterpret_cast<__half*>(scales), flags);
}
