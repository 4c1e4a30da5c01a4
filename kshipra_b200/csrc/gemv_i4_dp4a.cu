// K4, one token row: INT4 decode linear with integer dot products.
//
// Replaces QuantizedLinear.forward (engine/quantization.py:394-396) for one
// row of x and INT4 per-group weights (dequantize, then F.linear).  The
// product is computed exactly in int32 and scaled in fp32:
//
// * x (RMSNorm folded in, the GEMV's rounding) is cut into 32-element
//   vectors; each vector gets its own power-of-two scale 2^E (largest |x| just
//   below 2^21) and X = rint(x * 2^E) is stored as three balanced signed
//   8-bit digits, X = d0 + 256 d1 + 65536 d2, in shared memory -- once per
//   CTA, in the byte order of the unpacked weights (elements 0,2,4,6 then
//   1,3,5,7 of every 8), one 112-byte record per vector (the digits, 8 sum X
//   and 2^-E) so a vector costs seven conflict-free 16-byte shared loads;
// * a weight word of 8 nibbles becomes two words of q + 8 (0..15) with one or
//   two logic operations, and dp4a multiplies them with the digits: per
//   vector sum (q + 8) X = sum_p 256^p sum (q + 8) d_p in int32, minus the
//   stored 8 sum X, is sum q X exactly (|.| < 2^31);
// * the int32 result is converted once per vector and accumulated with the
//   group scale times 2^-E in fp32;
// * each warp owns two weight rows (gate and up for SwiGLU), so one load of
//   the digits serves both; lanes stride over the row's 16-byte vectors with
//   four vectors per row in flight (the remainder one at a time, no per-vector
//   bounds tests in the main loop), and each warp keeps an L2 bulk prefetch of
//   its next rows (weights and group scales) running; group scales are read
//   through the read-only cache.
//
// Against the CUDA-core fp32 GEMV (a byte permute, a float add and an FMA per
// weight, fp32 x re-read per row) this is about 1.5 instructions per weight,
// which a decode GEMV streaming INT4 at HBM speed can afford.

#include <math.h>
#include <stdlib.h>

#include <algorithm>

#include "linear.cuh"

namespace ksh {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kUnroll = 4;      // 16-byte vectors per lane and row in flight
constexpr int kPfItems = 4;     // row items a warp keeps prefetched ahead
constexpr int kRec = 7;         // 16-byte words per vector record (6 digit words + meta)

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
  return __dp4a(static_cast<int>(a), static_cast<int>(b), c);
}

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// q + 8 of the low / high nibbles of each byte (q two's complement)
__device__ __forceinline__ uint32_t u_lo(uint32_t w) { return (w & 0x0F0F0F0Fu) ^ 0x08080808u; }
__device__ __forceinline__ uint32_t u_hi(uint32_t w) { return ((w >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u; }

// sum (q + 8) * X over one 16-byte weight vector (32 elements), X given by
// its digit planes (two uint4 halves per plane)
__device__ __forceinline__ int vec_dot(const uint4& w, const uint4 (&d)[6]) {
  int p0 = 0, p1 = 0, p2 = 0;
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t lo = u_lo(ws[j]), hi = u_hi(ws[j]);
    const uint4& h0 = d[j >> 1];            // plane 0, half j / 2
    const uint4& h1 = d[2 + (j >> 1)];
    const uint4& h2 = d[4 + (j >> 1)];
    const uint32_t a0 = (j & 1) ? h0.z : h0.x, b0 = (j & 1) ? h0.w : h0.y;
    const uint32_t a1 = (j & 1) ? h1.z : h1.x, b1 = (j & 1) ? h1.w : h1.y;
    const uint32_t a2 = (j & 1) ? h2.z : h2.x, b2 = (j & 1) ? h2.w : h2.y;
    p0 = dp4a(lo, a0, p0);
    p0 = dp4a(hi, b0, p0);
    p1 = dp4a(lo, a1, p1);
    p1 = dp4a(hi, b1, p1);
    p2 = dp4a(lo, a2, p2);
    p2 = dp4a(hi, b2, p2);
  }
  return p0 + 256 * p1 + 65536 * p2;
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 2)
gemv_i4_dp4a_kernel(LinArgs a, int64_t items_per_cta) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int nv = static_cast<int>(a.kp / 32);
  // per 32-element vector one 112-byte record: the three digit planes (two
  // 16-byte halves each), then {8 sum X, 2^-E bits, 0, 0}; 28 words apart, so
  // the lanes of a quarter warp read their records from distinct banks
  uint4* rec = reinterpret_cast<uint4*>(smem);              // [nv][kRec]
  __shared__ float red[kWarps];
  __shared__ float inv_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // items: STORE -> a pair of consecutive rows; SWIGLU -> (gate row j, up row j)
  const int64_t nrows_out = EPI == EPI_SWIGLU ? a.inter : a.n;
  const int64_t nitems = EPI == EPI_SWIGLU ? nrows_out : (nrows_out + 1) / 2;
  const int64_t i_begin = static_cast<int64_t>(blockIdx.x) * items_per_cta;
  const int64_t i_end = min(i_begin + items_per_cta, nitems);
  const int64_t rb = a.kp / 2;
  const char* W = static_cast<const char*>(a.w);
  auto rows_of = [&](int64_t it, int64_t& r0, int64_t& r1) {
    if (EPI == EPI_SWIGLU) {
      r0 = it;
      r1 = it + a.inter;
    } else {
      r0 = 2 * it;
      r1 = 2 * it + 1 < a.n ? 2 * it + 1 : -1;
    }
  };
  auto prefetch_item = [&](int64_t it) {
    int64_t r0, r1;
    rows_of(it, r0, r1);
    const int64_t sb = 2 * (a.kp / a.g);                    // scale bytes per row
    if (EPI == EPI_SWIGLU) {
      prefetch_range_l2(W + r0 * rb, rb, lane, 32);
      prefetch_range_l2(W + r1 * rb, rb, lane, 32);
      if (lane == 31) {
        prefetch_range_l2(a.scales + r0 * (a.kp / a.g), sb, 0, 1);
        prefetch_range_l2(a.scales + r1 * (a.kp / a.g), sb, 0, 1);
      }
    } else {
      prefetch_range_l2(W + r0 * rb, (r1 >= 0 ? 2 : 1) * rb, lane, 32);
      if (lane == 31) prefetch_range_l2(a.scales + r0 * (a.kp / a.g), (r1 >= 0 ? 2 : 1) * sb, 0, 1);
    }
  };

  // ---- constant data before the dependency wait: the first rows to L2 ----
  for (int j = 0; j < kPfItems; ++j) {
    const int64_t it = i_begin + warp + static_cast<int64_t>(j) * kWarps;
    if (it < i_end) prefetch_item(it);
  }
  grid_dep_wait();
  grid_dep_launch();

  // ---- 1/rms of x (LlamaRMSNorm, the GEMV's reduction order) ----
  float inv = 1.0f;
  if (a.norm_w) {
    float s = 0.0f;
    for (int64_t e = tid; e < a.k; e += kThreads) {
      const float v = a.x[e];
      s = fmaf(v, v, s);
    }
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (tid == 0) {
      float t = 0.0f;
      for (int w = 0; w < kWarps; ++w) t += red[w];
      const float var = __fdiv_rn(t, static_cast<float>(a.k));
      inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, a.norm_eps)));
    }
    __syncthreads();
    inv = inv_s;
  }

  // ---- digits of x: four threads per 32-element vector, 8 elements each ----
  // With Y = X + 0x808080 (|X| < 2^23), the balanced digits of X are the
  // bytes of Y with the top bit flipped: X = sum_p 256^p ((byte_p(Y) ^ 0x80)
  // as a signed byte).  A thread's 8 elements give word 2q (elements 8q +
  // 0,2,4,6) and word 2q + 1 (8q + 1,3,5,7) of every plane, gathered with
  // byte permutes.
  for (int base = 0; base < 4 * nv; base += kThreads) {
    const int it = base + tid;
    const int v = it >> 2, q = it & 3;
    const bool act = v < nv;                     // all 4 threads of a vector agree
    float xv[8];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t e = static_cast<int64_t>(v) * 32 + q * 8 + i;
      float t = 0.0f;
      if (act && e < a.k) {
        t = a.x[e];
        if (a.norm_w) t = __fmul_rn(a.norm_w[e], __fmul_rn(t, inv));
      }
      xv[i] = t;
      amax = fmaxf(amax, fabsf(t));
    }
    // the vector's maximum over its 4 threads (consecutive lanes)
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    int E = 0;
    if (amax > 0.0f && isfinite(amax)) {
      int ex;
      frexpf(amax, &ex);                    // amax < 2^ex
      E = max(-120, min(21 - ex, 120));
    }
    const float sc = ldexpf(1.0f, E);
    uint32_t y[8];
    int sumx = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int X = __float2int_rn(xv[i] * sc);       // exact scaling, |X| <= 2^21
      sumx += X;
      y[i] = static_cast<uint32_t>(X + 0x808080);
    }
    sumx += __shfl_xor_sync(0xffffffffu, sumx, 1);
    sumx += __shfl_xor_sync(0xffffffffu, sumx, 2);
    if (act) {
      uint32_t* rw = reinterpret_cast<uint32_t*>(rec + static_cast<size_t>(v) * kRec);
#pragma unroll
      for (int p = 0; p < 3; ++p) {
        // byte p of each y, elements (0,2,4,6) and (1,3,5,7)
        const uint32_t sel = static_cast<uint32_t>(p) | (static_cast<uint32_t>(p + 4) << 4);
        const uint32_t e02 = __byte_perm(y[0], y[2], sel), e46 = __byte_perm(y[4], y[6], sel);
        const uint32_t e13 = __byte_perm(y[1], y[3], sel), e57 = __byte_perm(y[5], y[7], sel);
        const uint32_t even = __byte_perm(e02, e46, 0x5410) ^ 0x80808080u;
        const uint32_t odd = __byte_perm(e13, e57, 0x5410) ^ 0x80808080u;
        // words 2q, 2q + 1 of plane p: half q / 2, words (2q) % 4 and + 1
        uint32_t* h = rw + (p * 2 + (q >> 1)) * 4 + 2 * (q & 1);
        h[0] = even;
        h[1] = odd;
      }
      if (q == 0) {
        rw[24] = static_cast<uint32_t>(8 * sumx);
        rw[25] = __float_as_uint(ldexpf(1.0f, -E));
      }
    }
  }
  __syncthreads();

  // ---- rows: warp w takes items i_begin + w, + kWarps, ... ----
  const int64_t ng = a.kp / a.g;
  const uint32_t g = static_cast<uint32_t>(a.g);
  const bool g_pow2 = (g & (g - 1)) == 0;
  const int g_shift = __ffs(g) - 1;
  for (int64_t it = i_begin + warp; it < i_end; it += kWarps) {
    {
      const int64_t ahead = it + static_cast<int64_t>(kPfItems) * kWarps;
      if (ahead < i_end) prefetch_item(ahead);
    }
    int64_t r0, r1;
    rows_of(it, r0, r1);
    const uint4* w0 = reinterpret_cast<const uint4*>(W + r0 * rb);
    const uint4* w1 = reinterpret_cast<const uint4*>(W + (r1 >= 0 ? r1 : r0) * rb);
    const __half* s0 = a.scales + r0 * ng;
    const __half* s1 = a.scales + (r1 >= 0 ? r1 : r0) * ng;
    float acc0 = 0.0f, acc1 = 0.0f;
    // one vector: its digit record is shared by the two rows
    auto vec = [&](int v, const uint4& wa, const uint4& wb) {
      const uint4* rc = rec + static_cast<size_t>(v) * kRec;
      uint4 d[6];
#pragma unroll
      for (int h = 0; h < 6; ++h) d[h] = rc[h];
      const uint4 meta = rc[6];
      const uint32_t e0 = static_cast<uint32_t>(v) * 32u;
      const uint32_t grp = g_pow2 ? (e0 >> g_shift) : e0 / g;
      const float e = __uint_as_float(meta.y);
      const int c = static_cast<int>(meta.x);
      const int t0 = vec_dot(wa, d) - c;
      const int t1 = vec_dot(wb, d) - c;
      acc0 = fmaf(__int2float_rn(t0), __half2float(__ldg(s0 + grp)) * e, acc0);
      acc1 = fmaf(__int2float_rn(t1), __half2float(__ldg(s1 + grp)) * e, acc1);
    };
    int v0 = lane;
    for (; v0 + 32 * (kUnroll - 1) < nv; v0 += 32 * kUnroll) {
      uint4 wa[kUnroll], wb[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        wa[u] = ld_stream(w0 + v0 + 32 * u);
        wb[u] = ld_stream(w1 + v0 + 32 * u);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) vec(v0 + 32 * u, wa[u], wb[u]);
    }
    for (; v0 < nv; v0 += 32) vec(v0, ld_stream(w0 + v0), ld_stream(w1 + v0));
    acc0 = warp_sum(acc0);
    acc1 = warp_sum(acc1);
    if (lane == 0) {
      if constexpr (EPI == EPI_SWIGLU) {
        a.y[r0] = silu_f(acc0) * acc1;
      } else {
        float v0 = acc0;
        if (a.bias) v0 += a.bias[r0];
        if (a.residual) v0 = a.residual[r0] + v0;
        if (a.y) a.y[r0] = v0;
        if (r1 >= 0) {
          float v1 = acc1;
          if (a.bias) v1 += a.bias[r1];
          if (a.residual) v1 = a.residual[r1] + v1;
          if (a.y) a.y[r1] = v1;
        }
      }
    }
  }
}

// 0 off, 1 on (one-row INT4 linears); KSH_GEMV_DP4A=0 in the environment turns it off
int g_dp4a_mode = [] {
  const char* v = getenv("KSH_GEMV_DP4A");
  return (v && *v) ? (atoi(v) != 0 ? 1 : 0) : 1;
}();

size_t dp4a_smem(const LinArgs& a) { return static_cast<size_t>(a.kp / 32) * kRec * 16; }

}  // namespace

int set_gemv_dp4a_mode(int mode) {
  const int prev = g_dp4a_mode;
  g_dp4a_mode = mode ? 1 : 0;
  return prev;
}

bool gemv_i4_dp4a_eligible(int wk, int epi, const LinArgs& a) {
  if (g_dp4a_mode == 0 || wk != WK_I4 || a.m != 1 || a.argmax_out) return false;
  if (a.g % 32 != 0 || a.kp % 32 != 0 || (reinterpret_cast<uintptr_t>(a.w) & 15) != 0) return false;
  if (epi == EPI_SWIGLU && !a.y) return false;
  // the digits of x live in shared memory (112 bytes per 32 elements)
  return dp4a_smem(a) <= 100 * 1024;
}

int launch_gemv_i4_dp4a(int epi, const LinArgs& a, cudaStream_t stream) {
  const int64_t nrows_out = epi == EPI_SWIGLU ? a.inter : a.n;
  const int64_t nitems = epi == EPI_SWIGLU ? nrows_out : (nrows_out + 1) / 2;
  const size_t smem = dp4a_smem(a);
  if (nitems <= 0) return KSH_OK;
  const int64_t ctas = std::min<int64_t>(nitems, static_cast<int64_t>(num_sms()) * 2);
  const int64_t per = (nitems + ctas - 1) / ctas;
  const int64_t grid = (nitems + per - 1) / per;
  if (epi == EPI_SWIGLU) {
    auto kern = gemv_i4_dp4a_kernel<EPI_SWIGLU>;
    if (smem > 32 * 1024 && set_smem_optin(reinterpret_cast<const void*>(kern), smem) != KSH_OK)
      return KSH_ERR_CUDA;
    return launch(kern, dim3(static_cast<unsigned>(grid)), dim3(kThreads), smem, stream, a, per);
  }
  auto kern = gemv_i4_dp4a_kernel<EPI_STORE>;
  if (smem > 32 * 1024 && set_smem_optin(reinterpret_cast<const void*>(kern), smem) != KSH_OK)
    return KSH_ERR_CUDA;
  return launch(kern, dim3(static_cast<unsigned>(grid)), dim3(kThreads), smem, stream, a, per);
}

}  // namespace ksh
