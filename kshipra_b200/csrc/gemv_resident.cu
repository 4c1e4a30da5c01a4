// Latency-optimised decode GEMV for small weight matrices (M <= 4 rows).
//
// Same contract as gemv.cu (QuantizedLinear.forward, engine/quantization.py:
// 394-396, optional fused RMSNorm / residual / SwiGLU), specialised for the
// regime where every CTA's share of the weight matrix fits in registers --
// the q/k/v, o, gate/up and down projections of decode steps at small batch.
// There the time is latency, not bandwidth, so:
//
// * the grid is at most one CTA per SM; each warp owns `rw` consecutive rows
//   and loads ALL of their weight vectors (VPL 16-byte vectors per lane and
//   row) into registers before the programmatic-launch wait, together with
//   the RMSNorm weights it will need -- constant data, so the DRAM latency
//   overlaps the previous kernel;
// * after the wait a single pass loads x (one L2 round trip), accumulates the
//   row sums of squares and stages x into swizzled shared memory; the norm is
//   applied in shared memory;
// * each warp folds its register-resident rows, reduces with shuffles and
//   writes the epilogue (scale, bias, residual, SwiGLU).
// With registers capped at 128 per thread the CTA leaves room on the SM for
// the next kernel of the chain to become resident early.

#include <float.h>

#include <algorithm>

#include "linear.cuh"

namespace ksh {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kCap = 20;              // weight vectors per lane held in registers

template <int WK>
struct VecR;
template <>
struct VecR<WK_I8> {
  static constexpr int E = 16;
};
template <>
struct VecR<WK_I4> {
  static constexpr int E = 32;
};

template <int WK>
__device__ __forceinline__ int swz(int c) {
  if constexpr (WK == WK_I8) return (c & ~3) | ((c & 3) ^ ((c >> 3) & 3));
  return (c & ~7) | ((c & 7) ^ ((c >> 3) & 7));
}

__device__ __forceinline__ uint4 ld_w(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <int WK>
__device__ __forceinline__ float dot_vec(const uint4& w, int v, const float4* xr) {
  float s0 = 0.0f, s1 = 0.0f;
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  if constexpr (WK == WK_I8) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 x = xr[swz<WK>(4 * v + j)];
      const uint32_t wb = bias_i8(ws[j]);
      s0 = fmaf(dq_i8(wb, 0), x.x, s0);
      s1 = fmaf(dq_i8(wb, 1), x.y, s1);
      s0 = fmaf(dq_i8(wb, 2), x.z, s0);
      s1 = fmaf(dq_i8(wb, 3), x.w, s1);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 xa = xr[swz<WK>(8 * v + 2 * j)];
      const float4 xb = xr[swz<WK>(8 * v + 2 * j + 1)];
      const uint32_t lo = nib_lo(ws[j]), hi = nib_hi(ws[j]);
      const float q[8] = {dq_i4(lo, 0), dq_i4(hi, 0), dq_i4(lo, 1), dq_i4(hi, 1),
                          dq_i4(lo, 2), dq_i4(hi, 2), dq_i4(lo, 3), dq_i4(hi, 3)};
      s0 = fmaf(q[0], xa.x, s0);
      s1 = fmaf(q[1], xa.y, s1);
      s0 = fmaf(q[2], xa.z, s0);
      s1 = fmaf(q[3], xa.w, s1);
      s0 = fmaf(q[4], xb.x, s0);
      s1 = fmaf(q[5], xb.y, s1);
      s0 = fmaf(q[6], xb.z, s0);
      s1 = fmaf(q[7], xb.w, s1);
    }
  }
  return s0 + s1;
}

template <int WK, int EPI, int MT, int VPL>
__global__ void __launch_bounds__(kThreads, 2)
gemv_resident_kernel(LinArgs a, int rw) {
  constexpr int E = VecR<WK>::E;
  constexpr int F = EPI == EPI_SWIGLU ? 2 : 1;          // weight rows per output row
  constexpr int RWMAX = kCap / (VPL * F) > 0 ? kCap / (VPL * F) : 1;
  extern __shared__ float4 xs[];
  __shared__ float red[kWarps][MT];
  __shared__ float inv_rms[MT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nrg = EPI == EPI_SWIGLU ? a.inter : a.n;
  const int64_t keff = WK == WK_I4 ? a.kp : a.k;
  const int nv_row = static_cast<int>(keff / E);
  const int ktv = static_cast<int>(keff / 4);
  const int64_t rb = WK == WK_I8 ? a.k : a.kp / 2;
  const int64_t r_base = (static_cast<int64_t>(blockIdx.x) * kWarps + warp) * rw;

  // ---- constant data before the dependency wait: weights and norm weights ----
  uint4 w[RWMAX * F * VPL];
#pragma unroll
  for (int j = 0; j < RWMAX; ++j) {
    const int64_t r = r_base + j;
#pragma unroll
    for (int h = 0; h < F; ++h) {
      const char* rowp = static_cast<const char*>(a.w) + (r + h * a.inter) * rb;
#pragma unroll
      for (int v = 0; v < VPL; ++v) {
        const int vec = lane + 32 * v;
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (j < rw && r < nrg && vec < nv_row) val = ld_w(rowp + static_cast<int64_t>(vec) * 16);
        w[(j * F + h) * VPL + v] = val;
      }
    }
  }
  float* xf = reinterpret_cast<float*>(xs);
  float* nws = xf + MT * keff;                  // norm weights [keff]
  if (a.norm_w)
    for (int e = threadIdx.x; e < a.k; e += kThreads) nws[e] = a.norm_w[e];
  grid_dep_wait();
  grid_dep_launch();

  // ---- one pass over x: stage raw values, accumulate row sums of squares ----
  float ss[MT];
#pragma unroll
  for (int mm = 0; mm < MT; ++mm) {
    ss[mm] = 0.0f;
    for (int e = threadIdx.x; e < keff; e += kThreads) {
      float v = 0.0f;
      if (mm < a.m && e < a.k) v = a.x[mm * a.k + e];
      ss[mm] = fmaf(v, v, ss[mm]);
      xf[(mm * ktv + swz<WK>(e >> 2)) * 4 + (e & 3)] = v;
    }
  }
  if (a.norm_w) {
#pragma unroll
    for (int mm = 0; mm < MT; ++mm) {
      const float s = warp_sum(ss[mm]);
      if (lane == 0) red[warp][mm] = s;
    }
    __syncthreads();
    if (threadIdx.x < MT) {
      float t = 0.0f;
      for (int q = 0; q < kWarps; ++q) t += red[q][threadIdx.x];
      inv_rms[threadIdx.x] =
          __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, static_cast<float>(a.k)), a.norm_eps)));
    }
    __syncthreads();
#pragma unroll
    for (int mm = 0; mm < MT; ++mm) {
      const float inv = inv_rms[mm];
      if (mm < a.m)
        for (int e = threadIdx.x; e < a.k; e += kThreads) {
          float* p = &xf[(mm * ktv + swz<WK>(e >> 2)) * 4 + (e & 3)];
          *p = __fmul_rn(nws[e], __fmul_rn(*p, inv));
        }
    }
  }
  __syncthreads();

  // ---- fold the register-resident rows ----
  const int64_t ng = WK == WK_I4 ? a.kp / a.g : 0;
#pragma unroll
  for (int j = 0; j < RWMAX; ++j) {
    const int64_t r = r_base + j;
    if (j < rw && r < nrg) {
      float acc[F][MT];
#pragma unroll
      for (int h = 0; h < F; ++h)
#pragma unroll
        for (int mm = 0; mm < MT; ++mm) acc[h][mm] = 0.0f;
#pragma unroll
      for (int h = 0; h < F; ++h) {
        const int64_t rr = r + h * a.inter;
#pragma unroll
        for (int v = 0; v < VPL; ++v) {
          const int vec = lane + 32 * v;
          if (vec < nv_row) {
            float sc = 1.0f;
            if constexpr (WK == WK_I4) {
              const uint32_t e0 = static_cast<uint32_t>(vec) * E, g = static_cast<uint32_t>(a.g);
              sc = __half2float(
                  a.scales[rr * ng + ((g & (g - 1)) == 0 ? (e0 >> (__ffs(g) - 1)) : e0 / g)]);
            }
#pragma unroll
            for (int mm = 0; mm < MT; ++mm) {
              const float d = dot_vec<WK>(w[(j * F + h) * VPL + v], vec, xs + mm * ktv);
              if constexpr (WK == WK_I4) acc[h][mm] = fmaf(d, sc, acc[h][mm]);
              else acc[h][mm] += d;
            }
          }
        }
      }
#pragma unroll
      for (int h = 0; h < F; ++h)
#pragma unroll
        for (int mm = 0; mm < MT; ++mm) acc[h][mm] = warp_sum(acc[h][mm]);
#pragma unroll
      for (int mm = 0; mm < MT; ++mm) {
        if (lane == mm && mm < a.m) {
          if constexpr (EPI == EPI_STORE) {
            float v = acc[0][mm];
            if constexpr (WK == WK_I8) v *= __half2float(a.scales[r]);
            if (a.bias) v += a.bias[r];
            if (a.residual) v = a.residual[mm * a.n + r] + v;
            a.y[mm * a.n + r] = v;
          } else {
            float g = acc[0][mm], u = acc[1][mm];
            if constexpr (WK == WK_I8) {
              g *= __half2float(a.scales[r]);
              u *= __half2float(a.scales[r + a.inter]);
            }
            a.y[mm * a.inter + r] = silu_f(g) * u;
          }
        }
      }
    }
  }
}

template <int WK, int EPI, int MT, int VPL>
int launch_r(const LinArgs& a, int rw, cudaStream_t stream) {
  const int64_t keff = WK == WK_I4 ? a.kp : a.k;
  const size_t smem = static_cast<size_t>(MT + 1) * keff * 4;
  auto kern = gemv_resident_kernel<WK, EPI, MT, VPL>;
  if (smem > 32 * 1024 && set_smem_optin(reinterpret_cast<const void*>(kern), smem) != KSH_OK)
    return KSH_ERR_CUDA;
  const int64_t nrg = EPI == EPI_SWIGLU ? a.inter : a.n;
  const int64_t grid = (nrg + static_cast<int64_t>(kWarps) * rw - 1) / (static_cast<int64_t>(kWarps) * rw);
  return launch(kern, dim3(static_cast<unsigned>(grid)), dim3(kThreads), smem, stream, a, rw);
}

template <int WK, int EPI, int MT>
int dispatch_vpl(const LinArgs& a, int vpl, int rw, cudaStream_t s) {
  switch (vpl) {
    case 1: return launch_r<WK, EPI, MT, 1>(a, rw, s);
    case 2: return launch_r<WK, EPI, MT, 2>(a, rw, s);
    case 4: return launch_r<WK, EPI, MT, 4>(a, rw, s);
    case 8: return launch_r<WK, EPI, MT, 8>(a, rw, s);
    default: return launch_r<WK, EPI, MT, 16>(a, rw, s);
  }
}

template <int WK, int EPI>
int dispatch_mt(const LinArgs& a, int vpl, int rw, cudaStream_t s) {
  if (a.m <= 1) return dispatch_vpl<WK, EPI, 1>(a, vpl, rw, s);
  if (a.m <= 2) return dispatch_vpl<WK, EPI, 2>(a, vpl, rw, s);
  return dispatch_vpl<WK, EPI, 4>(a, vpl, rw, s);
}

}  // namespace

// Returns true (and launches) when the matrix fits the register-resident
// scheme: M <= 4, x fits one pass, and each warp's rows fit in kCap vectors.
bool launch_gemv_resident(int wk, int epi, const LinArgs& a, cudaStream_t stream, int* status) {
  if (a.m > 4 || (wk != WK_I8 && wk != WK_I4)) return false;
  if (a.argmax_out) return false;
  const int E = wk == WK_I8 ? 16 : 32;
  const int64_t keff = wk == WK_I4 ? a.kp : a.k;
  if (keff % E != 0 || (a.m + 1) * keff * 4 > 96 * 1024) return false;
  if (wk == WK_I4 && a.g % 32 != 0) return false;
  const int64_t nv_row = keff / E;
  int vpl = 1;
  while (vpl * 32 < nv_row) vpl *= 2;
  if (vpl > 16) return false;
  const int f = epi == EPI_SWIGLU ? 2 : 1;
  const int64_t nrg = epi == EPI_SWIGLU ? a.inter : a.n;
  const int64_t rw = (nrg + static_cast<int64_t>(kWarps) * num_sms() - 1) /
                     (static_cast<int64_t>(kWarps) * num_sms());
  if (vpl * f > kCap) return false;
  const int rwmax = kCap / (vpl * f);
  if (rw > rwmax) return false;
  const int r = static_cast<int>(rw);
  if (wk == WK_I8) *status = epi == EPI_SWIGLU ? dispatch_mt<WK_I8, EPI_SWIGLU>(a, vpl, r, stream)
                                               : dispatch_mt<WK_I8, EPI_STORE>(a, vpl, r, stream);
  else *status = epi == EPI_SWIGLU ? dispatch_mt<WK_I4, EPI_SWIGLU>(a, vpl, r, stream)
                                   : dispatch_mt<WK_I4, EPI_STORE>(a, vpl, r, stream);
  return true;
}

}  // namespace ksh
