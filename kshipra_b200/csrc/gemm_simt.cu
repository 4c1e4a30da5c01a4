// Generic CUDA-core linear layer for any shape (ragged k, odd group sizes,
// any m).  It dequantizes each weight tile into shared memory exactly as the
// reference does (fp32(q) * fp32(scale), engine/quantization.py:226-230,
// :321-344) and runs a 64x64 register-tiled fp32 GEMM.  It is the path for
// shapes the vectorised GEMV and the tensor-core GEMM do not take.

#include "linear.cuh"

namespace ksh {
namespace {

constexpr int BM = 64, BN = 64, BK = 16, TH = 256;

template <int WK>
__device__ __forceinline__ float load_w(const LinArgs& a, int64_t r, int64_t kk) {
  if (kk >= a.k) return 0.0f;
  if constexpr (WK == WK_F32) {
    return static_cast<const float*>(a.w)[r * a.k + kk];
  } else if constexpr (WK == WK_I8) {
    const int8_t q = static_cast<const int8_t*>(a.w)[r * a.k + kk];
    return static_cast<float>(q) * __half2float(a.scales[r]);
  } else {
    const uint8_t b = static_cast<const uint8_t*>(a.w)[r * (a.kp / 2) + (kk >> 1)];
    const int u = (kk & 1) ? (b >> 4) : (b & 0xF);
    const int q = (u ^ 8) - 8;
    return static_cast<float>(q) * __half2float(a.scales[r * (a.kp / a.g) + kk / a.g]);
  }
}

template <int WK, int EPI>
__global__ void __launch_bounds__(TH) gemm_simt_kernel(LinArgs a) {
  __shared__ float xs[BK][BM + 4];
  __shared__ float ws0[BK][BN + 4];
  __shared__ float ws1[EPI == EPI_SWIGLU ? BK : 1][BN + 4];
  grid_dep_wait();
  grid_dep_launch();
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * BN;
  const int64_t ncols = EPI == EPI_SWIGLU ? a.inter : a.n;
  // Optional RMSNorm of the x rows (LlamaRMSNorm), one warp per row, fixed order.
  __shared__ float inv_rms[BM];
  if (a.norm_w) {
    const int lane = tid & 31, wid = tid >> 5;
    for (int r = wid; r < BM; r += TH / 32) {
      const int64_t mm = m0 + r;
      float s = 0.0f;
      if (mm < a.m)
        for (int64_t e = lane; e < a.k; e += 32) {
          const float v = a.x[mm * a.k + e];
          s = fmaf(v, v, s);
        }
      s = warp_sum(s);
      if (lane == 0)
        inv_rms[r] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, static_cast<float>(a.k)),
                                                          a.norm_eps)));
    }
    __syncthreads();
  }
  float acc0[4][4] = {}, acc1[4][4] = {};
  for (int64_t k0 = 0; k0 < a.k; k0 += BK) {
#pragma unroll
    for (int i = 0; i < (BM * BK) / TH; ++i) {
      const int e = tid + i * TH, r = e / BK, c = e % BK;
      const int64_t mm = m0 + r, kk = k0 + c;
      float xv = (mm < a.m && kk < a.k) ? a.x[mm * a.k + kk] : 0.0f;
      if (a.norm_w && mm < a.m && kk < a.k) xv = __fmul_rn(a.norm_w[kk], __fmul_rn(xv, inv_rms[r]));
      xs[c][r] = xv;
      const int64_t nn = n0 + r;
      ws0[c][r] = nn < ncols ? load_w<WK>(a, nn, kk) : 0.0f;
      if constexpr (EPI == EPI_SWIGLU) ws1[c][r] = nn < ncols ? load_w<WK>(a, nn + a.inter, kk) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < BK; ++c) {
      float xa[4], wb[4], wc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) xa[i] = xs[c][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        wb[j] = ws0[c][tx + 16 * j];
        if constexpr (EPI == EPI_SWIGLU) wc[j] = ws1[c][tx + 16 * j];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc0[i][j] = fmaf(xa[i], wb[j], acc0[i][j]);
          if constexpr (EPI == EPI_SWIGLU) acc1[i][j] = fmaf(xa[i], wc[j], acc1[i][j]);
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t mm = m0 + ty + 16 * i;
    if (mm >= a.m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t nn = n0 + tx + 16 * j;
      if (nn >= ncols) continue;
      if constexpr (EPI == EPI_SWIGLU) {
        a.y[mm * a.inter + nn] = silu_f(acc0[i][j]) * acc1[i][j];
      } else {
        float v = acc0[i][j];
        if (a.bias) v += a.bias[nn];
        if (a.residual) v = a.residual[mm * a.n + nn] + v;
        a.y[mm * a.n + nn] = v;
      }
    }
  }
}

template <int WK, int EPI>
int launch_t(const LinArgs& a, cudaStream_t stream) {
  const int64_t ncols = EPI == EPI_SWIGLU ? a.inter : a.n;
  const int64_t gx = (ncols + BN - 1) / BN, gy = (a.m + BM - 1) / BM;
  if (gx > INT32_MAX || gy > 65535) return KSH_ERR_UNSUPPORTED;
  return launch(gemm_simt_kernel<WK, EPI>, dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)),
                dim3(TH), 0, stream, a);
}

}  // namespace

int launch_gemm_simt(int wk, int epi, const LinArgs& a, cudaStream_t stream) {
  switch (wk * 2 + epi) {
    case WK_F32 * 2 + EPI_STORE: return launch_t<WK_F32, EPI_STORE>(a, stream);
    case WK_F32 * 2 + EPI_SWIGLU: return launch_t<WK_F32, EPI_SWIGLU>(a, stream);
    case WK_I8 * 2 + EPI_STORE: return launch_t<WK_I8, EPI_STORE>(a, stream);
    case WK_I8 * 2 + EPI_SWIGLU: return launch_t<WK_I8, EPI_SWIGLU>(a, stream);
    case WK_I4 * 2 + EPI_STORE: return launch_t<WK_I4, EPI_STORE>(a, stream);
    case WK_I4 * 2 + EPI_SWIGLU: return launch_t<WK_I4, EPI_SWIGLU>(a, stream);
    default: return KSH_ERR_UNSUPPORTED;
  }
}

}  // namespace ksh
