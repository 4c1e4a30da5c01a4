// K3 / K4 / K11: decode-time linear layers on CUDA cores (M <= 16 rows).
//
// Replaces QuantizedLinear.forward (engine/quantization.py:394-396), which
// materialises dequant(W) and calls F.linear, and the fp32 lm_head
// (engine/model.py:151).  Weight-only quantized decode is HBM-bound: every
// weight byte is read once per step, so the kernel is built around the
// weight stream:
//
// * each warp owns one output row (two for the fused gate/up + SwiGLU);
//   lanes read the row with 128-bit non-allocating loads and reduce with
//   warp shuffles;
// * the first row's weight vectors (up to kHoist per lane) are loaded into
//   registers BEFORE the programmatic-launch wait: weights never depend on
//   the previous kernel, so their DRAM latency overlaps the tail of the
//   previous kernel (or, without PDL, the activation staging);
// * the activation rows (fp32) are staged once per CTA in shared memory with
//   an XOR swizzle that makes the per-lane float4 reads bank-conflict free;
//   an optional RMSNorm (LlamaRMSNorm arithmetic, deterministic per-row
//   reduction) is applied while staging, which removes the separate norm
//   kernel in front of q/k/v, gate/up and lm_head;
// * dequantization happens in registers: INT8 sums x*q and applies the
//   per-row fp16 scale once; INT4 sums x*q per 32-nibble vector (one group
//   slice) and applies the group scale per vector;
// * the lm_head variant fuses the greedy argmax (first index of the maximum)
//   with a last-CTA reduction over per-CTA partials.

#include <float.h>

#include <algorithm>

#include "linear.cuh"

namespace ksh {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
// Weight vectors per lane held in registers: the register budget scales with
// the number of staged-x values one vector consumes (4 fp32 / 16 int8 / 32
// int4 elements), so the counts are sized by elements, about 64 per lane and
// row.  Bandwidth for long rows comes from the bulk L2 prefetch of the CTA's
// rows, not from deep register pipelining.
template <int WK>
constexpr int unroll_count() { return WK == WK_F32 ? 4 : 2; }
template <int WK, int EPI, int MT>
constexpr int hoist_count() {
  return (WK == WK_F32 ? 8 : (WK == WK_I8 ? 4 : 2)) / (EPI == EPI_SWIGLU || MT > 4 ? 2 : 1);
}

template <int WK>
struct Vec;
template <>
struct Vec<WK_F32> {
  static constexpr int E = 4;
};
template <>
struct Vec<WK_I8> {
  static constexpr int E = 16;
};
template <>
struct Vec<WK_I4> {
  static constexpr int E = 32;
};

// Physical float4 slot of logical float4 index c inside a staged x row.
template <int WK>
__device__ __forceinline__ int swz(int c) {
  if constexpr (WK == WK_I8) return (c & ~3) | ((c & 3) ^ ((c >> 3) & 3));
  if constexpr (WK == WK_I4) return (c & ~7) | ((c & 7) ^ ((c >> 3) & 7));
  return c;
}

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Dot product of one 16-byte weight vector (local vector index v within the
// staged tile) with one staged x row.
template <int WK>
__device__ __forceinline__ float vec_dot(const uint4& w, int v, const float4* xr) {
  float s = 0.0f;
  if constexpr (WK == WK_F32) {
    const float4 x = xr[swz<WK>(v)];
    s = fmaf(__uint_as_float(w.x), x.x, s);
    s = fmaf(__uint_as_float(w.y), x.y, s);
    s = fmaf(__uint_as_float(w.z), x.z, s);
    s = fmaf(__uint_as_float(w.w), x.w, s);
  } else if constexpr (WK == WK_I8) {
    const uint32_t ws[4] = {bias_i8(w.x), bias_i8(w.y), bias_i8(w.z), bias_i8(w.w)};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 x = xr[swz<WK>(4 * v + j)];
      s = fmaf(dq_i8(ws[j], 0), x.x, s);
      s = fmaf(dq_i8(ws[j], 1), x.y, s);
      s = fmaf(dq_i8(ws[j], 2), x.z, s);
      s = fmaf(dq_i8(ws[j], 3), x.w, s);
    }
  } else {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 xa = xr[swz<WK>(8 * v + 2 * j)];
      const float4 xb = xr[swz<WK>(8 * v + 2 * j + 1)];
      const uint32_t lo = nib_lo(ws[j]), hi = nib_hi(ws[j]);
      s = fmaf(dq_i4(lo, 0), xa.x, s);
      s = fmaf(dq_i4(hi, 0), xa.y, s);
      s = fmaf(dq_i4(lo, 1), xa.z, s);
      s = fmaf(dq_i4(hi, 1), xa.w, s);
      s = fmaf(dq_i4(lo, 2), xb.x, s);
      s = fmaf(dq_i4(hi, 2), xb.y, s);
      s = fmaf(dq_i4(lo, 3), xb.z, s);
      s = fmaf(dq_i4(hi, 3), xb.w, s);
    }
  }
  return s;
}

template <int WK>
__device__ __forceinline__ int64_t row_bytes(const LinArgs& a) {
  if constexpr (WK == WK_F32) return a.k * 4;
  if constexpr (WK == WK_I8) return a.k;
  return a.kp / 2;
}

// Per-row 1/rms of x (LlamaRMSNorm: 1 / sqrt(mean(x^2) + eps)), reduced in a
// fixed order (lanes, then warps) so results are run-to-run deterministic.
template <int MT>
__device__ __forceinline__ void row_inv_rms(const LinArgs& a, float (*red)[MT], float* inv) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int mm = 0; mm < MT; ++mm) {
    float s = 0.0f;
    if (mm < a.m)
      for (int64_t e = threadIdx.x; e < a.k; e += kThreads) {
        const float v = a.x[mm * a.k + e];
        s = fmaf(v, v, s);
      }
    s = warp_sum(s);
    if (lane == 0) red[warp][mm] = s;
  }
  __syncthreads();
  if (threadIdx.x < MT) {
    float t = 0.0f;
    for (int w = 0; w < kWarps; ++w) t += red[w][threadIdx.x];
    const float var = __fdiv_rn(t, static_cast<float>(a.k));
    inv[threadIdx.x] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, a.norm_eps)));
  }
  __syncthreads();
}

// Stage x[:, k0 : k0 + kl] (kl multiple of 4) into xs, zero-filled beyond the
// logical k and beyond m; RMSNorm applied when a.norm_w is set.
template <int WK, int MT>
__device__ __forceinline__ void stage_x(const LinArgs& a, float4* xs, int ktv, int64_t k0,
                                        int kl, const float* inv) {
  float* xf = reinterpret_cast<float*>(xs);
  const int nel = MT * kl;
  for (int i = threadIdx.x; i < nel; i += kThreads) {
    const int mm = i / kl, e = i - mm * kl;
    const int64_t kk = k0 + e;
    float v = 0.0f;
    if (mm < a.m && kk < a.k) {
      v = a.x[mm * a.k + kk];
      if (a.norm_w) v = __fmul_rn(a.norm_w[kk], __fmul_rn(v, inv[mm]));
    }
    xf[(mm * ktv + swz<WK>(e >> 2)) * 4 + (e & 3)] = v;
  }
}

// Fold one weight vector (local index v) of rows r0 / r1 into the accumulators.
template <int WK, int EPI, int MT>
__device__ __forceinline__ void fold_vec(const LinArgs& a, const float4* xs, int ktv,
                                         int64_t r0, int64_t r1, int64_t k0, int v,
                                         const uint4& w0, const uint4& w1, float (&acc0)[MT],
                                         float (&acc1)[MT]) {
  constexpr int E = Vec<WK>::E;
  float s0 = 1.0f, s1 = 1.0f;
  if constexpr (WK == WK_I4) {
    // group of this vector's first element; a shift for power-of-two groups
    const int64_t ng = a.kp / a.g;
    const uint32_t e0 = static_cast<uint32_t>(k0) + static_cast<uint32_t>(v) * E;
    const uint32_t g = static_cast<uint32_t>(a.g);
    const int64_t grp = (g & (g - 1)) == 0 ? (e0 >> (__ffs(g) - 1)) : e0 / g;
    s0 = __half2float(a.scales[r0 * ng + grp]);
    if constexpr (EPI == EPI_SWIGLU) s1 = __half2float(a.scales[r1 * ng + grp]);
  }
#pragma unroll
  for (int mm = 0; mm < MT; ++mm) {
    const float4* xr = xs + mm * ktv;
    const float d0 = vec_dot<WK>(w0, v, xr);
    if constexpr (WK == WK_I4) acc0[mm] = fmaf(d0, s0, acc0[mm]);
    else acc0[mm] += d0;
    if constexpr (EPI == EPI_SWIGLU) {
      const float d1 = vec_dot<WK>(w1, v, xr);
      if constexpr (WK == WK_I4) acc1[mm] = fmaf(d1, s1, acc1[mm]);
      else acc1[mm] += d1;
    }
  }
}

// Accumulate rows r0 (and r1 for SwiGLU) over local vectors [v_begin, nv) of
// the staged tile, kUnroll vectors in flight per lane.
template <int WK, int EPI, int MT>
__device__ __forceinline__ void accumulate(const LinArgs& a, const float4* xs, int ktv,
                                           int64_t r0, int64_t r1, int64_t k0, int kl,
                                           int v_begin, float (&acc0)[MT], float (&acc1)[MT]) {
  constexpr int E = Vec<WK>::E;
  const int lane = threadIdx.x & 31;
  const int64_t rb = row_bytes<WK>(a);
  const char* w0 = static_cast<const char*>(a.w) + r0 * rb + (k0 / E) * 16;
  const char* w1 = static_cast<const char*>(a.w) + r1 * rb + (k0 / E) * 16;
  const int nv = kl / E;
  constexpr int kUnroll = unroll_count<WK>();
  for (int v0 = v_begin + lane; v0 < nv; v0 += 32 * kUnroll) {
    uint4 wv0[kUnroll], wv1[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int v = v0 + 32 * u;
      if (v < nv) {
        wv0[u] = ld_stream(w0 + static_cast<int64_t>(v) * 16);
        if constexpr (EPI == EPI_SWIGLU) wv1[u] = ld_stream(w1 + static_cast<int64_t>(v) * 16);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int v = v0 + 32 * u;
      if (v < nv) fold_vec<WK, EPI, MT>(a, xs, ktv, r0, r1, k0, v, wv0[u], wv1[u], acc0, acc1);
    }
  }
}

struct Best {
  float v;
  int32_t i;
};
__device__ __forceinline__ bool better(float v, int32_t i, float bv, int32_t bi) {
  return v > bv || (v == bv && i < bi);
}

// Reduce the row sums over the warp and write the epilogue for row group rg.
template <int WK, int EPI, int MT, bool ARGMAX>
__device__ __forceinline__ void finish_row(const LinArgs& a, int64_t rg, float (&acc0)[MT],
                                           float (&acc1)[MT], Best (&best)[MT]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int mm = 0; mm < MT; ++mm) {
    acc0[mm] = warp_sum(acc0[mm]);
    if constexpr (EPI == EPI_SWIGLU) acc1[mm] = warp_sum(acc1[mm]);
  }
  if constexpr (EPI == EPI_STORE) {
    const int64_t r = rg;
    float sc = 1.0f;
    if constexpr (WK == WK_I8) sc = __half2float(a.scales[r]);
    const float b = a.bias ? a.bias[r] : 0.0f;
#pragma unroll
    for (int mm = 0; mm < MT; ++mm) {
      if (lane == mm && mm < a.m) {
        float v = acc0[mm] * sc;
        if (a.bias) v += b;
        if (a.residual) v = a.residual[mm * a.n + r] + v;
        if (a.y) a.y[mm * a.n + r] = v;
        if constexpr (ARGMAX) {
          if (better(v, static_cast<int32_t>(r), best[mm].v, best[mm].i)) {
            best[mm].v = v;
            best[mm].i = static_cast<int32_t>(r);
          }
        }
      }
    }
  } else {
    const int64_t j = rg;
    float s0 = 1.0f, s1 = 1.0f;
    if constexpr (WK == WK_I8) {
      s0 = __half2float(a.scales[j]);
      s1 = __half2float(a.scales[j + a.inter]);
    }
#pragma unroll
    for (int mm = 0; mm < MT; ++mm) {
      if (lane == mm && mm < a.m) {
        const float g = acc0[mm] * s0;
        const float u = acc1[mm] * s1;
        a.y[mm * a.inter + j] = silu_f(g) * u;
      }
    }
  }
}

template <int WK, int EPI, int MT, bool ARGMAX>
__global__ void __launch_bounds__(kThreads, (WK == WK_F32 && MT <= 2) ? 3 : 2)
gemv_kernel(LinArgs a, int kt, int prefetch) {
  constexpr int E = Vec<WK>::E;
  extern __shared__ float4 xs[];
  __shared__ float red[kWarps][MT];
  __shared__ float inv_rms[MT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nrg = EPI == EPI_SWIGLU ? a.inter : a.n;
  const int64_t keff = WK == WK_I4 ? a.kp : a.k;
  const int ktv = kt / 4;
  const bool single = keff <= kt;
  const int64_t rb = row_bytes<WK>(a);
  const int nv_row = static_cast<int>(keff / E);
  // This CTA owns the contiguous row groups [g_begin, g_end) (8 rows each,
  // warp w takes row w of a group).
  const int64_t ngroups = (nrg + kWarps - 1) / kWarps;
  const int64_t gpc = (ngroups + gridDim.x - 1) / gridDim.x;
  const int64_t g_begin = static_cast<int64_t>(blockIdx.x) * gpc;
  const int64_t g_end = g_begin + gpc < ngroups ? g_begin + gpc : ngroups;
  const int64_t rg0 = g_begin * kWarps + warp;
  // rows of the first half (SwiGLU: gate rows; the up rows follow at +inter)
  auto prefetch_groups = [&](int64_t ga, int64_t gb, int tid, int nthr) {
    if (ga >= gb) return;
    const int64_t r_lo = ga * kWarps;
    const int64_t r_hi = gb * kWarps < nrg ? gb * kWarps : nrg;
    const char* base = static_cast<const char*>(a.w) + r_lo * rb;
    prefetch_range_l2(base, static_cast<size_t>((r_hi - r_lo) * rb), tid, nthr);
    if constexpr (EPI == EPI_SWIGLU)
      prefetch_range_l2(base + a.inter * rb, static_cast<size_t>((r_hi - r_lo) * rb), tid, nthr);
  };
  // L2 prefetch distance: about kPrefetchBytes of this CTA's rows ahead.
  constexpr int64_t kPrefetchBytes = 96 * 1024;
  const int64_t group_bytes = kWarps * rb * (EPI == EPI_SWIGLU ? 2 : 1);
  const int64_t pf_dist = kPrefetchBytes / group_bytes > 1 ? kPrefetchBytes / group_bytes : 1;

  // ---- constant data, safe before the dependency wait ----
  constexpr int kHoist = hoist_count<WK, EPI, MT>();
  uint4 h0[kHoist], h1[kHoist];
  if (single && rg0 < nrg) {
    const char* w0 = static_cast<const char*>(a.w) + rg0 * rb;
    const char* w1 = static_cast<const char*>(a.w) + (rg0 + a.inter) * rb;
#pragma unroll
    for (int u = 0; u < kHoist; ++u) {
      const int v = lane + 32 * u;
      if (v < nv_row) {
        h0[u] = ld_stream(w0 + static_cast<int64_t>(v) * 16);
        if constexpr (EPI == EPI_SWIGLU) h1[u] = ld_stream(w1 + static_cast<int64_t>(v) * 16);
      }
    }
  }
  if (prefetch) {
    const int64_t ge = g_begin + pf_dist < g_end ? g_begin + pf_dist : g_end;
    if (ge > g_begin + 1 || nv_row > 32 * kHoist) prefetch_groups(g_begin, ge, threadIdx.x, kThreads);
  }
  grid_dep_wait();
  grid_dep_launch();

  if (a.norm_w) row_inv_rms<MT>(a, red, inv_rms);

  Best best[MT];
#pragma unroll
  for (int mm = 0; mm < MT; ++mm) best[mm] = Best{-FLT_MAX, INT32_MAX};

  if (single) {
    stage_x<WK, MT>(a, xs, ktv, 0, static_cast<int>(keff), inv_rms);
    __syncthreads();
    for (int64_t gi = g_begin; gi < g_end; ++gi) {
      // keep the L2 prefetch pf_dist groups ahead (warp 0)
      if (prefetch && warp == 0 && gi + pf_dist < g_end)
        prefetch_groups(gi + pf_dist, gi + pf_dist + 1, lane, 32);
      const int64_t rg = gi * kWarps + warp;
      if (rg >= nrg) break;
      float acc0[MT], acc1[MT];
#pragma unroll
      for (int mm = 0; mm < MT; ++mm) acc0[mm] = acc1[mm] = 0.0f;
      const int64_t r1 = EPI == EPI_SWIGLU ? rg + a.inter : rg;
      int v_begin = 0;
      if (rg == rg0) {
#pragma unroll
        for (int u = 0; u < kHoist; ++u) {
          const int v = lane + 32 * u;
          if (v < nv_row) fold_vec<WK, EPI, MT>(a, xs, ktv, rg, r1, 0, v, h0[u], h1[u], acc0, acc1);
        }
        v_begin = 32 * kHoist;
      }
      accumulate<WK, EPI, MT>(a, xs, ktv, rg, r1, 0, static_cast<int>(keff), v_begin, acc0, acc1);
      finish_row<WK, EPI, MT, ARGMAX>(a, rg, acc0, acc1, best);
    }
  } else {
    // x does not fit shared memory at once: every group streams the x tiles
    // (the loop bounds are CTA-uniform; the barriers inside are reached by
    // all threads).
    for (int64_t gi = g_begin; gi < g_end; ++gi) {
      if (prefetch && warp == 0 && gi + pf_dist < g_end)
        prefetch_groups(gi + pf_dist, gi + pf_dist + 1, lane, 32);
      const int64_t rg = gi * kWarps + warp;
      const bool active = rg < nrg;
      const int64_t r1 = EPI == EPI_SWIGLU ? rg + a.inter : rg;
      float acc0[MT], acc1[MT];
#pragma unroll
      for (int mm = 0; mm < MT; ++mm) acc0[mm] = acc1[mm] = 0.0f;
      for (int64_t k0 = 0; k0 < keff; k0 += kt) {
        const int kl = static_cast<int>(keff - k0 < kt ? keff - k0 : kt);
        __syncthreads();
        stage_x<WK, MT>(a, xs, ktv, k0, kl, inv_rms);
        __syncthreads();
        if (active) accumulate<WK, EPI, MT>(a, xs, ktv, rg, r1, k0, kl, 0, acc0, acc1);
      }
      if (active) finish_row<WK, EPI, MT, ARGMAX>(a, rg, acc0, acc1, best);
    }
  }

  if constexpr (ARGMAX) {
    // CTA reduce: lane mm of each warp holds the warp's best for row mm.
    __shared__ Best sb[kWarps][MT];
    __shared__ bool is_last;
#pragma unroll
    for (int mm = 0; mm < MT; ++mm)
      if (lane == mm) sb[warp][mm] = best[mm];
    __syncthreads();
    if (threadIdx.x < a.m && threadIdx.x < MT) {
      const int mm = threadIdx.x;
      Best b = sb[0][mm];
      for (int w = 1; w < kWarps; ++w)
        if (better(sb[w][mm].v, sb[w][mm].i, b.v, b.i)) b = sb[w][mm];
      a.part_val[static_cast<int64_t>(blockIdx.x) * a.m + mm] = b.v;
      a.part_idx[static_cast<int64_t>(blockIdx.x) * a.m + mm] = b.i;
      __threadfence();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned prev = atomicAdd(a.counter, 1u);
      is_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (is_last) {
      __threadfence();
      // warp mm reduces row mm over all CTA partials
      for (int mm = warp; mm < a.m; mm += kWarps) {
        float bv = -FLT_MAX;
        int32_t bi = INT32_MAX;
        for (int c = lane; c < static_cast<int>(gridDim.x); c += 32) {
          const float v = __ldcg(a.part_val + static_cast<int64_t>(c) * a.m + mm);
          const int32_t i = __ldcg(a.part_idx + static_cast<int64_t>(c) * a.m + mm);
          if (better(v, i, bv, bi)) {
            bv = v;
            bi = i;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if (lane == 0) a.argmax_out[mm] = bi;
      }
      if (threadIdx.x == 0) *a.counter = 0u;
    }
  }
}

template <int WK, int EPI, int MT, bool ARGMAX>
int launch_t(const LinArgs& a, cudaStream_t stream) {
  const int64_t keff = WK == WK_I4 ? a.kp : a.k;
  // Shared-memory budget for the staged x tile: up to 96 KB.
  int64_t kt = (96 * 1024) / (MT * 4);
  kt = kt / 256 * 256;
  if (keff <= kt) kt = (keff + 255) / 256 * 256;
  const size_t smem = static_cast<size_t>(MT) * kt * 4;
  auto kern = gemv_kernel<WK, EPI, MT, ARGMAX>;
  if (smem > 32 * 1024) {
    if (set_smem_optin(reinterpret_cast<const void*>(kern), smem) != KSH_OK) return KSH_ERR_CUDA;
  }
  const int64_t nrg = EPI == EPI_SWIGLU ? a.inter : a.n;
  // Contiguous row blocks per CTA, exactly one resident wave.  At most 8
  // CTAs of 256 threads fit an SM, so the grid never exceeds
  // gemv_argmax_grid(), which sizes the argmax partials.
  const int per_sm = resident_ctas(reinterpret_cast<const void*>(kern), kThreads, smem);
  const int64_t grid = std::min((nrg + kWarps - 1) / kWarps,
                                static_cast<int64_t>(num_sms()) * std::min(std::max(per_sm, 1), 8));
  if (grid > INT32_MAX) return KSH_ERR_UNSUPPORTED;
  return launch(kern, dim3(static_cast<unsigned>(grid)), dim3(kThreads), smem, stream, a,
                static_cast<int>(kt), prefetch_enabled() ? 1 : 0);
}

template <int WK, int EPI, bool ARGMAX>
int dispatch_m(const LinArgs& a, cudaStream_t stream) {
  if (a.m <= 1) return launch_t<WK, EPI, 1, ARGMAX>(a, stream);
  if (a.m <= 2) return launch_t<WK, EPI, 2, ARGMAX>(a, stream);
  if (a.m <= 4) return launch_t<WK, EPI, 4, ARGMAX>(a, stream);
  if (a.m <= 8) return launch_t<WK, EPI, 8, ARGMAX>(a, stream);
  return launch_t<WK, EPI, 16, ARGMAX>(a, stream);
}

}  // namespace

// Grid size the lm_head argmax variant will use (for workspace sizing).
int64_t gemv_argmax_grid(int64_t n) {
  const int64_t g = (n + kWarps - 1) / kWarps;
  return std::min<int64_t>(g, static_cast<int64_t>(num_sms()) * 8);
}

int launch_gemv(int wk, int epi, const LinArgs& a, cudaStream_t stream) {
  const bool am = a.argmax_out != nullptr;
  if (epi == EPI_SWIGLU && am) return KSH_ERR_UNSUPPORTED;
  int st = KSH_OK;
  if (gemv_resident_enabled() && launch_gemv_resident(wk, epi, a, stream, &st)) return st;
  switch (wk * 4 + epi * 2 + (am ? 1 : 0)) {
    case WK_F32 * 4 + 0: return dispatch_m<WK_F32, EPI_STORE, false>(a, stream);
    case WK_F32 * 4 + 1: return dispatch_m<WK_F32, EPI_STORE, true>(a, stream);
    case WK_F32 * 4 + 2: return dispatch_m<WK_F32, EPI_SWIGLU, false>(a, stream);
    case WK_I8 * 4 + 0: return dispatch_m<WK_I8, EPI_STORE, false>(a, stream);
    case WK_I8 * 4 + 2: return dispatch_m<WK_I8, EPI_SWIGLU, false>(a, stream);
    case WK_I4 * 4 + 0: return dispatch_m<WK_I4, EPI_STORE, false>(a, stream);
    case WK_I4 * 4 + 2: return dispatch_m<WK_I4, EPI_SWIGLU, false>(a, stream);
    default: return KSH_ERR_UNSUPPORTED;
  }
}

}  // namespace ksh
