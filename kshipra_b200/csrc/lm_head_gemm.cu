// lm_head for a batch of rows (17 .. 64 per launch): fused final RMSNorm,
// fp32 GEMM against the [vocab, hidden] weight and greedy argmax.
//
// Replaces, for a decode step over many sequences, the final norm, the fp32
// lm_head and torch.argmax of the reference's generate loop
// (engine/model.py:180-200; the logits of every batch row).  The GEMV path
// reads the whole weight once per 16 rows; here every weight byte is read
// once per launch and reused across all rows from shared memory:
//
// * one CTA per SM pair slot loops over vocabulary tiles of 128 rows; the
//   producer thread streams 128 x 32-float weight tiles with TMA
//   (128B-swizzled) through a ring of stages;
// * the x tile (64 rows x 32 floats) is loaded by all threads one step
//   ahead, normalised on the way (w * (x * 1/rms), the GEMV's rounding), and
//   stored swizzled;
// * each thread accumulates 4 vocabulary rows x 8 batch rows in fp32 FMAs,
//   k in increasing order;
// * per tile: optional logits store, then the first-index maximum per batch
//   row, kept per CTA; per-CTA partials are reduced by the last CTA to
//   finish (the same scheme as the GEMV's argmax epilogue).
//
// 1/rms per row comes from a small kernel before (fixed reduction order).

#include <float.h>

#include <algorithm>

#include "linear.cuh"
#include "tc_common.cuh"

namespace ksh {
namespace {

using namespace tc;

constexpr int kBN = 128;        // vocabulary rows per tile
constexpr int kBM = 64;         // batch rows per launch
constexpr int kBK = 32;         // floats of k per step (one 128-byte swizzle row)
constexpr int kNS = 4;          // weight stages
constexpr int kThr = 256;
constexpr int kCtasPerSm = 2;

struct LmArgs {
  const float* x;          // [m, k]
  const float* norm_w;     // [k] or nullptr
  const float* inv_rms;    // [m] (when norm_w)
  float* logits;           // [m, vocab] or nullptr
  int64_t* tokens;         // [m] or nullptr
  float* part_val;         // [gridDim.x, m]
  int32_t* part_idx;
  uint32_t* counter;       // zero on entry, reset by the last CTA
  uint32_t* error;         // set when a stage wait gave up; the last CTA then
                           // writes token -1 for every row and clears it
  int m;
  int k;
  int vocab;
  int ntiles;
};

__device__ __forceinline__ bool better(float v, int32_t i, float bv, int32_t bi) {
  return v > bv || (v == bv && i < bi);
}

// 1/rms per row (LlamaRMSNorm: 1 / sqrt(mean(x^2) + eps)); one CTA per row,
// strided partial sums, then lanes and warps in a fixed order.
__global__ void __launch_bounds__(256) lm_inv_rms_kernel(const float* __restrict__ x, int k,
                                                         float eps, float* __restrict__ inv) {
  grid_dep_wait();
  grid_dep_launch();
  const float* row = x + static_cast<int64_t>(blockIdx.x) * k;
  float s = 0.0f;
  for (int e = threadIdx.x; e < k; e += 256) s = fmaf(row[e], row[e], s);
  s = warp_sum(s);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int w = 0; w < 8; ++w) t += red[w];
    inv[blockIdx.x] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, static_cast<float>(k)), eps)));
  }
}

// float offset of 16-byte chunk c of row r in a 128B-swizzled [rows][32] tile
__device__ __forceinline__ int swz(int r, int c) { return r * kBK + ((c ^ (r & 7)) << 2); }

__global__ void __launch_bounds__(kThr, kCtasPerSm)
lm_gemm_kernel(const __grid_constant__ CUtensorMap wmap, LmArgs a) {
  extern __shared__ __align__(128) float4 sm4[];
  float* sm = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(sm4) + 1023) & ~uintptr_t(1023));
  float* Ws = sm;                                   // [kNS][kBN][kBK], swizzled
  float* Xs = Ws + kNS * kBN * kBK;                 // [2][kBM][kBK], swizzled
  uint64_t* full = reinterpret_cast<uint64_t*>(Xs + 2 * kBM * kBK);
  __shared__ float best_v[kBM];
  __shared__ int32_t best_i[kBM];
  __shared__ float cand_v[2][kBM];
  __shared__ int32_t cand_i[2][kBM];
  __shared__ float inv_s[kBM];
  __shared__ bool is_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tn = (lane & 15) + 16 * (warp & 1);     // vocabulary rows tn + 32 i
  const int tm = (lane >> 4) + 2 * (warp >> 1);    // batch rows tm + 8 j
  const int ksteps = (a.k + kBK - 1) / kBK;
  const int my_tiles = a.ntiles > static_cast<int>(blockIdx.x)
                           ? (a.ntiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                           : 0;
  const int total = my_tiles * ksteps;              // (tile, step) pairs of this CTA, in order

  auto issue = [&](int q) {                         // weight tile of pair q into stage q % kNS
    const int t = static_cast<int>(blockIdx.x) + (q / ksteps) * static_cast<int>(gridDim.x);
    const int s = q % kNS;
    mbar_arrive_expect_tx(&full[s], kBN * kBK * 4);
    tma_load_2d(Ws + s * kBN * kBK, &wmap, &full[s], (q % ksteps) * kBK, t * kBN);
  };
  if (tid == 0) {
    for (int s = 0; s < kNS; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
    prefetch_tmap(&wmap);
    for (int q = 0; q < total && q < kNS; ++q) issue(q);   // weights: written before any launch
  }
  if (tid < kBM) {
    best_v[tid] = -FLT_MAX;
    best_i[tid] = INT32_MAX;
  }
  grid_dep_wait();
  grid_dep_launch();
  if (tid < kBM) inv_s[tid] = (a.norm_w && tid < a.m) ? a.inv_rms[tid] : 1.0f;
  __syncthreads();

  // x staging: thread -> rows xr, xr + 32, 16-byte chunk xc of the step
  const int xr = tid >> 3, xc = tid & 7;
  float4 xv[2];
  auto load_x = [&](int step) {
    const int k0 = step * kBK + xc * 4;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int r = xr + 32 * u;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < a.m && k0 < a.k) {
        v = *reinterpret_cast<const float4*>(a.x + static_cast<int64_t>(r) * a.k + k0);
        if (a.norm_w) {
          const float ir = inv_s[r];
          const float4 nw = *reinterpret_cast<const float4*>(a.norm_w + k0);
          v.x = __fmul_rn(nw.x, __fmul_rn(v.x, ir));
          v.y = __fmul_rn(nw.y, __fmul_rn(v.y, ir));
          v.z = __fmul_rn(nw.z, __fmul_rn(v.z, ir));
          v.w = __fmul_rn(nw.w, __fmul_rn(v.w, ir));
        }
      }
      xv[u] = v;
    }
  };
  auto store_x = [&](int buf) {
#pragma unroll
    for (int u = 0; u < 2; ++u)
      *reinterpret_cast<float4*>(Xs + buf * kBM * kBK + swz(xr + 32 * u, xc)) = xv[u];
  };

  bool aborted = false;
  int q = 0;
  for (int it = 0; it < my_tiles && !aborted; ++it) {
    const int tile = static_cast<int>(blockIdx.x) + it * static_cast<int>(gridDim.x);
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
    load_x(0);
    store_x(0);
    __syncthreads();
    for (int step = 0; step < ksteps; ++step, ++q) {
      const int s = q % kNS;
      if (step + 1 < ksteps) load_x(step + 1);
      const bool arrived = mbar_wait(&full[s], (q / kNS) & 1);
      if (arrived) {
        const float* W = Ws + s * kBN * kBK;
        const float* X = Xs + (step & 1) * kBM * kBK;
#pragma unroll
        for (int c = 0; c < kBK / 4; ++c) {
          float4 wv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) wv[i] = *reinterpret_cast<const float4*>(W + swz(tn + 32 * i, c));
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 xq = *reinterpret_cast<const float4*>(X + swz(tm + 8 * j, c));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              acc[i][j] = fmaf(wv[i].x, xq.x, acc[i][j]);
              acc[i][j] = fmaf(wv[i].y, xq.y, acc[i][j]);
              acc[i][j] = fmaf(wv[i].z, xq.z, acc[i][j]);
              acc[i][j] = fmaf(wv[i].w, xq.w, acc[i][j]);
            }
          }
        }
      }
      if (step + 1 < ksteps) store_x((step + 1) & 1);
      // stage s and x buffer step & 1 are free; a failed wait ends the CTA's work
      if (__syncthreads_or(!arrived)) {
        aborted = true;
        break;
      }
      if (tid == 0 && q + kNS < total) issue(q + kNS);
    }
    if (aborted) break;

    // ---- epilogue of the tile ----
    const int n0 = tile * kBN;
    if (a.logits) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = tm + 8 * j;
        if (r < a.m)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int n = n0 + tn + 32 * i;
            if (n < a.vocab) a.logits[static_cast<int64_t>(r) * a.vocab + n] = acc[i][j];
          }
      }
    }
    if (a.tokens) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float bv = -FLT_MAX;
        int32_t bi = INT32_MAX;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int n = n0 + tn + 32 * i;
          if (n < a.vocab && better(acc[i][j], n, bv, bi)) {
            bv = acc[i][j];
            bi = n;
          }
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) {          // the 16 lanes holding batch row tm + 8 j
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if ((lane & 15) == 0) {
          cand_v[warp & 1][tm + 8 * j] = bv;
          cand_i[warp & 1][tm + 8 * j] = bi;
        }
      }
      __syncthreads();
      if (tid < kBM) {
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (better(cand_v[h][tid], cand_i[h][tid], best_v[tid], best_i[tid])) {
            best_v[tid] = cand_v[h][tid];
            best_i[tid] = cand_i[h][tid];
          }
      }
      // the next tile's candidates are written after at least one more barrier
    }
  }
  if (aborted && tid == 0) atomicOr(a.error, 1u);
  if (!a.tokens) return;

  __syncthreads();
  if (tid < a.m) {
    a.part_val[static_cast<int64_t>(blockIdx.x) * a.m + tid] = best_v[tid];
    a.part_idx[static_cast<int64_t>(blockIdx.x) * a.m + tid] = best_i[tid];
    __threadfence();
  }
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const bool failed = __ldcg(a.error) != 0u;
  for (int r = warp; r < a.m; r += kThr / 32) {
    float bv = -FLT_MAX;
    int32_t bi = INT32_MAX;
    for (int c = lane; c < static_cast<int>(gridDim.x); c += 32) {
      const float v = __ldcg(a.part_val + static_cast<int64_t>(c) * a.m + r);
      const int32_t i = __ldcg(a.part_idx + static_cast<int64_t>(c) * a.m + r);
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
    if (lane == 0) a.tokens[r] = failed ? -1 : bi;
  }
  __syncthreads();
  if (tid == 0) {
    *a.counter = 0u;
    *a.error = 0u;
  }
}

constexpr size_t kSmem = (static_cast<size_t>(kNS) * kBN * kBK + 2 * kBM * kBK) * 4 + kNS * 8 + 1024;

}  // namespace

int64_t lm_gemm_grid(int64_t vocab) {
  const int64_t tiles = (vocab + kBN - 1) / kBN;
  return std::min<int64_t>(tiles, static_cast<int64_t>(num_sms()) * kCtasPerSm);
}

bool lm_gemm_ok(int64_t m, int64_t k, int64_t vocab, const float* x, const float* norm_w,
                const float* w) {
  return m > 0 && m <= kBM && k % 4 == 0 && vocab <= INT32_MAX - kBN && k <= INT32_MAX &&
         (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(norm_w) & 15) == 0;
}

// ws: [0, 4) counter, [4, 8) error word, [256, 512) 1/rms rows, then partials (grid x m values
// and indices).  Callers check lm_gemm_ok and the workspace size first.
int launch_lm_gemm(const float* x, int64_t m, int64_t k, const float* norm_w, float eps,
                   const float* w, int64_t vocab, float* logits, int64_t* tokens, char* ws,
                   cudaStream_t stream) {
  CUtensorMap map;
  if (!make_tensor_map_2d(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w, static_cast<uint64_t>(k),
                          static_cast<uint64_t>(vocab), static_cast<uint64_t>(k) * 4, kBK, kBN,
                          CU_TENSOR_MAP_SWIZZLE_128B))
    return KSH_ERR_UNSUPPORTED;
  float* inv = reinterpret_cast<float*>(ws + 256);
  // Completion counter and error word must start at zero whatever the
  // workspace held; the last CTA leaves both at zero for the next launch.
  const cudaError_t e = cudaMemsetAsync(ws, 0, 2 * sizeof(uint32_t), stream);
  if (e != cudaSuccess) return record_cuda_error(e);
  if (norm_w) {
    int st = launch(lm_inv_rms_kernel, dim3(static_cast<unsigned>(m)), dim3(256), 0, stream, x,
                    static_cast<int>(k), eps, inv);
    if (st != KSH_OK) return st;
  }
  if (set_smem_optin(reinterpret_cast<const void*>(lm_gemm_kernel), kSmem) != KSH_OK)
    return KSH_ERR_CUDA;
  const int64_t grid = lm_gemm_grid(vocab);
  LmArgs a = {};
  a.x = x;
  a.norm_w = norm_w;
  a.inv_rms = inv;
  a.logits = logits;
  a.tokens = tokens;
  a.counter = reinterpret_cast<uint32_t*>(ws);
  a.error = reinterpret_cast<uint32_t*>(ws + 4);
  a.part_val = reinterpret_cast<float*>(ws + 512);
  a.part_idx = reinterpret_cast<int32_t*>(ws + 512 + grid * m * 4);
  a.m = static_cast<int>(m);
  a.k = static_cast<int>(k);
  a.vocab = static_cast<int>(vocab);
  a.ntiles = static_cast<int>((vocab + kBN - 1) / kBN);
  return launch(lm_gemm_kernel, dim3(static_cast<unsigned>(grid)), dim3(kThr), kSmem, stream, map, a);
}

int64_t lm_gemm_workspace_size(int64_t m, int64_t vocab) {
  return 512 + lm_gemm_grid(vocab) * std::min<int64_t>(std::max<int64_t>(m, 1), kBM) * 8;
}

}  // namespace ksh
