// K5: prefill / batched quantized GEMM on the tcgen05 tensor cores.
//
// Replaces QuantizedLinear.forward (engine/quantization.py:394-396) for
// M > 16 rows.  y[m, n] = sum_k x[m, k] * q[n, k] * s[n(, g)] (+ bias,
// + residual, or SwiGLU over gate/up rows), x fp32.
//
// Precision scheme (the reference computes in fp32):
//   * x is split per row into two fp16 terms after an exact power-of-two row
//     scaling (x * 2^e = hi + lo, |x * 2^e| < 2^15), i.e. ~22 significant bits;
//   * the quantized weights are small integers, exact in fp16;
//   * D = hi * q^T + lo * q^T accumulates in fp32 in TMEM (two MMAs per K step);
//   * scales are applied in fp32 outside the MMA: per output channel at the
//     end (INT8), or per 128-wide K group by promoting each group's TMEM
//     partial into register accumulators (INT4); the row factor 2^-e last.
//
// CTA = one 128 x 128 output tile (SwiGLU: 64 gate + 64 up rows of W), K
// walked in 64-wide tiles through a 3-stage shared-memory ring:
//   warp 0  : TMA producer (x hi / lo tiles with 128B swizzle, raw weight tile)
//   warp 1  : TMEM allocation + single-thread tcgen05.mma issue
//   warps 2-5: dequantize the raw weight tile to fp16 in the UMMA K-major
//             128B-swizzled layout, then the epilogue (tcgen05.ld -> scales ->
//             bias / residual / SwiGLU -> global)
// For M >= kPreMinRows (a prefill chunk of many token tiles) the weight tile
// would be dequantized once per token tile; instead a pass before the GEMM
// widens the whole weight to fp16 q (exact, unscaled) in the workspace and the
// GEMM (PRE) loads fp16 tiles by TMA straight into the MMA's B operand: warps
// 2-5 only apply the scales (INT4 group promotion) and run the epilogue.
// Split-K over CTAs writes fp32 partial tiles to the workspace; the last CTA
// of a tile sums them in split order (deterministic) and runs the epilogue.
// Every mbarrier wait is bounded; a timeout raises KSH_FLAG_TIMEOUT in the
// status word and the CTA unwinds (TMEM is always released).

#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "linear.cuh"
#include "tc_common.cuh"

namespace ksh {
namespace {

using namespace tc;

constexpr int BM = 128, BN = 128, BK = 64;
constexpr int NS = 4;                      // TMA stages (x hi/lo + raw weights)
constexpr int NB = 2;                      // dequantized fp16 B tiles
constexpr int kThreads = 192;
constexpr int kMaxSplits = 8;
constexpr uint32_t kTmemCols = 2 * BN;
constexpr int A_BYTES = BM * BK * 2;       // one fp16 term
constexpr int BH_BYTES = BN * BK * 2;      // dequantized fp16 B tile
constexpr int BRAW_BYTES = BN * BK;        // int8 raw tile (int4 uses half)
constexpr int STAGE_BYTES = 2 * A_BYTES + BRAW_BYTES;
constexpr int RING_BYTES = NS * STAGE_BYTES + NB * BH_BYTES;
constexpr int OUT_LD = BN + 4;             // staging tile row stride (floats)
static_assert(BM * OUT_LD * 4 <= NS * STAGE_BYTES, "output staging reuses the TMA ring");
constexpr size_t SMEM_BYTES = 1024 + static_cast<size_t>(RING_BYTES) + 2 * BN * 4 + BN * 4 + 512;
// PRE: a stage holds x hi, x lo and the fp16 weight tile
constexpr int PRE_STAGE_BYTES = 2 * A_BYTES + BH_BYTES;
constexpr int PRE_RING_BYTES = NS * PRE_STAGE_BYTES;
static_assert(BM * OUT_LD * 4 <= PRE_RING_BYTES, "output staging reuses the PRE ring");
constexpr size_t PRE_SMEM_BYTES = 1024 + static_cast<size_t>(PRE_RING_BYTES) + 2 * BN * 4 + BN * 4 + 512;

struct TcArgs {
  const __half* scales;
  const float* bias;
  const float* residual;
  const float* inv_row;     // [M] 2^-e per x row
  float* y;
  float* part;              // split-K partial tiles
  uint32_t* counters;       // per output tile, zero on entry
  int32_t* flags;
  int m, n, inter, kt_total, kt_per_split, kt_per_group, ngroups_row, g;
};

// int8 byte pair -> fp16 bits, exact: 0x6400 | (b ^ 0x80) = 1024 + b + 128.
__device__ __forceinline__ uint32_t i8x2_to_h2(uint32_t w, int byte0) {
  const uint32_t x = w ^ 0x80808080u;
  const uint32_t sel = static_cast<uint32_t>(byte0) | (4u << 4) |
                       (static_cast<uint32_t>(byte0 + 1) << 8) | (5u << 12);
  const uint32_t h = __byte_perm(x, 0x64646464u, sel);
  __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h),
                      __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));
  return *reinterpret_cast<uint32_t*>(&r);
}
// two int4 nibbles (k, k+1) -> fp16 bits: 0x6400 | (u ^ 8) = 1024 + q + 8.
__device__ __forceinline__ uint32_t i4x2_to_h2(uint32_t w, int nib0) {
  const uint32_t lo = ((w >> (4 * nib0)) & 0xFu) ^ 0x8u;
  const uint32_t hi = ((w >> (4 * nib0 + 4)) & 0xFu) ^ 0x8u;
  const uint32_t h = (lo | 0x6400u) | ((hi | 0x6400u) << 16);
  __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h),
                      __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));
  return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int WK, int EPI, bool PRE>
__global__ void __launch_bounds__(kThreads, 1)
qgemm_tc_kernel(const __grid_constant__ CUtensorMap map_xh, const __grid_constant__ CUtensorMap map_xl,
                const __grid_constant__ CUtensorMap map_w, TcArgs a) {
  constexpr int SB = PRE ? PRE_STAGE_BYTES : STAGE_BYTES;
  constexpr int RB = PRE ? PRE_RING_BYTES : RING_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bh_base = smem + NS * SB;
  float* sc_s = reinterpret_cast<float*>(smem + RB);             // [2][BN] weight scales per group
  float* bias_s = sc_s + 2 * BN;                                  // [BN]
  uint64_t* bars = reinterpret_cast<uint64_t*>(bias_s + BN);
  uint64_t* full = bars;                       // [NS]  TMA landed
  uint64_t* empty = full + NS;                 // [NS]  MMA done with the stage
  uint64_t* bready = empty + NS;               // [NB]  fp16 B tile written
  uint64_t* bfree = bready + NB;               // [NB]  MMA done with the fp16 B tile
  uint64_t* acc_full = bfree + NB;             // [2]
  uint64_t* acc_empty = acc_full + 2;          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y, split = blockIdx.z;
  const int m0 = m_tile * BM;
  const int kt_begin = split * a.kt_per_split;
  const int kt_end = min(kt_begin + a.kt_per_split, a.kt_total);
  const int ntl = max(kt_end - kt_begin, 0);
  const int ktpg = WK == WK_I4 ? a.kt_per_group : max(ntl, 1);
  const int ngl = (ntl + ktpg - 1) / ktpg;

  auto stage_ah = [&](int s) { return smem + s * SB; };
  auto stage_al = [&](int s) { return smem + s * SB + A_BYTES; };
  auto stage_br = [&](int s) { return smem + s * SB + 2 * A_BYTES; };   // raw or (PRE) fp16 tile
  auto tile_bh = [&](int b) { return bh_base + b * BH_BYTES; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&bready[b], 128);
      mbar_init(&bfree[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_xh);
    prefetch_tmap(&map_xl);
    prefetch_tmap(&map_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Inputs (x split, weights) may be produced by the previous kernel.
  grid_dep_wait();

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t bytes = 2 * A_BYTES + (PRE ? BH_BYTES : (WK == WK_I8 ? BN * BK : BN * BK / 2));
      for (int i = 0; i < ntl && !*abort_flag; ++i) {
        const int s = i % NS;
        if (i >= NS && !mbar_wait(&empty[s], ((i / NS) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], bytes);
        const int kg = (kt_begin + i) * BK;
        tma_load_2d(stage_ah(s), &map_xh, &full[s], kg, m0);
        tma_load_2d(stage_al(s), &map_xl, &full[s], kg, m0);
        const int xw = (PRE || WK == WK_I8) ? kg : kg / 2;
        if (EPI == EPI_SWIGLU) {
          const int half_bytes = (PRE ? 2 * BK : (WK == WK_I8 ? BK : BK / 2)) * (BN / 2);
          tma_load_2d(stage_br(s), &map_w, &full[s], xw, n_tile * (BN / 2));
          tma_load_2d(stage_br(s) + half_bytes, &map_w, &full[s], xw, a.inter + n_tile * (BN / 2));
        } else {
          tma_load_2d(stage_br(s), &map_w, &full[s], xw, n_tile * BN);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(BM, BN);
      for (int i = 0; i < ntl && !*abort_flag; ++i) {
        const int s = i % NS, b = i % NB;
        const int gl = i / ktpg, buf = gl & 1;
        const bool first = (i % ktpg) == 0;
        if (first && gl >= 2 && !mbar_wait(&acc_empty[buf], ((gl >> 1) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        // PRE: the fp16 tile came with the stage; else the converters' barrier
        // implies full[s] completed
        if (!mbar_wait(PRE ? &full[s] : &bready[b], PRE ? (i / NS) & 1 : (i / NB) & 1)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t ah = smem_u32(stage_ah(s)), al = smem_u32(stage_al(s)),
                       bh = smem_u32(PRE ? stage_br(s) : tile_bh(b));
        const uint32_t d = tmem + buf * BN;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t bd = desc_k_sw128(bh + kk * 32);
          mma_f16(d, desc_k_sw128(ah + kk * 32), bd, idesc, (first && kk == 0) ? 0u : 1u);
          mma_f16(d, desc_k_sw128(al + kk * 32), bd, idesc, 1u);
        }
        mma_commit(&empty[s]);
        if (!PRE) mma_commit(&bfree[b]);
        if ((i % ktpg) == ktpg - 1 || i == ntl - 1) mma_commit(&acc_full[buf]);
      }
    }
  } else {
    // ---------------- converter + epilogue warps (128 threads) ----------------
    const int t = threadIdx.x - 64;          // B tile row this thread converts
    const int q = warp & 3;                  // TMEM lane quadrant of this warp
    const int row_local = q * 32 + lane;     // accumulator row (TMEM lane)
    // weight row feeding accumulator column / B row t
    const int wrow_t = [&]() -> int {
      if (EPI == EPI_SWIGLU) {
        const int c = n_tile * (BN / 2) + (t & (BN / 2 - 1));
        if (c >= a.inter) return -1;
        return t < BN / 2 ? c : a.inter + c;
      }
      const int r = n_tile * BN + t;
      return r < a.n ? r : -1;
    }();
    if (EPI == EPI_STORE) bias_s[t] = (a.bias && wrow_t >= 0) ? a.bias[wrow_t] : 0.0f;
    float acc[BN];
#pragma unroll
    for (int j = 0; j < BN; ++j) acc[j] = 0.0f;

    auto promote = [&](int gl) -> bool {
      const int buf = gl & 1;
      epi_bar();                              // every thread's scale for group gl is visible
      if (!mbar_wait(&acc_full[buf], (gl >> 1) & 1)) return false;
      tc_fence_after();
      const float* sc = sc_s + buf * BN;
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld_32x32b_x32(tmem + buf * BN + c * 32 + (static_cast<uint32_t>(q * 32) << 16), v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[c * 32 + j] = fmaf(v[j], sc[c * 32 + j], acc[c * 32 + j]);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      epi_bar();                              // scale slot `buf` may be rewritten after this
      return true;
    };

    auto group_scale = [&](int gl) {       // scale of row t for group gl, into slot gl & 1
      float scv = 0.0f;
      if (wrow_t >= 0) {
        if (WK == WK_I8) scv = __half2float(a.scales[wrow_t]);
        else scv = __half2float(a.scales[static_cast<int64_t>(wrow_t) * a.ngroups_row +
                                         (kt_begin + gl * ktpg) / ktpg]);
      }
      sc_s[(gl & 1) * BN + t] = scv;
    };
    bool ok = true;
    if (PRE) {
      // the weight tiles need no conversion: scales and promotion only
      for (int gl = 0; gl < ngl && ok; ++gl) {
        if (*abort_flag) {
          ok = false;
          break;
        }
        group_scale(gl);
        if (gl >= 1 && !promote(gl - 1)) ok = false;
      }
    }
    for (int i = 0; i < (PRE ? 0 : ntl) && ok; ++i) {
      const int s = i % NS, b = i % NB;
      const int gl = i / ktpg;
      if (*abort_flag || !mbar_wait(&full[s], (i / NS) & 1)) {
        ok = false;
        break;
      }
      if (i >= NB && !mbar_wait(&bfree[b], ((i / NB) - 1) & 1)) {
        ok = false;
        break;
      }
      if ((i % ktpg) == 0) group_scale(gl);
      // dequantize row t of the raw tile (TMA-swizzled) into the 128B-swizzled fp16 tile
      uint8_t* dst_row = tile_bh(b) + (t >> 3) * 1024 + (t & 7) * 128;
      const uint32_t rsw = static_cast<uint32_t>(t & 7);
      if (WK == WK_I8) {
        // raw rows are 64 B, TMA 64B swizzle: chunk c at c ^ ((t >> 1) & 3)
        const uint8_t* src = stage_br(s) + t * BK;
        const uint32_t rs = static_cast<uint32_t>((t >> 1) & 3);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 w = *reinterpret_cast<const uint4*>(src + ((static_cast<uint32_t>(j) ^ rs) << 4));
          uint4 o0, o1;
          o0.x = i8x2_to_h2(w.x, 0); o0.y = i8x2_to_h2(w.x, 2);
          o0.z = i8x2_to_h2(w.y, 0); o0.w = i8x2_to_h2(w.y, 2);
          o1.x = i8x2_to_h2(w.z, 0); o1.y = i8x2_to_h2(w.z, 2);
          o1.z = i8x2_to_h2(w.w, 0); o1.w = i8x2_to_h2(w.w, 2);
          *reinterpret_cast<uint4*>(dst_row + (((2 * j) ^ rsw) << 4)) = o0;
          *reinterpret_cast<uint4*>(dst_row + (((2 * j + 1) ^ rsw) << 4)) = o1;
        }
      } else {
        // raw rows are 32 B, TMA 32B swizzle: chunk c at c ^ ((t >> 2) & 1)
        const uint8_t* src = stage_br(s) + t * (BK / 2);
        const uint32_t rs = static_cast<uint32_t>((t >> 2) & 1);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const uint4 w = *reinterpret_cast<const uint4*>(src + ((static_cast<uint32_t>(j) ^ rs) << 4));
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {      // 8 nibbles -> one 16-byte chunk
            uint4 o;
            o.x = i4x2_to_h2(ws[e], 0);
            o.y = i4x2_to_h2(ws[e], 2);
            o.z = i4x2_to_h2(ws[e], 4);
            o.w = i4x2_to_h2(ws[e], 6);
            *reinterpret_cast<uint4*>(dst_row + ((static_cast<uint32_t>(4 * j + e) ^ rsw) << 4)) = o;
          }
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&bready[b]);
      if (WK == WK_I4 && (i % ktpg) == ktpg - 1 && gl >= 1 && !promote(gl - 1)) ok = false;
    }
    if (ok && ntl > 0 && !*abort_flag) ok = promote(ngl - 1);
    if (!ok) {
      *abort_flag = 1;
      raise_flag(a.flags, KSH_FLAG_TIMEOUT);
    }

    // ---------------- output: stage the tile in shared memory ----------------
    // The TMA ring is idle now (every stage was consumed by the MMA).
    float* stile = reinterpret_cast<float*>(smem);            // [BM][OUT_LD]
    float* rowp = stile + row_local * OUT_LD;
#pragma unroll
    for (int j = 0; j < BN; j += 4)
      *reinterpret_cast<float4*>(rowp + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
  }

  // ---------------- split-K reduction through distributed shared memory ----------------
  // The splits of one output tile form a thread-block cluster along z; rank r
  // sums rows [r * BM / splits, (r + 1) * BM / splits) of every rank's staged
  // tile in rank order (deterministic) and writes those rows.
  __syncthreads();
  const int splits = static_cast<int>(gridDim.z);
  if (splits > 1) cluster_sync();
  if (warp >= 2) {
    const int t = threadIdx.x - 64;
    float* stile = reinterpret_cast<float*>(smem);
    const int rows_per = (BM + splits - 1) / splits;
    const int r_lo = split * rows_per, r_hi = min(BM, r_lo + rows_per);
    const uint32_t sbase = smem_u32(stile);
    auto row_sum = [&](int r, int c4) -> float4 {
      if (splits == 1) return reinterpret_cast<const float4*>(stile + r * OUT_LD)[c4];
      const uint32_t off = static_cast<uint32_t>((r * OUT_LD + 4 * c4) * 4);
      float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
      float4 v[kMaxSplits];
#pragma unroll
      for (int sp = 0; sp < kMaxSplits; ++sp)
        if (sp < splits) v[sp] = ld_cluster_f32x4(map_rank(sbase + off, static_cast<uint32_t>(sp)));
#pragma unroll
      for (int sp = 0; sp < kMaxSplits; ++sp)
        if (sp < splits) {
          s4.x += v[sp].x; s4.y += v[sp].y; s4.z += v[sp].z; s4.w += v[sp].w;
        }
      return s4;
    };
    if (EPI == EPI_SWIGLU) {
      // columns [0, 64) gate, [64, 128) up; 16 float4 outputs per row
      const int oc4 = t & 15, orr = t >> 4;                 // rows r_lo + orr + 8i
      const int c = n_tile * (BN / 2) + 4 * oc4;
      for (int r = r_lo + orr; r < r_hi; r += 8) {
        const int m = m0 + r;
        if (m >= a.m) continue;
        const float inv = a.inv_row[m];
        const float4 gv = row_sum(r, oc4);
        const float4 uv = row_sum(r, oc4 + BN / 8);
        float o[4] = {silu_f(gv.x * inv) * (uv.x * inv), silu_f(gv.y * inv) * (uv.y * inv),
                      silu_f(gv.z * inv) * (uv.z * inv), silu_f(gv.w * inv) * (uv.w * inv)};
        float* yr = a.y + static_cast<int64_t>(m) * a.inter;
        if (c + 3 < a.inter && (a.inter & 3) == 0) {
          *reinterpret_cast<float4*>(yr + c) = make_float4(o[0], o[1], o[2], o[3]);
        } else {
          for (int e = 0; e < 4; ++e)
            if (c + e < a.inter) yr[c + e] = o[e];
        }
      }
    } else {
      const int c4 = t & 31, rr0 = t >> 5;                  // float4 column, rows r_lo + rr0 + 4i
      const int c = n_tile * BN + 4 * c4;
      const bool vec = (a.n & 3) == 0 && c + 3 < a.n;
      for (int r = r_lo + rr0; r < r_hi; r += 4) {
        const int m = m0 + r;
        if (m >= a.m) continue;
        const float inv = a.inv_row[m];
        const float4 v = row_sum(r, c4);
        float o[4] = {v.x * inv + bias_s[4 * c4], v.y * inv + bias_s[4 * c4 + 1],
                      v.z * inv + bias_s[4 * c4 + 2], v.w * inv + bias_s[4 * c4 + 3]};
        float* yr = a.y + static_cast<int64_t>(m) * a.n;
        const float* rres = a.residual ? a.residual + static_cast<int64_t>(m) * a.n : nullptr;
        if (vec) {
          if (rres) {
            const float4 rv = *reinterpret_cast<const float4*>(rres + c);
            o[0] = rv.x + o[0]; o[1] = rv.y + o[1]; o[2] = rv.z + o[2]; o[3] = rv.w + o[3];
          }
          *reinterpret_cast<float4*>(yr + c) = make_float4(o[0], o[1], o[2], o[3]);
        } else {
          for (int e = 0; e < 4; ++e)
            if (c + e < a.n) yr[c + e] = rres ? rres[c + e] + o[e] : o[e];
        }
      }
    }
  }
  if (splits > 1) cluster_sync();     // every rank's tile stays alive until all have read it

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  grid_dep_launch();
}

// x fp32 [m, k] -> hi, lo fp16 [m, k] with a per-row power-of-two scale so
// that max |x| * 2^e lies in [2^14, 2^15); inv_row[m] = 2^-e.  With norm_w
// set, x is first RMSNorm-ed (LlamaRMSNorm arithmetic, fixed-order reduction).
__device__ __forceinline__ float norm_val(const float* xr, const float* norm_w, float inv,
                                          int64_t j) {
  const float v = xr[j];
  return norm_w ? __fmul_rn(norm_w[j], __fmul_rn(v, inv)) : v;
}

// PERM stores each aligned 8-element chunk in the order [0,2,4,6,1,3,5,7] (the
// order in which the INT4 decode kernels unpack nibbles).
template <bool PERM>
__global__ void __launch_bounds__(256)
split_x_kernel(const float* __restrict__ x, int64_t k, __half* __restrict__ xh,
               __half* __restrict__ xl, float* __restrict__ inv_row,
               const float* __restrict__ norm_w, float eps) {
  __shared__ float red[2][8];
  grid_dep_wait();
  grid_dep_launch();
  const int64_t r = blockIdx.x;
  const float* xr = x + r * k;
  // One pass for both reductions: the sum of squares (RMSNorm) and the row
  // maximum of |norm_w * x|, scaled by 1/rms afterwards.  That maximum can
  // differ from the maximum of the normalised values by an ulp or two, which
  // at most shifts the power-of-two exponent by one: the largest scaled value
  // stays below 2^15 (1 + 2^-22), well inside fp16.
  float ss = 0.0f, mx = 0.0f;
  for (int64_t j = threadIdx.x; j < k; j += blockDim.x) {
    const float v = xr[j];
    ss = fmaf(v, v, ss);
    mx = fmaxf(mx, fabsf(norm_w ? norm_w[j] * v : v));
  }
  ss = warp_sum(ss);
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = ss;
    red[1][threadIdx.x >> 5] = mx;
  }
  __syncthreads();
  ss = 0.0f;
  mx = 0.0f;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {     // fixed order
    ss += red[0][w];
    mx = fmaxf(mx, red[1][w]);
  }
  float inv = 1.0f;
  if (norm_w) {
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(k)), eps)));
    mx *= inv;
  }
  int e = 0;
  if (mx > 0.0f && isfinite(mx)) {
    int ex;
    frexpf(mx, &ex);                 // mx = f * 2^ex, f in [0.5, 1)
    e = 15 - ex;                     // mx * 2^e in [2^14, 2^15)
    e = max(-100, min(e, 100));
  }
  const float sc = ldexpf(1.0f, e);
  if (threadIdx.x == 0) inv_row[r] = ldexpf(1.0f, -e);
  for (int64_t j = threadIdx.x; j < k; j += blockDim.x) {
    const float v = norm_val(xr, norm_w, inv, j) * sc;
    const __half h = __float2half_rn(v);
    // element e of a chunk goes to position (e & 1) * 4 + (e >> 1)
    const int64_t pos = PERM && (j | 7) < k ? (j & ~int64_t{7}) + ((j & 1) << 2) + ((j & 7) >> 1) : j;
    xh[r * k + pos] = h;
    xl[r * k + pos] = __float2half_rn(v - __half2float(h));
  }
}

// The same split, vectorised for k % 8 == 0 and k <= 8 * kSxChunks * kSxThreads:
// each thread loads its 8-element chunks once (two float4 each) and keeps them
// in registers for both passes; 16 warps per row; hi and lo leave as one
// 16-byte store per chunk.  Results equal split_x_kernel's up to the order of
// the row reductions (fixed here too).
constexpr int kSxThreads = 512;
constexpr int kSxChunks = 4;

template <bool PERM>
__global__ void __launch_bounds__(kSxThreads)
split_x_vec_kernel(const float* __restrict__ x, int64_t k, __half* __restrict__ xh,
                   __half* __restrict__ xl, float* __restrict__ inv_row,
                   const float* __restrict__ norm_w, float eps) {
  __shared__ float red[2][kSxThreads / 32];
  grid_dep_wait();
  grid_dep_launch();
  const int64_t r = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + r * k);
  const float4* nw4 = reinterpret_cast<const float4*>(norm_w);
  const int nchunk = static_cast<int>(k / 8);
  float v[kSxChunks][8];
  float ss = 0.0f, mx = 0.0f;
#pragma unroll
  for (int j = 0; j < kSxChunks; ++j) {
    const int c = threadIdx.x + j * kSxThreads;
    if (c < nchunk) {
      const float4 a0 = xr[2 * c], a1 = xr[2 * c + 1];
      v[j][0] = a0.x; v[j][1] = a0.y; v[j][2] = a0.z; v[j][3] = a0.w;
      v[j][4] = a1.x; v[j][5] = a1.y; v[j][6] = a1.z; v[j][7] = a1.w;
      float w8[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
      if (norm_w) {
        const float4 b0 = nw4[2 * c], b1 = nw4[2 * c + 1];
        w8[0] = b0.x; w8[1] = b0.y; w8[2] = b0.z; w8[3] = b0.w;
        w8[4] = b1.x; w8[5] = b1.y; w8[6] = b1.z; w8[7] = b1.w;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        ss = fmaf(v[j][e], v[j][e], ss);
        mx = fmaxf(mx, fabsf(norm_w ? w8[e] * v[j][e] : v[j][e]));
      }
    }
  }
  ss = warp_sum(ss);
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = ss;
    red[1][threadIdx.x >> 5] = mx;
  }
  __syncthreads();
  ss = 0.0f;
  mx = 0.0f;
#pragma unroll
  for (int w = 0; w < kSxThreads / 32; ++w) {     // fixed order
    ss += red[0][w];
    mx = fmaxf(mx, red[1][w]);
  }
  float inv = 1.0f;
  if (norm_w) {
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(k)), eps)));
    mx *= inv;
  }
  int e = 0;
  if (mx > 0.0f && isfinite(mx)) {
    int ex;
    frexpf(mx, &ex);
    e = max(-100, min(15 - ex, 100));
  }
  const float sc = ldexpf(1.0f, e);
  if (threadIdx.x == 0) inv_row[r] = ldexpf(1.0f, -e);
#pragma unroll
  for (int j = 0; j < kSxChunks; ++j) {
    const int c = threadIdx.x + j * kSxThreads;
    if (c < nchunk) {
      float w8[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
      if (norm_w) {
        const float4 b0 = nw4[2 * c], b1 = nw4[2 * c + 1];
        w8[0] = b0.x; w8[1] = b0.y; w8[2] = b0.z; w8[3] = b0.w;
        w8[4] = b1.x; w8[5] = b1.y; w8[6] = b1.z; w8[7] = b1.w;
      }
      __align__(16) __half hv[8], lv[8];
#pragma unroll
      for (int el = 0; el < 8; ++el) {
        const float nv = norm_w ? __fmul_rn(w8[el], __fmul_rn(v[j][el], inv)) : v[j][el];
        const float t = nv * sc;
        const __half h = __float2half_rn(t);
        // PERM: element el of the chunk goes to position (el & 1) * 4 + (el >> 1)
        const int pos = PERM ? ((el & 1) << 2) + (el >> 1) : el;
        hv[pos] = h;
        lv[pos] = __float2half_rn(t - __half2float(h));
      }
      *reinterpret_cast<uint4*>(xh + r * k + 8 * c) = *reinterpret_cast<const uint4*>(hv);
      *reinterpret_cast<uint4*>(xl + r * k + 8 * c) = *reinterpret_cast<const uint4*>(lv);
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

int launch_split(const float* x, int64_t m, int64_t k, __half* xh, __half* xl, float* inv,
                 const float* norm_w, float eps, bool perm, cudaStream_t stream) {
  const bool vec = k % 8 == 0 && k <= 8LL * kSxChunks * kSxThreads &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(norm_w) |
                     reinterpret_cast<uintptr_t>(xh) | reinterpret_cast<uintptr_t>(xl)) & 15) == 0;
  if (vec) {
    auto kern = perm ? split_x_vec_kernel<true> : split_x_vec_kernel<false>;
    return launch(kern, dim3(static_cast<unsigned>(m)), dim3(kSxThreads), 0, stream, x, k, xh,
                  xl, inv, norm_w, eps);
  }
  auto kern = perm ? split_x_kernel<true> : split_x_kernel<false>;
  return launch(kern, dim3(static_cast<unsigned>(m)), dim3(256), 0, stream, x, k, xh, xl, inv,
                norm_w, eps);
}


int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }

int max_splits(int64_t m, int64_t n) {
  const int64_t tiles = ((n + BN - 1) / BN) * ((m + BM - 1) / BM);
  const int64_t want = (num_sms() + tiles - 1) / tiles;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, kMaxSplits)));
}

// Rows of x from which the prefill GEMM widens the weight once per call
// (KSH_GEMM_PREDEQ_MIN in the environment sets it; 0 turns it off).
int64_t g_pre_min = [] {
  const char* v = getenv("KSH_GEMM_PREDEQ_MIN");
  return (v && *v) ? static_cast<int64_t>(atoll(v)) : static_cast<int64_t>(512);
}();

bool use_pre(int64_t m) { return g_pre_min > 0 && m >= g_pre_min; }

struct WsLayout {
  int64_t xh, xl, inv, wq, total;
};

// Workspace: the fp16 hi / lo split of x and the per-row factors, and for
// the PRE path the fp16 copy of the weight (rows x K rounded up to a group of
// 128).  (Split-K partial sums never leave the SMs: they are reduced over the
// cluster.)
WsLayout ws_layout(int64_t m, int64_t k, int64_t n_rows) {
  WsLayout w = {};
  w.xh = 0;
  w.xl = w.xh + align256(m * k * 2);
  w.inv = w.xl + align256(m * k * 2);
  w.wq = w.inv + align256(m * 4);
  w.total = w.wq + (use_pre(m) && n_rows > 0 ? align256(n_rows * ((k + 127) / 128 * 128) * 2) : 0);
  return w;
}

// Packed weight -> fp16 q (exact, unscaled), row-major [rows, keff]; one
// 16-byte payload chunk per thread (INT8: 16 values, INT4: 32, low nibble =
// even k).
template <int WK>
__global__ void __launch_bounds__(256)
dequant_w_kernel(const uint8_t* __restrict__ w, int64_t rows, int64_t row_bytes, int64_t keff,
                 __half* __restrict__ out) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t chunks_row = row_bytes / 16;
  const int64_t total = rows * chunks_row;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = c / chunks_row, j = c - r * chunks_row;
    const uint4 v = *reinterpret_cast<const uint4*>(w + r * row_bytes + j * 16);
    const uint32_t ws[4] = {v.x, v.y, v.z, v.w};
    __half* dst = out + r * keff + j * (WK == WK_I8 ? 16 : 32);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      uint4 o;
      if (WK == WK_I8) {
        o.x = i8x2_to_h2(ws[e], 0);
        o.y = i8x2_to_h2(ws[e], 2);
        reinterpret_cast<uint2*>(dst)[e] = make_uint2(o.x, o.y);
      } else {
        o.x = i4x2_to_h2(ws[e], 0);
        o.y = i4x2_to_h2(ws[e], 2);
        o.z = i4x2_to_h2(ws[e], 4);
        o.w = i4x2_to_h2(ws[e], 6);
        reinterpret_cast<uint4*>(dst)[e] = o;
      }
    }
  }
}

struct TcPlan {
  int tiles_n, tiles_m, kt_total, kt_per_group, splits, kt_per_split;
};

TcPlan plan(int wk, int64_t m, int64_t keff, int64_t n_rows, int64_t g) {
  TcPlan p = {};
  p.tiles_n = static_cast<int>((n_rows + BN - 1) / BN);
  p.tiles_m = static_cast<int>((m + BM - 1) / BM);
  p.kt_total = static_cast<int>((keff + BK - 1) / BK);
  p.kt_per_group = wk == WK_I4 ? static_cast<int>(g / BK) : 1;
  int splits = max_splits(m, n_rows);
  // at least 4 K tiles per split, split boundaries on group boundaries
  splits = std::min(splits, std::max(1, p.kt_total / 4));
  int kps = (p.kt_total + splits - 1) / splits;
  kps = (kps + p.kt_per_group - 1) / p.kt_per_group * p.kt_per_group;
  p.kt_per_split = kps;
  p.splits = (p.kt_total + kps - 1) / kps;
  return p;
}

template <int WK, int EPI>
int launch_tc(const LinArgs& a, char* ws, cudaStream_t stream) {
  const int64_t keff = WK == WK_I4 ? a.kp : a.k;
  const int64_t n_rows = a.n;   // SwiGLU: 2 * inter rows
  const TcPlan p = plan(WK, a.m, keff, n_rows, a.g);
  const WsLayout L = ws_layout(a.m, a.k, n_rows);
  __half* xh = reinterpret_cast<__half*>(ws + L.xh);
  __half* xl = reinterpret_cast<__half*>(ws + L.xl);
  float* inv = reinterpret_cast<float*>(ws + L.inv);
  int st = launch_split(a.x, a.m, a.k, xh, xl, inv, a.norm_w, a.norm_eps, false, stream);
  if (st != KSH_OK) return st;
  CUtensorMap mxh, mxl, mw;
  if (!make_tensor_map_2d(&mxh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh, a.k, a.m, a.k * 2, BK, BM,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tensor_map_2d(&mxl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xl, a.k, a.m, a.k * 2, BK, BM,
                CU_TENSOR_MAP_SWIZZLE_128B))
    return KSH_ERR_CUDA;
  const uint32_t box_rows = EPI == EPI_SWIGLU ? BN / 2 : BN;
  // the workspace's fp16 weight region holds rows x (K rounded up to 128)
  const bool pre = use_pre(a.m) && keff <= (a.k + 127) / 128 * 128;
  bool ok;
  if (pre) {
    // widen the whole weight once to fp16 q; the GEMM loads 128-byte rows of
    // it (128B swizzle, the MMA's K-major operand layout) straight by TMA
    __half* wq = reinterpret_cast<__half*>(ws + L.wq);
    const int64_t row_bytes = WK == WK_I8 ? a.k : a.kp / 2;
    const int64_t chunks = n_rows * (row_bytes / 16);
    const int64_t blocks = std::min<int64_t>((chunks + 255) / 256, static_cast<int64_t>(num_sms()) * 8);
    st = launch(WK == WK_I8 ? dequant_w_kernel<WK_I8> : dequant_w_kernel<WK_I4>,
                dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream,
                static_cast<const uint8_t*>(a.w), n_rows, row_bytes, keff, wq);
    if (st != KSH_OK) return st;
    ok = make_tensor_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, wq, keff, n_rows, keff * 2, BK,
                            box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    // raw weight tiles: 64-byte (int8) / 32-byte (int4) rows, TMA-swizzled so
    // the dequantizing threads read them without bank conflicts
    ok = WK == WK_I8
             ? make_tensor_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, a.k, n_rows, a.k, BK,
                                  box_rows, CU_TENSOR_MAP_SWIZZLE_64B)
             : make_tensor_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, a.kp / 2, n_rows,
                                  a.kp / 2, BK / 2, box_rows, CU_TENSOR_MAP_SWIZZLE_32B);
  }
  if (!ok) return KSH_ERR_CUDA;
  TcArgs t = {};
  t.scales = a.scales;
  t.bias = a.bias;
  t.residual = a.residual;
  t.inv_row = inv;
  t.y = a.y;
  t.flags = nullptr;
  t.m = static_cast<int>(a.m);
  t.n = static_cast<int>(a.n);
  t.inter = static_cast<int>(a.inter);
  t.kt_total = p.kt_total;
  t.kt_per_split = p.kt_per_split;
  t.kt_per_group = p.kt_per_group;
  t.ngroups_row = WK == WK_I4 ? static_cast<int>(a.kp / a.g) : 1;
  t.g = static_cast<int>(a.g);
  auto kern = pre ? qgemm_tc_kernel<WK, EPI, true> : qgemm_tc_kernel<WK, EPI, false>;
  const size_t smem_bytes = pre ? PRE_SMEM_BYTES : SMEM_BYTES;
  if (set_smem_optin(reinterpret_cast<const void*>(kern), smem_bytes) != KSH_OK) return KSH_ERR_CUDA;
  const unsigned gx = EPI == EPI_SWIGLU ? static_cast<unsigned>((a.inter + BN / 2 - 1) / (BN / 2))
                                        : static_cast<unsigned>(p.tiles_n);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gx, static_cast<unsigned>(p.tiles_m), static_cast<unsigned>(p.splits));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;      // the splits of a tile = one cluster
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = static_cast<unsigned>(p.splits);
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mxh, mxl, mw, t);
  if (e == cudaSuccess) count_launch();
  return e == cudaSuccess ? KSH_OK : record_cuda_error(e);
}

}  // namespace

int launch_split_x(const LinArgs& a, char* ws, bool perm, __half** xh, __half** xl, float** inv,
                   cudaStream_t stream) {
  const WsLayout L = ws_layout(a.m, a.k, a.n);
  *xh = reinterpret_cast<__half*>(ws + L.xh);
  *xl = reinterpret_cast<__half*>(ws + L.xl);
  *inv = reinterpret_cast<float*>(ws + L.inv);
  return launch_split(a.x, a.m, a.k, *xh, *xl, *inv, a.norm_w, a.norm_eps, perm, stream);
}

int64_t split_x_workspace_size(int64_t m, int64_t k) { return ws_layout(m, k, 0).total; }

int64_t set_gemm_predeq_min(int64_t rows) {
  const int64_t prev = g_pre_min;
  g_pre_min = rows > 0 ? rows : 0;
  return prev;
}

int64_t gemm_tc_workspace_size(int64_t m, int64_t k, int64_t n) {
  if (m <= 16) return 0;
  return ws_layout(m, k, n).total;
}

int launch_gemm_tc(int wk, int epi, const LinArgs& a, void* ws, int64_t ws_bytes,
                   cudaStream_t stream, bool* taken) {
  *taken = false;
  if (wk != WK_I8 && wk != WK_I4) return KSH_OK;
  if (a.m > 65535 * BM || a.n > INT32_MAX) return KSH_OK;
  if ((reinterpret_cast<uintptr_t>(a.w) & 15) != 0) return KSH_OK;
  if (wk == WK_I8 && a.k % 16 != 0) return KSH_OK;
  if (wk == WK_I4 && (a.g % BK != 0 || (a.kp / 2) % 16 != 0)) return KSH_OK;
  if (a.k % 8 != 0) return KSH_OK;
  if (!tensor_map_encoder_available()) return KSH_OK;
  const WsLayout L = ws_layout(a.m, a.k, a.n);
  if (!ws || ws_bytes < L.total || (reinterpret_cast<uintptr_t>(ws) & 255) != 0) return KSH_OK;
  *taken = true;
  char* w = static_cast<char*>(ws);
  if (wk == WK_I8) return epi == EPI_SWIGLU ? launch_tc<WK_I8, EPI_SWIGLU>(a, w, stream)
                                            : launch_tc<WK_I8, EPI_STORE>(a, w, stream);
  return epi == EPI_SWIGLU ? launch_tc<WK_I4, EPI_SWIGLU>(a, w, stream)
                           : launch_tc<WK_I4, EPI_STORE>(a, w, stream);
}

}  // namespace ksh
