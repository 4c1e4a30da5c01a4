// K6: decode-time quantized linear layers on the tcgen05 tensor cores (M <= 16).
//
// Replaces QuantizedLinear.forward (engine/quantization.py:394-396) for the
// decode regime of a few token rows against a large weight matrix.  On CUDA
// cores that product is issue-bound, not memory-bound: every weight element
// costs a dequantize plus one FMA per token row.  Here the tensor cores do
// the multiply-adds and the CUDA cores only convert weights, about one
// instruction per element, so the kernel can run at HBM speed:
//
// * swap-AB: the MMA's M side (128 TMEM lanes) is 128 weight rows, its N side
//   the token rows: N = 16 (up to 8 tokens) or 32 (up to 16), column m holding
//   the high fp16 half of token m and column MP + m the low half;
// * x is split in-kernel: per CTA K-slice, a power-of-two scale per token row
//   (max |x * 2^e| in [2^14, 2^15)), x * 2^e = hi + lo in fp16 (~22 bits); the
//   quantized weights are exact in fp16 and the accumulation is fp32 (TMEM);
// * a fused RMSNorm multiplies x by the norm weight while splitting and
//   applies 1/rms to the result; each CTA adds up sum(x^2) over its K-slice
//   and the slices are summed in rank order, so results are deterministic;
// * raw int8 / int4 weight tiles arrive by TMA (64 / 32-byte swizzle, no bank
//   conflicts for the converters) through a ring whose first stages are
//   issued before the programmatic-launch wait (weights are constant);
// * INT8 scales are applied per row (= TMEM lane) at the end; INT4 group
//   scales by promoting each 128-wide group's TMEM partial into registers
//   (double-buffered accumulator, so the MMAs of group g+1 overlap);
// * split-K over a thread-block cluster, reduced through distributed shared
//   memory in rank order; the epilogue adds bias / residual or applies SwiGLU
//   (tile = 64 gate rows + the 64 matching up rows).
//
// INT4 detail: the MMA sums over k, so any permutation of k applied to both
// operands leaves the result unchanged.  Each 8-element chunk is stored in the
// order [0,2,4,6,1,3,5,7], which turns the nibble unpacking into one byte
// permute per two elements.
//
// Every mbarrier wait is bounded; a timeout raises KSH_FLAG_TIMEOUT (when a
// status word is given) and the CTA unwinds through the same barriers, always
// releasing its TMEM.

#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "linear.cuh"
#include "tc_common.cuh"

namespace ksh {
namespace {

using namespace tc;

constexpr int BW = 128;            // weight rows per tile (MMA M)
constexpr int BK = 64;             // K per stage
constexpr int NA = 2;              // fp16 operand slots (A + B)
constexpr int kThreads = 192;
constexpr int kMaxSplits = 8;
constexpr int A_BYTES = BW * BK * 2;

template <int WK>
constexpr int raw_bytes() { return WK == WK_I8 ? BW * BK : BW * BK / 2; }
template <int WK>
constexpr int n_stages() { return WK == WK_I8 ? 4 : 8; }

struct GvArgs {
  const float* x;
  const float* norm_w;
  const __half* scales;
  const float* bias;
  const float* residual;
  float* y;
  int32_t* flags;
  float eps;
  int m, k, n, inter;
  int kt_total, kt_per_split, kt_per_group, ngroups_row;
};

template <int WK, int MP>
struct Layout {
  static constexpr int NCOL = 2 * MP;
  static constexpr int NS = n_stages<WK>();
  static constexpr int RAW = raw_bytes<WK>();
  static constexpr int B_BYTES = NCOL * 128;
  static constexpr int RAW_OFF = 0;
  static constexpr int A_OFF = RAW_OFF + NS * RAW;
  static constexpr int B_OFF = A_OFF + NA * A_BYTES;
  static constexpr int TILE_OFF = B_OFF + NA * B_BYTES;         // [BW][MP] partial outputs
  static constexpr int SMALL_OFF = TILE_OFF + BW * MP * 4;
  // small region: escale[MP], einv[MP], ss_part[MP], inv_s[MP], red_mx[4][MP], red_ss[4][MP]
  static constexpr int BAR_OFF = SMALL_OFF + (4 + 8) * MP * 4;
  static constexpr int BYTES = BAR_OFF + 256;
  // followed by this CTA's x slice (x * norm weight, fp32): m rows of
  // kt_per_split * BK floats, sized at launch
  static constexpr int XS_OFF = BYTES;
  static size_t smem(int m, int kt_per_split) {
    return 1024 + static_cast<size_t>(BYTES) + static_cast<size_t>(m) * kt_per_split * BK * 4;
  }
  static constexpr uint32_t TMEM_COLS = 2 * NCOL < 32 ? 32 : 2 * NCOL;
};

__device__ __forceinline__ void conv_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// int8 byte pair -> fp16 bits, exact: 0x6400 | (b ^ 0x80) = 1024 + q + 128.
__device__ __forceinline__ uint32_t i8pair_h2(uint32_t wb, uint32_t sel) {
  const uint32_t h = __byte_perm(wb, 0x64646464u, sel);
  __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h),
                      __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));
  return *reinterpret_cast<uint32_t*>(&r);
}
// biased nibble bytes (u = q + 8 in the low 4 bits of each byte) -> fp16 pair
// of bytes b0, b1: 0x6400 | u = 1024 + q + 8.
__device__ __forceinline__ uint32_t i4pair_h2(uint32_t nb, uint32_t sel) {
  const uint32_t h = __byte_perm(nb, 0x64646464u, sel);
  __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h),
                      __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));
  return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
  return static_cast<uint32_t>(__half_as_ushort(a)) |
         (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
}


// Pass over this CTA's K-slice of x (128 converter threads, t = 0..127):
// stores x * norm_w (fp32) in xs[m][0 .. slice_len) unless xs is null, zero
// past k_hi; per token
// row the power-of-two factor 2^e with max |x * norm_w * 2^e| in
// [2^(target-1), 2^target) (escale, einv = 2^-e) and the slice's sum of x^2
// (ss_part, fixed reduction order).  Ends with the converters synchronised.
template <int MP>
__device__ __forceinline__ void x_slice_prologue(const GvArgs& a, float* xs, int xs_ld, int k_lo,
                                                 int k_hi, int slice_len, int t, float* red_mx,
                                                 float* red_ss, float* escale, float* einv,
                                                 float* ss_part, int target) {
  const int lane = t & 31, cw = t >> 5;
#pragma unroll
  for (int m = 0; m < MP; ++m) {
    float mx = 0.0f, ss = 0.0f;
    if (m < a.m)
      for (int kl = t; kl < slice_len; kl += 128) {
        const int kk = k_lo + kl;
        float v = 0.0f, vn = 0.0f;
        if (kk < k_hi) {
          v = a.x[static_cast<int64_t>(m) * a.k + kk];
          vn = a.norm_w ? v * a.norm_w[kk] : v;
        }
        ss = fmaf(v, v, ss);
        mx = fmaxf(mx, fabsf(vn));
        if (xs) xs[m * xs_ld + kl] = vn;
      }
    mx = warp_max(mx);
    ss = warp_sum(ss);
    if (lane == 0) {
      red_mx[cw * MP + m] = mx;
      red_ss[cw * MP + m] = ss;
    }
  }
  conv_bar();
  if (t < MP) {
    float m4 = 0.0f, s4 = 0.0f;
    for (int w = 0; w < 4; ++w) {
      m4 = fmaxf(m4, red_mx[w * MP + t]);
      s4 += red_ss[w * MP + t];
    }
    int e = 0;
    if (m4 > 0.0f && isfinite(m4)) {
      int ex;
      frexpf(m4, &ex);
      e = max(-100, min(target - ex, 100));
    }
    escale[t] = ldexpf(1.0f, e);
    einv[t] = ldexpf(1.0f, -e);
    ss_part[t] = s4;
  }
  conv_bar();
}

// Split-K reduction over the thread-block cluster (the CTAs of blockIdx.y) and
// the epilogue.  tile[BW][MP] holds this CTA's partial outputs per TMEM lane
// (= weight row of the tile), ss_part[MP] its partial sums of x^2.  Rank r
// sums, in rank order, the rows [r * rows / splits, ...) of every rank's tile
// and writes them: 1/rms (fused norm), bias, residual, or SwiGLU over the
// gate rows [0, 64) and up rows [64, 128).
template <int EPI, int MP, int NT>
__device__ __forceinline__ void splitk_epilogue(const GvArgs& a, const float* tile,
                                                const float* ss_part, float* inv_s, int n_tile,
                                                int split) {
  __syncthreads();
  const int splits = static_cast<int>(gridDim.y);
  if (splits > 1) cluster_sync();
  const uint32_t tile_u32 = smem_u32(tile);
  const uint32_t ss_u32 = smem_u32(ss_part);
  // sum over ranks in rank order; all ranks' values are loaded before the
  // first add, so the distributed-shared-memory round trips overlap
  auto cl_sum = [&](const float* local, uint32_t base, int idx) -> float {
    if (splits == 1) return local[idx];
    float v[kMaxSplits];
#pragma unroll
    for (int sp = 0; sp < kMaxSplits; ++sp)
      v[sp] = sp < splits ? ld_cluster_f32(map_rank(base + static_cast<uint32_t>(idx) * 4,
                                                    static_cast<uint32_t>(sp)))
                          : 0.0f;
    float s = 0.0f;
#pragma unroll
    for (int sp = 0; sp < kMaxSplits; ++sp)
      if (sp < splits) s += v[sp];
    return s;
  };
  auto inv_of = [&](int m) -> float {
    if (!a.norm_w) return 1.0f;
    const float ssum = cl_sum(ss_part, ss_u32, m);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ssum, static_cast<float>(a.k)), a.eps)));
  };
  constexpr int OUT_ROWS = EPI == EPI_SWIGLU ? BW / 2 : BW;
  const int rows_per = (OUT_ROWS + splits - 1) / splits;
  const int r_lo = split * rows_per, r_hi = min(OUT_ROWS, r_lo + rows_per);
  const int nr = max(r_hi - r_lo, 0);
  for (int it = threadIdx.x; it < nr * a.m; it += NT) {
    const int m = it / nr, j = r_lo + it % nr;
    if (EPI == EPI_SWIGLU) {
      const int c = n_tile * (BW / 2) + j;
      if (c >= a.inter) continue;
      const float gs = cl_sum(tile, tile_u32, j * MP + m);
      const float us = cl_sum(tile, tile_u32, (j + BW / 2) * MP + m);
      const float inv = inv_of(m);
      a.y[static_cast<int64_t>(m) * a.inter + c] = silu_f(gs * inv) * (us * inv);
    } else {
      const int c = n_tile * BW + j;
      if (c >= a.n) continue;
      const float bias = a.bias ? a.bias[c] : 0.0f;
      const float res = a.residual ? a.residual[static_cast<int64_t>(m) * a.n + c] : 0.0f;
      float o = cl_sum(tile, tile_u32, j * MP + m) * inv_of(m);
      if (a.bias) o += bias;
      if (a.residual) o = res + o;
      a.y[static_cast<int64_t>(m) * a.n + c] = o;
    }
  }
  if (splits > 1) cluster_sync();     // every rank's tile stays alive until all have read it
}

template <int WK, int EPI, int MP>
__global__ void __launch_bounds__(kThreads, 1)
qgemv_tc_kernel(const __grid_constant__ CUtensorMap map_w, GvArgs a) {
  using L = Layout<WK, MP>;
  constexpr int NCOL = L::NCOL;
  constexpr int NS = L::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* tile = reinterpret_cast<float*>(smem + L::TILE_OFF);
  float* escale = reinterpret_cast<float*>(smem + L::SMALL_OFF);
  float* einv = escale + MP;
  float* ss_part = einv + MP;
  float* inv_s = ss_part + MP;
  float* red_mx = inv_s + MP;          // [4][MP]
  float* red_ss = red_mx + 4 * MP;     // [4][MP]
  float* xs = reinterpret_cast<float*>(smem + L::XS_OFF);    // [m][xs_ld]
  const int xs_ld = a.kt_per_split * BK;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;               // [NS] raw tile landed
  uint64_t* empty = full + NS;         // [NS] converters done with the raw tile
  uint64_t* aready = empty + NS;       // [NA] fp16 operands written
  uint64_t* afree = aready + NA;       // [NA] MMAs done with the operands
  uint64_t* acc_full = afree + NA;     // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, split = blockIdx.y;
  const int kt_begin = split * a.kt_per_split;
  const int kt_end = min(kt_begin + a.kt_per_split, a.kt_total);
  const int ntl = max(kt_end - kt_begin, 0);
  const int ktpg = WK == WK_I4 ? a.kt_per_group : max(ntl, 1);
  const int ngl = (ntl + ktpg - 1) / ktpg;
  auto raw_tile = [&](int s) { return smem + L::RAW_OFF + s * L::RAW; };
  auto a_tile = [&](int b) { return smem + L::A_OFF + b * A_BYTES; };
  auto b_tile = [&](int b) { return smem + L::B_OFF + b * L::B_BYTES; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 128);
    }
    for (int b = 0; b < NA; ++b) {
      mbar_init(&aready[b], 128);
      mbar_init(&afree[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer: raw weight tiles ----------------
    if (lane == 0) {
      const int pre = min(NS, ntl);
      auto issue = [&](int i) {
        const int s = i % NS;
        mbar_arrive_expect_tx(&full[s], L::RAW);
        const int kg = (kt_begin + i) * BK;
        const int xw = WK == WK_I8 ? kg : kg / 2;
        if (EPI == EPI_SWIGLU) {
          const int half_bytes = L::RAW / 2;
          tma_load_2d(raw_tile(s), &map_w, &full[s], xw, n_tile * (BW / 2));
          tma_load_2d(raw_tile(s) + half_bytes, &map_w, &full[s], xw, a.inter + n_tile * (BW / 2));
        } else {
          tma_load_2d(raw_tile(s), &map_w, &full[s], xw, n_tile * BW);
        }
      };
      // weights are constant: the first stages go out before the dependency wait
      for (int i = 0; i < pre; ++i) issue(i);
      grid_dep_wait();
      grid_dep_launch();
      int issued = pre;
      for (int i = pre; i < ntl && !*abort_flag; ++i) {
        const int s = i % NS;
        if (!mbar_wait(&empty[s], ((i / NS) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        issue(i);
        issued = i + 1;
      }
      // after an abort, let the copies still in flight land before the CTA
      // exits (bounded; every earlier stage was reused, so it has landed)
      if (*abort_flag)
        for (int i = max(0, issued - NS); i < issued; ++i) mbar_wait(&full[i % NS], (i / NS) & 1);
    } else {
      grid_dep_wait();
      grid_dep_launch();
    }
  } else if (warp == 1) {
    // ---------------- single-thread MMA issue ----------------
    grid_dep_wait();
    grid_dep_launch();
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(BW, NCOL);
      for (int i = 0; i < ntl && !*abort_flag; ++i) {
        const int b = i % NA;
        const int gl = i / ktpg, buf = gl & 1;
        const bool first = (i % ktpg) == 0;
        if (first && gl >= 2 && !mbar_wait(&acc_empty[buf], ((gl >> 1) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        if (!mbar_wait(&aready[b], (i / NA) & 1)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t ad = smem_u32(a_tile(b)), bd = smem_u32(b_tile(b));
        const uint32_t d = tmem + buf * NCOL;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          mma_f16(d, desc_k_sw128(ad + kk * 32), desc_k_sw128(bd + kk * 32), idesc,
                  (first && kk == 0) ? 0u : 1u);
        mma_commit(&afree[b]);
        if ((i % ktpg) == ktpg - 1 || i == ntl - 1) mma_commit(&acc_full[buf]);
      }
    }
  } else {
    // ---------------- converters + epilogue (128 threads) ----------------
    grid_dep_wait();
    grid_dep_launch();
    const int t = threadIdx.x - 64;               // raw / A row this thread converts
    const int q = warp & 3;                       // TMEM lane quadrant
    const int row_local = q * 32 + lane;          // accumulator row (TMEM lane)
    const int k_lo = kt_begin * BK;
    const int k_hi = min(kt_end * BK, a.k);

    // weight row behind TMEM lane row_local (-1: outside the matrix)
    const int wrow = [&]() -> int {
      if (EPI == EPI_SWIGLU) {
        const int c = n_tile * (BW / 2) + (row_local & (BW / 2 - 1));
        if (c >= a.inter) return -1;
        return row_local < BW / 2 ? c : a.inter + c;
      }
      const int r = n_tile * BW + row_local;
      return r < a.n ? r : -1;
    }();

    // ---- this CTA's slice of x: scaled copy in shared memory, per-row factors ----
    x_slice_prologue<MP>(a, xs, xs_ld, k_lo, k_hi, ntl * BK, t, red_mx, red_ss, escale, einv, ss_part, 15);
    // token rows >= m stay zero in both operand slots
    for (int i = t; i < NA * L::B_BYTES / 16; i += 128) {
      const int bsl = i / (L::B_BYTES / 16), rem = i % (L::B_BYTES / 16);
      const int r = rem / 8;
      if ((r % MP) >= a.m)
        reinterpret_cast<uint4*>(b_tile(bsl))[rem] = make_uint4(0u, 0u, 0u, 0u);
    }
    conv_bar();

    // INT4 scale of this lane's weight row for local group gl
    auto group_scale = [&](int gl) -> float {
      if (wrow < 0) return 0.0f;
      if (WK == WK_I8) return __half2float(a.scales[wrow]);
      return __half2float(a.scales[static_cast<int64_t>(wrow) * a.ngroups_row +
                                   (kt_begin + gl * ktpg) / ktpg]);
    };
    float acc[NCOL];
#pragma unroll
    for (int j = 0; j < NCOL; ++j) acc[j] = 0.0f;
    float sc_next = WK == WK_I4 ? group_scale(0) : 0.0f;

    auto promote = [&](int gl) -> bool {
      const int buf = gl & 1;
      const float sc = WK == WK_I4 ? sc_next : group_scale(0);
      if (WK == WK_I4 && gl + 1 < ngl) sc_next = group_scale(gl + 1);
      if (!mbar_wait(&acc_full[buf], (gl >> 1) & 1)) return false;
      tc_fence_after();
      const uint32_t taddr = tmem + buf * NCOL + (static_cast<uint32_t>(q * 32) << 16);
      if constexpr (NCOL == 16) {
        float v[16];
        tmem_ld_32x32b_x16(taddr, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = fmaf(v[j], sc, acc[j]);
      } else {
        float v[32];
        tmem_ld_32x32b_x32(taddr, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = fmaf(v[j], sc, acc[j]);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      return true;
    };

    bool ok = true;
    for (int i = 0; i < ntl && ok; ++i) {
      const int s = i % NS, b = i % NA;
      const int gl = i / ktpg;
      if (*abort_flag || !mbar_wait(&full[s], (i / NS) & 1)) {
        ok = false;
        break;
      }
      if (i >= NA && !mbar_wait(&afree[b], ((i / NA) - 1) & 1)) {
        ok = false;
        break;
      }
      // ---- raw row t -> fp16 A row t (128B swizzle) ----
      uint8_t* dst_row = a_tile(b) + (t >> 3) * 1024 + (t & 7) * 128;
      const uint32_t rsw = static_cast<uint32_t>(t & 7);
      if (WK == WK_I8) {
        const uint8_t* src = raw_tile(s) + t * BK;                // TMA 64B swizzle
        const uint32_t rs = static_cast<uint32_t>((t >> 1) & 3);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 w = *reinterpret_cast<const uint4*>(src + ((static_cast<uint32_t>(j) ^ rs) << 4));
          const uint32_t wx = w.x ^ 0x80808080u, wy = w.y ^ 0x80808080u, wz = w.z ^ 0x80808080u,
                         ww = w.w ^ 0x80808080u;
          uint4 o0, o1;
          o0.x = i8pair_h2(wx, 0x5140u); o0.y = i8pair_h2(wx, 0x5342u);
          o0.z = i8pair_h2(wy, 0x5140u); o0.w = i8pair_h2(wy, 0x5342u);
          o1.x = i8pair_h2(wz, 0x5140u); o1.y = i8pair_h2(wz, 0x5342u);
          o1.z = i8pair_h2(ww, 0x5140u); o1.w = i8pair_h2(ww, 0x5342u);
          *reinterpret_cast<uint4*>(dst_row + (((2 * j) ^ rsw) << 4)) = o0;
          *reinterpret_cast<uint4*>(dst_row + (((2 * j + 1) ^ rsw) << 4)) = o1;
        }
      } else {
        const uint8_t* src = raw_tile(s) + t * (BK / 2);          // TMA 32B swizzle
        const uint32_t rs = static_cast<uint32_t>((t >> 2) & 1);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const uint4 w = *reinterpret_cast<const uint4*>(src + ((static_cast<uint32_t>(j) ^ rs) << 4));
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {          // one word = 8 elements = one 16-byte chunk
            const uint32_t lo = nib_lo(ws[e]), hi = nib_hi(ws[e]);
            uint4 o;                             // element order [0,2,4,6,1,3,5,7]
            o.x = i4pair_h2(lo, 0x5140u);
            o.y = i4pair_h2(lo, 0x5342u);
            o.z = i4pair_h2(hi, 0x5140u);
            o.w = i4pair_h2(hi, 0x5342u);
            *reinterpret_cast<uint4*>(dst_row + ((static_cast<uint32_t>(4 * j + e) ^ rsw) << 4)) = o;
          }
        }
      }
      mbar_arrive(&empty[s]);
      // ---- x chunk of this K step -> B rows m (hi) and MP + m (lo) ----
      {
        for (int it = t; it < a.m * 8; it += 128) {
          const int m = it >> 3, c = it & 7;
          const float4* xr = reinterpret_cast<const float4*>(xs + m * xs_ld + i * BK + c * 8);
          const float4 x0 = xr[0], x1 = xr[1];
          const float es = escale[m];
          const float v[8] = {x0.x * es, x0.y * es, x0.z * es, x0.w * es,
                              x1.x * es, x1.y * es, x1.z * es, x1.w * es};
          __half h[8], l[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int src = WK == WK_I4 ? ((j & 3) * 2 + (j >> 2)) : j;
            h[j] = __float2half_rn(v[src]);
            l[j] = __float2half_rn(v[src] - __half2float(h[j]));
          }
          const uint4 hv = make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(h[4], h[5]),
                                      pack_h2(h[6], h[7]));
          const uint4 lv = make_uint4(pack_h2(l[0], l[1]), pack_h2(l[2], l[3]), pack_h2(l[4], l[5]),
                                      pack_h2(l[6], l[7]));
          const int rh = m, rl = MP + m;
          *reinterpret_cast<uint4*>(b_tile(b) + (rh >> 3) * 1024 + (rh & 7) * 128 +
                                    ((c ^ (rh & 7)) << 4)) = hv;
          *reinterpret_cast<uint4*>(b_tile(b) + (rl >> 3) * 1024 + (rl & 7) * 128 +
                                    ((c ^ (rl & 7)) << 4)) = lv;
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&aready[b]);
      if (WK == WK_I4 && (i % ktpg) == ktpg - 1 && gl >= 1 && !promote(gl - 1)) ok = false;
    }
    if (ok && ntl > 0 && !*abort_flag) ok = promote(ngl - 1);
    if (!ok) {
      *abort_flag = 1;
      raise_flag(a.flags, KSH_FLAG_TIMEOUT);
    }
    // ---- partial outputs of this K-slice: unscale hi + lo, stage by TMEM lane ----
#pragma unroll
    for (int m = 0; m < MP; ++m)
      tile[row_local * MP + m] = wrow >= 0 ? (acc[m] + acc[MP + m]) * einv[m] : 0.0f;
  }

  splitk_epilogue<EPI, MP, kThreads>(a, tile, ss_part, inv_s, n_tile, split);

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
  grid_dep_launch();
}


// ---------------------------------------------------------------------------
// INT8: kind::i8 MMAs straight on the TMA-loaded weight tiles
// ---------------------------------------------------------------------------
//
// int8 weights are already an MMA operand: a 128-row x 128-byte TMA box with
// 128-byte swizzle is the K-major layout tcgen05 reads, so nothing is
// converted.  The token rows enter as fixed point: per CTA slice and token,
// X = rint(x * w_norm * 2^e) with |X| < 2^22, written as three balanced signed
// 8-bit digits X = c0 + 2^8 c1 + 2^16 c2 (B columns d * MP + m).  The int32
// accumulation is exact; the epilogue forms (D0 + 2^8 D1 + 2^16 D2) * 2^-e *
// scale in fp32.
constexpr int BK8 = 128;                          // K bytes per stage
constexpr int A8_BYTES = BW * BK8;                // 16 KB

template <int MP, int AT>
struct LayoutI8 {
  // AT swizzle atoms (128 K bytes each) per stage: 128 * AT contiguous bytes
  // of every weight row per TMA stage
  static constexpr int NCOL = (3 * MP + 15) / 16 * 16;
  static constexpr int NS = AT == 1 ? 4 : 2;      // TMA stages
  static constexpr int KS = BK8 * AT;             // K bytes per stage
  static constexpr int A_STAGE = A8_BYTES * AT;
  static constexpr int B_ATOM = NCOL * 128;
  static constexpr int B_BYTES = B_ATOM * AT;
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = A_OFF + NS * A_STAGE;
  static constexpr int TILE_OFF = B_OFF + NS * B_BYTES;
  static constexpr int SMALL_OFF = TILE_OFF + BW * MP * 4;
  static constexpr int BAR_OFF = SMALL_OFF + (4 + 8) * MP * 4;
  static constexpr int BAR_BYTES = 256;
  static constexpr int BYTES = BAR_OFF + BAR_BYTES;
  static size_t smem(int, int) { return 1024 + static_cast<size_t>(BYTES); }
  // Consecutive MMAs rotate over NC accumulator copies: an MMA that adds into
  // the accumulator the previous one wrote waits for it, and with N this
  // small that latency, not the math, would set the pace.
  static constexpr int NC = 4;
  static constexpr uint32_t TMEM_COLS = NC * NCOL <= 64 ? 64 : (NC * NCOL <= 128 ? 128 : 256);
};

template <int EPI, int MP, int AT>
__global__ void __launch_bounds__(kThreads, 1)
qgemv_i8_kernel(const __grid_constant__ CUtensorMap map_w, GvArgs a) {
  using L = LayoutI8<MP, AT>;
  constexpr int NCOL = L::NCOL;
  constexpr int NS = L::NS;
  constexpr int KS = L::KS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* tile = reinterpret_cast<float*>(smem + L::TILE_OFF);
  float* escale = reinterpret_cast<float*>(smem + L::SMALL_OFF);
  float* einv = escale + MP;
  float* ss_part = einv + MP;
  float* inv_s = ss_part + MP;
  float* red_mx = inv_s + MP;
  float* red_ss = red_mx + 4 * MP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;               // [NS] weight tile landed (TMA)
  uint64_t* bready = full + NS;        // [NS] token digits written
  uint64_t* empty = bready + NS;       // [NS] MMAs done with the stage
  uint64_t* acc_full = empty + NS;     // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, split = blockIdx.y;
  const int kt_begin = split * a.kt_per_split;
  const int kt_end = min(kt_begin + a.kt_per_split, a.kt_total);
  const int ntl = max(kt_end - kt_begin, 0);
  auto a_tile = [&](int s) { return smem + L::A_OFF + s * L::A_STAGE; };
  auto b_tile = [&](int s) { return smem + L::B_OFF + s * L::B_BYTES; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&bready[s], 128);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer: weight tiles ----------------
    if (lane == 0) {
      const int pre = min(NS, ntl);
      auto issue = [&](int i) {
        const int s = i % NS;
        mbar_arrive_expect_tx(&full[s], L::A_STAGE);
#pragma unroll
        for (int at = 0; at < AT; ++at) {
          const int kg = (kt_begin + i) * KS + at * BK8;
          uint8_t* dst = a_tile(s) + at * A8_BYTES;
          if (EPI == EPI_SWIGLU) {
            tma_load_2d(dst, &map_w, &full[s], kg, n_tile * (BW / 2));
            tma_load_2d(dst + A8_BYTES / 2, &map_w, &full[s], kg, a.inter + n_tile * (BW / 2));
          } else {
            tma_load_2d(dst, &map_w, &full[s], kg, n_tile * BW);
          }
        }
      };
      for (int i = 0; i < pre; ++i) issue(i);      // constant data: before the wait
      grid_dep_wait();
      grid_dep_launch();
      int issued = pre;
      for (int i = pre; i < ntl && !*abort_flag; ++i) {
        const int s = i % NS;
        if (!mbar_wait(&empty[s], ((i / NS) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        issue(i);
        issued = i + 1;
      }
      if (*abort_flag)
        for (int i = max(0, issued - NS); i < issued; ++i) mbar_wait(&full[i % NS], (i / NS) & 1);
    } else {
      grid_dep_wait();
      grid_dep_launch();
    }
  } else if (warp == 1) {
    // ---------------- single-thread MMA issue ----------------
    grid_dep_wait();
    grid_dep_launch();
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8_s32(BW, NCOL);
      bool ok = true;
      for (int i = 0; i < ntl && ok && !*abort_flag; ++i) {
        const int s = i % NS;
        if (!mbar_wait(&full[s], (i / NS) & 1) || !mbar_wait(&bready[s], (i / NS) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ad = smem_u32(a_tile(s)), bd = smem_u32(b_tile(s));
#pragma unroll
        for (int at = 0; at < AT; ++at)
#pragma unroll
          for (int kk = 0; kk < BK8 / 32; ++kk) {
            const int u = (i * AT + at) * (BK8 / 32) + kk;      // MMA index in this CTA
            mma_i8(tmem + (u % L::NC) * NCOL, desc_k_sw128(ad + at * A8_BYTES + kk * 32),
                   desc_k_sw128(bd + at * L::B_ATOM + kk * 32), idesc, u >= L::NC ? 1u : 0u);
          }
        mma_commit(&empty[s]);
      }
      if (!ok) *abort_flag = 1;
      mma_commit(acc_full);         // also after an abort: the waiters must not hang
    }
  } else {
    // ---------------- token digits + epilogue (128 threads) ----------------
    grid_dep_wait();
    grid_dep_launch();
    const int t = threadIdx.x - 64;
    const int q = warp & 3;
    const int row_local = q * 32 + lane;
    const int k_lo = kt_begin * KS;
    const int k_hi = min(kt_end * KS, a.k);
    const int wrow = [&]() -> int {
      if (EPI == EPI_SWIGLU) {
        const int c = n_tile * (BW / 2) + (row_local & (BW / 2 - 1));
        if (c >= a.inter) return -1;
        return row_local < BW / 2 ? c : a.inter + c;
      }
      const int r = n_tile * BW + row_local;
      return r < a.n ? r : -1;
    }();
    const float wscale = wrow >= 0 ? __half2float(a.scales[wrow]) : 0.0f;
    x_slice_prologue<MP>(a, nullptr, 0, k_lo, k_hi, ntl * KS, t, red_mx, red_ss, escale, einv, ss_part, 22);
    // digit rows of tokens >= m, and padding rows >= 3 * MP, stay zero
    for (int i = t; i < NS * L::B_BYTES / 16; i += 128) {
      const int st = i / (L::B_BYTES / 16), rem = i % (L::B_BYTES / 16);
      const int r = (rem % (L::B_ATOM / 16)) / 8;      // row within its atom
      if (r >= 3 * MP || (r % MP) >= a.m)
        reinterpret_cast<uint4*>(b_tile(st))[rem] = make_uint4(0u, 0u, 0u, 0u);
    }
    conv_bar();

    bool ok = true;
    for (int i = 0; i < ntl && ok; ++i) {
      const int s = i % NS;
      if (*abort_flag || (i >= NS && !mbar_wait(&empty[s], ((i / NS) - 1) & 1))) {
        ok = false;
        break;
      }
      // (token m, 16-element chunk c): three digit rows, 16 bytes each
      // (x comes from L2: the writers run up to NS stages ahead of the MMAs)
      for (int it = t; it < a.m * 8 * AT; it += 128) {
        const int m = it / (8 * AT), cg = it % (8 * AT), c = cg & 7;
        const int kb = (kt_begin + i) * KS + cg * 16;   // a.k % 16 == 0: chunks are whole
        float4 xv[4] = {};
        if (kb < a.k) {
          const float4* xr = reinterpret_cast<const float4*>(a.x + static_cast<int64_t>(m) * a.k + kb);
#pragma unroll
          for (int w = 0; w < 4; ++w) xv[w] = xr[w];
          if (a.norm_w) {
            const float4* nr = reinterpret_cast<const float4*>(a.norm_w + kb);
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              const float4 nv = nr[w];
              xv[w].x *= nv.x; xv[w].y *= nv.y; xv[w].z *= nv.z; xv[w].w *= nv.w;
            }
          }
        }
        const float es = escale[m];
        uint32_t d0[4], d1[4], d2[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const float4 v = xv[w];
          const float vv[4] = {v.x, v.y, v.z, v.w};
          uint32_t b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // rint(v * 2^e) through the 1.5 * 2^23 magic constant (|X| < 2^22)
            const int X = __float_as_int(fmaf(vv[j], es, 12582912.0f)) - 0x4B400000;
            const int c0 = ((X + 128) & 255) - 128;
            const int X1 = (X - c0) >> 8;
            const int c1 = ((X1 + 128) & 255) - 128;
            const int c2 = (X1 - c1) >> 8;
            b0 |= (static_cast<uint32_t>(c0) & 0xFFu) << (8 * j);
            b1 |= (static_cast<uint32_t>(c1) & 0xFFu) << (8 * j);
            b2 |= (static_cast<uint32_t>(c2) & 0xFFu) << (8 * j);
          }
          d0[w] = b0;
          d1[w] = b1;
          d2[w] = b2;
        }
        uint8_t* bt = b_tile(s) + (cg >> 3) * L::B_ATOM;
        const int r0 = m, r1 = MP + m, r2 = 2 * MP + m;
        *reinterpret_cast<uint4*>(bt + (r0 >> 3) * 1024 + (r0 & 7) * 128 + ((c ^ (r0 & 7)) << 4)) =
            make_uint4(d0[0], d0[1], d0[2], d0[3]);
        *reinterpret_cast<uint4*>(bt + (r1 >> 3) * 1024 + (r1 & 7) * 128 + ((c ^ (r1 & 7)) << 4)) =
            make_uint4(d1[0], d1[1], d1[2], d1[3]);
        *reinterpret_cast<uint4*>(bt + (r2 >> 3) * 1024 + (r2 & 7) * 128 + ((c ^ (r2 & 7)) << 4)) =
            make_uint4(d2[0], d2[1], d2[2], d2[3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&bready[s]);
    }
    if (!ok) {
      *abort_flag = 1;
      raise_flag(a.flags, KSH_FLAG_TIMEOUT);
    }
    // ---- combine the digit columns: (D0 + 2^8 D1 + 2^16 D2) * 2^-e * scale ----
    float out[MP];
#pragma unroll
    for (int m = 0; m < MP; ++m) out[m] = 0.0f;
    if (ntl > 0 && mbar_wait(acc_full, 0)) {
      tc_fence_after();
      int dd[NCOL];
#pragma unroll
      for (int j = 0; j < NCOL; ++j) dd[j] = 0;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16);
      const int used = min(L::NC, ntl * AT * (BK8 / 32));     // copies that were written
      for (int cp = 0; cp < used; ++cp) {
#pragma unroll
        for (int c = 0; c < NCOL / 16; ++c) {
          float v[16];
          tmem_ld_32x32b_x16(taddr + cp * NCOL + c * 16, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) dd[c * 16 + j] += __float_as_int(v[j]);
        }
      }
#pragma unroll
      for (int m = 0; m < MP; ++m)
        out[m] = fmaf(65536.0f, static_cast<float>(dd[2 * MP + m]),
                      fmaf(256.0f, static_cast<float>(dd[MP + m]), static_cast<float>(dd[m]))) *
                 einv[m] * wscale;
    } else if (ntl > 0) {
      raise_flag(a.flags, KSH_FLAG_TIMEOUT);
    }
#pragma unroll
    for (int m = 0; m < MP; ++m) tile[row_local * MP + m] = wrow >= 0 ? out[m] : 0.0f;
  }

  splitk_epilogue<EPI, MP, kThreads>(a, tile, ss_part, inv_s, n_tile, split);

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
  grid_dep_launch();
}


// ---------------------------------------------------------------------------
// INT4: kind::i8 MMAs on nibbles sign-extended to bytes, per-group promotion
// ---------------------------------------------------------------------------
//
// One 128-wide K step is one quantization group (G = 128).  Converter warps
// widen each raw 64-byte row (128 nibbles) to 128 signed bytes; within every
// 16-element chunk the byte order is [0,2,4,6,1,3,5,7,8,10,12,14,9,11,13,15]
// (low nibbles, then high nibbles, of each 32-bit word), and the token digits
// use the same order.  Each group's MMAs accumulate into their own TMEM
// buffer (two, alternating); the converter warps read it back (int32, |D| <=
// 2^17, converted exactly through the 1.5 * 2^23 constant) and add it, times
// the group scale, to register accumulators.  A seventh warp writes the
// token digits, running ahead of the MMAs.
constexpr int kThreadsI4 = 224;
constexpr int RAW4_BYTES = BW * BK8 / 2;          // 8 KB: 128 rows x 64 bytes

template <int MP>
struct LayoutI4 {
  static constexpr int NCOL = (3 * MP + 15) / 16 * 16;
  static constexpr int RS = 4;                    // raw TMA stages
  static constexpr int NA4 = 3;                   // widened operand slots
  static constexpr int NB4 = 3;                   // token digit slots
  static constexpr int B_BYTES = NCOL * 128;
  static constexpr int RAW_OFF = 0;
  static constexpr int A_OFF = RAW_OFF + RS * RAW4_BYTES;
  static constexpr int B_OFF = A_OFF + NA4 * A8_BYTES;
  static constexpr int TILE_OFF = B_OFF + NB4 * B_BYTES;
  static constexpr int SMALL_OFF = TILE_OFF + BW * MP * 4;
  static constexpr int BAR_OFF = SMALL_OFF + (4 + 8) * MP * 4;
  static constexpr int BAR_BYTES = 256;
  static constexpr int BYTES = BAR_OFF + BAR_BYTES;
  static size_t smem(int, int) { return 1024 + static_cast<size_t>(BYTES); }
  static constexpr uint32_t TMEM_COLS = 2 * NCOL <= 32 ? 32 : (2 * NCOL <= 64 ? 64 : 128);
};

__device__ __forceinline__ uint32_t s4_lo_bytes(uint32_t w) {
  return ((((w & 0x0F0F0F0Fu) ^ 0x08080808u) + 0x78787878u) ^ 0x80808080u);
}
__device__ __forceinline__ uint32_t s4_hi_bytes(uint32_t w) {
  return (((((w >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u) + 0x78787878u) ^ 0x80808080u);
}
// exact int -> float for |v| < 2^22
__device__ __forceinline__ float i2f_small(int v) {
  return __int_as_float(v + 0x4B400000) - 12582912.0f;
}

template <int EPI, int MP>
__global__ void __launch_bounds__(kThreadsI4, 1)
qgemv_i4_kernel(const __grid_constant__ CUtensorMap map_w, GvArgs a) {
  using L = LayoutI4<MP>;
  constexpr int NCOL = L::NCOL;
  constexpr int RS = L::RS, NA4 = L::NA4, NB4 = L::NB4;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* tile = reinterpret_cast<float*>(smem + L::TILE_OFF);
  float* escale = reinterpret_cast<float*>(smem + L::SMALL_OFF);
  float* einv = escale + MP;
  float* ss_part = einv + MP;
  float* inv_s = ss_part + MP;
  float* red_mx = inv_s + MP;
  float* red_ss = red_mx + 4 * MP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;               // [RS]  raw tile landed
  uint64_t* rempty = full + RS;        // [RS]  converters done with the raw tile
  uint64_t* aready = rempty + RS;      // [NA4] widened weights written
  uint64_t* afree = aready + NA4;      // [NA4] MMAs done with them
  uint64_t* bready = afree + NA4;      // [NB4] token digits written
  uint64_t* bfree = bready + NB4;      // [NB4] MMAs done with them
  uint64_t* acc_full = bfree + NB4;    // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* xready = acc_empty + 2;    // [1]   per-token scales known
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xready + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  static_assert((2 * RS + 2 * NA4 + 2 * NB4 + 4 + 1) * 8 + 8 <= L::BAR_BYTES, "barrier region");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, split = blockIdx.y;
  const int kt_begin = split * a.kt_per_split;
  const int kt_end = min(kt_begin + a.kt_per_split, a.kt_total);
  const int ntl = max(kt_end - kt_begin, 0);
  auto raw_tile = [&](int s) { return smem + L::RAW_OFF + s * RAW4_BYTES; };
  auto a_tile = [&](int s) { return smem + L::A_OFF + s * A8_BYTES; };
  auto b_tile = [&](int s) { return smem + L::B_OFF + s * L::B_BYTES; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < RS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&rempty[s], 128);
    }
    for (int s = 0; s < NA4; ++s) {
      mbar_init(&aready[s], 128);
      mbar_init(&afree[s], 1);
    }
    for (int s = 0; s < NB4; ++s) {
      mbar_init(&bready[s], 32);
      mbar_init(&bfree[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(xready, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer: raw int4 tiles ----------------
    if (lane == 0) {
      const int pre = min(RS, ntl);
      auto issue = [&](int i) {
        const int s = i % RS;
        mbar_arrive_expect_tx(&full[s], RAW4_BYTES);
        const int xb = (kt_begin + i) * (BK8 / 2);
        if (EPI == EPI_SWIGLU) {
          tma_load_2d(raw_tile(s), &map_w, &full[s], xb, n_tile * (BW / 2));
          tma_load_2d(raw_tile(s) + RAW4_BYTES / 2, &map_w, &full[s], xb, a.inter + n_tile * (BW / 2));
        } else {
          tma_load_2d(raw_tile(s), &map_w, &full[s], xb, n_tile * BW);
        }
      };
      for (int i = 0; i < pre; ++i) issue(i);      // constant data: before the wait
      grid_dep_wait();
      grid_dep_launch();
      int issued = pre;
      for (int i = pre; i < ntl && !*abort_flag; ++i) {
        const int s = i % RS;
        if (!mbar_wait(&rempty[s], ((i / RS) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        issue(i);
        issued = i + 1;
      }
      if (*abort_flag)
        for (int i = max(0, issued - RS); i < issued; ++i) mbar_wait(&full[i % RS], (i / RS) & 1);
    } else {
      grid_dep_wait();
      grid_dep_launch();
    }
  } else if (warp == 1) {
    // ---------------- single-thread MMA issue ----------------
    grid_dep_wait();
    grid_dep_launch();
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_s8_s32(BW, NCOL);
      bool ok = true;
      for (int i = 0; i < ntl && !*abort_flag; ++i) {
        const int sa = i % NA4, sb = i % NB4, buf = i & 1;
        if ((i >= 2 && !mbar_wait(&acc_empty[buf], ((i >> 1) - 1) & 1)) ||
            !mbar_wait(&aready[sa], (i / NA4) & 1) || !mbar_wait(&bready[sb], (i / NB4) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ad = smem_u32(a_tile(sa)), bd = smem_u32(b_tile(sb));
        const uint32_t d = tmem + buf * NCOL;
#pragma unroll
        for (int kk = 0; kk < BK8 / 32; ++kk)
          mma_i8(d, desc_k_sw128(ad + kk * 32), desc_k_sw128(bd + kk * 32), idesc, kk ? 1u : 0u);
        mma_commit(&afree[sa]);
        mma_commit(&bfree[sb]);
        mma_commit(&acc_full[buf]);
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 6) {
    // ---------------- token digits (32 threads) ----------------
    grid_dep_wait();
    grid_dep_launch();
    bool ok = mbar_wait(xready, 0);
    for (int i = 0; i < ntl && ok; ++i) {
      const int sb = i % NB4;
      if (*abort_flag || (i >= NB4 && !mbar_wait(&bfree[sb], ((i / NB4) - 1) & 1))) {
        ok = false;
        break;
      }
      for (int it = lane; it < a.m * 8; it += 32) {
        const int m = it >> 3, c = it & 7;
        const int kb = (kt_begin + i) * BK8 + c * 16;
        float xv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) xv[j] = 0.0f;
        if (kb + 16 <= a.k) {
          const float4* xr = reinterpret_cast<const float4*>(a.x + static_cast<int64_t>(m) * a.k + kb);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const float4 v = xr[w];
            xv[4 * w] = v.x; xv[4 * w + 1] = v.y; xv[4 * w + 2] = v.z; xv[4 * w + 3] = v.w;
          }
        } else {
          for (int j = 0; j < 16; ++j)
            if (kb + j < a.k) xv[j] = a.x[static_cast<int64_t>(m) * a.k + kb + j];
        }
        if (a.norm_w) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (kb + j < a.k) xv[j] *= a.norm_w[kb + j];
        }
        const float es = escale[m];
        uint32_t d0[4] = {}, d1[4] = {}, d2[4] = {};
#pragma unroll
        for (int p = 0; p < 16; ++p) {
          // byte p holds element [0,2,4,6,1,3,5,7,...] of the chunk
          const int e = (p & 8) + ((p & 3) << 1) + ((p >> 2) & 1);
          const int X = __float_as_int(fmaf(xv[e], es, 12582912.0f)) - 0x4B400000;
          const int c0 = ((X + 128) & 255) - 128;
          const int X1 = (X - c0) >> 8;
          const int c1 = ((X1 + 128) & 255) - 128;
          const int c2 = (X1 - c1) >> 8;
          d0[p >> 2] |= (static_cast<uint32_t>(c0) & 0xFFu) << (8 * (p & 3));
          d1[p >> 2] |= (static_cast<uint32_t>(c1) & 0xFFu) << (8 * (p & 3));
          d2[p >> 2] |= (static_cast<uint32_t>(c2) & 0xFFu) << (8 * (p & 3));
        }
        uint8_t* bt = b_tile(sb);
        const int r0 = m, r1 = MP + m, r2 = 2 * MP + m;
        *reinterpret_cast<uint4*>(bt + (r0 >> 3) * 1024 + (r0 & 7) * 128 + ((c ^ (r0 & 7)) << 4)) =
            make_uint4(d0[0], d0[1], d0[2], d0[3]);
        *reinterpret_cast<uint4*>(bt + (r1 >> 3) * 1024 + (r1 & 7) * 128 + ((c ^ (r1 & 7)) << 4)) =
            make_uint4(d1[0], d1[1], d1[2], d1[3]);
        *reinterpret_cast<uint4*>(bt + (r2 >> 3) * 1024 + (r2 & 7) * 128 + ((c ^ (r2 & 7)) << 4)) =
            make_uint4(d2[0], d2[1], d2[2], d2[3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(&bready[sb]);
    }
    if (!ok) {
      *abort_flag = 1;
      raise_flag(a.flags, KSH_FLAG_TIMEOUT);
    }
  } else {
    // ---------------- converters + promotion + epilogue (128 threads) ----------------
    grid_dep_wait();
    grid_dep_launch();
    const int t = threadIdx.x - 64;
    const int q = warp & 3;
    const int row_local = q * 32 + lane;
    const int k_lo = kt_begin * BK8;
    const int k_hi = min(kt_end * BK8, a.k);
    const int wrow = [&]() -> int {
      if (EPI == EPI_SWIGLU) {
        const int c = n_tile * (BW / 2) + (row_local & (BW / 2 - 1));
        if (c >= a.inter) return -1;
        return row_local < BW / 2 ? c : a.inter + c;
      }
      const int r = n_tile * BW + row_local;
      return r < a.n ? r : -1;
    }();
    x_slice_prologue<MP>(a, nullptr, 0, k_lo, k_hi, ntl * BK8, t, red_mx, red_ss, escale, einv, ss_part, 22);
    for (int i = t; i < NB4 * L::B_BYTES / 16; i += 128) {
      const int st = i / (L::B_BYTES / 16), rem = i % (L::B_BYTES / 16);
      const int r = rem / 8;
      if (r >= 3 * MP || (r % MP) >= a.m)
        reinterpret_cast<uint4*>(b_tile(st))[rem] = make_uint4(0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
    conv_bar();
    if (t == 0) mbar_arrive(xready);

    auto group_scale = [&](int i) -> float {
      return wrow >= 0 ? __half2float(a.scales[static_cast<int64_t>(wrow) * a.ngroups_row + kt_begin + i])
                       : 0.0f;
    };
    float acc[NCOL];
#pragma unroll
    for (int j = 0; j < NCOL; ++j) acc[j] = 0.0f;
    float sc_next = ntl > 0 ? group_scale(0) : 0.0f;
    auto promote = [&](int i) -> bool {
      const int buf = i & 1;
      const float sc = sc_next;
      if (i + 1 < ntl) sc_next = group_scale(i + 1);
      if (!mbar_wait(&acc_full[buf], (i >> 1) & 1)) return false;
      tc_fence_after();
      const uint32_t taddr = tmem + buf * NCOL + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll
      for (int c = 0; c < NCOL / 16; ++c) {
        float v[16];
        tmem_ld_32x32b_x16(taddr + c * 16, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[c * 16 + j] = fmaf(i2f_small(__float_as_int(v[j])), sc, acc[c * 16 + j]);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      return true;
    };

    bool ok = true;
    for (int i = 0; i < ntl && ok; ++i) {
      const int s = i % RS, sa = i % NA4;
      if (*abort_flag || !mbar_wait(&full[s], (i / RS) & 1) ||
          (i >= NA4 && !mbar_wait(&afree[sa], ((i / NA4) - 1) & 1))) {
        ok = false;
        break;
      }
      // raw row t (64 bytes, TMA 64B swizzle: chunk j at j ^ ((t >> 1) & 3)) ->
      // 128 signed bytes (128B swizzle: chunk c at c ^ (t & 7))
      const uint8_t* src = raw_tile(s) + t * 64;
      uint8_t* dst = a_tile(sa) + (t >> 3) * 1024 + (t & 7) * 128;
      const uint32_t rs = static_cast<uint32_t>((t >> 1) & 3), rsw = static_cast<uint32_t>(t & 7);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 w = *reinterpret_cast<const uint4*>(src + ((static_cast<uint32_t>(j) ^ rs) << 4));
        const uint4 o0 = make_uint4(s4_lo_bytes(w.x), s4_hi_bytes(w.x), s4_lo_bytes(w.y), s4_hi_bytes(w.y));
        const uint4 o1 = make_uint4(s4_lo_bytes(w.z), s4_hi_bytes(w.z), s4_lo_bytes(w.w), s4_hi_bytes(w.w));
        *reinterpret_cast<uint4*>(dst + (((2 * j) ^ rsw) << 4)) = o0;
        *reinterpret_cast<uint4*>(dst + (((2 * j + 1) ^ rsw) << 4)) = o1;
      }
      fence_proxy_async_smem();
      mbar_arrive(&aready[sa]);
      mbar_arrive(&rempty[s]);
      if (i >= 1 && !promote(i - 1)) ok = false;
    }
    if (ok && ntl > 0 && !*abort_flag) ok = promote(ntl - 1);
    if (!ok) {
      *abort_flag = 1;
      raise_flag(a.flags, KSH_FLAG_TIMEOUT);
    }
#pragma unroll
    for (int m = 0; m < MP; ++m)
      tile[row_local * MP + m] =
          wrow >= 0 ? fmaf(65536.0f, acc[2 * MP + m], fmaf(256.0f, acc[MP + m], acc[m])) * einv[m] : 0.0f;
  }

  splitk_epilogue<EPI, MP, kThreadsI4>(a, tile, ss_part, inv_s, n_tile, split);

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

// 0: off; 1: auto (by scheme, token count and matrix size); 2: every eligible
// shape; 3: as 2, through the fp16-operand kernel (for tests)
std::atomic<int> g_gemv_tc{-1};

struct GvPlan {
  int tiles, kt_total, kt_per_group, splits, kt_per_split;
};

// Split-K that minimises (waves x K steps per CTA) on the resident CTA slots
// (slots(kt_per_split, split): CTAs the GPU holds at once at that split's
// shared-memory size, in clusters of the split),
// split boundaries on group boundaries, at most kMaxSplits (one cluster).
template <typename SlotsFn>
GvPlan gv_plan(int epi, int64_t keff, int64_t n_rows, int bk, int kt_per_group, SlotsFn slots_of) {
  GvPlan p = {};
  const int64_t rows_per_tile = epi == EPI_SWIGLU ? BW / 2 : BW;
  const int64_t out_rows = epi == EPI_SWIGLU ? n_rows / 2 : n_rows;
  p.tiles = static_cast<int>((out_rows + rows_per_tile - 1) / rows_per_tile);
  p.kt_total = static_cast<int>((keff + bk - 1) / bk);
  p.kt_per_group = kt_per_group;
  const int groups = (p.kt_total + p.kt_per_group - 1) / p.kt_per_group;
  double best = 1e30;
  for (int s = 1; s <= kMaxSplits && s <= groups; ++s) {
    const int gps = (groups + s - 1) / s;
    const int kps = gps * p.kt_per_group;
    const int real = (p.kt_total + kps - 1) / kps;
    if (real != s) continue;
    const int64_t slots = slots_of(kps, s);
    if (slots <= 0) continue;
    const int64_t ctas = static_cast<int64_t>(p.tiles) * s;
    const int64_t waves = (ctas + slots - 1) / slots;
    // per-CTA fixed cost (prologue, pipeline fill, reduction) ~ 3 K steps
    const double cost = static_cast<double>(waves) * (kps + 3);
    if (cost < best - 1e-9) {
      best = cost;
      p.splits = s;
      p.kt_per_split = kps;
    }
  }
  return p;
}

constexpr size_t kMaxSmem = 227 * 1024;

// CTAs of `kern` resident on the GPU at `smem` bytes in clusters of
// `cluster`: the smaller of the occupancy query and the shared-memory bound
// (both CTAs' reservations) per SM, and of the cluster-placement query.
int64_t gv_slots(const void* kern, size_t smem, int cluster, int threads = kThreads) {
  if (smem > kMaxSmem) return 0;
  const int by_smem = static_cast<int>((228 * 1024) / (smem + 1024));
  const int occ = resident_ctas(kern, threads, smem);
  const int64_t per_sm = static_cast<int64_t>(num_sms()) * std::max(1, std::min(by_smem, std::max(occ, 1)));
  return cluster > 1 ? std::min(per_sm, cluster_slots(kern, threads, smem, cluster)) : per_sm;
}

GvArgs gv_args(const LinArgs& a, const GvPlan& p, int ngroups_row) {
  GvArgs g = {};
  g.x = a.x;
  g.norm_w = a.norm_w;
  g.scales = a.scales;
  g.bias = a.bias;
  g.residual = a.residual;
  g.y = a.y;
  g.flags = nullptr;
  g.eps = a.norm_eps;
  g.m = static_cast<int>(a.m);
  g.k = static_cast<int>(a.k);
  g.n = static_cast<int>(a.n);
  g.inter = static_cast<int>(a.inter);
  g.kt_total = p.kt_total;
  g.kt_per_split = p.kt_per_split;
  g.kt_per_group = p.kt_per_group;
  g.ngroups_row = ngroups_row;
  return g;
}

// One launch: grid (tiles, splits), the splits of a tile as one cluster.
template <typename Kern>
int gv_launch(Kern kern, const GvPlan& p, size_t smem, cudaStream_t stream, const CUtensorMap& mw,
              const GvArgs& g, int threads = kThreads) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.tiles), static_cast<unsigned>(p.splits), 1);
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(p.splits);
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mw, g);
  if (e == cudaSuccess) count_launch();
  return e == cudaSuccess ? KSH_OK : record_cuda_error(e);
}

// fp16 operand kernel (INT4; INT8 in test mode 3)
template <int WK, int EPI, int MP>
int launch_gv(const LinArgs& a, cudaStream_t stream) {
  using L = Layout<WK, MP>;
  auto kern = qgemv_tc_kernel<WK, EPI, MP>;
  const void* kp = reinterpret_cast<const void*>(kern);
  if (set_smem_optin(kp, kMaxSmem) != KSH_OK) return KSH_ERR_CUDA;
  const int64_t keff = WK == WK_I4 ? a.kp : a.k;
  const int m = static_cast<int>(a.m);
  const GvPlan p = gv_plan(EPI, keff, a.n, BK, WK == WK_I4 ? static_cast<int>(a.g / BK) : 1,
                           [&](int kps, int sp) { return gv_slots(kp, L::smem(m, kps), sp); });
  if (p.splits < 1) return KSH_ERR_UNSUPPORTED;
  CUtensorMap mw;
  const uint32_t box_rows = EPI == EPI_SWIGLU ? BW / 2 : BW;
  const bool ok = WK == WK_I8
                      ? make_tensor_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, a.k, a.n, a.k,
                                           BK, box_rows, CU_TENSOR_MAP_SWIZZLE_64B)
                      : make_tensor_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, a.kp / 2, a.n,
                                           a.kp / 2, BK / 2, box_rows, CU_TENSOR_MAP_SWIZZLE_32B);
  if (!ok) return KSH_ERR_CUDA;
  return gv_launch(kern, p, L::smem(m, p.kt_per_split), stream, mw,
                   gv_args(a, p, WK == WK_I4 ? static_cast<int>(a.kp / a.g) : 1));
}

// kind::i8 kernel (INT8)
template <int EPI, int MP>
int launch_gv_i8(const LinArgs& a, cudaStream_t stream) {
  constexpr int AT = 2;              // 256 contiguous bytes of each weight row per stage
  using L = LayoutI8<MP, AT>;
  auto kern = qgemv_i8_kernel<EPI, MP, AT>;
  const void* kp = reinterpret_cast<const void*>(kern);
  if (set_smem_optin(kp, kMaxSmem) != KSH_OK) return KSH_ERR_CUDA;
  const int m = static_cast<int>(a.m);
  const GvPlan p = gv_plan(EPI, a.k, a.n, L::KS, 1,
                           [&](int kps, int sp) { return gv_slots(kp, L::smem(m, kps), sp); });
  if (p.splits < 1) return KSH_ERR_UNSUPPORTED;
  CUtensorMap mw;
  const uint32_t box_rows = EPI == EPI_SWIGLU ? BW / 2 : BW;
  if (!make_tensor_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, a.k, a.n, a.k, BK8, box_rows,
                          CU_TENSOR_MAP_SWIZZLE_128B))
    return KSH_ERR_CUDA;
  return gv_launch(kern, p, L::smem(m, p.kt_per_split), stream, mw, gv_args(a, p, 1));
}

// kind::i8 kernel for INT4 (group size 128)
template <int EPI, int MP>
int launch_gv_i4(const LinArgs& a, cudaStream_t stream) {
  using L = LayoutI4<MP>;
  auto kern = qgemv_i4_kernel<EPI, MP>;
  const void* kp = reinterpret_cast<const void*>(kern);
  if (set_smem_optin(kp, kMaxSmem) != KSH_OK) return KSH_ERR_CUDA;
  const GvPlan p = gv_plan(EPI, a.kp, a.n, BK8, 1,
                           [&](int kps, int sp) { return gv_slots(kp, L::smem(0, kps), sp, kThreadsI4); });
  if (p.splits < 1) return KSH_ERR_UNSUPPORTED;
  CUtensorMap mw;
  const uint32_t box_rows = EPI == EPI_SWIGLU ? BW / 2 : BW;
  if (!make_tensor_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, a.kp / 2, a.n, a.kp / 2, BK8 / 2,
                          box_rows, CU_TENSOR_MAP_SWIZZLE_64B))
    return KSH_ERR_CUDA;
  return gv_launch(kern, p, L::smem(0, 0), stream, mw, gv_args(a, p, static_cast<int>(a.kp / a.g)),
                   kThreadsI4);
}

template <int EPI>
int launch_gv_i4_m(const LinArgs& a, cudaStream_t stream) {
  if (a.m <= 5) return launch_gv_i4<EPI, 5>(a, stream);
  if (a.m <= 10) return launch_gv_i4<EPI, 10>(a, stream);
  return launch_gv_i4<EPI, 16>(a, stream);
}

template <int WK, int EPI>
int launch_gv_m(const LinArgs& a, cudaStream_t stream) {
  if (a.m <= 8) return launch_gv<WK, EPI, 8>(a, stream);
  return launch_gv<WK, EPI, 16>(a, stream);
}

template <int EPI>
int launch_gv_i8_m(const LinArgs& a, cudaStream_t stream) {
  if (a.m <= 5) return launch_gv_i8<EPI, 5>(a, stream);
  if (a.m <= 10) return launch_gv_i8<EPI, 10>(a, stream);
  return launch_gv_i8<EPI, 16>(a, stream);
}

}  // namespace

int gemv_tc_mode() {
  int v = g_gemv_tc.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* e = getenv("KSH_GEMV_TC");
    v = (e && *e) ? std::min(std::max(atoi(e), 0), 3) : 1;
    g_gemv_tc.store(v);
  }
  return v;
}

int set_gemv_tc_mode(int mode) {
  const int prev = gemv_tc_mode();
  g_gemv_tc.store(std::min(std::max(mode, 0), 3));
  return prev;
}

// Whether the tensor-core decode path takes this linear: quantized weights,
// M <= 16, shapes the TMA tiles and the in-kernel x split support, and a
// matrix large enough that its weight stream (not latency) dominates.
bool gemv_tc_eligible(int wk, int epi, const LinArgs& a) {
  const int mode = gemv_tc_mode();
  if (mode == 0) return false;
  if (wk != WK_I8 && wk != WK_I4) return false;
  if (a.m < 1 || a.m > 16 || a.argmax_out) return false;
  if (a.k > INT32_MAX / 2 || a.n > INT32_MAX || a.m * a.k > INT32_MAX) return false;
  if ((reinterpret_cast<uintptr_t>(a.w) & 15) != 0) return false;
  if (wk == WK_I8 && a.k % 16 != 0) return false;
  if (wk == WK_I4 && (a.g % BK != 0 || (a.kp / 2) % 16 != 0)) return false;
  if (epi == EPI_SWIGLU && a.n != 2 * a.inter) return false;
  if ((reinterpret_cast<uintptr_t>(a.x) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(a.norm_w) & 15) != 0)
    return false;
  if (!tensor_map_encoder_available()) return false;
  const int64_t keff = wk == WK_I4 ? a.kp : a.k;
  // the x slice of the largest split must fit shared memory (bound over both kernels)
  const int64_t k_split = (keff + kMaxSplits - 1) / kMaxSplits + 2 * BK8;
  const size_t worst = 1024 + static_cast<size_t>(std::max(Layout<WK_I4, 16>::BYTES, LayoutI8<16, 2>::BYTES)) +
                       static_cast<size_t>(a.m) * k_split * 4;
  if (worst > kMaxSmem) return false;
  if (mode >= 2) return true;
  // auto: where the measured tensor-core path beats the CUDA-core GEMV.  Its
  // fixed cost (~5 us: cluster launch, TMEM, x prologue, split-K exchange)
  // pays off once the matrix or the token count is large enough.
  const int64_t wbytes = wk == WK_I8 ? a.n * keff : a.n * keff / 2;
  constexpr int64_t MiB = int64_t{1} << 20;
  if (wk == WK_I8) {
    if (a.m <= 2) return wbytes >= 16 * MiB;
    if (a.m <= 7) return wbytes >= 2 * MiB;
    return wbytes >= MiB / 2;
  }
  // INT4 (integer-MMA kernel for G = 128)
  if (a.m <= 2) return wbytes >= 24 * MiB;
  if (a.m <= 7) return wbytes >= 2 * MiB;
  return wbytes >= MiB;
}

int launch_gemv_tc(int wk, int epi, const LinArgs& a, cudaStream_t stream) {
  if (wk == WK_I8) {
    if (gemv_tc_mode() == 3)
      return epi == EPI_SWIGLU ? launch_gv_m<WK_I8, EPI_SWIGLU>(a, stream)
                               : launch_gv_m<WK_I8, EPI_STORE>(a, stream);
    return epi == EPI_SWIGLU ? launch_gv_i8_m<EPI_SWIGLU>(a, stream)
                             : launch_gv_i8_m<EPI_STORE>(a, stream);
  }
  if (gemv_tc_mode() != 3 && a.g == BK8)
    return epi == EPI_SWIGLU ? launch_gv_i4_m<EPI_SWIGLU>(a, stream)
                             : launch_gv_i4_m<EPI_STORE>(a, stream);
  return epi == EPI_SWIGLU ? launch_gv_m<WK_I4, EPI_SWIGLU>(a, stream)
                           : launch_gv_m<WK_I4, EPI_STORE>(a, stream);
}

}  // namespace ksh
