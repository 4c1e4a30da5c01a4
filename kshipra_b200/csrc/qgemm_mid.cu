// K7: quantized linear layers for batches of 17..64 token rows on tcgen05.
//
// Replaces QuantizedLinear.forward (engine/quantization.py:394-396) for the
// batched decode regime (continuous batching, large decode batches): a few
// dozen token rows against a large weight matrix.  Tokens on the MMA's M side
// (the prefill GEMM) leave most of each 128-row tile empty; here the roles are
// swapped:
//
// * swap-AB: the MMA's M side (128 TMEM lanes) is 128 weight rows, its N side
//   the MP = 32 or 64 token rows (zero-filled past m by TMA);
// * x is split once per call (split_x_kernel: optional RMSNorm, a power-of-two
//   row scale, x * 2^e = hi + lo in fp16).  INT8: the lo tile sits right
//   after the hi tile, so one MMA of N = 2 * MP takes both terms into
//   separate TMEM columns (an M = 128 tcgen05.mma takes max(~45, N / 2)
//   cycles); INT4: two MMAs of N = MP add both terms into the same columns,
//   which leaves TMEM room for two accumulator buffers;
// * raw int8 / int4 weight tiles arrive by TMA and converter warps widen them
//   to fp16 (exact) straight into TMEM (tcgen05.st, one weight row per lane),
//   where the MMAs take them as the A operand: only the x tiles are read from
//   shared memory by the tensor core.  (With both operands in shared memory
//   an N = 128 MMA alone reads 128 bytes per cycle, the whole shared-memory
//   bandwidth, and the TMA and converter traffic came on top of it.)  INT4
//   chunks are widened in the order [0,2,4,6,1,3,5,7], and split_x stores x
//   in the same order (a permutation of k applied to both operands leaves
//   the sum as is);
// * a CTA covers NT = 2 tiles of 128 weight rows, so each x stage fetched from
//   L2 feeds every tile's MMAs; one warp issues them all, converged, from
//   one elected lane (an M = 128 tcgen05.mma with A in TMEM takes ~34 cycles
//   at N = 64 and ~64 at N = 128; a lone lane-0 thread of a diverged warp
//   issues one only every ~67 cycles), waiting once per stage;
// * INT4 group scales are applied by promoting each group's TMEM partial into
//   register accumulators (double-buffered TMEM, an FMA per token and row);
//   INT8 accumulates the whole K-slice in TMEM and scales once;
// * split-K over a thread-block cluster, reduced through distributed shared
//   memory in rank order (deterministic); the epilogue applies the row factor
//   2^-e, bias, residual or SwiGLU (tile = 64 gate rows + the 64 matching up
//   rows) with vectorised stores.
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

int launch_split_x(const LinArgs& a, char* ws, bool perm, __half** xh, __half** xl, float** inv,
                   cudaStream_t stream);
int64_t split_x_workspace_size(int64_t m, int64_t k);

namespace {

using namespace tc;

constexpr int BW = 128;                 // weight rows per tile (MMA M)
constexpr int BK = 64;                  // K per sub-stage (one 128-byte fp16 row)
constexpr int NT = 2;                   // weight tiles per CTA
// warp 0: TMA; warp 1: MMAs of every tile (the whole warp converged, one
// elected lane issuing); warps 2 .. 1 + 4 NT: converters
constexpr int kConvWarp0 = 2;
constexpr int kThreads = 32 * (kConvWarp0 + 4 * NT);
constexpr int kMaxSplits = 8;

// SK sub-stages of BK per pipeline stage: every barrier round trip (~200
// cycles on a completed phase) and the per-stage bookkeeping of the MMA and
// converter warps are paid once per SK * BK of K.
template <int WK, int MP, int SK>
struct MidLayout {
  static constexpr int BKS = SK * BK;                         // K per stage
  static constexpr int XT = MP * BK * 2;                      // one x term sub-tile
  static constexpr int RAWT = BW * (WK == WK_I8 ? BK : BK / 2);  // one tile's raw sub-tile
  // stage: [x hi k][x lo k] for every sub-stage k (the lo rows right after
  // the hi rows: one INT8 B operand of 2 MP rows), then tile j's raw
  // sub-tiles [j][k]
  static constexpr int XSUB = 2 * XT;
  static constexpr int STAGE = SK * XSUB + NT * SK * RAWT;
  static constexpr int NS = std::min(8, (200 * 1024) / STAGE);
  static constexpr int RING = NS * STAGE;
  static constexpr int BAR_OFF = RING;
  static constexpr int BYTES = BAR_OFF + 512;
  static constexpr int OUT_LD = NT * BW;                      // staged partials [MP][NT * BW]
  // TMEM columns.  Accumulators from column 0, per tile and buffer: INT4 MP
  // columns (the hi- and lo-term MMAs add into the same ones), two buffers
  // (one group promoted while the next accumulates); INT8 [hi: MP][lo: MP],
  // one buffer.  From A_COL the fp16 weight operands: per buffer and tile
  // BKS / 2 columns (two K-consecutive halves per column, one row per lane).
  static constexpr uint32_t ACC_COLS = WK == WK_I4 ? MP : 2 * MP;
  static constexpr uint32_t A_COL = 256;
  static constexpr uint32_t A_COLS = BKS / 2;
  static constexpr int NA = static_cast<int>(256 / (NT * A_COLS));  // operand buffers
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(NS >= 3 && NA >= 2, "pipeline depth");
  static_assert(MP * OUT_LD * 4 <= RING, "staged partials reuse the TMA ring");
  static_assert(XT % 1024 == 0 && STAGE % 1024 == 0 && RAWT % 1024 == 0, "swizzle alignment");
  static_assert((WK == WK_I4 ? 2 : 1) * NT * ACC_COLS <= A_COL, "accumulator columns");
  static_assert(A_COL + NA * NT * A_COLS <= TMEM_COLS, "operand columns");
  static constexpr size_t smem() { return 1024 + static_cast<size_t>(BYTES); }
};

struct MidArgs {
  const __half* scales;
  const float* bias;
  const float* residual;
  const float* inv_row;     // [m] 2^-e per x row
  float* y;
  int32_t* flags;
  int m, n, inter;
  int kt_total, kt_per_split, kt_per_group, ngroups_row;
};

// int8 byte pair -> fp16 bits, exact: 0x6400 | (b ^ 0x80) = 1024 + q + 128.
__device__ __forceinline__ uint32_t i8pair_h2(uint32_t wb, uint32_t sel) {
  const uint32_t h = __byte_perm(wb, 0x64646464u, sel);
  __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h),
                      __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));
  return *reinterpret_cast<uint32_t*>(&r);
}
// biased nibble bytes (u = q + 8) -> fp16 pair of bytes b0, b1: 1024 + q + 8 - 1032.
__device__ __forceinline__ uint32_t i4pair_h2(uint32_t nb, uint32_t sel) {
  const uint32_t h = __byte_perm(nb, 0x64646464u, sel);
  __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h),
                      __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408)));
  return *reinterpret_cast<uint32_t*>(&r);
}

template <int WK, int EPI, int MP, int SK>
__global__ void __launch_bounds__(kThreads, 1)
qgemm_mid_kernel(const __grid_constant__ CUtensorMap map_xh, const __grid_constant__ CUtensorMap map_xl,
                 const __grid_constant__ CUtensorMap map_w, MidArgs a) {
  using L = MidLayout<WK, MP, SK>;
  constexpr int NS = L::NS, NA = L::NA;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;               // [NS] x tiles + raw weight tiles landed
  uint64_t* empty = full + NS;         // [NS] MMAs and converters done with the stage
  uint64_t* aready = empty + NS;       // [NA][NT] fp16 weights of a tile in TMEM
  uint64_t* afree = aready + NA * NT;  // [NA][NT] the tile's MMAs done with them
  uint64_t* acc_full = afree + NA * NT;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta_tile = blockIdx.x * NT, split = blockIdx.y;
  const int kt_begin = split * a.kt_per_split;
  const int kt_end = min(kt_begin + a.kt_per_split, a.kt_total);
  const int ntl = max(kt_end - kt_begin, 0);
  const int ktpg = WK == WK_I4 ? a.kt_per_group : max(ntl, 1);
  const int ngl = (ntl + ktpg - 1) / ktpg;
  auto xh_tile = [&](int s, int k) { return smem + s * L::STAGE + k * L::XSUB; };
  auto xl_tile = [&](int s, int k) { return smem + s * L::STAGE + k * L::XSUB + L::XT; };
  auto raw_tile = [&](int s, int j, int k) {
    return smem + s * L::STAGE + SK * L::XSUB + (j * SK + k) * L::RAWT;
  };
  auto a_col = [&](int b, int j) { return L::A_COL + static_cast<uint32_t>(b * NT + j) * L::A_COLS; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + NT * 4);             // the MMAs + every converter warp
    }
    for (int b = 0; b < NA * NT; ++b) {
      mbar_init(&aready[b], 4);                     // the tile's four converter warps
      mbar_init(&afree[b], 1);
    }
    for (int b = 0; b < 2; ++b) mbar_init(&acc_full[b], 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_xh);
    prefetch_tmap(&map_xl);
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
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const int pre = min(NS, ntl);
      auto issue_w = [&](int i) {
        const int s = i % NS;
        mbar_arrive_expect_tx(&full[s], L::STAGE);
#pragma unroll
        for (int k = 0; k < SK; ++k) {
          const int kg = (kt_begin + i) * L::BKS + k * BK;
          const int xw = WK == WK_I8 ? kg : kg / 2;
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            if (EPI == EPI_SWIGLU) {
              const int r0 = (cta_tile + j) * (BW / 2);
              tma_load_2d(raw_tile(s, j, k), &map_w, &full[s], xw, r0);
              tma_load_2d(raw_tile(s, j, k) + L::RAWT / 2, &map_w, &full[s], xw, a.inter + r0);
            } else {
              tma_load_2d(raw_tile(s, j, k), &map_w, &full[s], xw, (cta_tile + j) * BW);
            }
          }
        }
      };
      auto issue_x = [&](int i) {
        const int s = i % NS;
#pragma unroll
        for (int k = 0; k < SK; ++k) {
          const int kg = (kt_begin + i) * L::BKS + k * BK;
          tma_load_2d(xh_tile(s, k), &map_xh, &full[s], kg, 0);
          tma_load_2d(xl_tile(s, k), &map_xl, &full[s], kg, 0);
        }
      };
      // weights are constant: their first stages go out before the dependency
      // wait; x is written by the preceding split kernel
      for (int i = 0; i < pre; ++i) issue_w(i);
      grid_dep_wait();
      grid_dep_launch();
      for (int i = 0; i < pre; ++i) issue_x(i);
      int issued = pre;
      for (int i = pre; i < ntl && !*abort_flag; ++i) {
        const int s = i % NS;
        if (!mbar_wait(&empty[s], ((i / NS) - 1) & 1)) {
          *abort_flag = 1;
          break;
        }
        issue_w(i);
        issue_x(i);
        issued = i + 1;
      }
      // after an abort, let the copies still in flight land before the CTA exits
      if (*abort_flag)
        for (int i = max(0, issued - NS); i < issued; ++i) mbar_wait(&full[i % NS], (i / NS) & 1);
    } else {
      grid_dep_wait();
      grid_dep_launch();
    }
  } else if (warp == 1) {
    // ---------------- MMA issue: the whole warp, one elected lane ----------------
    grid_dep_wait();
    grid_dep_launch();
    // INT4: N = MP, the hi- and lo-term MMAs into the same columns; INT8:
    // N = 2 MP, the lo tile follows the hi tile in shared memory, so one B
    // operand of 2 MP rows carries both terms into separate columns
    constexpr uint32_t idesc = idesc_f16_f32(BW, WK == WK_I4 ? MP : 2 * MP);
    // group and position in it, counted (no division by the runtime group length)
    int gl = 0, kin = 0;
    for (int i = 0; i < ntl; ++i, (++kin == ktpg) ? (kin = 0, ++gl) : 0) {
      const int s = i % NS, b = i % NA;
      const int buf = WK == WK_I4 ? (gl & 1) : 0;
      const bool first = kin == 0;
      // Lane 1 waits for every tile's converters (they arrive after
      // observing this stage's TMA barrier and, in program order, after
      // promoting the group whose TMEM buffer this stage's MMAs overwrite,
      // fenced with tcgen05.fence::before_thread_sync).
      static_assert(NT == 2, "the ready test covers two tiles");
      int got = 1;
      if (lane == 1) {
        const uint32_t ph = (i / NA) & 1;
        // a non-blocking test in a bounded loop: a blocking try_wait may
        // suspend the thread past the converters' arrival
        got = 0;
        for (uint32_t it = 0; it < (1u << 22); ++it) {
          if (mbar_test2(&aready[b * NT], ph, &aready[b * NT + 1], ph)) {
            got = 1;
            break;
          }
          if ((it & 1023u) == 1023u && *abort_flag) break;
        }
        if (!got) *abort_flag = 1;
      }
      if (!__shfl_sync(0xffffffffu, got, 1)) break;
      tc_fence_after();
      if (elect_one()) {
        // a 32-byte step along K adds 2 to the descriptor's start-address
        // field and 8 columns to the TMEM operand address
#pragma unroll
        for (int k = 0; k < SK; ++k) {
          const uint64_t bh = desc_k_sw128(smem_u32(xh_tile(s, k)));
          const uint64_t bl = desc_k_sw128(smem_u32(xl_tile(s, k)));
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const uint32_t at = tmem + a_col(b, j) + static_cast<uint32_t>(k * (BK / 2));
            const uint32_t d = tmem + static_cast<uint32_t>(buf * NT + j) * L::ACC_COLS;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              mma_f16_ts(d, at + 8 * kk, bh + 2 * kk, idesc, (first && k == 0 && kk == 0) ? 0u : 1u);
              if (WK == WK_I4) mma_f16_ts(d, at + 8 * kk, bl + 2 * kk, idesc, 1u);
            }
          }
        }
        mma_commit(&empty[s]);
#pragma unroll
        for (int j = 0; j < NT; ++j) mma_commit(&afree[b * NT + j]);
        if (kin == ktpg - 1 || i == ntl - 1) mma_commit(&acc_full[buf]);
      }
      __syncwarp();
    }
  } else {
    // ---------------- converters + promotion (NT * 128 threads) ----------------
    grid_dep_wait();
    grid_dep_launch();
    const int cw = warp - kConvWarp0;
    const int j = cw >> 2;                          // weight tile of this warp
    const int q = warp & 3;                         // TMEM lane quadrant
    const int row = q * 32 + lane;                  // tile row = TMEM lane
    const int wrow = [&]() -> int {
      if (EPI == EPI_SWIGLU) {
        const int c = (cta_tile + j) * (BW / 2) + (row & (BW / 2 - 1));
        if (c >= a.inter) return -1;
        return row < BW / 2 ? c : a.inter + c;
      }
      const int r = (cta_tile + j) * BW + row;
      return r < a.n ? r : -1;
    }();
    auto group_scale = [&](int gl) -> float {
      if (wrow < 0) return 0.0f;
      if (WK == WK_I8) return __half2float(a.scales[wrow]);
      return __half2float(a.scales[static_cast<int64_t>(wrow) * a.ngroups_row + kt_begin / ktpg + gl]);
    };
    float acc[MP];
#pragma unroll
    for (int c = 0; c < MP; ++c) acc[c] = 0.0f;
    float sc_next = group_scale(0);

    auto promote = [&](int gl) -> bool {
      const int buf = WK == WK_I4 ? (gl & 1) : 0;
      const float sc = sc_next;
      if (WK == WK_I4 && gl + 1 < ngl) sc_next = group_scale(gl + 1);
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (gl >> 1) & 1))) return false;
      tc_fence_after();
      const uint32_t taddr = tmem + static_cast<uint32_t>(buf * NT + j) * L::ACC_COLS +
                             (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll
      for (int c = 0; c < MP / 32; ++c) {
        float vh[32], vl[32];
        tmem_ld_32x32b_x32(taddr + c * 32, vh);
        if (WK == WK_I8) tmem_ld_32x32b_x32(taddr + MP + c * 32, vl);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          acc[c * 32 + e] = fmaf(WK == WK_I8 ? vh[e] + vl[e] : vh[e], sc, acc[c * 32 + e]);
      }
      tc_fence_before();     // TMEM reads ordered before the next aready arrival
      return true;
    };

    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    // Software-pipelined: stage i + 1's barriers are tested and its raw
    // words loaded while stage i's TMEM store is in flight.
    constexpr int RW = WK == WK_I8 ? 4 : 2;         // 16-byte raw chunks per row and sub-stage
    uint4 rw[SK][RW];
    // stage i's TMA data landed and its operand buffer free (warp-uniform:
    // the TMEM store and loads are .sync.aligned)
    auto wait_stage = [&](int i) -> bool {
      const int s = i % NS, b = i % NA;
      bool got;
      if (i < NA) {
        got = mbar_wait(&full[s], (i / NS) & 1);
      } else {
        const uint32_t pf = (i / NS) & 1, pa = ((i / NA) - 1) & 1;
        got = mbar_test2(&full[s], pf, &afree[b * NT + j], pa) ||
              (!*abort_flag && mbar_wait(&full[s], pf) && mbar_wait(&afree[b * NT + j], pa));
      }
      return __all_sync(0xffffffffu, got);
    };
    auto load_raw = [&](int i) {
      const int s = i % NS;
#pragma unroll
      for (int k = 0; k < SK; ++k) {
        if (WK == WK_I8) {
          const uint8_t* src = raw_tile(s, j, k) + row * BK;        // TMA 64B swizzle
          const uint32_t rs = static_cast<uint32_t>((row >> 1) & 3);
#pragma unroll
          for (int c = 0; c < RW; ++c)
            rw[k][c] = *reinterpret_cast<const uint4*>(src + ((static_cast<uint32_t>(c) ^ rs) << 4));
        } else {
          const uint8_t* src = raw_tile(s, j, k) + row * (BK / 2);  // TMA 32B swizzle
          const uint32_t rs = static_cast<uint32_t>((row >> 2) & 1);
#pragma unroll
          for (int c = 0; c < RW; ++c)
            rw[k][c] = *reinterpret_cast<const uint4*>(src + ((static_cast<uint32_t>(c) ^ rs) << 4));
        }
      }
    };
    bool ok = ntl == 0 || wait_stage(0);
    if (ok && ntl > 0) load_raw(0);
    int gl = 0, kin = 0;
    for (int i = 0; i < ntl && ok; ++i, (++kin == ktpg) ? (kin = 0, ++gl) : 0) {
      const int s = i % NS, b = i % NA;
      tc_fence_after();      // the MMAs that read this operand buffer have completed
#pragma unroll
      for (int k = 0; k < SK; ++k) {
        // raw row -> 32 columns of fp16 pairs (this row's 64 K elements of sub-stage k)
        uint32_t h[32];
        if (WK == WK_I8) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t wx = rw[k][c].x ^ 0x80808080u, wy = rw[k][c].y ^ 0x80808080u,
                           wz = rw[k][c].z ^ 0x80808080u, ww = rw[k][c].w ^ 0x80808080u;
            h[8 * c + 0] = i8pair_h2(wx, 0x5140u); h[8 * c + 1] = i8pair_h2(wx, 0x5342u);
            h[8 * c + 2] = i8pair_h2(wy, 0x5140u); h[8 * c + 3] = i8pair_h2(wy, 0x5342u);
            h[8 * c + 4] = i8pair_h2(wz, 0x5140u); h[8 * c + 5] = i8pair_h2(wz, 0x5342u);
            h[8 * c + 6] = i8pair_h2(ww, 0x5140u); h[8 * c + 7] = i8pair_h2(ww, 0x5342u);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint32_t ws[4] = {rw[k][c].x, rw[k][c].y, rw[k][c].z, rw[k][c].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {      // one word = 8 elements = four columns
              const uint32_t lo = nib_lo(ws[e]), hi = nib_hi(ws[e]);
              const int o = 4 * (4 * c + e);   // element order [0,2,4,6,1,3,5,7]
              h[o + 0] = i4pair_h2(lo, 0x5140u);
              h[o + 1] = i4pair_h2(lo, 0x5342u);
              h[o + 2] = i4pair_h2(hi, 0x5140u);
              h[o + 3] = i4pair_h2(hi, 0x5342u);
            }
          }
        }
        tmem_st_32x32b_x32(tmem + lane_base + a_col(b, j) + static_cast<uint32_t>(k * (BK / 2)), h);
      }
      const bool next = i + 1 < ntl;
      const bool next_ok = !next || wait_stage(i + 1);
      if (next && next_ok) load_raw(i + 1);
      tmem_wait_st();
      tc_fence_before();
      // one arrival per warp (the barriers count warps)
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&aready[b * NT + j]);
        mbar_arrive(&empty[s]);
      }
      if (!next_ok) {
        ok = false;
        break;
      }
      if (WK == WK_I4 && kin == ktpg - 1 && gl >= 1 && !promote(gl - 1)) ok = false;
    }
    if (ok && ntl > 0 && __all_sync(0xffffffffu, !*abort_flag)) ok = promote(ngl - 1);
    if (!ok) {
      *abort_flag = 1;
      raise_flag(a.flags, KSH_FLAG_TIMEOUT);
    }
    // Stage this K-slice's partials as [token][tile row] over the TMA ring:
    // every load has landed and the last MMA (which read the last x tiles)
    // has completed before the final promotion returned.
    float* stile = reinterpret_cast<float*>(smem);
    const int orow = j * BW + row;
#pragma unroll
    for (int c = 0; c < MP; ++c) stile[c * L::OUT_LD + orow] = acc[c];
  }

  // ---------------- split-K reduction over the cluster + epilogue ----------------
  __syncthreads();
  const int splits = static_cast<int>(gridDim.y);
  if (splits > 1) cluster_sync();
  {
    const float* stile = reinterpret_cast<const float*>(smem);
    const uint32_t sbase = smem_u32(stile);
    auto col_sum = [&](int mrow, int r4) -> float4 {
      const int off = mrow * L::OUT_LD + 4 * r4;
      if (splits == 1) return *reinterpret_cast<const float4*>(stile + off);
      float4 v[kMaxSplits];
#pragma unroll
      for (int sp = 0; sp < kMaxSplits; ++sp)
        if (sp < splits) v[sp] = ld_cluster_f32x4(map_rank(sbase + static_cast<uint32_t>(off * 4), static_cast<uint32_t>(sp)));
      float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int sp = 0; sp < kMaxSplits; ++sp)
        if (sp < splits) {
          s4.x += v[sp].x; s4.y += v[sp].y; s4.z += v[sp].z; s4.w += v[sp].w;
        }
      return s4;
    };
    // output float4 columns of this CTA, divided among the ranks
    constexpr int OUT4 = EPI == EPI_SWIGLU ? NT * BW / 8 : NT * BW / 4;
    const int per = (OUT4 + splits - 1) / splits;
    const int u_lo = split * per, u_hi = min(OUT4, u_lo + per);
    const int nu = max(u_hi - u_lo, 0);
    for (int it = threadIdx.x; it < nu * a.m; it += kThreads) {
      const int mrow = it / nu, u = u_lo + it % nu;
      const float inv = a.inv_row[mrow];
      float o[4];
      int c;
      int64_t ld;
      if (EPI == EPI_SWIGLU) {
        const int jt = u / (BW / 8), r4 = u % (BW / 8);
        c = (cta_tile + jt) * (BW / 2) + 4 * r4;
        ld = a.inter;
        if (c >= a.inter) continue;
        const float4 g = col_sum(mrow, (jt * BW) / 4 + r4);
        const float4 up = col_sum(mrow, (jt * BW + BW / 2) / 4 + r4);
        o[0] = silu_f(g.x * inv) * (up.x * inv);
        o[1] = silu_f(g.y * inv) * (up.y * inv);
        o[2] = silu_f(g.z * inv) * (up.z * inv);
        o[3] = silu_f(g.w * inv) * (up.w * inv);
      } else {
        c = cta_tile * BW + 4 * u;
        ld = a.n;
        if (c >= a.n) continue;
        const float4 v = col_sum(mrow, u);
        o[0] = v.x * inv; o[1] = v.y * inv; o[2] = v.z * inv; o[3] = v.w * inv;
        if (a.bias)
          for (int e = 0; e < 4; ++e) o[e] += c + e < a.n ? a.bias[c + e] : 0.0f;
      }
      float* yr = a.y + static_cast<int64_t>(mrow) * ld;
      const float* rr = (EPI == EPI_STORE && a.residual) ? a.residual + static_cast<int64_t>(mrow) * ld : nullptr;
      if ((ld & 3) == 0 && c + 3 < ld) {
        if (rr) {
          const float4 rv = *reinterpret_cast<const float4*>(rr + c);
          o[0] = rv.x + o[0]; o[1] = rv.y + o[1]; o[2] = rv.z + o[2]; o[3] = rv.w + o[3];
        }
        *reinterpret_cast<float4*>(yr + c) = make_float4(o[0], o[1], o[2], o[3]);
      } else {
        for (int e = 0; e < 4; ++e)
          if (c + e < ld) yr[c + e] = rr ? rr[c + e] + o[e] : o[e];
      }
    }
  }
  if (splits > 1) cluster_sync();     // every rank's partials stay alive until all have read them

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
  grid_dep_launch();
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

// 0: off; 1: on for eligible shapes (KSH_GEMM_MID in the environment sets it at load)
std::atomic<int> g_mid_mode{-1};

int mid_mode() {
  int v = g_mid_mode.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* e = getenv("KSH_GEMM_MID");
    v = (e && *e) ? (atoi(e) != 0 ? 1 : 0) : 1;
    g_mid_mode.store(v);
  }
  return v;
}

struct MidPlan {
  int ctas, kt_total, kt_per_group, splits, kt_per_split;
};

// Split-K minimising (waves x K steps per CTA) on the CTAs the GPU holds at
// once in clusters of that split (slots_of(s)), split boundaries on group
// boundaries, at most kMaxSplits (one cluster).  Counting the SMs alone
// misjudged cluster placement: 16 clusters of 8 at one CTA per SM ran as two
// waves (the down projection of the 8B shape at M = 64, SMs resident 47 % of
// the kernel's time).
template <typename SlotsFn>
MidPlan mid_plan(int epi, int64_t keff, int64_t n_rows, int bks, int kt_per_group, SlotsFn slots_of) {
  MidPlan p = {};
  const int64_t rows_per_tile = epi == EPI_SWIGLU ? BW / 2 : BW;
  const int64_t out_rows = epi == EPI_SWIGLU ? n_rows / 2 : n_rows;
  const int64_t tiles = (out_rows + rows_per_tile - 1) / rows_per_tile;
  p.ctas = static_cast<int>((tiles + NT - 1) / NT);
  p.kt_total = static_cast<int>((keff + bks - 1) / bks);
  p.kt_per_group = kt_per_group;
  const int groups = (p.kt_total + kt_per_group - 1) / kt_per_group;
  double best = 1e30;
  for (int s = 1; s <= kMaxSplits && s <= groups; ++s) {
    const int kps = (groups + s - 1) / s * kt_per_group;
    if ((p.kt_total + kps - 1) / kps != s) continue;
    const int64_t slots = std::max<int64_t>(s, slots_of(s));
    const int64_t waves = (static_cast<int64_t>(p.ctas) * s + slots - 1) / slots;
    const double cost = static_cast<double>(waves) * (kps * (bks / BK) + 3);   // in BK steps
    if (cost < best - 1e-9) {
      best = cost;
      p.splits = s;
      p.kt_per_split = kps;
    }
  }
  return p;
}

template <int WK, int EPI, int MP, int SK>
int launch_mid(const LinArgs& a, char* ws, cudaStream_t stream) {
  using L = MidLayout<WK, MP, SK>;
  const int64_t keff = WK == WK_I4 ? a.kp : a.k;
  auto kern = qgemm_mid_kernel<WK, EPI, MP, SK>;
  if (set_smem_optin(reinterpret_cast<const void*>(kern), L::smem()) != KSH_OK) return KSH_ERR_CUDA;
  const MidPlan p = mid_plan(EPI, keff, a.n, L::BKS, WK == WK_I4 ? static_cast<int>(a.g / L::BKS) : 1,
                             [&](int s) {
                               return cluster_slots(reinterpret_cast<const void*>(kern), kThreads,
                                                    L::smem(), s);
                             });
  if (p.splits < 1) return KSH_ERR_UNSUPPORTED;
  __half *xh = nullptr, *xl = nullptr;
  float* inv = nullptr;
  int st = launch_split_x(a, ws, WK == WK_I4, &xh, &xl, &inv, stream);
  if (st != KSH_OK) return st;
  CUtensorMap mxh, mxl, mw;
  if (!make_tensor_map_2d(&mxh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xh, a.k, a.m, a.k * 2, BK, MP,
                          CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tensor_map_2d(&mxl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xl, a.k, a.m, a.k * 2, BK, MP,
                          CU_TENSOR_MAP_SWIZZLE_128B))
    return KSH_ERR_CUDA;
  const uint32_t box_rows = EPI == EPI_SWIGLU ? BW / 2 : BW;
  const bool ok = WK == WK_I8
                      ? make_tensor_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, a.k, a.n, a.k, BK,
                                           box_rows, CU_TENSOR_MAP_SWIZZLE_64B)
                      : make_tensor_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, a.kp / 2, a.n,
                                           a.kp / 2, BK / 2, box_rows, CU_TENSOR_MAP_SWIZZLE_32B);
  if (!ok) return KSH_ERR_CUDA;
  MidArgs t = {};
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
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.ctas), static_cast<unsigned>(p.splits), 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::smem();
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (p.splits > 1) {                                     // the splits of a CTA's tiles = one cluster
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = static_cast<unsigned>(p.splits);
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  ++na;
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mxh, mxl, mw, t);
  if (e == cudaSuccess) count_launch();
  return e == cudaSuccess ? KSH_OK : record_cuda_error(e);
}

// INT4 with groups of whole 128-wide stages: two sub-stages per stage (the
// promotion once per stage).  INT8 keeps 64-wide stages: its 64 KB stages of
// two sub-stages leave room for three in the ring, too shallow to cover the
// weight stream (40.7 -> 46.8 us at 4096 x 28672, M = 64).
template <int WK, int EPI>
int launch_mid_m(const LinArgs& a, char* ws, cudaStream_t stream) {
  if constexpr (WK == WK_I4) {
    if (a.g % (2 * BK) == 0)
      return a.m <= 32 ? launch_mid<WK, EPI, 32, 2>(a, ws, stream) : launch_mid<WK, EPI, 64, 2>(a, ws, stream);
  }
  return a.m <= 32 ? launch_mid<WK, EPI, 32, 1>(a, ws, stream) : launch_mid<WK, EPI, 64, 1>(a, ws, stream);
}

}  // namespace

int set_gemm_mid_mode(int mode) {
  const int prev = mid_mode();
  g_mid_mode.store(mode != 0 ? 1 : 0);
  return prev;
}

// Whether this kernel takes the linear: 17..64 rows, quantized weights, the
// shapes its TMA tiles support, and a workspace for the split x.
bool gemm_mid_eligible(int wk, int epi, const LinArgs& a, const void* ws, int64_t ws_bytes) {
  if (mid_mode() == 0) return false;
  if (wk != WK_I8 && wk != WK_I4) return false;
  if (a.m <= 16 || a.m > 64 || a.argmax_out) return false;
  if (a.k > INT32_MAX / 2 || a.n > INT32_MAX || a.k % 8 != 0) return false;
  if ((reinterpret_cast<uintptr_t>(a.w) & 15) != 0) return false;
  if (wk == WK_I8 && a.k % 16 != 0) return false;
  if (wk == WK_I4 && (a.g % BK != 0 || (a.kp / 2) % 16 != 0)) return false;
  if (epi == EPI_SWIGLU && a.n != 2 * a.inter) return false;
  if (!tensor_map_encoder_available()) return false;
  if (!ws || ws_bytes < split_x_workspace_size(a.m, a.k) || (reinterpret_cast<uintptr_t>(ws) & 255) != 0)
    return false;
  return true;
}

int launch_gemm_mid(int wk, int epi, const LinArgs& a, void* ws, cudaStream_t stream) {
  char* w = static_cast<char*>(ws);
  if (wk == WK_I8) return epi == EPI_SWIGLU ? launch_mid_m<WK_I8, EPI_SWIGLU>(a, w, stream)
                                            : launch_mid_m<WK_I8, EPI_STORE>(a, w, stream);
  return epi == EPI_SWIGLU ? launch_mid_m<WK_I4, EPI_SWIGLU>(a, w, stream)
                           : launch_mid_m<WK_I4, EPI_STORE>(a, w, stream);
}

}  // namespace ksh
