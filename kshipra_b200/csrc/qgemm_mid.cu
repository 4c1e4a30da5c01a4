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
//   row scale, x * 2^e = hi + lo in fp16); the lo tile sits right after the hi
//   tile, so one MMA of N = 2 * MP takes both terms into separate TMEM columns
//   (an M = 128 tcgen05.mma takes max(~45, N / 2) cycles, so the wider MMA
//   costs little more than one of the two narrow ones);
// * raw int8 / int4 weight tiles arrive by TMA and converter warps widen them
//   to fp16 (exact) in the 128B-swizzled K-major layout; INT4 chunks are
//   widened in the order [0,2,4,6,1,3,5,7], and split_x stores x in the same
//   order (a permutation of k applied to both operands leaves the sum as is);
// * a CTA covers NT = 2 tiles of 128 weight rows, so each x stage fetched from
//   L2 feeds NT * 4 MMAs; each tile has its own MMA-issuing thread (one thread
//   issues a tcgen05.mma only every ~70 cycles once commits are counted), and
//   that thread waits once per stage, on the converters' barrier alone (an
//   mbarrier wait stalls the issuing thread until its MMAs in flight finish);
// * INT4 group scales are applied by promoting each group's TMEM partial into
//   register accumulators (double-buffered TMEM, an add and an FMA per token
//   and row); INT8 accumulates the whole K-slice in TMEM and scales once;
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
constexpr int BK = 64;                  // K per stage (one 128-byte fp16 row)
constexpr int NT = 2;                   // weight tiles per CTA
constexpr int NA = 2;                   // fp16 weight operand buffers
// warp 0: TMA; warp 1: MMAs of tile 0; warps 2 .. 1 + 4 NT: converters;
// warps 2 + 4 NT ..: MMAs of tiles 1 .. NT - 1 (one issuing thread per tile:
// a single thread issues a tcgen05.mma only every ~70 cycles, slower than the
// tensor core runs these N = 64 / 128 MMAs)
constexpr int kConvWarp0 = 2;
constexpr int kMmaWarpHi = kConvWarp0 + 4 * NT;
constexpr int kThreads = 32 * (kMmaWarpHi + NT - 1);
constexpr int kMaxSplits = 8;
constexpr int A_TILE = BW * BK * 2;     // 16 KB

template <int WK, int MP>
struct MidLayout {
  static constexpr int XT = MP * BK * 2;                      // one x term tile
  static constexpr int RAWT = BW * (WK == WK_I8 ? BK : BK / 2);
  static constexpr int STAGE = 2 * XT + NT * RAWT;
  static constexpr int ABUF = NT * A_TILE;
  static constexpr int NS = std::min(8, (200 * 1024 - NA * ABUF) / STAGE);
  static constexpr int RING = NS * STAGE;
  static constexpr int A_OFF = RING;
  static constexpr int BAR_OFF = A_OFF + NA * ABUF;
  static constexpr int BYTES = BAR_OFF + 512;
  static constexpr int OUT_LD = NT * BW;                      // staged partials [MP][NT * BW]
  // per tile and buffer: [hi-term columns: MP][lo-term columns: MP]
  static constexpr uint32_t TMEM_COLS = (WK == WK_I4 ? 2 : 1) * NT * 2 * MP;
  static_assert(NS >= 3, "pipeline depth");
  static_assert(MP * OUT_LD * 4 <= RING, "staged partials reuse the TMA ring");
  static_assert(XT % 1024 == 0 && STAGE % 1024 == 0 && RAWT % 1024 == 0, "swizzle alignment");
  static_assert(TMEM_COLS >= 32 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM allocation");
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

template <int WK, int EPI, int MP>
__global__ void __launch_bounds__(kThreads, 1)
qgemm_mid_kernel(const __grid_constant__ CUtensorMap map_xh, const __grid_constant__ CUtensorMap map_xl,
                 const __grid_constant__ CUtensorMap map_w, MidArgs a) {
  using L = MidLayout<WK, MP>;
  constexpr int NS = L::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* full = bars;               // [NS] x tiles + raw weight tiles landed
  uint64_t* empty = full + NS;         // [NS] MMAs and converters done with the stage
  uint64_t* aready = empty + NS;       // [NA] fp16 weights written
  uint64_t* afree = aready + NA;       // [NA] MMAs done with them
  uint64_t* acc_full = afree + NA;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta_tile = blockIdx.x * NT, split = blockIdx.y;
  const int kt_begin = split * a.kt_per_split;
  const int kt_end = min(kt_begin + a.kt_per_split, a.kt_total);
  const int ntl = max(kt_end - kt_begin, 0);
  const int ktpg = WK == WK_I4 ? a.kt_per_group : max(ntl, 1);
  const int ngl = (ntl + ktpg - 1) / ktpg;
  auto xh_tile = [&](int s) { return smem + s * L::STAGE; };
  auto xl_tile = [&](int s) { return smem + s * L::STAGE + L::XT; };
  auto raw_tile = [&](int s, int j) { return smem + s * L::STAGE + 2 * L::XT + j * L::RAWT; };
  auto a_tile = [&](int b, int j) { return smem + L::A_OFF + b * L::ABUF + j * A_TILE; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NT + NT * 128);          // every tile's MMAs + the converters
    }
    for (int b = 0; b < NA; ++b) {
      mbar_init(&aready[b], NT * 128);
      mbar_init(&afree[b], NT);
    }
    for (int b = 0; b < 2; ++b) mbar_init(&acc_full[b], NT);
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
        const int kg = (kt_begin + i) * BK;
        const int xw = WK == WK_I8 ? kg : kg / 2;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          if (EPI == EPI_SWIGLU) {
            const int r0 = (cta_tile + j) * (BW / 2);
            tma_load_2d(raw_tile(s, j), &map_w, &full[s], xw, r0);
            tma_load_2d(raw_tile(s, j) + L::RAWT / 2, &map_w, &full[s], xw, a.inter + r0);
          } else {
            tma_load_2d(raw_tile(s, j), &map_w, &full[s], xw, (cta_tile + j) * BW);
          }
        }
      };
      auto issue_x = [&](int i) {
        const int s = i % NS;
        const int kg = (kt_begin + i) * BK;
        tma_load_2d(xh_tile(s), &map_xh, &full[s], kg, 0);
        tma_load_2d(xl_tile(s), &map_xl, &full[s], kg, 0);
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
  } else if (warp == 1 || warp >= kMmaWarpHi) {
    // ---------------- MMA issue: one thread per weight tile ----------------
    grid_dep_wait();
    grid_dep_launch();
    if (lane == 0) {
      const int j = warp == 1 ? 0 : warp - kMmaWarpHi + 1;
      constexpr uint32_t idesc = idesc_f16_f32(BW, 2 * MP);   // N: x hi rows, then lo rows
      for (int i = 0; i < ntl && !*abort_flag; ++i) {
        const int s = i % NS, b = i % NA;
        const int gl = i / ktpg, buf = WK == WK_I4 ? (gl & 1) : 0;
        const bool first = (i % ktpg) == 0;
        // One wait per stage: an mbarrier wait in this thread stalls until
        // the MMAs it has in flight complete (a few hundred cycles), so it
        // waits on the converters' barrier alone.  The converters arrive there
        // after observing this stage's TMA barrier (x tiles landed) and, in
        // program order, after promoting the group whose TMEM buffer this
        // stage's MMAs overwrite (fenced with tcgen05.fence::before_thread_sync).
        if (!mbar_wait(&aready[b], (i / NA) & 1)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        // The lo tile follows the hi tile in shared memory, so one B operand
        // of 2 * MP rows carries both terms: one MMA per K step.  A 32-byte
        // step along K adds 2 to the descriptors' start-address field.
        const uint64_t bdesc = desc_k_sw128(smem_u32(xh_tile(s)));
        const uint64_t adesc = desc_k_sw128(smem_u32(a_tile(b, j)));
        const uint32_t d = tmem + static_cast<uint32_t>((buf * NT + j) * 2 * MP);
        mma_f16(d, adesc, bdesc, idesc, first ? 0u : 1u);
#pragma unroll
        for (int kk = 1; kk < BK / 16; ++kk)
          mma_f16(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, 1u);
        mma_commit(&empty[s]);
        mma_commit(&afree[b]);
        if ((i % ktpg) == ktpg - 1 || i == ntl - 1) mma_commit(&acc_full[buf]);
      }
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
      return __half2float(a.scales[static_cast<int64_t>(wrow) * a.ngroups_row + (kt_begin + gl * ktpg) / ktpg]);
    };
    float acc[MP];
#pragma unroll
    for (int c = 0; c < MP; ++c) acc[c] = 0.0f;
    float sc_next = group_scale(0);

    auto promote = [&](int gl) -> bool {
      const int buf = WK == WK_I4 ? (gl & 1) : 0;
      const float sc = sc_next;
      if (WK == WK_I4 && gl + 1 < ngl) sc_next = group_scale(gl + 1);
      if (!mbar_wait(&acc_full[buf], (gl >> 1) & 1)) return false;
      tc_fence_after();
      const uint32_t taddr = tmem + static_cast<uint32_t>((buf * NT + j) * 2 * MP) + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll
      for (int c = 0; c < MP / 32; ++c) {
        float vh[32], vl[32];
        tmem_ld_32x32b_x32(taddr + c * 32, vh);
        tmem_ld_32x32b_x32(taddr + MP + c * 32, vl);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) acc[c * 32 + e] = fmaf(vh[e] + vl[e], sc, acc[c * 32 + e]);
      }
      tc_fence_before();     // TMEM reads ordered before the next aready arrival
      return true;
    };

    bool ok = true;
    for (int i = 0; i < ntl && ok; ++i) {
      const int s = i % NS, b = i % NA;
      const int gl = i / ktpg;
      if (*abort_flag || !mbar_wait(&full[s], (i / NS) & 1) ||
          (i >= NA && !mbar_wait(&afree[b], ((i / NA) - 1) & 1))) {
        ok = false;
        break;
      }
      // raw row -> fp16 row of the 128B-swizzled K-major operand
      uint8_t* dst = a_tile(b, j) + (row >> 3) * 1024 + (row & 7) * 128;
      const uint32_t rsw = static_cast<uint32_t>(row & 7);
      if (WK == WK_I8) {
        const uint8_t* src = raw_tile(s, j) + row * BK;             // TMA 64B swizzle
        const uint32_t rs = static_cast<uint32_t>((row >> 1) & 3);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 w = *reinterpret_cast<const uint4*>(src + ((static_cast<uint32_t>(c) ^ rs) << 4));
          const uint32_t wx = w.x ^ 0x80808080u, wy = w.y ^ 0x80808080u, wz = w.z ^ 0x80808080u,
                         ww = w.w ^ 0x80808080u;
          uint4 o0, o1;
          o0.x = i8pair_h2(wx, 0x5140u); o0.y = i8pair_h2(wx, 0x5342u);
          o0.z = i8pair_h2(wy, 0x5140u); o0.w = i8pair_h2(wy, 0x5342u);
          o1.x = i8pair_h2(wz, 0x5140u); o1.y = i8pair_h2(wz, 0x5342u);
          o1.z = i8pair_h2(ww, 0x5140u); o1.w = i8pair_h2(ww, 0x5342u);
          *reinterpret_cast<uint4*>(dst + (((2 * c) ^ rsw) << 4)) = o0;
          *reinterpret_cast<uint4*>(dst + (((2 * c + 1) ^ rsw) << 4)) = o1;
        }
      } else {
        const uint8_t* src = raw_tile(s, j) + row * (BK / 2);       // TMA 32B swizzle
        const uint32_t rs = static_cast<uint32_t>((row >> 2) & 1);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint4 w = *reinterpret_cast<const uint4*>(src + ((static_cast<uint32_t>(c) ^ rs) << 4));
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {        // one word = 8 elements = one 16-byte chunk
            const uint32_t lo = nib_lo(ws[e]), hi = nib_hi(ws[e]);
            uint4 o;                           // element order [0,2,4,6,1,3,5,7]
            o.x = i4pair_h2(lo, 0x5140u);
            o.y = i4pair_h2(lo, 0x5342u);
            o.z = i4pair_h2(hi, 0x5140u);
            o.w = i4pair_h2(hi, 0x5342u);
            *reinterpret_cast<uint4*>(dst + ((static_cast<uint32_t>(4 * c + e) ^ rsw) << 4)) = o;
          }
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&aready[b]);
      mbar_arrive(&empty[s]);
      if (WK == WK_I4 && (i % ktpg) == ktpg - 1 && gl >= 1 && !promote(gl - 1)) ok = false;
    }
    if (ok && ntl > 0 && !*abort_flag) ok = promote(ngl - 1);
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

// Split-K minimising (waves x K steps per CTA) at one CTA per SM, split
// boundaries on group boundaries, at most kMaxSplits (one cluster).
MidPlan mid_plan(int epi, int64_t keff, int64_t n_rows, int kt_per_group) {
  MidPlan p = {};
  const int64_t rows_per_tile = epi == EPI_SWIGLU ? BW / 2 : BW;
  const int64_t out_rows = epi == EPI_SWIGLU ? n_rows / 2 : n_rows;
  const int64_t tiles = (out_rows + rows_per_tile - 1) / rows_per_tile;
  p.ctas = static_cast<int>((tiles + NT - 1) / NT);
  p.kt_total = static_cast<int>((keff + BK - 1) / BK);
  p.kt_per_group = kt_per_group;
  const int groups = (p.kt_total + kt_per_group - 1) / kt_per_group;
  const int64_t slots = num_sms();
  double best = 1e30;
  for (int s = 1; s <= kMaxSplits && s <= groups; ++s) {
    const int kps = (groups + s - 1) / s * kt_per_group;
    if ((p.kt_total + kps - 1) / kps != s) continue;
    const int64_t waves = (static_cast<int64_t>(p.ctas) * s + slots - 1) / slots;
    const double cost = static_cast<double>(waves) * (kps + 3);
    if (cost < best - 1e-9) {
      best = cost;
      p.splits = s;
      p.kt_per_split = kps;
    }
  }
  return p;
}

template <int WK, int EPI, int MP>
int launch_mid(const LinArgs& a, char* ws, cudaStream_t stream) {
  using L = MidLayout<WK, MP>;
  const int64_t keff = WK == WK_I4 ? a.kp : a.k;
  const MidPlan p = mid_plan(EPI, keff, a.n, WK == WK_I4 ? static_cast<int>(a.g / BK) : 1);
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
  auto kern = qgemm_mid_kernel<WK, EPI, MP>;
  if (set_smem_optin(reinterpret_cast<const void*>(kern), L::smem()) != KSH_OK) return KSH_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.ctas), static_cast<unsigned>(p.splits), 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::smem();
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;      // the splits of a CTA's tiles = one cluster
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(p.splits);
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mxh, mxl, mw, t);
  if (e == cudaSuccess) count_launch();
  return e == cudaSuccess ? KSH_OK : record_cuda_error(e);
}

template <int WK, int EPI>
int launch_mid_m(const LinArgs& a, char* ws, cudaStream_t stream) {
  if (a.m <= 32) return launch_mid<WK, EPI, 32>(a, ws, stream);
  return launch_mid<WK, EPI, 64>(a, ws, stream);
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
