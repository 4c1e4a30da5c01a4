// lm_head for batches of rows on tcgen05 tensor cores: fused final RMSNorm,
// fp32-accurate GEMM against the [vocab, hidden] weight, optional logits and
// the greedy first-index argmax.
//
// Replaces, for a decode step over many sequences (and for the L-row logits of
// the drop-in forward), the final norm, the fp32 lm_head and torch.argmax of
// the reference (engine/model.py:150-151, 187, 200).  The fp32 product is
// carried by fp16 tensor-core MMAs on split operands:
//
// * the weight is split once (ksh_lm_head_split_weight): per vocabulary row
//   a power-of-two scale 2^s puts max |w| * 2^s in [2^14, 2^15), and
//   w * 2^s = hi + lo with hi = fp16(w * 2^s), lo = fp16(w * 2^s - hi);
//   inv[v] = 2^-s.  The two fp16 matrices take the fp32 weight's 4 bytes per
//   element, so one launch streams the same bytes as the fp32 GEMV;
// * x is split per call the same way per batch row (split_x: RMSNorm folded
//   in, 2^e row scale);
// * per 128-row vocabulary tile and K step of 16, two MMAs accumulate in one
//   TMEM tile: W_hi x [x_hi | x_lo] (N = 128: columns 0..63 take x_hi, 64..127
//   x_lo) and W_lo x x_hi (N = 64, into columns 0..63).  Only lo * lo (about
//   2^-22 of the product) is dropped; logit = (col c + col 64 + c) * 2^-s * 2^-e;
// * each K chunk of 256 goes to a fresh (double-buffered) TMEM accumulator
//   and the epilogue warps add the chunks in fp32 registers, so no tensor-core
//   accumulation chain is longer than 16 MMA steps;
// * swap-AB: vocabulary rows are the MMA's M side (TMEM lanes), the 64 batch
//   rows (zero-filled by TMA past m) its N side;
// * persistent CTAs (one per SM) loop over vocabulary tiles; warp 0 streams
//   the weight tiles and the x tiles (L2-resident) by TMA through a 4-stage
//   ring, one thread of warp 1 issues the MMAs, four epilogue warps read the
//   double-buffered TMEM accumulator, store logits (coalesced along the
//   vocabulary) and keep each batch row's first-index maximum, as an ordered
//   integer key and a warp max-reduce;
// * per-CTA (key, index) partials are reduced by the last CTA to finish.
//
// Every mbarrier wait is bounded; a wait that gives up sets the workspace
// error word, the CTA unwinds (letting its copies and MMAs land before the
// TMEM is released) and the last CTA writes token -1 for every row.

#include <cudaTypedefs.h>
#include <float.h>

#include <algorithm>

#include "linear.cuh"
#include "tc_common.cuh"

namespace ksh {

int launch_split_x(const LinArgs& a, char* ws, bool perm, __half** xh, __half** xl, float** inv,
                   cudaStream_t stream);
int64_t split_x_workspace_size(int64_t m, int64_t k);

namespace {

using namespace tc;

constexpr int BV = 128;                 // vocabulary rows per tile (MMA M)
constexpr int BK = 64;                  // K per stage (one 128-byte fp16 row)
constexpr int MP = 64;                  // batch rows per launch (MMA N per term)
constexpr int NS = 4;                   // pipeline stages
constexpr int kThreads = 192;           // warp 0 TMA, warp 1 MMA, warps 2..5 epilogue
constexpr int A_TILE = BV * BK * 2;     // 16 KB
constexpr int X_TILE = MP * BK * 2;     // 8 KB
constexpr int STAGE = 2 * A_TILE + 2 * X_TILE;
constexpr int RING = NS * STAGE;
constexpr int BAR_OFF = RING;
constexpr int SMEM = 1024 + RING + 1024;
constexpr uint32_t TMEM_COLS = 2 * 2 * MP;   // two buffers of [x_hi cols | x_lo cols]
constexpr uint32_t kPolls = 1u << 22;
constexpr int PROMO = 4;                // K stages per TMEM accumulator chunk (K = 256)

struct TcArgs {
  const float* x_inv;      // [m_total] 2^-e per batch row (split_x), rows r0 ..
  const float* w_inv;      // [vocab] 2^-s per vocabulary row
  float* logits;           // [m, vocab] (rows r0 ..) or nullptr
  int64_t* tokens;         // [m] or nullptr
  uint32_t* part_key;      // [gridDim.x, MP]
  int32_t* part_idx;
  uint32_t* counter;       // zero on entry (cleared by the entry point)
  uint32_t* error;
  int m;                   // rows of this launch (<= MP)
  int r0;                  // first batch row of this launch in the split x
  int k;
  int vocab;
  int ntiles;
};

// Barrier over the 128 epilogue threads (named barrier 1) that also ORs a
// predicate across them, so that every one of them takes the same branch.
__device__ __forceinline__ bool epi_bar_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}

// Order-preserving key of a float (larger float -> larger key; -0 == +0; a
// NaN compares above +inf, as torch.argmax takes NaN as the maximum).
__device__ __forceinline__ uint32_t fkey(float v) {
  const uint32_t b = __float_as_uint(v + 0.0f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void __launch_bounds__(kThreads, 1)
lm_tc_kernel(const __grid_constant__ CUtensorMap map_wh, const __grid_constant__ CUtensorMap map_wl,
             const __grid_constant__ CUtensorMap map_xh, const __grid_constant__ CUtensorMap map_xl,
             TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* full = bars;               // [NS] weight + x tiles landed
  uint64_t* empty = full + NS;         // [NS] MMAs done with the stage
  uint64_t* acc_full = empty + NS;     // [2] tile accumulated
  uint64_t* acc_empty = acc_full + 2;  // [2] epilogue read the accumulator
  uint64_t* drained = acc_empty + 2;   // [1] every MMA of this CTA completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ uint32_t cand_key[2][4][MP];
  __shared__ int32_t cand_idx[2][4][MP];
  __shared__ float xinv_s[MP];
  __shared__ bool is_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = (a.k + BK - 1) / BK;
  const int my_tiles = a.ntiles > static_cast<int>(blockIdx.x)
                           ? (a.ntiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                           : 0;
  const int total = my_tiles * kt;
  auto wh_tile = [&](int s) { return smem + s * STAGE; };
  auto wl_tile = [&](int s) { return smem + s * STAGE + A_TILE; };
  auto xh_tile = [&](int s) { return smem + s * STAGE + 2 * A_TILE; };   // x_lo follows x_hi

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(drained, 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&map_wh);
    prefetch_tmap(&map_wl);
    prefetch_tmap(&map_xh);
    prefetch_tmap(&map_xl);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      auto tile_of = [&](int q) { return static_cast<int>(blockIdx.x) + (q / kt) * static_cast<int>(gridDim.x); };
      auto issue_w = [&](int q) {
        const int s = q % NS;
        mbar_arrive_expect_tx(&full[s], STAGE);
        const int k0 = (q % kt) * BK, v0 = tile_of(q) * BV;
        tma_load_2d(wh_tile(s), &map_wh, &full[s], k0, v0);
        tma_load_2d(wl_tile(s), &map_wl, &full[s], k0, v0);
      };
      auto issue_x = [&](int q) {
        const int s = q % NS;
        const int k0 = (q % kt) * BK;
        tma_load_2d(xh_tile(s), &map_xh, &full[s], k0, a.r0);
        tma_load_2d(xh_tile(s) + X_TILE, &map_xl, &full[s], k0, a.r0);
      };
      const int pre = min(NS, total);
      // the weight split is constant: its first stages go out before the
      // dependency wait; x comes from the split kernel just before
      for (int q = 0; q < pre; ++q) issue_w(q);
      grid_dep_wait();
      grid_dep_launch();
      for (int q = 0; q < pre; ++q) issue_x(q);
      int issued = pre;
      for (int q = pre; q < total && !*abort_flag; ++q) {
        const int s = q % NS;
        if (!mbar_wait(&empty[s], ((q / NS) - 1) & 1, kPolls)) {
          *abort_flag = 1;
          break;
        }
        issue_w(q);
        issue_x(q);
        issued = q + 1;
      }
      if (*abort_flag)      // let the copies in flight land before the CTA exits
        for (int q = max(0, issued - NS); q < issued; ++q) mbar_wait(&full[q % NS], (q / NS) & 1, kPolls);
    } else {
      grid_dep_wait();
      grid_dep_launch();
    }
  } else if (warp == 1) {
    // ---------------- MMA issue ----------------
    grid_dep_wait();
    grid_dep_launch();
    if (lane == 0) {
      constexpr uint32_t idesc_hl = idesc_f16_f32(BV, 2 * MP);   // W_hi x [x_hi | x_lo]
      constexpr uint32_t idesc_h = idesc_f16_f32(BV, MP);        // W_lo x x_hi
      int q = 0;
      // The tile's K range runs in chunks of PROMO stages, each into a fresh
      // TMEM accumulator (double-buffered); the epilogue adds the chunks in
      // fp32 registers.  The tensor core's accumulation over a long K chain
      // loses low bits (measured: 3e-5 of the largest logit over K = 4096 in
      // one accumulator); over 16 MMA steps per chunk it stays near 1e-6.
      const int nch = (kt + PROMO - 1) / PROMO;
      int g = 0;
      bool ok = true;
      for (int t = 0; t < my_tiles && ok; ++t) {
        for (int ch = 0; ch < nch && ok; ++ch, ++g) {
          const int buf = g & 1;
          if (*abort_flag || (g >= 2 && !mbar_wait(&acc_empty[buf], ((g >> 1) - 1) & 1, kPolls))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + static_cast<uint32_t>(buf * 2 * MP);
          const int k_end = min(kt, (ch + 1) * PROMO);
          for (int kk = ch * PROMO; kk < k_end; ++kk, ++q) {
            const int s = q % NS;
            if (*abort_flag || !mbar_wait(&full[s], (q / NS) & 1, kPolls)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t ah = desc_k_sw128(smem_u32(wh_tile(s)));
            const uint64_t al = desc_k_sw128(smem_u32(wl_tile(s)));
            const uint64_t bx = desc_k_sw128(smem_u32(xh_tile(s)));
#pragma unroll
            for (int k16 = 0; k16 < BK / 16; ++k16) {
              mma_f16(d, ah + 2 * k16, bx + 2 * k16, idesc_hl,
                      (kk > ch * PROMO || k16 > 0) ? 1u : 0u);
              mma_f16(d, al + 2 * k16, bx + 2 * k16, idesc_h, 1u);
            }
            mma_commit(&empty[s]);
          }
          if (ok) mma_commit(&acc_full[buf]);
        }
      }
      if (!ok) *abort_flag = 1;
      // every MMA of this thread completes before the TMEM is released
      mma_commit(drained);
      mbar_wait(drained, 0, kPolls);
    }
  } else {
    // ---------------- epilogue (128 threads, TMEM lane = vocabulary row) ----------------
    grid_dep_wait();
    grid_dep_launch();
    const int et = threadIdx.x - 64;                 // 0 .. 127
    const int quad = warp & 3;                       // TMEM lane quadrant of this warp
    const int row = quad * 32 + lane;
    if (et < MP) xinv_s[et] = et < a.m ? a.x_inv[a.r0 + et] : 0.0f;
    epi_bar_or(false);
    uint32_t best_key = 0u;                          // thread et < m keeps batch row et
    int32_t best_idx = INT32_MAX;
    const int nch = (kt + PROMO - 1) / PROMO;
    int g = 0;
    bool ok = true;
    for (int t = 0; t < my_tiles && ok; ++t) {
      const int tile = static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x);
      // columns 0..63: W_hi x_hi + W_lo x_hi; 64..127: W_hi x_lo, summed over
      // the tile's K chunks in registers
      float acc[MP];
#pragma unroll
      for (int c = 0; c < MP; ++c) acc[c] = 0.0f;
      for (int ch = 0; ch < nch; ++ch, ++g) {
        const int buf = g & 1;
        // all 128 threads agree on giving up, so none is left at a barrier
        const bool fail = *abort_flag || !mbar_wait(&acc_full[buf], (g >> 1) & 1, kPolls);
        if (epi_bar_or(fail)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem + static_cast<uint32_t>(buf * 2 * MP) + (static_cast<uint32_t>(quad * 32) << 16);
#pragma unroll
        for (int half = 0; half < MP / 32; ++half) {
          float vh[32], vl[32];                      // valid only after tcgen05.wait::ld
          tmem_ld_32x32b_x32(taddr + half * 32, vh);
          tmem_ld_32x32b_x32(taddr + MP + half * 32, vl);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[half * 32 + e] += vh[e] + vl[e];
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);                // the accumulator may be overwritten
      }
      if (!ok) break;
      const int v = tile * BV + row;
      const bool live = v < a.vocab;
      const float winv = live ? a.w_inv[v] : 0.0f;
      const int cb = t & 1;
#pragma unroll
      for (int c = 0; c < MP; ++c) {
        if (c < a.m) {
          const float val = acc[c] * (winv * xinv_s[c]);
          if (a.logits && live) a.logits[static_cast<int64_t>(c) * a.vocab + v] = val;
          const uint32_t key = live ? fkey(val) : 0u;
          const uint32_t wmax = __reduce_max_sync(0xffffffffu, key);
          const uint32_t hit = __ballot_sync(0xffffffffu, key == wmax);
          if (lane == __ffs(hit) - 1) {              // lowest lane = lowest vocabulary index
            cand_key[cb][quad][c] = wmax;
            cand_idx[cb][quad][c] = v;
          }
        }
      }
      epi_bar_or(false);
      if (et < a.m) {
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {             // quadrants in increasing row order
          const uint32_t k2 = cand_key[cb][qd][et];
          const int32_t i2 = cand_idx[cb][qd][et];
          if (k2 > best_key || (k2 == best_key && i2 < best_idx)) {
            best_key = k2;
            best_idx = i2;
          }
        }
      }
      // candidates of tile t + 1 go to the other buffer; tile t + 2 reuses
      // this one only after the next barrier
    }
    if (!ok) *abort_flag = 1;
    if (a.tokens && et < a.m) {
      a.part_key[static_cast<int64_t>(blockIdx.x) * MP + et] = best_key;
      a.part_idx[static_cast<int64_t>(blockIdx.x) * MP + et] = best_idx;
    }
  }

  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) atomicOr(a.error, 1u);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  if (!a.tokens) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const bool failed = __ldcg(a.error) != 0u;
  for (int r = warp; r < a.m; r += kThreads / 32) {
    uint32_t bk = 0u;
    int32_t bi = INT32_MAX;
    for (int c = lane; c < static_cast<int>(gridDim.x); c += 32) {
      const uint32_t k2 = __ldcg(a.part_key + static_cast<int64_t>(c) * MP + r);
      const int32_t i2 = __ldcg(a.part_idx + static_cast<int64_t>(c) * MP + r);
      if (k2 > bk || (k2 == bk && i2 < bi)) {
        bk = k2;
        bi = i2;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint32_t ok2 = __shfl_xor_sync(0xffffffffu, bk, o);
      const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ok2 > bk || (ok2 == bk && oi < bi)) {
        bk = ok2;
        bi = oi;
      }
    }
    if (lane == 0) a.tokens[r] = failed ? -1 : bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    *a.counter = 0u;
    *a.error = 0u;
  }
}

// Weight split, one CTA per vocabulary row: 2^s from the row maximum, then
// hi = fp16(w * 2^s), lo = fp16(w * 2^s - hi).  Non-finite values set the
// status bit and split as zero.
__global__ void __launch_bounds__(256)
lm_split_weight_kernel(const float* __restrict__ w, int64_t k, __half* __restrict__ wh,
                       __half* __restrict__ wl, float* __restrict__ winv, int32_t* flags) {
  __shared__ float red[8];
  grid_dep_wait();
  grid_dep_launch();
  const int64_t r = blockIdx.x;
  const float* wr = w + r * k;
  float mx = 0.0f;
  bool bad = false;
  for (int64_t j = threadIdx.x; j < k; j += blockDim.x) {
    const float v = wr[j];
    if (!isfinite(v)) bad = true;
    else mx = fmaxf(mx, fabsf(v));
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) raise_flag(flags, KSH_FLAG_NONFINITE);
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = 0.0f;
  for (int i = 0; i < 8; ++i) mx = fmaxf(mx, red[i]);
  int e = 0;
  if (mx > 0.0f) {
    int ex;
    frexpf(mx, &ex);
    e = max(-100, min(15 - ex, 100));
  }
  const float sc = ldexpf(1.0f, e);
  if (threadIdx.x == 0) winv[r] = ldexpf(1.0f, -e);
  for (int64_t j = threadIdx.x; j < k; j += blockDim.x) {
    const float v0 = wr[j];
    const float v = isfinite(v0) ? v0 * sc : 0.0f;
    const __half h = __float2half_rn(v);
    wh[r * k + j] = h;
    wl[r * k + j] = __float2half_rn(v - __half2float(h));
  }
}

bool map_f16(CUtensorMap* m, const void* base, int64_t inner, int64_t outer, uint32_t box_outer) {
  return make_tensor_map_2d(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, base, static_cast<uint64_t>(inner),
                            static_cast<uint64_t>(outer), static_cast<uint64_t>(inner) * 2, BK,
                            box_outer, CU_TENSOR_MAP_SWIZZLE_128B);
}

int64_t tc_grid(int64_t vocab) {
  const int64_t tiles = (vocab + BV - 1) / BV;
  return std::min<int64_t>(tiles, num_sms());
}

// ws: [0, 4) counter, [4, 8) error, [256, 256 + grid * MP * 8) partials, then the x split
int64_t part_bytes(int64_t vocab) { return (256 + tc_grid(vocab) * MP * 8 + 255) / 256 * 256; }

}  // namespace
}  // namespace ksh

using namespace ksh;

extern "C" int64_t ksh_lm_head_tc_workspace_size(int64_t m, int64_t hidden, int64_t vocab) {
  if (m <= 0 || hidden <= 0 || vocab <= 0) return 0;
  return part_bytes(vocab) + split_x_workspace_size(m, hidden);
}

extern "C" int ksh_lm_head_split_weight(const float* w, int64_t vocab, int64_t hidden,
                                        void* w_hi, void* w_lo, float* w_inv, int32_t* flags,
                                        void* stream) {
  KSH_CHECK_ARG(vocab > 0 && vocab <= INT32_MAX && hidden > 0 && w && w_hi && w_lo && w_inv);
  return launch(lm_split_weight_kernel, dim3(static_cast<unsigned>(vocab)), dim3(256), 0,
                static_cast<cudaStream_t>(stream), w, hidden, static_cast<__half*>(w_hi),
                static_cast<__half*>(w_lo), w_inv, flags);
}

extern "C" int ksh_lm_head_argmax_tc(const float* x, int64_t m, int64_t hidden,
                                     const float* norm_w, float norm_eps, const void* w_hi,
                                     const void* w_lo, const float* w_inv, int64_t vocab,
                                     float* logits, int64_t* tokens, void* workspace,
                                     int64_t workspace_bytes, void* stream) {
  KSH_CHECK_ARG(m >= 0 && m <= INT32_MAX && hidden > 0 && hidden <= INT32_MAX && vocab > 0 &&
                vocab <= INT32_MAX - BV && x && w_hi && w_lo && w_inv);
  KSH_CHECK_ARG(logits || tokens);
  if (m == 0) return KSH_OK;
  if (hidden % 8 != 0) return KSH_ERR_UNSUPPORTED;          // fp16 rows on 16-byte strides
  if (((reinterpret_cast<uintptr_t>(w_hi) | reinterpret_cast<uintptr_t>(w_lo)) & 15) != 0)
    return KSH_ERR_ALIGN;
  if (!tensor_map_encoder_available()) return KSH_ERR_UNSUPPORTED;
  const int64_t need = ksh_lm_head_tc_workspace_size(m, hidden, vocab);
  if (!workspace || workspace_bytes < need) return KSH_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return KSH_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const int64_t pb = part_bytes(vocab);
  // x -> (RMSNorm) -> 2^e (hi + lo), all m rows at once
  LinArgs la = {};
  la.x = x;
  la.m = m;
  la.k = hidden;
  la.kp = hidden;
  la.n = vocab;
  la.norm_w = norm_w;
  la.norm_eps = norm_eps;
  // Completion counter and error word start at zero whatever the workspace
  // held; each launch's last CTA leaves them at zero for the next chunk.
  const cudaError_t e = cudaMemsetAsync(ws, 0, 8, s);
  if (e != cudaSuccess) return record_cuda_error(e);
  __half *xh = nullptr, *xl = nullptr;
  float* xinv = nullptr;
  int st = launch_split_x(la, ws + pb, false, &xh, &xl, &xinv, s);
  if (st != KSH_OK) return st;
  CUtensorMap mwh, mwl, mxh, mxl;
  if (!map_f16(&mwh, w_hi, hidden, vocab, BV) || !map_f16(&mwl, w_lo, hidden, vocab, BV) ||
      !map_f16(&mxh, xh, hidden, m, MP) || !map_f16(&mxl, xl, hidden, m, MP))
    return KSH_ERR_UNSUPPORTED;
  if (set_smem_optin(reinterpret_cast<const void*>(lm_tc_kernel), SMEM) != KSH_OK)
    return KSH_ERR_CUDA;
  const int64_t grid = tc_grid(vocab);
  for (int64_t r0 = 0; r0 < m; r0 += MP) {
    TcArgs a = {};
    a.x_inv = xinv;
    a.w_inv = w_inv;
    a.logits = logits ? logits + r0 * vocab : nullptr;
    a.tokens = tokens ? tokens + r0 : nullptr;
    a.counter = reinterpret_cast<uint32_t*>(ws);
    a.error = reinterpret_cast<uint32_t*>(ws + 4);
    a.part_key = reinterpret_cast<uint32_t*>(ws + 256);
    a.part_idx = reinterpret_cast<int32_t*>(ws + 256 + grid * MP * 4);
    a.m = static_cast<int>(std::min<int64_t>(MP, m - r0));
    a.r0 = static_cast<int>(r0);
    a.k = static_cast<int>(hidden);
    a.vocab = static_cast<int>(vocab);
    a.ntiles = static_cast<int>((vocab + BV - 1) / BV);
    st = launch(lm_tc_kernel, dim3(static_cast<unsigned>(grid)), dim3(kThreads), SMEM, s, mwh, mwl,
                mxh, mxl, a);
    if (st != KSH_OK) return st;
  }
  return KSH_OK;
}
