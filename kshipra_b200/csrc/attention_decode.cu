// K6 + K7 fused: decode-step attention (one new token per sequence).
//
// Replaces, for the decode step of KshipraModel.forward, the RoPE at the
// token's absolute position (engine/model.py:47-55, 108, 121), the K/V write
// into the block pool (model.py:123-129) and chunked_attention with
// chunk_len = 1 (engine/chunked_prefill.py:93-140).
//
// One thread-block cluster per (sequence, kv head); its CTAs split the key
// range (tiles of 16 positions) evenly at run time from the sequence's
// current length.  Inside a CTA the warps specialise:
//
// * warp 0 streams the CTA's K/V tiles into a ring of shared-memory stages
//   with TMA (full / empty mbarrier pair per stage); the first stages are
//   requested BEFORE the programmatic-launch wait: those pool rows belong to
//   earlier positions, written by kernels that have completed (every kernel
//   of this library triggers its dependents only after its own wait), so the
//   K/V fetch overlaps the q/k/v projection still running;
// * after the wait all warps rotate the g query heads of the group; the CTA
//   holding the last tile also rotates k and writes k and v to the pool (for
//   later steps);
// * consumer warps 1..2 take whole tiles round-robin, each with its own
//   online-softmax state: scores (q . k) / sqrt(D) with the causal bound, the
//   reference's merge (running max with m_safe, exp, rescale) and P.V.  A
//   tile needs no CTA-wide barrier, so tiles of different warps overlap; the
//   warp holding the new token's tile patches that row in shared memory;
// * the warps' (m, l, acc) are merged per CTA, and the CTAs' in rank order
//   through distributed shared memory by cluster rank 0, which writes the
//   output.
//
// Bounds: block ids outside [0, num_blocks) raise KSH_FLAG_BAD_BLOCK (those
// keys are skipped); positions outside the RoPE table raise
// KSH_FLAG_BAD_POSITION; slots outside the pool KSH_FLAG_BAD_SLOT.  Every
// mbarrier wait is bounded (KSH_FLAG_TIMEOUT).

#include <math.h>
#include <stdlib.h>

#include <algorithm>

#include "tc_common.cuh"

namespace ksh {
namespace {

using namespace tc;

constexpr int kTK = 16;                          // keys per tile
constexpr int kConsumers = 2;                    // consumer warps per CTA
constexpr int kThreads = 32 * (kConsumers + 1);  // + the TMA producer warp
constexpr int kMaxCluster = 8;
// three CTAs per SM: 2 consumers and a 64 KB ring per CTA streamed 0.90 of
// measured HBM at the Llama-3-8B shape, 3 consumers and 96 KB (two CTAs per
// SM) 0.83, 2 consumers and 96 KB 0.71
constexpr int kRingBytes = 64 * 1024;

// 0: cluster size chosen per launch; KSH_DECODE_SPLIT=1..8 in the environment forces it
int g_forced_split = [] {
  const char* v = getenv("KSH_DECODE_SPLIT");
  const int c = (v && *v) ? atoi(v) : 0;
  return c >= 1 && c <= 8 ? c : 0;
}();

struct DecArgs {
  const float* qkv;          // [B, (hq + 2 hkv) * d]
  const int64_t* positions;  // [B]
  const int64_t* slots;      // [B]
  const float* rcos;         // [max_pos, d/2]
  const float* rsin;
  float* pool;               // [nb, L, 2, hkv, bs, d]
  const int32_t* block_tables;
  float* out;                // [B, hq, d]
  int32_t* flags;
  float* gpart;              // key split without a cluster: [items][splits][G][D + 4] partial states
  uint32_t* gcount;          // [items] CTAs finished per item (zero between launches)
  int64_t max_pos, num_blocks, num_layers, layer, hkv, hq, bs, max_blocks;
  int g;
  float scale;
};

// Staged K / V tiles: 16 rows x D floats as D/32 TMA boxes of 16 rows x 128 B,
// 128B-swizzled (16-byte chunk c of row r at chunk c ^ (r & 7)).  Float offset
// of float4 column d4 of row r:
template <int D>
__device__ __forceinline__ int tile_off(int r, int d4) {
  return (d4 >> 3) * (kTK * 32) + r * 32 + (((d4 & 7) ^ (r & 7)) << 2);
}

template <int D, int G>
struct DecLayout {
  static constexpr int D4 = D / 4;
  static constexpr int TILE_F = kTK * D;                 // floats per K (or V) tile
  static constexpr int STAGE_F = 2 * TILE_F;             // K tile then V tile
  // 4 stages (D 128) / 8 (D 64), a multiple of the consumer count: tile i
  // sits in stage i % NST and belongs to consumer i % kConsumers, so each
  // stage is only ever read by one consumer, which waits on it again only
  // after releasing it -- its full barrier is never more than one phase
  // behind that wait (with stages shared between consumers a fast consumer
  // could meet the completed phase of the stage's fill before last, which
  // has the same parity).
  static constexpr int NST = kRingBytes / (STAGE_F * 4) / kConsumers * kConsumers;
  static constexpr int QS = D + 4;                       // padded q row (odd heads, other banks)
  static constexpr int GP = (G + 3) & ~3;                // padded probability row
  static constexpr int PW = (kTK + 1) * GP;              // per-warp probabilities + corr row
  static constexpr int RING_F = NST * STAGE_F;
  static constexpr int Q_OFF = RING_F;
  static constexpr int P_OFF = Q_OFF + G * QS;
  static constexpr int BAR_OFF = P_OFF + kConsumers * PW; // floats, then 2 NST mbarriers
  static constexpr size_t SMEM = (BAR_OFF + 2 * NST * 2) * 4 + 1024;
  // after the main loop the ring holds the warps' states [kConsumers][G][D+4]
  // and, on cluster rank 0, every rank's state [kMaxCluster][G][D+4]
  static constexpr int WST_F = kConsumers * G * (D + 4);
  static constexpr int PART_F = kMaxCluster * G * (D + 4);
  static_assert(NST >= 2 * kConsumers && NST % kConsumers == 0, "stages per consumer");
  static_assert(WST_F + PART_F <= RING_F, "merge areas fit the ring");
  static_assert(BAR_OFF % 2 == 0 && Q_OFF % 4 == 0 && P_OFF % 4 == 0, "alignment");
};

// GS: the key split runs over independent CTAs (gridDim.x of them per item)
// instead of a cluster; each CTA leaves its state in a.gpart and the last of
// an item to finish (a.gcount) merges them in split order and writes the
// output.  Any split count then fills the SMs' resident slots, which a
// cluster split, tied to cluster placement, does not.
template <int D, int G, bool GS>
__global__ void __launch_bounds__(kThreads, 3)
decode_attn_kernel(const __grid_constant__ CUtensorMap pool_map, DecArgs a) {
  using Ly = DecLayout<D, G>;
  constexpr int D4 = Ly::D4, TILE_F = Ly::TILE_F, STAGE_F = Ly::STAGE_F, NST = Ly::NST;
  constexpr int QS = Ly::QS, GP = Ly::GP;
  constexpr int GH = (G + 1) / 2;        // heads per lane in the score phase
  constexpr int NACC = GH == 1 ? 4 : (GH == 2 ? 2 : 1);  // independent partial sums per head
  // D 128 with 4 heads per group (the Llama-3-8B shape): lanes split D instead
  // of keys for q.k (see the consumer loop)
  constexpr bool kBfly = D == 128 && G == 4;
  extern __shared__ __align__(128) float4 sm4[];
  // TMA 128B-swizzled destinations need 1024-byte alignment
  float* sm = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(sm4) + 1023) & ~uintptr_t(1023));
  float* ring = sm;                                   // [NST][K tile, V tile]
  float* Qs = sm + Ly::Q_OFF;                         // [G][QS]
  float* Ps = sm + Ly::P_OFF;                         // [kConsumers][kTK + 1][GP]
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Ly::BAR_OFF);   // [NST]
  uint64_t* empty = full + NST;                                     // [NST]
  __shared__ int tile_ok[NST];
  __shared__ float newk[D], newv[D];
  __shared__ int fail_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t rank = GS ? blockIdx.x : cluster_rank();
  const uint32_t csize = GS ? gridDim.x : cluster_size();
  const int item = blockIdx.y;                  // (b, hk)
  const int b = item / static_cast<int>(a.hkv);
  const int hk = item - b * static_cast<int>(a.hkv);

  // ---- sequence state (written by kernels that completed before this one started) ----
  const int64_t p = a.positions[b];
  const int total = static_cast<int>(p) + 1;                       // keys 0..p
  const int64_t cap = a.max_blocks * a.bs;
  const int total_c = static_cast<int>(min(static_cast<int64_t>(total), cap));
  const int ntiles = (total_c + kTK - 1) / kTK;
  const int tpc = (ntiles + static_cast<int>(csize) - 1) / static_cast<int>(csize);
  const int t_begin = static_cast<int>(rank) * tpc;
  const int t_end = min(t_begin + tpc, ntiles);
  const int ntl = max(t_end - t_begin, 0);
  const int64_t head_rows = a.hkv * a.bs;                         // rows between K and V
  const int32_t* bt = a.block_tables + static_cast<int64_t>(b) * a.max_blocks;

  // The producer lane stages local tile i into stage i % NST (D/32 boxes for
  // K and for V); an out-of-range block id marks the tile bad instead.
  auto issue = [&](int i) {
    const int s = i % NST;
    const int t = t_begin + i;
    const int64_t j = (static_cast<int64_t>(t) * kTK) / a.bs;
    const int64_t off = static_cast<int64_t>(t) * kTK - j * a.bs;
    const int64_t blk = j < a.max_blocks ? bt[j] : -1;
    if (blk < 0 || blk >= a.num_blocks) {
      tile_ok[s] = 0;
      mbar_arrive(&full[s]);
      return;
    }
    tile_ok[s] = 1;
    const int krow = static_cast<int>((((blk * a.num_layers + a.layer) * 2) * a.hkv + hk) * a.bs + off);
    const int vrow = krow + static_cast<int>(head_rows);
    float* st = ring + s * STAGE_F;
    mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(STAGE_F * 4));
#pragma unroll
    for (int cb = 0; cb < D / 32; ++cb) {
      tma_load_2d(st + cb * kTK * 32, &pool_map, &full[s], cb * 32, krow);
      tma_load_2d(st + TILE_F + cb * kTK * 32, &pool_map, &full[s], cb * 32, vrow);
    }
  };

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fail_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&pool_map);
    for (int i = 0; i < ntl && i < NST; ++i) issue(i);
  }

  grid_dep_wait();
  grid_dep_launch();

  // ---- RoPE of q (and of k for the owner of the last tile) ----
  const bool owner = ntl > 0 && t_end == ntiles && total == total_c;
  const int half = D / 2;
  int64_t pr = p;
  if (pr < 0 || pr >= a.max_pos) {
    if (tid == 0 && rank == 0) raise_flag(a.flags, KSH_FLAG_BAD_POSITION);
    pr = 0;
  }
  if (total != total_c && tid == 0 && rank == 0) raise_flag(a.flags, KSH_FLAG_BAD_LENGTH);
  const float* cr = a.rcos + pr * half;
  const float* sr = a.rsin + pr * half;
  const float* row = a.qkv + static_cast<int64_t>(b) * (a.hq + 2 * a.hkv) * D;
  for (int i = tid; i < (G + (owner ? 1 : 0)) * half; i += kThreads) {
    const int h = i / half, j = i - h * half;
    const float* src = h < G ? row + (static_cast<int64_t>(hk) * G + h) * D
                             : row + (a.hq + hk) * D;
    const float x1 = src[j], x2 = src[j + half];
    const float c = cr[j], s = sr[j];
    const float o1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(-x2, s));
    const float o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    if (h < G) {
      Qs[h * QS + j] = o1;
      Qs[h * QS + j + half] = o2;
    } else {
      newk[j] = o1;
      newk[j + half] = o2;
    }
  }
  if (owner) {
    const float* vsrc = row + (a.hq + a.hkv + hk) * D;
    for (int j = tid; j < D; j += kThreads) newv[j] = vsrc[j];
  }
  __syncthreads();
  if (owner) {
    const int64_t slot = a.slots[b];
    const int64_t sblk = slot >= 0 ? slot / a.bs : -1;
    if (sblk >= 0 && sblk < a.num_blocks) {
      float* kd = a.pool + ((((sblk * a.num_layers + a.layer) * 2) * a.hkv + hk) * a.bs + slot % a.bs) * D;
      float* vd = kd + head_rows * D;
      for (int j = tid; j < D; j += kThreads) {
        kd[j] = newk[j];
        vd[j] = newv[j];
      }
    } else if (tid == 0) {
      raise_flag(a.flags, KSH_FLAG_BAD_SLOT);
    }
  }

  const int cw = warp - 1;                       // consumer index (warp 0 produces)
  float4 acc[G];
#pragma unroll
  for (int h = 0; h < G; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
  float m_run[GH], l_run[GH];
#pragma unroll
  for (int u = 0; u < GH; ++u) {
    m_run[u] = -INFINITY;
    l_run[u] = 0.0f;
  }

  if (warp == 0) {
    // ---- producer: refill each stage once its consumer released it ----
    if (lane == 0) {
      for (int i = NST; i < ntl; ++i) {
        if (!mbar_wait(&empty[i % NST], ((i / NST) - 1) & 1)) {
          atomicOr(&fail_s, 1);
          break;
        }
        issue(i);
      }
    }
  } else {
    // ---- consumers: warp cw takes tiles cw, cw + kConsumers, ... ----
    const int r = lane & (kTK - 1), hg = lane >> 4;
    float* P = Ps + cw * Ly::PW;
    bool bad = false;
    float4 qf[kBfly ? G : 1];                    // this lane's 4-float column of every head's q
    if constexpr (kBfly) {
#pragma unroll
      for (int h = 0; h < G; ++h) qf[h] = *reinterpret_cast<const float4*>(Qs + h * QS + 4 * lane);
    }
    for (int i = cw; i < ntl; i += kConsumers) {
      const int s = i % NST;
      const bool arrived = mbar_wait(&full[s], (i / NST) & 1);
      if (__any_sync(0xffffffffu, !arrived)) {   // warp-uniform exit (shuffles below)
        if (lane == 0) atomicOr(&fail_s, 1);
        break;
      }
      float* Kt = ring + s * STAGE_F;
      float* Vt = Kt + TILE_F;
      const bool ok = tile_ok[s] != 0;
      bad |= !ok;
      if (owner && i == ntl - 1) {               // the new token's row, possibly stale in the pool copy
        const int rr = static_cast<int>(p) - (t_begin + i) * kTK;
        for (int j = lane; j < D; j += 32) {
          Kt[tile_off<D>(rr, j >> 2) + (j & 3)] = newk[j];
          Vt[tile_off<D>(rr, j >> 2) + (j & 3)] = newv[j];
        }
        __syncwarp();
      }
      if constexpr (kBfly) {
        // scores: lane -> 4-float column slice of D for all 16 keys x 4 heads
        // (q in registers, one conflict-free K row read per key); the 64
        // partial dot products are summed over the warp by a reduce-scatter
        // butterfly (round m keeps the half of the values that lane bit m
        // selects) that leaves lane l head l >> 3 at keys 2 (l & 7) + {0, 1}
        float v[4 * kTK];
#pragma unroll
        for (int rr = 0; rr < kTK; ++rr) {
          const float4 kv = *reinterpret_cast<const float4*>(Kt + tile_off<D>(rr, lane));
#pragma unroll
          for (int h = 0; h < 4; ++h)
            v[h * kTK + rr] = fmaf(qf[h].x, kv.x, fmaf(qf[h].y, kv.y, fmaf(qf[h].z, kv.z, qf[h].w * kv.w)));
        }
#pragma unroll
        for (int rd = 0; rd < 5; ++rd) {
          const int m = 16 >> rd, half = 32 >> rd;
          const bool upper = (lane & m) != 0;
#pragma unroll
          for (int j = 0; j < half; ++j) {
            const float keep = upper ? v[j + half] : v[j];
            const float send = upper ? v[j] : v[j + half];
            v[j] = keep + __shfl_xor_sync(0xffffffffu, send, m);
          }
        }
        // online softmax of head hh over the tile's keys (8 lanes x 2 keys)
        const int hh = lane >> 3, r0 = 2 * (lane & 7);
        const int kb = (t_begin + i) * kTK;
        const float s0 = (ok && kb + r0 < total_c) ? v[0] * a.scale : -INFINITY;
        const float s1 = (ok && kb + r0 + 1 < total_c) ? v[1] * a.scale : -INFINITY;
        float tmax = fmaxf(s0, s1);
#pragma unroll
        for (int o = 4; o >= 1; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
        const float m_new = fmaxf(m_run[0], tmax);
        const float m_safe = isinf(m_new) ? 0.0f : m_new;
        const float p0 = expf(s0 - m_safe), p1 = expf(s1 - m_safe);
        float psum = p0 + p1;
#pragma unroll
        for (int o = 4; o >= 1; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
        const float corr = expf(m_run[0] - m_safe);
        l_run[0] = __fadd_rn(__fmul_rn(l_run[0], corr), psum);
        m_run[0] = m_new;
        P[r0 * GP + hh] = p0;
        P[(r0 + 1) * GP + hh] = p1;
        if ((lane & 7) == 0) P[kTK * GP + hh] = corr;
      } else {
        const bool valid = ok && (t_begin + i) * kTK + r < total_c;
        // scores: lane -> key r, heads hg, hg + 2, ...
        float dot[GH][NACC];
#pragma unroll
        for (int u = 0; u < GH; ++u)
#pragma unroll
          for (int e = 0; e < NACC; ++e) dot[u][e] = 0.0f;
#pragma unroll
        for (int d4 = 0; d4 < D4; ++d4) {
          const float4 kv = *reinterpret_cast<const float4*>(Kt + tile_off<D>(r, d4));
#pragma unroll
          for (int u = 0; u < GH; ++u) {
            const int h = hg + 2 * u;
            if (G % 2 == 0 || h < G) {
              const float4 qv = *reinterpret_cast<const float4*>(Qs + h * QS + 4 * d4);
              float& dd = dot[u][d4 % NACC];
              dd = fmaf(qv.x, kv.x, dd);
              dd = fmaf(qv.y, kv.y, dd);
              dd = fmaf(qv.z, kv.z, dd);
              dd = fmaf(qv.w, kv.w, dd);
            }
          }
        }
        // online softmax over the tile's 16 keys (the lanes of one half-warp)
#pragma unroll
        for (int u = 0; u < GH; ++u) {
          const int h = hg + 2 * u;
          float sc = dot[u][0];
#pragma unroll
          for (int e = 1; e < NACC; ++e) sc += dot[u][e];
          const float sv = (valid && h < G) ? sc * a.scale : -INFINITY;
          float tmax = sv;
#pragma unroll
          for (int o = 8; o >= 1; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
          const float m_new = fmaxf(m_run[u], tmax);
          const float m_safe = isinf(m_new) ? 0.0f : m_new;
          const float pj = expf(sv - m_safe);
          float psum = pj;
#pragma unroll
          for (int o = 8; o >= 1; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
          const float corr = expf(m_run[u] - m_safe);
          l_run[u] = __fadd_rn(__fmul_rn(l_run[u], corr), psum);
          m_run[u] = m_new;
          if (h < G) {
            P[r * GP + h] = pj;
            if (r == 0) P[kTK * GP + h] = corr;
          }
        }
      }
      __syncwarp();
      // acc[h][c4] = acc * corr[h] + sum_keys p[h][key] V[key][c4]
      {
        float pr4[GP];
#pragma unroll
        for (int q = 0; q < GP / 4; ++q) {
          const float4 t = reinterpret_cast<const float4*>(P + kTK * GP)[q];
          pr4[4 * q] = t.x; pr4[4 * q + 1] = t.y; pr4[4 * q + 2] = t.z; pr4[4 * q + 3] = t.w;
        }
#pragma unroll
        for (int h = 0; h < G; ++h) {
          acc[h].x *= pr4[h];
          acc[h].y *= pr4[h];
          acc[h].z *= pr4[h];
          acc[h].w *= pr4[h];
        }
      }
      constexpr int KSTEP = D == 128 ? 1 : 2;    // D 64: the half-warps take alternate keys
      const int c4 = D == 128 ? lane : (lane & 15);
      const int k0 = D == 128 ? 0 : (lane >> 4);
#pragma unroll 4
      for (int kk = k0; kk < kTK; kk += KSTEP) {
        const float4 v = *reinterpret_cast<const float4*>(Vt + tile_off<D>(kk, c4));
        float pk[GP];
#pragma unroll
        for (int q = 0; q < GP / 4; ++q) {
          const float4 t = reinterpret_cast<const float4*>(P + kk * GP)[q];
          pk[4 * q] = t.x; pk[4 * q + 1] = t.y; pk[4 * q + 2] = t.z; pk[4 * q + 3] = t.w;
        }
#pragma unroll
        for (int h = 0; h < G; ++h) {
          acc[h].x = fmaf(pk[h], v.x, acc[h].x);
          acc[h].y = fmaf(pk[h], v.y, acc[h].y);
          acc[h].z = fmaf(pk[h], v.z, acc[h].z);
          acc[h].w = fmaf(pk[h], v.w, acc[h].w);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (D == 64) {
#pragma unroll
      for (int h = 0; h < G; ++h) {
        acc[h].x += __shfl_xor_sync(0xffffffffu, acc[h].x, 16);
        acc[h].y += __shfl_xor_sync(0xffffffffu, acc[h].y, 16);
        acc[h].z += __shfl_xor_sync(0xffffffffu, acc[h].z, 16);
        acc[h].w += __shfl_xor_sync(0xffffffffu, acc[h].w, 16);
      }
    }
    if (bad && lane == 0) atomicOr(&fail_s, 2);
  }
  __syncthreads();                               // every stage consumed: the ring is free
  if (tid == 0) {
    if (fail_s & 1) raise_flag(a.flags, KSH_FLAG_TIMEOUT);
    if (fail_s & 2) raise_flag(a.flags, KSH_FLAG_BAD_BLOCK);
  }

  // ---- per-CTA merge of the consumer warps' states ----
  float* wst = ring;                              // [kConsumers][G][D + 4]: m, l, pad, pad, acc
  if (warp > 0) {
    const int r = lane & (kTK - 1), hg = lane >> 4;
    if (D == 128 || lane < 16) {                 // D 64: both half-warps hold the sum
#pragma unroll
      for (int h = 0; h < G; ++h)
        reinterpret_cast<float4*>(wst + (cw * G + h) * (D + 4) + 4)[lane] = acc[h];
    }
    if constexpr (kBfly) {
      if ((lane & 7) == 0) {                     // lane l ran head l >> 3
        wst[(cw * G + (lane >> 3)) * (D + 4)] = m_run[0];
        wst[(cw * G + (lane >> 3)) * (D + 4) + 1] = l_run[0];
      }
    } else if (r == 0) {
#pragma unroll
      for (int u = 0; u < GH; ++u) {
        const int h = hg + 2 * u;
        if (h < G) {
          wst[(cw * G + h) * (D + 4)] = m_run[u];
          wst[(cw * G + h) * (D + 4) + 1] = l_run[u];
        }
      }
    }
  }
  __syncthreads();
  float* part = ring + Ly::WST_F;                 // [kMaxCluster][G][D + 4] on rank 0
  if (!GS && csize > 1) cluster_sync();           // every rank is done with its ring
  const uint32_t slot0 = smem_u32(part + static_cast<int>(rank) * G * (D + 4));
  const uint32_t dst = (!GS && csize > 1) ? map_rank(slot0, 0u) : slot0;
  float* gdst = GS ? a.gpart + (static_cast<int64_t>(item) * csize + rank) * G * (D + 4) : nullptr;
  for (int w = tid; w < G * D4; w += kThreads) {
    const int h = w / D4, c = w - h * D4;
    float M = -INFINITY;
#pragma unroll
    for (int q = 0; q < kConsumers; ++q) M = fmaxf(M, wst[(q * G + h) * (D + 4)]);
    const float Ms = isinf(M) ? 0.0f : M;
    float Lsum = 0.0f;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < kConsumers; ++q) {
      const float* ws_ = wst + (q * G + h) * (D + 4);
      const float wgt = expf(ws_[0] - Ms);
      Lsum = fmaf(ws_[1], wgt, Lsum);
      const float4 ar = reinterpret_cast<const float4*>(ws_ + 4)[c];
      A.x = fmaf(ar.x, wgt, A.x);
      A.y = fmaf(ar.y, wgt, A.y);
      A.z = fmaf(ar.z, wgt, A.z);
      A.w = fmaf(ar.w, wgt, A.w);
    }
    if (GS) {
      reinterpret_cast<float4*>(gdst + h * (D + 4) + 4)[c] = A;
      if (c == 0) {
        gdst[h * (D + 4)] = M;
        gdst[h * (D + 4) + 1] = Lsum;
      }
    } else {
      st_cluster_f32x4(dst + static_cast<uint32_t>((h * (D + 4) + 4 + 4 * c) * 4), A);
      if (c == 0) {
        st_cluster_f32(dst + static_cast<uint32_t>(h * (D + 4) * 4), M);
        st_cluster_f32(dst + static_cast<uint32_t>((h * (D + 4) + 1) * 4), Lsum);
      }
    }
  }
  const float* src_part = part;
  if (GS) {
    // the last CTA of the item to finish merges every split's state
    __shared__ int last_s;
    __threadfence();
    __syncthreads();
    if (tid == 0) last_s = atomicAdd(a.gcount + item, 1u) == csize - 1u;
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    src_part = a.gpart + static_cast<int64_t>(item) * csize * G * (D + 4);
  } else {
    if (csize > 1) cluster_sync();                // all ranks' states have landed in rank 0
    else __syncthreads();
    if (rank != 0) return;
  }
  // the states: in global memory (GS, written by other CTAs: read past L1)
  // or in this CTA's shared memory (cluster rank 0)
  auto ld1 = [](const float* q) -> float {
    if constexpr (GS) return __ldcg(q);
    else return *q;
  };
  auto ld4 = [](const float4* q) -> float4 {
    if constexpr (GS) return __ldcg(q);
    else return *q;
  };
  for (int w = tid; w < G * D4; w += kThreads) {
    const int h = w / D4, c = w - h * D4;
    float M = -INFINITY;
    for (uint32_t r = 0; r < csize; ++r) M = fmaxf(M, ld1(src_part + (r * G + h) * (D + 4)));
    const float Ms = isinf(M) ? 0.0f : M;
    float L = 0.0f;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t r = 0; r < csize; ++r) {
      const float* pr_ = src_part + (r * G + h) * (D + 4);
      const float wgt = expf(ld1(pr_) - Ms);
      L = fmaf(ld1(pr_ + 1), wgt, L);
      const float4 ar = ld4(reinterpret_cast<const float4*>(pr_ + 4) + c);
      A.x = fmaf(ar.x, wgt, A.x);
      A.y = fmaf(ar.y, wgt, A.y);
      A.z = fmaf(ar.z, wgt, A.z);
      A.w = fmaf(ar.w, wgt, A.w);
    }
    float4 o;
    o.x = __fdiv_rn(A.x, L);
    o.y = __fdiv_rn(A.y, L);
    o.z = __fdiv_rn(A.z, L);
    o.w = __fdiv_rn(A.w, L);
    reinterpret_cast<float4*>(a.out + (static_cast<int64_t>(b) * a.hq + hk * G + h) * D)[c] = o;
  }
  if (GS && tid == 0) a.gcount[item] = 0u;       // ready for the next launch
}

// Cluster size (key split) for a launch: the estimated time of
// ceil(CTAs / resident CTAs) waves of (tiles per CTA + a ramp of two tiles),
// minimised over 1..8, the smaller size on ties.
template <class K>
int choose_split(K kern, size_t smem, int64_t items, int64_t tiles, int* resident) {
  int best = 1;
  double best_cost = 0.0;
  const int cmax = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(kMaxCluster, tiles / 2)));
  for (int c = 1; c <= cmax; ++c) {
    if (resident[c] == 0) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(c), 1, 1);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = static_cast<unsigned>(c);
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = std::max(1, num_sms() / c);
      }
      resident[c] = n;
    }
    const int64_t slots = static_cast<int64_t>(resident[c]) * c;
    const int64_t waves = (items * c + slots - 1) / slots;
    const double cost = static_cast<double>(waves) * (static_cast<double>((tiles + c - 1) / c) + 2.0);
    if (c == 1 || cost < best_cost) {
      best = c;
      best_cost = cost;
    }
  }
  return best;
}

// Key split over independent CTAs (with a workspace for the partial
// states): the estimated time of ceil(CTAs / resident CTAs) waves of (tiles
// per CTA + 4 tiles for the prologue, the ramp and the merge), minimised
// over 1..8, the smaller split on ties.
int choose_gsplit(int resident_ctas, int64_t items, int64_t tiles) {
  int best = 1;
  double best_cost = 0.0;
  const int64_t slots = static_cast<int64_t>(resident_ctas) * num_sms();
  const int smax = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(kMaxCluster, tiles / 2)));
  for (int sp = 1; sp <= smax; ++sp) {
    const int64_t waves = (items * sp + slots - 1) / slots;
    const double cost = static_cast<double>(waves) * (static_cast<double>((tiles + sp - 1) / sp) + 4.0);
    if (sp == 1 || cost < best_cost) {
      best = sp;
      best_cost = cost;
    }
  }
  return best;
}

// 0: split chosen per launch; KSH_DECODE_GSPLIT=1..8 forces the workspace path's split
int g_forced_gsplit = [] {
  const char* v = getenv("KSH_DECODE_GSPLIT");
  const int c = (v && *v) ? atoi(v) : 0;
  return c >= 1 && c <= 8 ? c : 0;
}();

template <int D, int G>
int launch_dec(const CUtensorMap& map, const DecArgs& a, int64_t B, int64_t max_total_len,
               cudaStream_t stream) {
  using Ly = DecLayout<D, G>;
  const int64_t items = B * a.hkv;
  const int64_t tiles = (max_total_len + kTK - 1) / kTK;
  if (a.gpart && items <= 65535) {
    auto gkern = decode_attn_kernel<D, G, true>;
    if (set_smem_optin(reinterpret_cast<const void*>(gkern), Ly::SMEM) != KSH_OK) return KSH_ERR_CUDA;
    const int per_sm = resident_ctas(reinterpret_cast<const void*>(gkern), kThreads, Ly::SMEM);
    const int sp = g_forced_gsplit > 0 ? g_forced_gsplit : choose_gsplit(per_sm, items, tiles);
    if (sp > 1)
      return launch(gkern, dim3(static_cast<unsigned>(sp), static_cast<unsigned>(items)),
                    dim3(kThreads), Ly::SMEM, stream, map, a);
  }
  auto kern = decode_attn_kernel<D, G, false>;
  if (set_smem_optin(reinterpret_cast<const void*>(kern), Ly::SMEM) != KSH_OK) return KSH_ERR_CUDA;
  static int resident[kMaxCluster + 1] = {};     // resident clusters per cluster size
  const int cluster = g_forced_split > 0 ? g_forced_split
                                         : choose_split(kern, Ly::SMEM, items, tiles, resident);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(cluster), static_cast<unsigned>(items), 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = Ly::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, map, a);
  if (e == cudaSuccess) count_launch();
  return e == cudaSuccess ? KSH_OK : record_cuda_error(e);
}

}  // namespace
}  // namespace ksh

using namespace ksh;

namespace {
constexpr int kGMaxSplit = kMaxCluster;

int64_t dec_counter_bytes(int64_t items) { return (items * 4 + 255) / 256 * 256; }

int decode_attention_impl(const float* qkv, int64_t batch, int64_t hq, int64_t hkv, int64_t d,
                          const int64_t* positions, const int64_t* slot_mapping,
                          const float* rope_cos, const float* rope_sin, int64_t max_pos,
                          float* pool, int64_t num_blocks, int64_t num_layers, int64_t layer,
                          int64_t block_size, const int32_t* block_tables, int64_t max_blocks,
                          int64_t max_total_len, float* out, void* workspace,
                          int64_t workspace_bytes, int32_t* flags, void* stream);
}  // namespace

extern "C" int64_t ksh_decode_attention_workspace_size(int64_t batch, int64_t hq, int64_t hkv,
                                                       int64_t d) {
  if (batch <= 0 || hq <= 0 || hkv <= 0 || hq % hkv != 0 || d <= 0) return 0;
  const int64_t items = batch * hkv;
  return dec_counter_bytes(items) + items * kGMaxSplit * (hq / hkv) * (d + 4) * 4;
}

extern "C" int ksh_decode_attention_ws(const float* qkv, int64_t batch, int64_t hq, int64_t hkv,
                                       int64_t d, const int64_t* positions,
                                       const int64_t* slot_mapping, const float* rope_cos,
                                       const float* rope_sin, int64_t max_pos, float* pool,
                                       int64_t num_blocks, int64_t num_layers, int64_t layer,
                                       int64_t block_size, const int32_t* block_tables,
                                       int64_t max_blocks, int64_t max_total_len, float* out,
                                       void* workspace, int64_t workspace_bytes, int32_t* flags,
                                       void* stream) {
  KSH_CHECK_ARG(workspace != nullptr);
  if (workspace_bytes < ksh_decode_attention_workspace_size(batch, hq, hkv, d))
    return KSH_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return KSH_ERR_ALIGN;
  return decode_attention_impl(qkv, batch, hq, hkv, d, positions, slot_mapping, rope_cos, rope_sin,
                               max_pos, pool, num_blocks, num_layers, layer, block_size,
                               block_tables, max_blocks, max_total_len, out, workspace,
                               workspace_bytes, flags, stream);
}

extern "C" int ksh_decode_attention(const float* qkv, int64_t batch, int64_t hq, int64_t hkv,
                                    int64_t d, const int64_t* positions,
                                    const int64_t* slot_mapping, const float* rope_cos,
                                    const float* rope_sin, int64_t max_pos, float* pool,
                                    int64_t num_blocks, int64_t num_layers, int64_t layer,
                                    int64_t block_size, const int32_t* block_tables,
                                    int64_t max_blocks, int64_t max_total_len, float* out,
                                    int32_t* flags, void* stream) {
  return decode_attention_impl(qkv, batch, hq, hkv, d, positions, slot_mapping, rope_cos, rope_sin,
                               max_pos, pool, num_blocks, num_layers, layer, block_size,
                               block_tables, max_blocks, max_total_len, out, nullptr, 0, flags,
                               stream);
}

namespace {
int decode_attention_impl(const float* qkv, int64_t batch, int64_t hq, int64_t hkv, int64_t d,
                          const int64_t* positions, const int64_t* slot_mapping,
                          const float* rope_cos, const float* rope_sin, int64_t max_pos,
                          float* pool, int64_t num_blocks, int64_t num_layers, int64_t layer,
                          int64_t block_size, const int32_t* block_tables, int64_t max_blocks,
                          int64_t max_total_len, float* out, void* workspace,
                          int64_t workspace_bytes, int32_t* flags, void* stream) {
  (void)workspace_bytes;
  KSH_CHECK_ARG(batch > 0 && hq > 0 && hkv > 0 && hq % hkv == 0 && max_pos > 0);
  KSH_CHECK_ARG(num_blocks > 0 && num_layers > 0 && layer >= 0 && layer < num_layers);
  KSH_CHECK_ARG(max_blocks > 0 && max_total_len > 0 && batch * hkv <= 65535);
  KSH_CHECK_ARG(qkv && positions && slot_mapping && rope_cos && rope_sin && pool && block_tables &&
                out);
  const int64_t g = hq / hkv;
  if (block_size % kTK != 0 || (d != 64 && d != 128) ||
      (reinterpret_cast<uintptr_t>(pool) & 15) != 0 || (reinterpret_cast<uintptr_t>(out) & 15) != 0)
    return KSH_ERR_UNSUPPORTED;
  DecArgs a = {};
  a.qkv = qkv;
  a.positions = positions;
  a.slots = slot_mapping;
  a.rcos = rope_cos;
  a.rsin = rope_sin;
  a.pool = pool;
  a.block_tables = block_tables;
  a.out = out;
  a.flags = flags;
  a.max_pos = max_pos;
  a.num_blocks = num_blocks;
  a.num_layers = num_layers;
  a.layer = layer;
  a.hkv = hkv;
  a.hq = hq;
  a.bs = block_size;
  a.max_blocks = max_blocks;
  a.g = static_cast<int>(g);
  a.scale = static_cast<float>(1.0 / sqrt(static_cast<double>(d)));
  if (workspace) {
    a.gcount = static_cast<uint32_t*>(workspace);
    a.gpart = reinterpret_cast<float*>(static_cast<char*>(workspace) + dec_counter_bytes(batch * hkv));
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the pool as a 2-D tensor of token rows (D floats each) for TMA
  const int64_t rows = num_blocks * num_layers * 2 * hkv * block_size;
  if (rows >= (int64_t(1) << 31)) return KSH_ERR_UNSUPPORTED;
  CUtensorMap map;
  if (!make_tensor_map_2d(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, pool, static_cast<uint64_t>(d),
                          static_cast<uint64_t>(rows), static_cast<uint64_t>(d) * 4, 32, kTK,
                          CU_TENSOR_MAP_SWIZZLE_128B))
    return KSH_ERR_UNSUPPORTED;
#define KSH_DEC(DD, GG) \
  if (d == DD && g == GG) return launch_dec<DD, GG>(map, a, batch, max_total_len, st);
  KSH_DEC(64, 1) KSH_DEC(64, 2) KSH_DEC(64, 4) KSH_DEC(64, 7) KSH_DEC(64, 8)
  KSH_DEC(128, 1) KSH_DEC(128, 2) KSH_DEC(128, 4) KSH_DEC(128, 8)
#undef KSH_DEC
  return KSH_ERR_UNSUPPORTED;
}
}  // namespace

extern "C" int ksh_set_decode_split(int clusters) {
  const int prev = g_forced_split;
  g_forced_split = clusters >= 1 && clusters <= kMaxCluster ? clusters : 0;
  return prev;
}

extern "C" int ksh_set_decode_gsplit(int splits) {
  const int prev = g_forced_gsplit;
  g_forced_gsplit = splits >= 1 && splits <= kGMaxSplit ? splits : 0;
  return prev;
}
