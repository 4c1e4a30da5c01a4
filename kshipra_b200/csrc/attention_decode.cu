// K6 + K7 fused: decode-step attention (one new token per sequence).
//
// Replaces, for the decode step of KshipraModel.forward, the RoPE at the
// token's absolute position (engine/model.py:47-55, 108, 121), the K/V write
// into the block pool (model.py:123-129) and chunked_attention with
// chunk_len = 1 (engine/chunked_prefill.py:93-140).
//
// One thread-block cluster per (sequence, kv head); its CTAs split the key
// range (tiles of 16 positions) evenly at run time from the sequence's
// current length:
//
// * each CTA streams its K/V tiles with 1-D bulk copies (cp.async.bulk) into
//   a ring of shared-memory stages guarded by mbarriers; the first stages are
//   requested BEFORE the programmatic-launch wait: those pool rows belong to
//   earlier positions, written by kernels that have completed (every kernel
//   of this library triggers its dependents only after its own wait), so the
//   K/V fetch overlaps the q/k/v projection still running;
// * after the wait each CTA rotates the g query heads of the group; the CTA
//   holding the last tile also rotates k, writes k and v to the pool (for
//   later steps) and patches its shared-memory copy of that row;
// * per tile: scores (q . k) / sqrt(D), the causal bound, and the reference's
//   online-softmax merge (running max with m_safe, exp, rescale);
// * the CTAs' (m, l, acc) are merged in rank order through distributed shared
//   memory by cluster rank 0, which writes the output.
//
// Bounds: block ids outside [0, num_blocks) raise KSH_FLAG_BAD_BLOCK (those
// keys are skipped); positions outside the RoPE table raise
// KSH_FLAG_BAD_POSITION; slots outside the pool KSH_FLAG_BAD_SLOT.  Every
// mbarrier wait is bounded (KSH_FLAG_TIMEOUT).

#include <math.h>

#include <algorithm>

#include "tc_common.cuh"

namespace ksh {
namespace {

using namespace tc;

constexpr int kTK = 16;          // keys per tile
constexpr int kThreads = 256;   // 8 warps: enough in flight per SM at one CTA per SM
constexpr int kMaxCluster = 8;

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
  int64_t max_pos, num_blocks, num_layers, layer, hkv, hq, bs, max_blocks;
  int g;
  float scale;
};

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Staged K / V tiles: 16 rows x D floats as D/32 TMA boxes of 16 rows x 128 B,
// 128B-swizzled (16-byte chunk c of row r at chunk c ^ (r & 7)).  Float4
// column d4 of row r:
template <int D>
__device__ __forceinline__ int tile_off(int r, int d4) {
  return (d4 >> 3) * (kTK * 32) + r * 32 + (((d4 & 7) ^ (r & 7)) << 2);
}

template <int D, int G, int NST>
__global__ void __launch_bounds__(kThreads)
decode_attn_kernel(const __grid_constant__ CUtensorMap pool_map, DecArgs a) {
  constexpr int D4 = D / 4;
  constexpr int TILE_F = kTK * D;               // floats per staged K (or V) tile
  constexpr int CH = NST / 2;                   // tiles per chunk (ring = 2 chunks)
  constexpr int CK = CH * kTK;                  // keys per chunk (64 or 128)
  constexpr int KW = CK / 32;                   // score warps along keys (one key per lane)
  static_assert(CK % 32 == 0 && KW >= 1 && KW <= kThreads / 32, "score mapping");
  static_assert((kThreads / (D / 4)) * G * D <= NST * kTK * D, "PV reduction fits the K ring");
  constexpr int HW = (kThreads / 32) / KW;      // score warps along heads
  constexpr int GH = (G + HW - 1) / HW;         // heads per score warp
  constexpr int KGS = kThreads / D4;            // PV key groups
  constexpr int KPG = CK / KGS;                 // keys per PV group and chunk
  extern __shared__ __align__(128) float4 sm4[];
  // TMA 128B-swizzled destinations need 1024-byte alignment
  float* sm = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(sm4) + 1023) & ~uintptr_t(1023));
  float* Kt = sm;                               // [NST][D/32][kTK][32], swizzled
  float* Vt = Kt + NST * TILE_F;                // [NST][D/32][kTK][32], swizzled
  float* Qs = Vt + NST * TILE_F;                // [G][D]
  float* Ss = Qs + G * D;                       // [G][CK + 1]
  float* corr_s = Ss + G * (CK + 1);            // [G]
  float* ms = corr_s + G;                       // [G] running max
  float* ls = ms + G;                           // [G] running sum
  // offsets so far: 2*NST*TILE_F + G*D + G*CK + 4G floats, a multiple of 4
  // [kMaxCluster][G][D + 4]: every rank's (m, l, pad, pad, acc), received by rank 0
  float* part = ls + G;
  uint64_t* full = reinterpret_cast<uint64_t*>(part + kMaxCluster * G * (D + 4));   // [NST]
  __shared__ int tile_ok[NST];
  __shared__ float newk[D], newv[D];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t rank = cluster_rank(), csize = cluster_size();
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

  // Thread 0 stages local tile i into stage i % NST with TMA (D/32 boxes for K
  // and for V); an out-of-range block id marks the tile bad instead.
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
    mbar_arrive_expect_tx(&full[s], 2u * TILE_F * 4u);
#pragma unroll
    for (int cb = 0; cb < D / 32; ++cb) {
      tma_load_2d(Kt + s * TILE_F + cb * kTK * 32, &pool_map, &full[s], cb * 32, krow);
      tma_load_2d(Vt + s * TILE_F + cb * kTK * 32, &pool_map, &full[s], cb * 32, vrow);
    }
  };

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) mbar_init(&full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&pool_map);
    for (int i = 0; i < ntl && i < NST; ++i) issue(i);
  }
  if (tid < G) {
    ms[tid] = -INFINITY;
    ls[tid] = 0.0f;
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
      Qs[h * D + j] = o1;
      Qs[h * D + j + half] = o2;
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

  // ---- chunks of CH tiles (CK = 64 keys) ----
  // PV ownership: float4 column c4 over the KPG keys kg*KPG .. of each chunk,
  // all G heads; partial sums stay per thread until the end.
  const int c4 = tid % D4, kg = tid / D4;
  float4 acc[G];
#pragma unroll
  for (int h = 0; h < G; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
  bool timed_out = false, bad_block = false;

  for (int c0 = 0; c0 < ntl && !timed_out; c0 += CH) {
    const int nt = min(CH, ntl - c0);
    for (int i = c0; i < c0 + nt; ++i) {
      if (!mbar_wait(&full[i % NST], (i / NST) & 1)) timed_out = true;
      if (!tile_ok[i % NST]) bad_block = true;
    }
    if (timed_out) break;
    if (owner && c0 + nt == ntl) {             // patch the new token's row
      const int i = ntl - 1, s = i % NST;
      const int rr = static_cast<int>(p) - (t_begin + i) * kTK;
      for (int j = tid; j < D; j += kThreads) {
        Kt[s * TILE_F + tile_off<D>(rr, j >> 2) + (j & 3)] = newk[j];
        Vt[s * TILE_F + tile_off<D>(rr, j >> 2) + (j & 3)] = newv[j];
      }
      __syncthreads();
    }
    const int kbase = (t_begin + c0) * kTK;    // absolute position of chunk key 0
    const int nk = nt * kTK;
    // scores: warp (kh, hh): lane -> key kh*32 + lane, heads hh*GH ..; q read as broadcast
    {
      const int kh = warp % KW, hh = warp / KW;
      const int j = kh * 32 + lane;
      const int s = (c0 + (j >> 4)) % NST;
      const bool valid = j < nk && kbase + j < total_c && tile_ok[s];
      const float* kt = Kt + s * TILE_F;
      const int r = j & (kTK - 1);
      float dot[GH];
#pragma unroll
      for (int u = 0; u < GH; ++u) dot[u] = 0.0f;
#pragma unroll
      for (int d4 = 0; d4 < D4; ++d4) {
        const float4 kv = *reinterpret_cast<const float4*>(kt + tile_off<D>(r, d4));
#pragma unroll
        for (int u = 0; u < GH; ++u) {
          const int h = hh * GH + u;
          if (h < G) {
            const float4 qv = reinterpret_cast<const float4*>(Qs + h * D)[d4];
            dot[u] = fmaf(qv.x, kv.x, dot[u]);
            dot[u] = fmaf(qv.y, kv.y, dot[u]);
            dot[u] = fmaf(qv.z, kv.z, dot[u]);
            dot[u] = fmaf(qv.w, kv.w, dot[u]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < GH; ++u) {
        const int h = hh * GH + u;
        if (h < G) Ss[h * (CK + 1) + j] = valid ? dot[u] * a.scale : -INFINITY;
      }
    }
    __syncthreads();
    // online softmax merge, one warp per head
    for (int h = warp; h < G; h += kThreads / 32) {
      float* srow = Ss + h * (CK + 1);
      float mx = -INFINITY;
      for (int j = lane; j < CK; j += 32) mx = fmaxf(mx, srow[j]);
      mx = warp_max(mx);
      const float m_old = ms[h];
      const float m_new = fmaxf(m_old, mx);
      const float m_safe = isinf(m_new) ? 0.0f : m_new;
      float psum = 0.0f;
      for (int j = lane; j < CK; j += 32) {
        const float pj = expf(srow[j] - m_safe);
        srow[j] = pj;
        psum += pj;
      }
      psum = warp_sum(psum);
      if (lane == 0) {
        const float corr = expf(m_old - m_safe);
        ls[h] = __fadd_rn(__fmul_rn(ls[h], corr), psum);
        ms[h] = m_new;
        corr_s[h] = corr;
      }
    }
    __syncthreads();
    // acc[h][c4] = acc * corr[h] + sum_{j in group} p[h][j] V[j][c4]
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float crr = corr_s[h];
      acc[h].x *= crr;
      acc[h].y *= crr;
      acc[h].z *= crr;
      acc[h].w *= crr;
    }
#pragma unroll 4
    for (int jj = 0; jj < KPG; ++jj) {
      const int j = kg * KPG + jj;
      if (j < nk) {
        const int s = (c0 + (j >> 4)) % NST;
        const float4 v =
            *reinterpret_cast<const float4*>(Vt + s * TILE_F + tile_off<D>(j & (kTK - 1), c4));
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float pj = Ss[h * (CK + 1) + j];
          acc[h].x = fmaf(pj, v.x, acc[h].x);
          acc[h].y = fmaf(pj, v.y, acc[h].y);
          acc[h].z = fmaf(pj, v.z, acc[h].z);
          acc[h].w = fmaf(pj, v.w, acc[h].w);
        }
      }
    }
    __syncthreads();                           // this chunk's stages are free
    if (tid == 0)
      for (int i = c0 + NST; i < min(c0 + NST + CH, ntl); ++i) issue(i);
  }
  if (tid == 0) {
    if (timed_out) raise_flag(a.flags, KSH_FLAG_TIMEOUT);
    if (bad_block) raise_flag(a.flags, KSH_FLAG_BAD_BLOCK);
  }

  // ---- reduce the PV key groups (the K ring is idle now) and send this CTA's
  // (m, l, acc) to cluster rank 0 with remote shared-memory stores ----
  float* red = Kt;                              // [KGS][G][D]
#pragma unroll
  for (int h = 0; h < G; ++h)
    reinterpret_cast<float4*>(red + (kg * G + h) * D)[c4] = acc[h];
  __syncthreads();
  const uint32_t slot0 = smem_u32(part + static_cast<int>(rank) * G * (D + 4));
  const uint32_t dst = csize > 1 ? map_rank(slot0, 0u) : slot0;
  for (int w = tid; w < G * D4; w += kThreads) {
    const int h = w / D4, c = w - h * D4;
    float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int g2 = 0; g2 < KGS; ++g2) {
      const float4 v = reinterpret_cast<const float4*>(red + (g2 * G + h) * D)[c];
      s4.x += v.x; s4.y += v.y; s4.z += v.z; s4.w += v.w;
    }
    st_cluster_f32x4(dst + static_cast<uint32_t>((h * (D + 4) + 4 + 4 * c) * 4), s4);
  }
  if (tid < G) {
    st_cluster_f32(dst + static_cast<uint32_t>(tid * (D + 4) * 4), ms[tid]);
    st_cluster_f32(dst + static_cast<uint32_t>((tid * (D + 4) + 1) * 4), ls[tid]);
  }
  if (csize > 1) cluster_sync();              // all ranks' states have landed in rank 0
  else __syncthreads();
  if (rank != 0) return;
  for (int w = tid; w < G * D4; w += kThreads) {
    const int h = w / D4, c = w - h * D4;
    float M = -INFINITY;
    for (uint32_t r = 0; r < csize; ++r) M = fmaxf(M, part[(r * G + h) * (D + 4)]);
    const float Ms = isinf(M) ? 0.0f : M;
    float L = 0.0f;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
    for (uint32_t r = 0; r < csize; ++r) {
      const float* pr_ = part + (r * G + h) * (D + 4);
      const float wgt = expf(pr_[0] - Ms);
      L = fmaf(pr_[1], wgt, L);
      const float4 ar = reinterpret_cast<const float4*>(pr_ + 4)[c];
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
}

template <int D, int G>
int launch_dec(const CUtensorMap& map, const DecArgs& a, int64_t B, int cluster,
               cudaStream_t stream) {
  constexpr int NST = D == 64 ? 16 : 8;           // two chunks of 128 / 64 keys
  constexpr int CK = (NST / 2) * kTK;
  const size_t smem = (2ull * NST * kTK * D + static_cast<size_t>(G) * D + G * (CK + 1) +
                       3 * G + static_cast<size_t>(kMaxCluster) * G * (D + 4)) * 4 + NST * 8 +
                      1024;
  auto kern = decode_attn_kernel<D, G, NST>;
  if (smem > 32 * 1024 && set_smem_optin(reinterpret_cast<const void*>(kern), smem) != KSH_OK)
    return KSH_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(cluster), static_cast<unsigned>(B * a.hkv), 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
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
  return e == cudaSuccess ? KSH_OK : record_cuda_error(e);
}

}  // namespace

int decode_attention_cluster(int64_t batch, int64_t hkv, int64_t max_total_len) {
  const int64_t items = batch * hkv;
  const int64_t tiles = (max_total_len + kTK - 1) / kTK;
  // enough CTAs for about four per SM (the key range split over a cluster)
  int64_t c = (4LL * num_sms() + items - 1) / items;
  c = std::min<int64_t>(c, std::max<int64_t>(1, tiles / 2));
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(c, kMaxCluster)));
}

}  // namespace ksh

using namespace ksh;

extern "C" int ksh_decode_attention(const float* qkv, int64_t batch, int64_t hq, int64_t hkv,
                                    int64_t d, const int64_t* positions,
                                    const int64_t* slot_mapping, const float* rope_cos,
                                    const float* rope_sin, int64_t max_pos, float* pool,
                                    int64_t num_blocks, int64_t num_layers, int64_t layer,
                                    int64_t block_size, const int32_t* block_tables,
                                    int64_t max_blocks, int64_t max_total_len, float* out,
                                    int32_t* flags, void* stream) {
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
  const int cl = decode_attention_cluster(batch, hkv, max_total_len);
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
  if (d == DD && g == GG) return launch_dec<DD, GG>(map, a, batch, cl, st);
  KSH_DEC(64, 1) KSH_DEC(64, 2) KSH_DEC(64, 4) KSH_DEC(64, 7) KSH_DEC(64, 8)
  KSH_DEC(128, 1) KSH_DEC(128, 2) KSH_DEC(128, 4) KSH_DEC(128, 8)
#undef KSH_DEC
  return KSH_ERR_UNSUPPORTED;
}
