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
constexpr int kThreads = 128;
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

template <int D, int G, int NST>
__global__ void __launch_bounds__(kThreads)
decode_attn_kernel(DecArgs a) {
  constexpr int D4 = D / 4;
  constexpr int TILE_F = kTK * D;               // floats per K (or V) tile
  constexpr int CH = NST / 2;                   // tiles per chunk (ring = 2 chunks)
  constexpr int CK = CH * kTK;                  // keys per chunk
  constexpr int NPV = (G * D4 + kThreads - 1) / kThreads;   // (head, float4 col) pairs per thread
  extern __shared__ __align__(128) float4 sm4[];
  float* sm = reinterpret_cast<float*>(sm4);
  float* Kt = sm;                               // [NST][kTK][D]
  float* Vt = Kt + NST * TILE_F;                // [NST][kTK][D]
  float* Qs = Vt + NST * TILE_F;                // [G][D]
  float* Ss = Qs + G * D;                       // [G][CK + 1]
  float* corr_s = Ss + G * (CK + 1);            // [G]
  float* ms = corr_s + G;                       // [G] running max
  float* ls = ms + G;                           // [G] running sum
  // offsets so far: 2*NST*TILE_F + G*D + G*CK + 4G floats, a multiple of 4
  float* part = ls + G;                         // [G][D + 4]: m, l, pad, pad, acc (16B aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(part + G * (D + 4));   // [NST]
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

  auto issue = [&](int i) {          // local tile i into stage i % NST (thread 0)
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
    const float* kp = a.pool + ((((blk * a.num_layers + a.layer) * 2) * a.hkv + hk) * a.bs + off) * D;
    const float* vp = kp + head_rows * D;
    mbar_arrive_expect_tx(&full[s], 2u * TILE_F * 4u);
    bulk_g2s(Kt + s * TILE_F, kp, TILE_F * 4u, &full[s]);
    bulk_g2s(Vt + s * TILE_F, vp, TILE_F * 4u, &full[s]);
  };

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) mbar_init(&full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
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

  // ---- chunks of CH tiles ----
  float4 acc[NPV];
#pragma unroll
  for (int u = 0; u < NPV; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
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
        Kt[s * TILE_F + rr * D + j] = newk[j];
        Vt[s * TILE_F + rr * D + j] = newv[j];
      }
      __syncthreads();
    }
    const int kbase = (t_begin + c0) * kTK;    // absolute position of chunk key 0
    const int nk = nt * kTK;
    // scores S[h][j] = (q_h . k_j) * scale, -inf beyond the causal bound
    for (int idx = tid; idx < G * CK; idx += kThreads) {
      const int h = idx / CK, j = idx - h * CK;
      float sc = -INFINITY;
      const int s = (c0 + j / kTK) % NST;
      if (j < nk && kbase + j < total_c && tile_ok[s]) {
        const float* kr = Kt + s * TILE_F + (j % kTK) * D;
        float dot = 0.0f;
#pragma unroll
        for (int cc = 0; cc < D4; ++cc) {
          const int c = (cc + j) & (D4 - 1);
          const float4 qv = reinterpret_cast<const float4*>(Qs + h * D)[c];
          const float4 kv = reinterpret_cast<const float4*>(kr)[c];
          dot = fmaf(qv.x, kv.x, dot);
          dot = fmaf(qv.y, kv.y, dot);
          dot = fmaf(qv.z, kv.z, dot);
          dot = fmaf(qv.w, kv.w, dot);
        }
        sc = dot * a.scale;
      }
      Ss[h * (CK + 1) + j] = sc;
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
    // acc[h][c4] = acc * corr[h] + sum_j p[h][j] V[j][c4]
#pragma unroll
    for (int u = 0; u < NPV; ++u) {
      const int idx = tid + u * kThreads;
      if (idx < G * D4) {
        const int h = idx / D4, c4 = idx - h * D4;
        const float* prow = Ss + h * (CK + 1);
        float4 pv = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int t = 0; t < nt; ++t) {
          const float* vt = Vt + ((c0 + t) % NST) * TILE_F;
#pragma unroll
          for (int jj = 0; jj < kTK; ++jj) {
            const float pj = prow[t * kTK + jj];
            const float4 v = reinterpret_cast<const float4*>(vt + jj * D)[c4];
            pv.x = fmaf(pj, v.x, pv.x);
            pv.y = fmaf(pj, v.y, pv.y);
            pv.z = fmaf(pj, v.z, pv.z);
            pv.w = fmaf(pj, v.w, pv.w);
          }
        }
        const float crr = corr_s[h];
        acc[u].x = __fadd_rn(__fmul_rn(acc[u].x, crr), pv.x);
        acc[u].y = __fadd_rn(__fmul_rn(acc[u].y, crr), pv.y);
        acc[u].z = __fadd_rn(__fmul_rn(acc[u].z, crr), pv.z);
        acc[u].w = __fadd_rn(__fmul_rn(acc[u].w, crr), pv.w);
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

  // ---- publish this CTA's state; every rank merges a slice of the outputs ----
  if (tid < G) {
    part[tid * (D + 4)] = ms[tid];
    part[tid * (D + 4) + 1] = ls[tid];
  }
#pragma unroll
  for (int u = 0; u < NPV; ++u) {
    const int idx = tid + u * kThreads;
    if (idx < G * D4) {
      const int h = idx / D4, c4 = idx - h * D4;
      reinterpret_cast<float4*>(part + h * (D + 4) + 4)[c4] = acc[u];
    }
  }
  __syncthreads();
  cluster_sync();
  {
    const uint32_t base = smem_u32(part);
    const int per_rank = (G * D4 + static_cast<int>(csize) - 1) / static_cast<int>(csize);
    for (int w = static_cast<int>(rank) * per_rank + tid;
         w < min((static_cast<int>(rank) + 1) * per_rank, G * D4); w += kThreads) {
      const int h = w / D4, c = w - h * D4;
      const uint32_t off = static_cast<uint32_t>(h * (D + 4)) * 4u;
      float mr[kMaxCluster], lr[kMaxCluster];
      float4 ar[kMaxCluster];
#pragma unroll
      for (int r = 0; r < kMaxCluster; ++r) {
        if (r < static_cast<int>(csize)) {
          const uint32_t pb = map_rank(base + off, static_cast<uint32_t>(r));
          mr[r] = ld_cluster_f32(pb);
          lr[r] = ld_cluster_f32(pb + 4);
          ar[r] = ld_cluster_f32x4(pb + 16u + static_cast<uint32_t>(c) * 16u);
        }
      }
      float M = -INFINITY;
#pragma unroll
      for (int r = 0; r < kMaxCluster; ++r)
        if (r < static_cast<int>(csize)) M = fmaxf(M, mr[r]);
      const float Ms = isinf(M) ? 0.0f : M;
      float L = 0.0f;
      float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < kMaxCluster; ++r) {
        if (r < static_cast<int>(csize)) {
          const float wgt = expf(mr[r] - Ms);
          L = fmaf(lr[r], wgt, L);
          A.x = fmaf(ar[r].x, wgt, A.x);
          A.y = fmaf(ar[r].y, wgt, A.y);
          A.z = fmaf(ar[r].z, wgt, A.z);
          A.w = fmaf(ar[r].w, wgt, A.w);
        }
      }
      float4 o;
      o.x = __fdiv_rn(A.x, L);
      o.y = __fdiv_rn(A.y, L);
      o.z = __fdiv_rn(A.z, L);
      o.w = __fdiv_rn(A.w, L);
      reinterpret_cast<float4*>(a.out + (static_cast<int64_t>(b) * a.hq + hk * G + h) * D)[c] = o;
    }
  }
  cluster_sync();      // keep every CTA's shared memory alive until all ranks have read it
}

template <int D, int G>
int launch_dec(const DecArgs& a, int64_t B, int cluster, cudaStream_t stream) {
  constexpr int NST = D == 128 ? 6 : 8;
  constexpr int CK = (NST / 2) * kTK;
  const size_t smem = (2ull * NST * kTK * D + static_cast<size_t>(G) * D + G * (CK + 1) +
                       3 * G + 4 + static_cast<size_t>(G) * (D + 4)) * 4 + NST * 8 + 16;
  auto kern = decode_attn_kernel<D, G, NST>;
  if (smem > 48 * 1024 && set_smem_optin(reinterpret_cast<const void*>(kern), smem) != KSH_OK)
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  return e == cudaSuccess ? KSH_OK : record_cuda_error(e);
}

}  // namespace

int decode_attention_cluster(int64_t batch, int64_t hkv, int64_t max_total_len) {
  const int64_t items = batch * hkv;
  const int64_t tiles = (max_total_len + kTK - 1) / kTK;
  int64_t c = (2LL * num_sms() + items - 1) / items;
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
#define KSH_DEC(DD, GG) \
  if (d == DD && g == GG) return launch_dec<DD, GG>(a, batch, cl, st);
  KSH_DEC(64, 1) KSH_DEC(64, 2) KSH_DEC(64, 4) KSH_DEC(64, 7) KSH_DEC(64, 8)
  KSH_DEC(128, 1) KSH_DEC(128, 2) KSH_DEC(128, 4) KSH_DEC(128, 8)
#undef KSH_DEC
  return KSH_ERR_UNSUPPORTED;
}
