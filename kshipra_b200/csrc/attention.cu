// K7 / K8: paged online-softmax attention over the block pool.
//
// Replaces chunked_attention (engine/chunked_prefill.py:93-140), batched over
// sequences.  One CTA owns (sequence, kv head, tile of query positions,
// split of the key range):
//
// * its rows are the g = hq / hkv query heads that share the kv head times
//   the query positions of the tile, so every K/V tile is read once per GQA
//   group (the reference repeats K/V per query head instead);
// * keys are walked in tiles of 16 positions gathered through the block table
//   (any block size); the next tile's K/V is loaded into registers while the
//   current one is consumed from shared memory;
// * per tile: scores s = (q . k) * 1/sqrt(D) with the causal mask
//   k_pos > q_pos -> -inf, then the reference's merge: m' = max(m, rowmax s),
//   m_safe = m' if finite else 0, p = exp(s - m_safe), l = l*exp(m - m_safe) +
//   sum p, acc = acc*exp(m - m_safe) + p V.  No score matrix is materialised;
// * when the key range is split over CTAs (decode, long contexts) each split
//   writes (m, l, acc) to the workspace and the last CTA of the group merges
//   them in split order (deterministic), then resets its counter.
//
// Block ids outside [0, num_blocks) and sequences longer than their block
// table raise KSH_FLAG_BAD_BLOCK / KSH_FLAG_BAD_LENGTH; the offending keys
// read as zeros.  No waits, no traps.

#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace ksh {
namespace {

constexpr int kTK = 16;          // keys per tile
constexpr int kThreads = 128;

struct AttnArgs {
  const float* q;          // [T, hq, d]
  const float* pool;       // [nb, L, 2, hkv, bs, d]
  const int32_t* block_tables;
  const int32_t* q_start;  // [S + 1]
  const int32_t* prefix_lens;
  float* out;              // [T, hq, d]
  uint32_t* counters;      // [items]
  float* part;             // [items, nsplit, rmax, d + 4]
  int32_t* flags;
  int64_t num_blocks, num_layers, layer, hkv, hq, bs, max_blocks;
  int g, qt, nqt, nsplit, tps, rmax;
  float scale;
};

// Row index (in units of d floats) of the K row of `pos` for (sequence s,
// kv head hk); -1 when the block-table entry is out of range.  The V row is
// hkv * bs rows further.
__device__ __forceinline__ int64_t token_row(const AttnArgs& a, int s, int hk, int pos) {
  const int64_t j = pos / a.bs;
  if (j >= a.max_blocks) return -1;
  const int64_t blk = a.block_tables[static_cast<int64_t>(s) * a.max_blocks + j];
  if (blk < 0 || blk >= a.num_blocks) return -1;
  const int64_t off = pos - j * a.bs;
  return (((blk * a.num_layers + a.layer) * 2) * a.hkv + hk) * a.bs + off;
}

template <int D, int RMAX>
__global__ void __launch_bounds__(kThreads) paged_attn_kernel(AttnArgs a) {
  constexpr int D4 = D / 4;
  constexpr int LD_PER_T = kTK * D4 / kThreads;   // float4 of K (and of V) per thread
  static_assert(LD_PER_T >= 1, "tile too small");
  extern __shared__ float4 smem4[];
  float4* Qs = smem4;                       // [RMAX][D4]
  float4* Ks = Qs + RMAX * D4;              // [kTK][D4]
  float4* Vs = Ks + kTK * D4;               // [kTK][D4]
  float* Ss = reinterpret_cast<float*>(Vs + kTK * D4);   // [RMAX][kTK + 1]
  float* corr_s = Ss + RMAX * (kTK + 1);    // [RMAX]
  float* l_s = corr_s + RMAX;               // [RMAX]
  float* m_s = l_s + RMAX;                  // [RMAX]
  __shared__ bool is_last;

  const int tid = threadIdx.x;
  const int item = blockIdx.x, sp = blockIdx.y;
  const int per_seq = static_cast<int>(a.hkv) * a.nqt;
  const int s = item / per_seq;
  const int hk = (item % per_seq) / a.nqt;
  const int qti = item % a.nqt;

  grid_dep_wait();
  grid_dep_launch();

  const int q0 = a.q_start[s];
  const int C = a.q_start[s + 1] - q0;
  const int prefix = a.prefix_lens[s];
  const int qa = qti * a.qt;
  if (qa >= C) return;                     // uniform over the item's splits
  const int nq = min(a.qt, C - qa);
  const int R = nq * a.g;
  int total = prefix + qa + nq;            // keys this tile needs
  const int64_t cap = a.max_blocks * a.bs;
  if (total > cap) {
    if (tid == 0) raise_flag(a.flags, KSH_FLAG_BAD_LENGTH);
    total = static_cast<int>(cap);
  }
  const int ntiles = (total + kTK - 1) / kTK;
  const int t_begin = sp * a.tps;
  const int t_end = min(t_begin + a.tps, ntiles);

  // q rows: r = qi * g + gi  ->  q[(q0 + qa + qi), hk * g + gi, :]
  for (int i = tid; i < RMAX * D4; i += kThreads) {
    const int r = i / D4, c = i - r * D4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < R) {
      const int qi = r / a.g, gi = r - qi * a.g;
      const int64_t row = (static_cast<int64_t>(q0 + qa + qi) * a.hq + hk * a.g + gi);
      v = reinterpret_cast<const float4*>(a.q + row * D)[c];
    }
    Qs[i] = v;
  }

  // Softmax state lives with thread r (< RMAX).
  float m_r = -INFINITY, l_r = 0.0f;
  // PV ownership: column float4 c4, rows r0 + RSTEP * i.
  constexpr int RSTEP = kThreads / D4;
  constexpr int NRPV = RMAX / RSTEP > 0 ? RMAX / RSTEP : 1;
  const int c4 = tid % D4, r0 = tid / D4;
  float4 acc[NRPV];
#pragma unroll
  for (int i = 0; i < NRPV; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);

  // Register prefetch of one K/V tile.
  float4 kreg[LD_PER_T], vreg[LD_PER_T];
  bool bad = false;
  auto load_tile = [&](int t) {
#pragma unroll
    for (int u = 0; u < LD_PER_T; ++u) {
      const int f = tid + u * kThreads;
      const int j = f / D4, c = f - j * D4;
      const int pos = t * kTK + j;
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (pos < total) {
        const int64_t row = token_row(a, s, hk, pos);
        if (row >= 0) {
          kv = reinterpret_cast<const float4*>(a.pool + row * D)[c];
          vv = reinterpret_cast<const float4*>(a.pool + (row + a.hkv * a.bs) * D)[c];
        } else {
          bad = true;
        }
      }
      kreg[u] = kv;
      vreg[u] = vv;
    }
  };

  if (t_begin < t_end) load_tile(t_begin);
  for (int t = t_begin; t < t_end; ++t) {
    __syncthreads();   // previous tile fully consumed (and Qs written on entry)
#pragma unroll
    for (int u = 0; u < LD_PER_T; ++u) {
      Ks[tid + u * kThreads] = kreg[u];
      Vs[tid + u * kThreads] = vreg[u];
    }
    __syncthreads();
    if (t + 1 < t_end) load_tile(t + 1);

    // scores
    {
      const int j = tid & (kTK - 1);
      const int kpos = t * kTK + j;
#pragma unroll
      for (int rr = tid >> 4; rr < RMAX; rr += kThreads / kTK) {
        float sc = -INFINITY;
        if (rr < R) {
          const int qpos = prefix + qa + rr / a.g;
          if (kpos <= qpos && kpos < total) {
            float dot = 0.0f;
#pragma unroll
            for (int cc = 0; cc < D4; ++cc) {
              const int c = (cc + j) & (D4 - 1);
              const float4 qv = Qs[rr * D4 + c];
              const float4 kv = Ks[j * D4 + c];
              dot = fmaf(qv.x, kv.x, dot);
              dot = fmaf(qv.y, kv.y, dot);
              dot = fmaf(qv.z, kv.z, dot);
              dot = fmaf(qv.w, kv.w, dot);
            }
            sc = dot * a.scale;
          }
        }
        Ss[rr * (kTK + 1) + j] = sc;
      }
    }
    __syncthreads();
    // online softmax, one thread per row
    if (tid < RMAX) {
      float* sr = Ss + tid * (kTK + 1);
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < kTK; ++j) mx = fmaxf(mx, sr[j]);
      const float m_new = fmaxf(m_r, mx);
      const float m_safe = isinf(m_new) ? 0.0f : m_new;
      float psum = 0.0f;
#pragma unroll
      for (int j = 0; j < kTK; ++j) {
        const float p = expf(sr[j] - m_safe);
        sr[j] = p;
        psum += p;
      }
      const float corr = expf(m_r - m_safe);
      l_r = __fadd_rn(__fmul_rn(l_r, corr), psum);
      m_r = m_new;
      corr_s[tid] = corr;
    }
    __syncthreads();
    // acc = acc * corr + P V
#pragma unroll
    for (int i = 0; i < NRPV; ++i) {
      const int r = r0 + RSTEP * i;
      if (r < RMAX) {
        const float* pr = Ss + r * (kTK + 1);
        float4 pv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < kTK; ++j) {
          const float p = pr[j];
          const float4 v = Vs[j * D4 + c4];
          pv.x = fmaf(p, v.x, pv.x);
          pv.y = fmaf(p, v.y, pv.y);
          pv.z = fmaf(p, v.z, pv.z);
          pv.w = fmaf(p, v.w, pv.w);
        }
        const float cr = corr_s[r];
        acc[i].x = __fadd_rn(__fmul_rn(acc[i].x, cr), pv.x);
        acc[i].y = __fadd_rn(__fmul_rn(acc[i].y, cr), pv.y);
        acc[i].z = __fadd_rn(__fmul_rn(acc[i].z, cr), pv.z);
        acc[i].w = __fadd_rn(__fmul_rn(acc[i].w, cr), pv.w);
      }
    }
  }
  if (bad) raise_flag(a.flags, KSH_FLAG_BAD_BLOCK);

  __syncthreads();
  if (tid < RMAX) {
    l_s[tid] = l_r;
    m_s[tid] = m_r;
  }
  __syncthreads();

  if (a.nsplit == 1) {
#pragma unroll
    for (int i = 0; i < NRPV; ++i) {
      const int r = r0 + RSTEP * i;
      if (r < R) {
        const int qi = r / a.g, gi = r - qi * a.g;
        const int64_t row = static_cast<int64_t>(q0 + qa + qi) * a.hq + hk * a.g + gi;
        const float l = l_s[r];
        float4 o;
        o.x = __fdiv_rn(acc[i].x, l);
        o.y = __fdiv_rn(acc[i].y, l);
        o.z = __fdiv_rn(acc[i].z, l);
        o.w = __fdiv_rn(acc[i].w, l);
        reinterpret_cast<float4*>(a.out + row * D)[c4] = o;
      }
    }
    return;
  }

  // Split-K: publish (m, l, acc) and let the last split of the item merge.
  const int64_t pstride = static_cast<int64_t>(RMAX) * (D + 4);
  float* mine = a.part + (static_cast<int64_t>(item) * a.nsplit + sp) * pstride;
#pragma unroll
  for (int i = 0; i < NRPV; ++i) {
    const int r = r0 + RSTEP * i;
    if (r < RMAX) reinterpret_cast<float4*>(mine + r * (D + 4) + 4)[c4] = acc[i];
  }
  // row layout: m, l, 2 pad floats, then acc (16-byte aligned)
  if (tid < RMAX) {
    mine[tid * (D + 4)] = m_s[tid];
    mine[tid * (D + 4) + 1] = l_s[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(a.counters + item, 1u);
    is_last = (prev == static_cast<unsigned>(a.nsplit) - 1u);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const float* base = a.part + static_cast<int64_t>(item) * a.nsplit * pstride;
  for (int i = tid; i < R * D4; i += kThreads) {
    const int r = i / D4, c = i - r * D4;
    float M = -INFINITY;
    for (int k = 0; k < a.nsplit; ++k) M = fmaxf(M, __ldcg(base + k * pstride + r * (D + 4)));
    const float Ms = isinf(M) ? 0.0f : M;
    float L = 0.0f;
    float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < a.nsplit; ++k) {
      const float* pk = base + k * pstride + r * (D + 4);
      const float mk = __ldcg(pk);
      const float w = expf(mk - Ms);
      L = fmaf(__ldcg(pk + 1), w, L);
      const float4 ak = __ldcg(reinterpret_cast<const float4*>(pk + 4) + c);
      A.x = fmaf(ak.x, w, A.x);
      A.y = fmaf(ak.y, w, A.y);
      A.z = fmaf(ak.z, w, A.z);
      A.w = fmaf(ak.w, w, A.w);
    }
    const int qi = r / a.g, gi = r - qi * a.g;
    const int64_t row = static_cast<int64_t>(q0 + qa + qi) * a.hq + hk * a.g + gi;
    float4 o;
    o.x = __fdiv_rn(A.x, L);
    o.y = __fdiv_rn(A.y, L);
    o.z = __fdiv_rn(A.z, L);
    o.w = __fdiv_rn(A.w, L);
    reinterpret_cast<float4*>(a.out + row * D)[c] = o;
  }
  if (tid == 0) a.counters[item] = 0u;
}

// Generic fallback for head dims other than 64 / 128: one warp per
// (query row, query head), keys walked one by one with the same merge.
__global__ void __launch_bounds__(32)
paged_attn_generic_kernel(AttnArgs a, int d, int max_q) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x;
  const int s = blockIdx.z, h = blockIdx.y, qi = blockIdx.x;
  const int q0 = a.q_start[s];
  const int C = a.q_start[s + 1] - q0;
  if (qi >= C) return;
  const int prefix = a.prefix_lens[s];
  const int hk = h / a.g;
  const int qpos = prefix + qi;
  const int64_t cap = a.max_blocks * a.bs;
  int total = qpos + 1;
  if (total > cap) {
    if (lane == 0) raise_flag(a.flags, KSH_FLAG_BAD_LENGTH);
    total = static_cast<int>(cap);
  }
  const float* qr = a.q + (static_cast<int64_t>(q0 + qi) * a.hq + h) * d;
  constexpr int kMaxPer = 8;   // d <= 256
  float acc[kMaxPer];
  for (int i = 0; i < kMaxPer; ++i) acc[i] = 0.0f;
  float m = -INFINITY, l = 0.0f;
  for (int pos = 0; pos < total; ++pos) {
    const int64_t j = pos / a.bs;
    const int64_t blk = a.block_tables[static_cast<int64_t>(s) * a.max_blocks + j];
    if (blk < 0 || blk >= a.num_blocks) {
      if (lane == 0) raise_flag(a.flags, KSH_FLAG_BAD_BLOCK);
      continue;
    }
    const int64_t off = pos - j * a.bs;
    const float* kp =
        a.pool + ((((blk * a.num_layers + a.layer) * 2) * a.hkv + hk) * a.bs + off) * d;
    const float* vp = kp + a.hkv * a.bs * d;
    float dot = 0.0f;
    for (int c = lane; c < d; c += 32) dot = fmaf(qr[c], kp[c], dot);
    dot = warp_sum(dot);
    const float sc = dot * a.scale;
    const float m_new = fmaxf(m, sc);
    const float m_safe = isinf(m_new) ? 0.0f : m_new;
    const float p = expf(sc - m_safe);
    const float corr = expf(m - m_safe);
    l = __fadd_rn(__fmul_rn(l, corr), p);
    for (int i = 0; i < kMaxPer; ++i) {
      const int c = lane + 32 * i;
      if (c < d) acc[i] = __fadd_rn(__fmul_rn(acc[i], corr), p * vp[c]);
    }
    m = m_new;
  }
  float* orow = a.out + (static_cast<int64_t>(q0 + qi) * a.hq + h) * d;
  for (int i = 0; i < kMaxPer; ++i) {
    const int c = lane + 32 * i;
    if (c < d) orow[c] = __fdiv_rn(acc[i], l);
  }
}

struct Plan {
  int rmax, qt, nqt, nsplit, tps;
  int64_t items;
  int64_t counter_bytes, part_bytes;
};

Plan make_plan(int64_t num_seqs, int64_t hq, int64_t hkv, int64_t d, int64_t max_q_len,
               int64_t max_total_len) {
  Plan p = {};
  const int g = static_cast<int>(hq / hkv);
  const bool decode = max_q_len <= 1;
  p.rmax = decode ? (g <= 8 ? 8 : (g <= 16 ? 16 : 64)) : 64;
  if (g > p.rmax) p.rmax = 64;
  p.qt = std::max(1, p.rmax / g);
  p.nqt = static_cast<int>((std::max<int64_t>(max_q_len, 1) + p.qt - 1) / p.qt);
  p.items = num_seqs * hkv * p.nqt;
  const int64_t max_tiles = std::max<int64_t>(1, (max_total_len + kTK - 1) / kTK);
  // Short chunks leave few items: split their keys finely (down to one
  // 16-key tile per CTA) so that about four CTAs per SM share the work and
  // each CTA's serial key walk stays short.
  const int64_t target = 4LL * num_sms();
  int64_t ns = (target + p.items - 1) / p.items;
  ns = std::min<int64_t>(ns, max_tiles);
  ns = std::max<int64_t>(1, std::min<int64_t>(ns, 64));
  p.tps = static_cast<int>((max_tiles + ns - 1) / ns);
  p.nsplit = static_cast<int>((max_tiles + p.tps - 1) / p.tps);
  p.counter_bytes = (p.items * 4 + 255) / 256 * 256;
  p.part_bytes = p.nsplit > 1 ? p.items * p.nsplit * p.rmax * (d + 4) * 4 : 0;
  (void)d;
  return p;
}

template <int D, int RMAX>
int launch_attn(const AttnArgs& a, const Plan& p, cudaStream_t stream) {
  constexpr int D4 = D / 4;
  const size_t smem = (static_cast<size_t>(RMAX) * D4 + 2 * kTK * D4) * 16 +
                      (static_cast<size_t>(RMAX) * (kTK + 1) + 3 * RMAX) * 4;
  auto kern = paged_attn_kernel<D, RMAX>;
  if (smem > 32 * 1024 && set_smem_optin(reinterpret_cast<const void*>(kern), smem) != KSH_OK)
    return KSH_ERR_CUDA;
  return launch(kern, dim3(static_cast<unsigned>(p.items), static_cast<unsigned>(p.nsplit)),
                dim3(kThreads), smem, stream, a);
}

}  // namespace
}  // namespace ksh

using namespace ksh;

extern "C" int64_t ksh_paged_attention_workspace_size(int64_t num_seqs, int64_t hq,
                                                      int64_t hkv, int64_t d,
                                                      int64_t max_q_len,
                                                      int64_t max_total_len) {
  if (num_seqs <= 0 || hq <= 0 || hkv <= 0 || hq % hkv != 0 || d <= 0) return 0;
  const Plan p = make_plan(num_seqs, hq, hkv, d, max_q_len, max_total_len);
  return p.counter_bytes + p.part_bytes;
}

extern "C" int ksh_paged_attention(const float* q, int64_t hq, int64_t d, const float* pool,
                                   int64_t num_blocks, int64_t num_layers, int64_t layer,
                                   int64_t hkv, int64_t block_size,
                                   const int32_t* block_tables, int64_t max_blocks,
                                   const int32_t* q_start, const int32_t* prefix_lens,
                                   int64_t num_seqs, int64_t max_q_len, int64_t max_total_len,
                                   float* out, void* workspace, int64_t workspace_bytes,
                                   int32_t* flags, void* stream) {
  KSH_CHECK_ARG(hq > 0 && hkv > 0 && hq % hkv == 0 && d > 0 && num_blocks > 0 &&
                num_layers > 0 && layer >= 0 && layer < num_layers && block_size > 0 &&
                max_blocks > 0 && num_seqs >= 0 && max_q_len >= 0 && max_total_len >= 0);
  KSH_CHECK_ARG(q && pool && block_tables && q_start && prefix_lens && out);
  if (num_seqs == 0 || max_q_len == 0) return KSH_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  AttnArgs a = {};
  a.q = q;
  a.pool = pool;
  a.block_tables = block_tables;
  a.q_start = q_start;
  a.prefix_lens = prefix_lens;
  a.out = out;
  a.flags = flags;
  a.num_blocks = num_blocks;
  a.num_layers = num_layers;
  a.layer = layer;
  a.hkv = hkv;
  a.hq = hq;
  a.bs = block_size;
  a.max_blocks = max_blocks;
  a.g = static_cast<int>(hq / hkv);
  a.scale = static_cast<float>(1.0 / sqrt(static_cast<double>(d)));
  const bool fast = (d == 64 || d == 128) && (reinterpret_cast<uintptr_t>(pool) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(q) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  if (!fast) {
    if (d > 256 || max_q_len > 65535 || hq > 65535 || num_seqs > 65535) return KSH_ERR_UNSUPPORTED;
    return launch(paged_attn_generic_kernel,
                  dim3(static_cast<unsigned>(max_q_len), static_cast<unsigned>(hq),
                       static_cast<unsigned>(num_seqs)),
                  dim3(32), 0, st, a, static_cast<int>(d), static_cast<int>(max_q_len));
  }
  const Plan p = make_plan(num_seqs, hq, hkv, d, max_q_len, max_total_len);
  if (p.items > INT32_MAX) return KSH_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < p.counter_bytes + p.part_bytes) return KSH_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return KSH_ERR_ALIGN;
  a.counters = static_cast<uint32_t*>(workspace);
  a.part = reinterpret_cast<float*>(static_cast<char*>(workspace) + p.counter_bytes);
  if (p.nsplit > 1) {
    // The split counters must start at zero.  The last CTA of each item
    // resets its counter, but the caller's workspace may hold anything on
    // its first use, so clear them here on the caller's stream.
    const cudaError_t e = cudaMemsetAsync(workspace, 0, static_cast<size_t>(p.items) * 4, st);
    if (e != cudaSuccess) return record_cuda_error(e);
  }
  a.qt = p.qt;
  a.nqt = p.nqt;
  a.nsplit = p.nsplit;
  a.tps = p.tps;
  a.rmax = p.rmax;
  if (d == 64) {
    if (p.rmax == 8) return launch_attn<64, 8>(a, p, st);
    if (p.rmax == 16) return launch_attn<64, 16>(a, p, st);
    return launch_attn<64, 64>(a, p, st);
  }
  if (p.rmax == 8) return launch_attn<128, 8>(a, p, st);
  if (p.rmax == 16) return launch_attn<128, 16>(a, p, st);
  return launch_attn<128, 64>(a, p, st);
}
