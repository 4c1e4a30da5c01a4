// Small per-token kernels of the forward: embedding gather, RMSNorm, RoPE +
// K/V scatter into the block pool, and the on-device greedy-decode
// bookkeeping that lets a decode step replay from a CUDA graph.

#include "common.cuh"

namespace ksh {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) red[wid] = v;
  __syncthreads();
  if (wid == 0) {
    float t = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0.0f;
    t = warp_sum(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

// HF Embedding lookup (engine/model.py:107).  Out-of-range ids raise
// KSH_FLAG_BAD_TOKEN and produce a zero row.
__global__ void __launch_bounds__(kThreads)
embedding_kernel(const int64_t* __restrict__ ids, const float* __restrict__ table,
                 int64_t vocab, int64_t hidden, float* __restrict__ out, int32_t* flags) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t t = blockIdx.x;
  const int64_t id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0) raise_flag(flags, KSH_FLAG_BAD_TOKEN);
  const float* src = table + (ok ? id : 0) * hidden;
  float* dst = out + t * hidden;
  for (int64_t j = threadIdx.x; j < hidden; j += blockDim.x) dst[j] = ok ? src[j] : 0.0f;
}

// LlamaRMSNorm (HF, called at engine/model.py:113,146,150):
//   h = x * rsqrt(mean(x^2) + eps); y = w * h
// rsqrt is 1 / sqrt with IEEE sqrt and division, as the CPU reference.
__global__ void __launch_bounds__(kThreads)
rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
               float* __restrict__ y, int64_t hidden, float eps) {
  __shared__ float red[32];
  grid_dep_wait();
  grid_dep_launch();
  const float* xr = x + static_cast<int64_t>(blockIdx.x) * hidden;
  float* yr = y + static_cast<int64_t>(blockIdx.x) * hidden;
  float ss = 0.0f;
  for (int64_t j = threadIdx.x; j < hidden; j += blockDim.x) ss = fmaf(xr[j], xr[j], ss);
  ss = block_sum(ss, red);
  const float var = __fdiv_rn(ss, static_cast<float>(hidden));
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  for (int64_t j = threadIdx.x; j < hidden; j += blockDim.x)
    yr[j] = __fmul_rn(w[j], __fmul_rn(xr[j], inv));
}

// RoPE at absolute positions + K/V scatter (engine/model.py:47-55, 121-129).
//   out[j]       = x[j] * cos_j - x[j + d/2] * sin_j
//   out[j + d/2] = x[j + d/2] * cos_j + x[j] * sin_j
// Products and sum are rounded separately (no FMA contraction), matching the
// reference's elementwise tensor ops.  One CTA per token.
__global__ void __launch_bounds__(kThreads)
rope_kv_kernel(const float* __restrict__ qkv, int64_t hq, int64_t hkv, int64_t d,
               const int64_t* __restrict__ positions, const int64_t* __restrict__ slots,
               const float* __restrict__ rcos, const float* __restrict__ rsin,
               int64_t max_pos, float* __restrict__ q_out, float* __restrict__ pool,
               int64_t num_blocks, int64_t num_layers, int64_t layer, int64_t bs,
               int32_t* flags) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t t = blockIdx.x;
  const int64_t half = d / 2;
  const int64_t width = (hq + 2 * hkv) * d;
  const float* row = qkv + t * width;
  int64_t pos = positions[t];
  const bool pos_ok = pos >= 0 && pos < max_pos;
  if (!pos_ok) {
    if (threadIdx.x == 0) raise_flag(flags, KSH_FLAG_BAD_POSITION);
    pos = 0;
  }
  const int64_t slot = slots[t];
  const int64_t blk = slot >= 0 ? slot / bs : -1;
  const int64_t off = slot >= 0 ? slot % bs : 0;
  const bool slot_ok = blk >= 0 && blk < num_blocks;
  if (!slot_ok && threadIdx.x == 0) raise_flag(flags, KSH_FLAG_BAD_SLOT);
  const float* cr = rcos + pos * half;
  const float* sr = rsin + pos * half;
  // pool[blk, layer, kv, h, off, :]
  const int64_t head_stride = bs * d;
  const int64_t kv_stride = hkv * head_stride;
  float* kbase = pool + ((blk * num_layers + layer) * 2) * kv_stride + off * d;
  // rotate q and k heads
  const int64_t nrot = (hq + hkv) * half;
  for (int64_t i = threadIdx.x; i < nrot; i += blockDim.x) {
    const int64_t h = i / half, j = i - h * half;
    const float* src = row + h * d;
    const float x1 = src[j], x2 = src[j + half];
    const float c = cr[j], s = sr[j];
    const float o1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(-x2, s));
    const float o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    if (h < hq) {
      float* dst = q_out + (t * hq + h) * d;
      dst[j] = o1;
      dst[j + half] = o2;
    } else if (slot_ok) {
      float* dst = kbase + (h - hq) * head_stride;
      dst[j] = o1;
      dst[j + half] = o2;
    }
  }
  if (slot_ok) {
    const float* vsrc = row + (hq + hkv) * d;
    float* vbase = kbase + kv_stride;
    for (int64_t i = threadIdx.x; i < hkv * d; i += blockDim.x) {
      const int64_t h = i / d, j = i - h * d;
      vbase[h * head_stride + j] = vsrc[i];
    }
  }
}

__global__ void decode_advance_kernel(const int64_t* __restrict__ next, int64_t batch,
                                      int64_t* ids, int64_t* positions, int32_t* prefix_lens,
                                      int64_t* slots, const int32_t* __restrict__ block_tables,
                                      int64_t max_blocks, int64_t bs, int64_t* history,
                                      int64_t hist_stride, int64_t* step, int32_t* flags) {
  grid_dep_wait();
  grid_dep_launch();
  const int64_t st = *step;
  for (int64_t b = threadIdx.x + static_cast<int64_t>(blockIdx.x) * blockDim.x; b < batch;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = next[b];
    ids[b] = tok;
    if (history && st < hist_stride) history[b * hist_stride + st] = tok;
    const int64_t p = positions[b] + 1;
    positions[b] = p;
    prefix_lens[b] = static_cast<int32_t>(p);
    const int64_t j = p / bs;
    int64_t slot = -1;
    if (j < max_blocks) {
      slot = static_cast<int64_t>(block_tables[b * max_blocks + j]) * bs + p % bs;
    } else {
      raise_flag(flags, KSH_FLAG_BAD_LENGTH);
    }
    slots[b] = slot;
  }
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x == 0) *step = st + 1;
}

}  // namespace
}  // namespace ksh

using namespace ksh;

extern "C" int ksh_embedding(const int64_t* ids, int64_t m, const float* table, int64_t vocab,
                             int64_t hidden, float* out, int32_t* flags, void* stream) {
  KSH_CHECK_ARG(m >= 0 && vocab > 0 && hidden > 0 && ids && table && out && m <= INT32_MAX);
  return launch(embedding_kernel, dim3(static_cast<unsigned>(m)), dim3(kThreads), 0,
                static_cast<cudaStream_t>(stream), ids, table, vocab, hidden, out, flags);
}

extern "C" int ksh_rmsnorm(const float* x, const float* w, float* y, int64_t m, int64_t hidden,
                           float eps, void* stream) {
  KSH_CHECK_ARG(m >= 0 && hidden > 0 && x && w && y && m <= INT32_MAX);
  return launch(rmsnorm_kernel, dim3(static_cast<unsigned>(m)), dim3(kThreads), 0,
                static_cast<cudaStream_t>(stream), x, w, y, hidden, eps);
}

extern "C" int ksh_rope_kv_write(const float* qkv, int64_t m, int64_t hq, int64_t hkv,
                                 int64_t d, const int64_t* positions,
                                 const int64_t* slot_mapping, const float* rope_cos,
                                 const float* rope_sin, int64_t max_pos, float* q_out,
                                 float* pool, int64_t num_blocks, int64_t num_layers,
                                 int64_t layer, int64_t block_size, int32_t* flags,
                                 void* stream) {
  KSH_CHECK_ARG(m >= 0 && hq > 0 && hkv > 0 && d > 0 && d % 2 == 0 && max_pos > 0);
  KSH_CHECK_ARG(num_blocks > 0 && num_layers > 0 && layer >= 0 && layer < num_layers &&
                block_size > 0 && m <= INT32_MAX);
  KSH_CHECK_ARG(qkv && positions && slot_mapping && rope_cos && rope_sin && q_out && pool);
  return launch(rope_kv_kernel, dim3(static_cast<unsigned>(m)), dim3(kThreads), 0,
                static_cast<cudaStream_t>(stream), qkv, hq, hkv, d, positions, slot_mapping,
                rope_cos, rope_sin, max_pos, q_out, pool, num_blocks, num_layers, layer,
                block_size, flags);
}

extern "C" int ksh_decode_advance(const int64_t* next, int64_t batch, int64_t* ids,
                                  int64_t* positions, int32_t* prefix_lens, int64_t* slots,
                                  const int32_t* block_tables, int64_t max_blocks,
                                  int64_t block_size, int64_t* history, int64_t hist_stride,
                                  int64_t* step, int32_t* flags, void* stream) {
  KSH_CHECK_ARG(batch > 0 && max_blocks > 0 && block_size > 0 && next && ids && positions &&
                prefix_lens && slots && block_tables && step);
  const int64_t nb = (batch + 255) / 256;
  KSH_CHECK_ARG(nb <= 1);  // single CTA: the step counter is bumped after a CTA barrier
  return launch(decode_advance_kernel, dim3(1), dim3(256), 0, static_cast<cudaStream_t>(stream),
                next, batch, ids, positions, prefix_lens, slots, block_tables, max_blocks,
                block_size, history, hist_stride, step, flags);
}
