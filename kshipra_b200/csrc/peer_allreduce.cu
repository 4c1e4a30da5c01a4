// Sum all-reduce of the row-parallel projections' partial sums over the peer
// memory of the tensor-parallel ranks (one process per GPU, NVLink).
//
// Replaces, for the decode step, the NCCL all-reduce after o_proj and
// down_proj of a tensor-parallel layer (the reference runs one process and
// has no collective; the split is this build's, model.py:111-148 summed over
// the ranks' heads and MLP columns).  Each rank's buffer (symmetric memory:
// the same size on every rank, every rank's buffer mapped into every rank's
// address space) holds
//
//   partial[2][n_max]  the producing GEMM's output, written in place,
//   reduced[2][n_max]  this rank's reduced slice,
//   flags[2][G][R]     one 32-bit word per (phase, CTA index, source rank),
//
// two of each buffer used alternately by consecutive calls.  A call (two
// phases, plain peer loads and stores, no multicast):
//
// 1. CTA c of every rank announces the call's epoch to CTA c of every peer,
//    waits until all peers have announced it (their partial sums are then
//    complete), sums sub-range c of its own slice of the n floats over all
//    ranks in rank order, and stores it in its reduced buffer;
// 2. it announces that, waits for all peers, and gathers sub-range c of every
//    rank's slice from the peers' reduced buffers into the output.
//
// With two ranks one phase does: after the first barrier every rank sums all
// n floats from both partial buffers itself (the reads of the second phase
// would cost as much as the extra reads, and a barrier more).
//
// Every rank gets the same bits (each slice is summed once, in rank order).
// A CTA only waits for the CTAs of the same index on the other GPUs, so no
// CTA of one GPU waits for another of the same GPU; the grid is small enough
// to be resident at once.  The alternate buffers make a call's writes safe:
// the partial (reduced) buffer a call reads is next written two calls later,
// after every rank has passed the first barrier of the call in between,
// which it can only do once it has finished this one.  Epochs are per-CTA
// counters in device memory, so the call can be captured in a CUDA graph and
// replayed.  Every wait is bounded: a peer that does not arrive within the
// limit raises KSH_FLAG_TIMEOUT and the kernel returns.

#include "common.cuh"

namespace ksh {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxRanks = 8;
constexpr int kGrid = 128;                // CTAs per call (every rank the same)
constexpr int kOneShotRanks = 2;          // up to this many ranks: one phase, every rank sums all
constexpr uint32_t kSpin = 1u << 22;      // polls of a flag before giving up (~0.3 s)

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct ArArgs {
  const uint64_t* peers;   // [R] base of every rank's buffer, in this process's address space
  float* out;              // [n]
  uint32_t* epochs;        // [kGrid] this rank's per-CTA call counters
  int32_t* flags;          // status word
  int64_t n, n_max;
  int rank, world, parity;
};

// Announce epoch e in phase ph to CTA blockIdx.x of every rank, then wait
// until every rank has announced it to this CTA.  false: a peer never came.
__device__ bool barrier_peers(const ArArgs& a, int ph, uint32_t e, int64_t flag_off) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) ok_s = 1;
  __syncthreads();
  const int R = a.world;
  if (threadIdx.x < R) {
    // the release store at system scope orders this CTA's earlier writes
    // (made visible to this thread by the barrier above) before the flag
    uint32_t* fl = reinterpret_cast<uint32_t*>(reinterpret_cast<float*>(a.peers[threadIdx.x]) + flag_off);
    st_release_sys(fl + (ph * kGrid + blockIdx.x) * R + a.rank, e);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(
                               reinterpret_cast<const float*>(a.peers[a.rank]) + flag_off) +
                           (ph * kGrid + blockIdx.x) * R + threadIdx.x;
    bool arrived = false;
    for (uint32_t it = 0; it < kSpin; ++it) {
      if (static_cast<int32_t>(ld_acquire_sys(mine) - e) >= 0) {
        arrived = true;
        break;
      }
      if (it >= 256) __nanosleep(64);         // poll fast first: the peers are usually close
    }
    if (!arrived) ok_s = 0;
  }
  __syncthreads();
  return ok_s != 0;
}

__global__ void __launch_bounds__(kThreads)
peer_allreduce_kernel(ArArgs a) {
  __shared__ uint32_t e_s;
  // the partial sums come from the kernel before this one
  grid_dep_wait();
  if (threadIdx.x == 0) e_s = a.epochs[blockIdx.x] + 1u;
  __syncthreads();
  const uint32_t e = e_s;
  const int R = a.world;
  const int64_t flag_off = 4 * a.n_max;
  const int64_t p_off = a.parity * a.n_max, r_off = 2 * a.n_max + a.parity * a.n_max;
  // float4 granularity: slice s of the n floats belongs to rank s, sub-range c to CTA c
  const int64_t n4 = a.n / 4;
  const int64_t slice4 = (n4 + R - 1) / R;
  const int64_t sub4 = (slice4 + kGrid - 1) / kGrid;
  bool ok = barrier_peers(a, 0, e, flag_off);
  if (ok && R <= kOneShotRanks) {
    // one shot: this CTA's 1/G of all n floats straight from every rank's
    // partial, summed in rank order -- one barrier, no second phase
    const int64_t per = (n4 + kGrid - 1) / kGrid;
    const int64_t lo = blockIdx.x * per, hi = min(lo + per, n4);
    float4* out4 = reinterpret_cast<float4*>(a.out);
    for (int64_t i = lo + threadIdx.x; i < hi; i += kThreads) {
      float4 v[kOneShotRanks];
#pragma unroll
      for (int r = 0; r < kOneShotRanks; ++r)
        if (r < R)
          v[r] = __ldcv(reinterpret_cast<const float4*>(
                            reinterpret_cast<const float*>(a.peers[r]) + p_off) + i);
      float4 s = v[0];
#pragma unroll
      for (int r = 1; r < kOneShotRanks; ++r)
        if (r < R) {
          s.x += v[r].x; s.y += v[r].y; s.z += v[r].z; s.w += v[r].w;
        }
      out4[i] = s;
    }
    grid_dep_launch();
    if (threadIdx.x == 0) a.epochs[blockIdx.x] = e;
    return;
  }
  if (ok) {
    // every rank's float4 of this position loaded before any is added, so
    // the peer round trips overlap; summed in rank order
    const int64_t lo = a.rank * slice4 + blockIdx.x * sub4;
    const int64_t hi = min(min(lo + sub4, (a.rank + 1) * slice4), n4);
    float4* red = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.peers[a.rank]) + r_off);
    for (int64_t i = lo + threadIdx.x; i < hi; i += kThreads) {
      float4 v[kMaxRanks];
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < R)
          v[r] = __ldcv(reinterpret_cast<const float4*>(
                            reinterpret_cast<const float*>(a.peers[r]) + p_off) + i);
      float4 s = v[0];
#pragma unroll
      for (int r = 1; r < kMaxRanks; ++r)
        if (r < R) {
          s.x += v[r].x; s.y += v[r].y; s.z += v[r].z; s.w += v[r].w;
        }
      red[i] = s;
    }
    ok = barrier_peers(a, 1, e, flag_off);
  }
  if (ok) {
    // sub-range c of every rank's slice: one float4 per rank in flight
    float4* out4 = reinterpret_cast<float4*>(a.out);
    for (int64_t j = threadIdx.x; j < sub4; j += kThreads) {
      float4 v[kMaxRanks];
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        const int64_t i = r * slice4 + blockIdx.x * sub4 + j;
        if (r < R && blockIdx.x * sub4 + j < slice4 && i < n4)
          v[r] = __ldcv(reinterpret_cast<const float4*>(
                            reinterpret_cast<const float*>(a.peers[r]) + r_off) + i);
      }
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        const int64_t i = r * slice4 + blockIdx.x * sub4 + j;
        if (r < R && blockIdx.x * sub4 + j < slice4 && i < n4) out4[i] = v[r];
      }
    }
  } else if (threadIdx.x == 0) {
    raise_flag(a.flags, KSH_FLAG_TIMEOUT);
  }
  grid_dep_launch();
  if (threadIdx.x == 0) a.epochs[blockIdx.x] = e;
}

}  // namespace
}  // namespace ksh

using namespace ksh;

extern "C" int64_t ksh_peer_allreduce_buffer_floats(int64_t n_max, int world) {
  if (n_max <= 0 || world < 1 || world > kMaxRanks) return 0;
  return 4 * n_max + (2 * kGrid * world + 3) / 4 * 4;
}

extern "C" int64_t ksh_peer_allreduce_epoch_words(void) { return kGrid; }

extern "C" int ksh_peer_allreduce_f32(const uint64_t* peer_buffers, int rank, int world,
                                      int64_t n, int64_t n_max, int parity, float* out,
                                      uint32_t* epochs, int32_t* flags, void* stream) {
  KSH_CHECK_ARG(peer_buffers && out && epochs && world >= 1 && world <= kMaxRanks && rank >= 0 &&
                rank < world && n > 0 && n <= n_max && n % 4 == 0 && n_max % 4 == 0 &&
                (parity == 0 || parity == 1));
  if ((reinterpret_cast<uintptr_t>(out) & 15) != 0) return KSH_ERR_ALIGN;
  ArArgs a = {};
  a.peers = peer_buffers;
  a.out = out;
  a.epochs = epochs;
  a.flags = flags;
  a.n = n;
  a.n_max = n_max;
  a.rank = rank;
  a.world = world;
  a.parity = parity;
  return launch(peer_allreduce_kernel, dim3(kGrid), dim3(kThreads), 0,
                static_cast<cudaStream_t>(stream), a);
}
