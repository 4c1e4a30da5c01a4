// Host-side runtime helpers: device properties, launch options, status text.

#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <unordered_map>
#include <utility>

#include <cudaTypedefs.h>

#include "linear.cuh"
#include "tc_common.cuh"

namespace ksh {

namespace {
std::atomic<int> g_last_cuda_error{0};

int env_flag(const char* name, int dflt) {
  const char* v = getenv(name);
  if (!v || !*v) return dflt;
  return atoi(v) != 0;
}
std::atomic<int> g_pdl{env_flag("KSH_PDL", 1)};
std::atomic<int> g_prefetch{env_flag("KSH_L2_PREFETCH", 1)};
std::atomic<int> g_resident{env_flag("KSH_GEMV_RESIDENT", 1)};
}  // namespace

int set_gemv_resident_enabled(int on) { return g_resident.exchange(on ? 1 : 0); }
bool gemv_resident_enabled() { return g_resident.load(std::memory_order_relaxed) != 0; }

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }
bool prefetch_enabled() { return g_prefetch.load(std::memory_order_relaxed) != 0; }

int record_cuda_error(cudaError_t e) {
  g_last_cuda_error.store(static_cast<int>(e));
  return KSH_ERR_CUDA;
}

namespace {
std::atomic<uint64_t> g_launches{0};
}  // namespace

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int num_sms() {
  static std::mutex mu;
  static std::unordered_map<int, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  cache[dev] = n;
  return n;
}

int set_smem_optin(const void* kernel, size_t bytes) {
  // cudaFuncSetAttribute is per device; cache (device, kernel) -> bytes set.
  static std::mutex mu;
  static std::unordered_map<const void*, std::unordered_map<int, size_t>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  size_t& cur = done[kernel][dev];
  if (cur >= bytes) return KSH_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(bytes));
  if (e != cudaSuccess) return record_cuda_error(e);
  cur = bytes;
  return KSH_OK;
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}
}  // namespace

bool tensor_map_encoder_available() { return encode_fn() != nullptr; }

bool make_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base,
                        uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
                        uint32_t box_outer, CUtensorMapSwizzle sw) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int resident_ctas(const void* kernel, int threads, size_t smem) {
  static std::mutex mu;
  struct Key {
    const void* k;
    int dev, threads;
    size_t smem;
    bool operator==(const Key& o) const {
      return k == o.k && dev == o.dev && threads == o.threads && smem == o.smem;
    }
  };
  struct Hash {
    size_t operator()(const Key& x) const {
      return std::hash<const void*>()(x.k) ^ (static_cast<size_t>(x.dev) << 1) ^
             (static_cast<size_t>(x.threads) << 8) ^ (x.smem << 20);
    }
  };
  static std::unordered_map<Key, int, Hash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const Key key{kernel, dev, threads, smem};
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess) {
    cudaGetLastError();
    n = 1;
  }
  n = n < 1 ? 1 : n;
  cache[key] = n;
  return n;
}

namespace {
// The library's two forms of device wait, run on something nothing will ever
// complete unless `arrive` is set: an mbarrier phase (as the TMA / tcgen05
// pipelines wait) and a flag word in global memory (as an inter-CTA or
// inter-GPU hand-off waits).  Each gives up after `polls` attempts with the
// same primitive the kernels use and raises KSH_FLAG_TIMEOUT; `where`
// records which wait gave up (1 = mbarrier, 2 = flag) for the host.
__global__ void bounded_wait_check_kernel(uint32_t polls, int arrive,
                                          const volatile int32_t* gflag, int32_t* flags,
                                          int32_t* where) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
  }
  __syncthreads();
  if (arrive && threadIdx.x == 0) tc::mbar_arrive(&bar);
  const bool ok_bar = tc::mbar_wait(&bar, 0, polls);
  bool ok_flag = arrive != 0;
  if (!arrive) {
    for (uint32_t i = 0; i < polls && !ok_flag; ++i) {
      ok_flag = *gflag != 0;
      if (!ok_flag) __nanosleep(32);
    }
  }
  if (threadIdx.x == 0) {
    if (!ok_bar || !ok_flag) raise_flag(flags, KSH_FLAG_TIMEOUT);
    if (where) *where = (ok_bar ? 0 : 1) | (ok_flag ? 0 : 2);
  }
}
}  // namespace

int64_t cluster_slots(const void* kernel, int threads, size_t smem, int cluster) {
  if (cluster <= 1) return static_cast<int64_t>(resident_ctas(kernel, threads, smem)) * num_sms();
  static std::mutex mu;
  struct Key {
    const void* k;
    int dev, threads, cluster;
    size_t smem;
    bool operator==(const Key& o) const {
      return k == o.k && dev == o.dev && threads == o.threads && cluster == o.cluster &&
             smem == o.smem;
    }
  };
  struct Hash {
    size_t operator()(const Key& x) const {
      return std::hash<const void*>()(x.k) ^ (static_cast<size_t>(x.dev) << 1) ^
             (static_cast<size_t>(x.threads) << 8) ^ (static_cast<size_t>(x.cluster) << 16) ^
             (x.smem << 24);
    }
  };
  static std::unordered_map<Key, int64_t, Hash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const Key key{kernel, dev, threads, cluster, smem};
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(cluster), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = static_cast<unsigned>(cluster);
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = std::max(1, num_sms() / cluster);
  }
  const int64_t slots = static_cast<int64_t>(n) * cluster;
  cache[key] = slots;
  return slots;
}

}  // namespace ksh

extern "C" int ksh_check_bounded_wait(int64_t polls, int arrive, const int32_t* wait_flag,
                                      int32_t* flags, int32_t* where, void* stream) {
  KSH_CHECK_ARG(polls > 0 && polls <= (1LL << 24) && wait_flag && flags);
  return ksh::launch(ksh::bounded_wait_check_kernel, dim3(1), dim3(32), 0,
                     static_cast<cudaStream_t>(stream), static_cast<uint32_t>(polls), arrive,
                     wait_flag, flags, where);
}

extern "C" int ksh_abi_version(void) { return 1; }

extern "C" int ksh_last_cuda_error(void) { return ksh::g_last_cuda_error.load(); }

extern "C" int ksh_set_pdl(int enabled) { return ksh::g_pdl.exchange(enabled ? 1 : 0); }

extern "C" int ksh_set_gemv_resident(int enabled) { return ksh::set_gemv_resident_enabled(enabled); }

extern "C" int ksh_set_gemv_tc(int mode) { return ksh::set_gemv_tc_mode(mode); }

extern "C" const char* ksh_status_string(int status) {
  switch (status) {
    case KSH_OK: return "ok";
    case KSH_ERR_SHAPE: return "invalid shape or size argument";
    case KSH_ERR_ALIGN: return "pointer not aligned as required";
    case KSH_ERR_CUDA: return "CUDA launch failed";
    case KSH_ERR_UNSUPPORTED: return "shape not supported by the kernels";
    case KSH_ERR_WORKSPACE: return "workspace missing or too small";
    case KSH_ERR_TOO_LARGE: return "size exceeds the fixed scratch array of this entry point";
    default: return "unknown status";
  }
}

extern "C" uint64_t ksh_kernel_launches(void) { return ksh::g_launches.load(); }
