// capi.cu — library-wide C entry points and the host launch helpers.
#include <atomic>
#include <mutex>
#include <unordered_map>

#include "common.cuh"

namespace dslpg {

namespace {
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices];  // 0 = not queried yet

struct OccKey {
  int dev;
  const void* fn;
  int block;
  size_t smem;
  bool operator==(const OccKey& o) const {
    return dev == o.dev && fn == o.fn && block == o.block && smem == o.smem;
  }
};
struct OccKeyHash {
  size_t operator()(const OccKey& k) const {
    size_t h = std::hash<const void*>()(k.fn);
    h ^= (static_cast<size_t>(k.dev) << 1) ^ (static_cast<size_t>(k.block) << 9) ^ (k.smem << 21);
    return h;
  }
};
std::mutex g_occ_mu;
// The kernel-shape override of dslpg_set_kernel_path: per host thread, so a
// test or benchmark that forces one shape never changes another thread's launches.
thread_local int g_path = DSLPG_PATH_AUTO;
struct SmemKey {
  int dev;
  const void* fn;
  bool operator==(const SmemKey& o) const { return dev == o.dev && fn == o.fn; }
};
struct SmemKeyHash {
  size_t operator()(const SmemKey& k) const { return std::hash<const void*>()(k.fn) ^ static_cast<size_t>(k.dev); }
};
std::unordered_map<SmemKey, size_t, SmemKeyHash> g_smem;
std::unordered_map<OccKey, int, OccKeyHash> g_occ;
}  // namespace

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  int n = g_sm_count[dev];
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev] = n;  // benign race: every writer stores the same value
  }
  return n;
}

int persistent_grid(const void* kernel, int block, size_t smem, int64_t work_ctas) {
  if (work_ctas <= 0) return 0;
  int dev = 0;
  cudaGetDevice(&dev);
  int occ = 0;
  {
    std::lock_guard<std::mutex> lk(g_occ_mu);
    auto it = g_occ.find(OccKey{dev, kernel, block, smem});
    if (it != g_occ.end()) occ = it->second;
  }
  if (occ == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, block, smem) != cudaSuccess ||
        occ <= 0)
      occ = 1;
    std::lock_guard<std::mutex> lk(g_occ_mu);
    g_occ[OccKey{dev, kernel, block, smem}] = occ;
  }
  int64_t full = static_cast<int64_t>(occ) * sm_count();
  return static_cast<int>(work_ctas < full ? work_ctas : full);
}

int max_active_clusters(const void* kernel, const cudaLaunchConfig_t& cfg, int cluster_size, int fallback) {
  int dev = 0;
  cudaGetDevice(&dev);
  // cached beside the occupancy figures; a negative block field marks a cluster count
  const OccKey key{dev, kernel, -(cluster_size * 4096 + static_cast<int>(cfg.blockDim.x)), cfg.dynamicSmemBytes};
  {
    std::lock_guard<std::mutex> lk(g_occ_mu);
    auto it = g_occ.find(key);
    if (it != g_occ.end()) return it->second;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n < 1) {
    cudaGetLastError();
    n = fallback;
  }
  if (n < 1) n = 1;
  std::lock_guard<std::mutex> lk(g_occ_mu);
  g_occ[key] = n;
  return n;
}

cudaError_t allow_dynamic_smem(const void* kernel, size_t bytes) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_occ_mu);
  auto it = g_smem.find(SmemKey{dev, kernel});
  if (it != g_smem.end() && it->second >= bytes) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e == cudaSuccess) {
    g_smem[SmemKey{dev, kernel}] = bytes;
    // occupancy depends on the attribute: forget cached figures for this kernel
    for (auto o = g_occ.begin(); o != g_occ.end();) {
      if (o->first.fn == kernel && o->first.dev == dev) o = g_occ.erase(o);
      else ++o;
    }
  }
  return e;
}

int kernel_path() { return g_path; }

}  // namespace dslpg

extern "C" int dslpg_set_kernel_path(int path) {
  if (path < DSLPG_PATH_AUTO || path > DSLPG_PATH_CLUSTER) return DSLPG_ERR_BAD_ARGUMENT;
  dslpg::g_path = path;
  return DSLPG_OK;
}

extern "C" int dslpg_get_kernel_path(void) { return dslpg::g_path; }

extern "C" unsigned int dslpg_take_wait_timeouts(void) {
  return dslpg::take_wait_timeouts_rownorm() + dslpg::take_wait_timeouts_rowstat() + dslpg::take_wait_timeouts_ff();
}

extern "C" int dslpg_version(void) { return (0 << 16) | 1; }

extern "C" const char* dslpg_error_string(int code) {
  switch (code) {
    case DSLPG_OK: return "success";
    case DSLPG_ERR_NULL_POINTER: return "dslpg: a required pointer is NULL";
    case DSLPG_ERR_BAD_SHAPE: return "dslpg: invalid shape (sizes must be positive and in range)";
    case DSLPG_ERR_BAD_DTYPE: return "dslpg: unsupported dtype code";
    case DSLPG_ERR_BAD_EPS: return "dslpg: eps must be finite and >= 0";
    case DSLPG_ERR_BAD_ARGUMENT: return "dslpg: invalid argument";
    case DSLPG_ERR_TOO_LARGE:
      return "dslpg: problem too large for dslpg_kernel_ff_static's static scratch "
             "(dslpg_kernel_ff_workspace_bytes(M, K) must be <= 16 MiB + 64 KiB); use dslpg_kernel_ff";
    default: break;
  }
  if (code > 0) return cudaGetErrorString(static_cast<cudaError_t>(code));
  return "dslpg: unknown error";
}
