// Library-level entry points: error string, device query, ABI self-description.
#include <cxxabi.h>
#include <map>
#include <mutex>
#include <stdlib.h>
#include <string.h>

#include "host_common.h"

namespace qb {

static thread_local char g_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_error[0] = '\0'; }

static thread_local const void* g_last_kernel = nullptr;
static thread_local char g_last_kernel_name[512] = "";

void note_launch(const void* kernel) { g_last_kernel = kernel; }

static constexpr int kMaxDevices = 64;
static DeviceFacts g_facts[kMaxDevices];
static bool g_facts_ready[kMaxDevices];
static std::mutex g_facts_mutex;

static const DeviceFacts* device_facts(int device) {
  if (device < 0 || device >= kMaxDevices) {
    set_error(QB_ERR_INVALID, "device ordinal %d out of range", device);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_facts_mutex);
  if (!g_facts_ready[device]) {
    DeviceFacts f;
    f.device = device;
    cudaError_t e = cudaDeviceGetAttribute(&f.sm_count, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&f.cc_major, cudaDevAttrComputeCapabilityMajor, device);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&f.cc_minor, cudaDevAttrComputeCapabilityMinor, device);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&f.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if (e != cudaSuccess) {
      set_error(QB_ERR_CUDA, "cudaDeviceGetAttribute(device %d): %s", device, cudaGetErrorString(e));
      return nullptr;
    }
    if (f.cc_major < 10) {
      set_error(QB_ERR_UNSUPPORTED,
                "device %d has compute capability %d.%d; this library is built for sm_100a only",
                device, f.cc_major, f.cc_minor);
      return nullptr;
    }
    g_facts[device] = f;
    g_facts_ready[device] = true;
  }
  return &g_facts[device];
}

int cached_occupancy(const void* kernel, int threads, size_t smem) {
  struct Key {
    const void* k; int t; size_t s; int dev;
    bool operator<(const Key& o) const {
      if (k != o.k) return k < o.k;
      if (t != o.t) return t < o.t;
      if (s != o.s) return s < o.s;
      return dev < o.dev;
    }
  };
  static std::map<Key, int> cache;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  const Key key{kernel, threads, smem, dev};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  if (smem > 32 * 1024) ensure_kernel_attributes(kernel, smem, 1);
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, smem) != cudaSuccess) {
    cudaGetLastError();
    occ = 1;
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = occ;
  return occ;
}

int cached_max_clusters(const void* kernel, int threads, size_t smem, int cluster_n) {
  struct Key {
    const void* k; int t; size_t s; int c; int dev;
    bool operator<(const Key& o) const {
      if (k != o.k) return k < o.k;
      if (t != o.t) return t < o.t;
      if (s != o.s) return s < o.s;
      if (c != o.c) return c < o.c;
      return dev < o.dev;
    }
  };
  static std::map<Key, int> cache;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  const Key key{kernel, threads, smem, cluster_n, dev};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  if (smem > 32 * 1024 || cluster_n > 8) ensure_kernel_attributes(kernel, smem, cluster_n);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(cluster_n), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster_n);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n < 1) {
    cudaGetLastError();
    n = 0;  // unknown: the caller falls back to resident CTAs / cluster size
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = n;
  return n;
}

int ensure_kernel_attributes(const void* kernel, size_t smem, int cluster_n) {
  struct Key {
    const void* k; int dev;
    bool operator<(const Key& o) const { return k != o.k ? k < o.k : dev < o.dev; }
  };
  struct Val { size_t smem; bool nonportable; };
  static std::map<Key, Val> cache;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  Val& v = cache[Key{kernel, dev}];
  if (smem > v.smem) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return static_cast<int>(e);
    v.smem = smem;
  }
  if (cluster_n > 8 && !v.nonportable) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return static_cast<int>(e);
    v.nonportable = true;
  }
  return 0;
}

// Counter of timed-out waits of the shared-memory ring kernels, one per device (the variable is
// part of the library image on every GPU; the host needs its device address).
__device__ unsigned int g_ring_timeouts;

unsigned int* ring_timeout_counter() {
  static unsigned int* ptrs[kMaxDevices];
  static std::mutex mu;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error(QB_ERR_CUDA, "ring: no current device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_ring_timeouts);
    if (e != cudaSuccess || p == nullptr) {
      set_error(QB_ERR_CUDA, "ring: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return nullptr;
    }
    ptrs[dev] = static_cast<unsigned int*>(p);
  }
  return ptrs[dev];
}

const DeviceFacts* current_device_facts() {
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) {
    set_error(QB_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    return nullptr;
  }
  return device_facts(device);
}

}  // namespace qb

using namespace qb;

extern "C" int qb_query_device(int32_t device, qb_device_info* info) {
  clear_error();
  if (info == nullptr) return set_error(QB_ERR_INVALID, "query_device: null info");
  const DeviceFacts* f = device < 0 ? current_device_facts() : device_facts(device);
  if (f == nullptr) return g_error[0] && strstr(g_error, "built for") ? QB_ERR_UNSUPPORTED : QB_ERR_CUDA;
  memset(info, 0, sizeof(*info));
  info->device = f->device;
  info->sm_count = f->sm_count;
  info->cc_major = f->cc_major;
  info->cc_minor = f->cc_minor;
  info->max_smem_optin = f->max_smem_optin;
  info->max_cluster = 16;
  return QB_OK;
}

extern "C" int qb_ring_timeouts(uint32_t* count) {
  clear_error();
  if (count == nullptr) return set_error(QB_ERR_INVALID, "ring_timeouts: null output");
  unsigned int* p = ring_timeout_counter();
  if (p == nullptr) return QB_ERR_CUDA;
  unsigned int v = 0;
  cudaError_t e = cudaMemcpy(&v, p, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess)
    return set_error(QB_ERR_CUDA, "ring_timeouts: cudaMemcpy: %s", cudaGetErrorString(e));
  *count = v;
  return QB_OK;
}

extern "C" const char* qb_last_error(void) { return g_error; }

extern "C" const char* qb_last_kernel(void) {
  g_last_kernel_name[0] = '\0';
  if (g_last_kernel == nullptr) return g_last_kernel_name;
  const char* mangled = nullptr;
  if (cudaFuncGetName(&mangled, g_last_kernel) != cudaSuccess || mangled == nullptr) {
    cudaGetLastError();
    return g_last_kernel_name;
  }
  int status = 0;
  char* pretty = abi::__cxa_demangle(mangled, nullptr, nullptr, &status);
  snprintf(g_last_kernel_name, sizeof(g_last_kernel_name), "%s", status == 0 && pretty ? pretty : mangled);
  free(pretty);
  return g_last_kernel_name;
}

extern "C" int qb_abi_version(void) { return QB_ABI_VERSION; }

extern "C" int qb_sizeof_args(int32_t which) {
  switch (which) {
    case 0: return (int)sizeof(qb_launch_cfg);
    case 1: return (int)sizeof(qb_norm_fwd_args);
    case 2: return (int)sizeof(qb_norm_bwd_args);
    case 3: return (int)sizeof(qb_colsum_args);
    case 4: return (int)sizeof(qb_softmax_fwd_args);
    case 5: return (int)sizeof(qb_softmax_bwd_args);
    case 6: return (int)sizeof(qb_ce_fwd_args);
    case 7: return (int)sizeof(qb_ce_bwd_args);
    case 8: return (int)sizeof(qb_ce_combine_args);
    case 9: return (int)sizeof(qb_device_info);
    case 10: return (int)sizeof(qb_norm_bwd_static_args);
    case 11: return (int)sizeof(qb_rms_final_reduce_args);
    case 12: return (int)sizeof(qb_topk_fwd_args);
    case 13: return (int)sizeof(qb_topk_bwd_args);
    case 14: return (int)sizeof(qb_colsum_allreduce_args);
    case 15: return (int)sizeof(qb_ce_combine_exchange_args);
    default: return -1;
  }
}
