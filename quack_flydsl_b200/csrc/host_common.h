// Host-side helpers shared by the launchers: error reporting, device facts, alignment-driven
// vector width, cluster launches.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include "quack_b200.h"

namespace qb {

// Records a message for qb_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);
void clear_error();

struct DeviceFacts {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
  int max_smem_optin = 0;
};
// Facts of the current device (cached per device ordinal).  Returns nullptr and sets the error
// on failure.
const DeviceFacts* current_device_facts();

inline bool is_float_dtype(int dt) { return dt == QB_F32 || dt == QB_F16 || dt == QB_BF16; }
inline int host_dtype_bytes(int dt) { return dt == QB_F32 ? 4 : 2; }
inline bool is_pow2(int64_t v) { return v > 0 && (v & (v - 1)) == 0; }
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int next_pow2(int64_t v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

// Tracks the widest vector (in elements, power of two <= 16 bytes / widest element) with which
// every registered tensor can be accessed: the chunk start addresses base + (row*stride + col)
// must be aligned to the chunk size in bytes for every row and every chunk-aligned column.
struct VecWidth {
  int vec = 8;
  void limit_elems(int64_t n) {  // n must be a multiple of vec (row length, row strides)
    while (vec > 1 && (n % vec) != 0) vec >>= 1;
  }
  void add_tensor(const void* base, int dt, int64_t row_stride) {
    if (base == nullptr) return;
    const int eb = host_dtype_bytes(dt);
    while (vec * eb > 16) vec >>= 1;
    while (vec > 1 && (reinterpret_cast<uintptr_t>(base) % (uintptr_t)(vec * eb)) != 0) vec >>= 1;
    limit_elems(row_stride);
  }
  // Small contiguous per-column tensors (weight, bias): an fp32 chunk wider than 16 bytes is read
  // as two 16-byte accesses, so only min(16, vec * bytes) alignment is needed.
  void add_param(const void* base, int dt) {
    if (base == nullptr) return;
    const int eb = host_dtype_bytes(dt);
    while (vec > 1) {
      const int need = vec * eb > 16 ? 16 : vec * eb;
      if ((reinterpret_cast<uintptr_t>(base) % (uintptr_t)need) == 0) break;
      vec >>= 1;
    }
  }
};

// Geometry of a kernel that keeps whole rows in registers: `tpr` threads (times cluster_n CTAs)
// share a row, each thread owning K chunks of `vec` elements spaced tpr chunks apart.
struct RowPlan {
  int vec = 0;
  int tpr = 0;
  int threads = 0;
  int rows_per_cta = 0;
  int cluster_n = 0;
  int K = 0;             // chunks per thread: 1, 2, 4, 8 (16 only when vec <= 4)
  int cols_per_cta = 0;  // columns owned by one CTA of the cluster
};

// Per-thread row-element capacity of a kernel as a function of the CTA size (what its register
// budget allows at the matching __launch_bounds__).
struct ElemCaps {
  int c256;   // CTAs of <= 256 threads
  int c512;   // CTAs of 257..512 threads
  int c1024;  // CTAs of 513..1024 threads
  int kmax = 0;  // largest instantiated K; 0 = default (16 for vec <= 4, else 8)
  int at(int threads) const { return threads > 512 ? c1024 : (threads > 256 ? c512 : c256); }
};

// Largest chunks-per-thread K (a power of two; 16 only exists for vec <= 4) for a CTA size.
inline int max_k(const ElemCaps& caps, int threads, int vec) {
  const int kmax = caps.kmax > 0 ? caps.kmax : (vec <= 4 ? 16 : 8);
  int k = 1;
  while (k * 2 <= kmax && k * 2 * vec <= caps.at(threads)) k <<= 1;
  return (k * vec <= caps.at(threads)) ? k : 0;
}

// Picks (cluster_n, tpr, threads, K) for a row of N elements accessed `vec` at a time.
// pref_elems_per_cta: a row longer than this is split over a cluster (up to 8 CTAs; 16 only if
// it would not fit otherwise).  k_target: preferred chunks per thread.  Launch overrides in cfg
// win where given; an over-clustered override is clamped so that every CTA of a cluster owns at
// least one chunk (reference: quack/reduction_base.py:28-40).
inline int plan_rows(const char* op, int64_t N, int vec, const ElemCaps& caps,
                     int64_t pref_elems_per_cta, int k_target, int default_threads,
                     const qb_launch_cfg& cfg, RowPlan* out) {
  if (cfg.cluster_n < 0 || cfg.threads_per_row < 0 || cfg.num_threads < 0 ||
      (cfg.cluster_n && !is_pow2(cfg.cluster_n)) || cfg.cluster_n > 16 ||
      (cfg.threads_per_row && !is_pow2(cfg.threads_per_row)) || cfg.threads_per_row > 1024 ||
      (cfg.num_threads && (!is_pow2(cfg.num_threads) || cfg.num_threads < 32)) ||
      cfg.num_threads > 1024)
    return set_error(QB_ERR_INVALID,
                     "%s: bad launch override (threads %d, threads_per_row %d, cluster %d)", op,
                     cfg.num_threads, cfg.threads_per_row, cfg.cluster_n);
  const int64_t chunks = N / vec;
  // Chunks one CTA can hold, over all CTA sizes.
  int64_t max_cap = 0;
  for (int t = 32; t <= 1024; t <<= 1) {
    const int64_t c = (int64_t)t * max_k(caps, t, vec);
    if (c > max_cap) max_cap = c;
  }
  int cluster_n = cfg.cluster_n;
  if (cluster_n == 0) {
    cluster_n = 1;
    int64_t pref = pref_elems_per_cta / vec;
    if (pref > max_cap) pref = max_cap;
    while (ceil_div(chunks, cluster_n) > pref && cluster_n < 8) cluster_n <<= 1;
    if (ceil_div(chunks, cluster_n) > max_cap) cluster_n = 16;
  }
  while (cluster_n > 1 && (int64_t)(cluster_n - 1) * ceil_div(chunks, cluster_n) >= chunks)
    cluster_n >>= 1;
  const int64_t cpc = ceil_div(chunks, cluster_n);  // chunks per CTA
  if (cpc > max_cap)
    return set_error(QB_ERR_UNSUPPORTED,
                     "%s: a row of %lld elements (vector width %d, cluster %d) does not fit in registers",
                     op, (long long)N, vec, cluster_n);
  int tpr = cfg.threads_per_row;
  int threads = cfg.num_threads;
  // A row shared by a cluster is owned by whole CTAs (one row per CTA tile).
  if (cluster_n > 1 && tpr == 0 && threads) tpr = threads;
  if (tpr == 0) {
    int want = next_pow2(ceil_div(cpc, k_target));
    const int lo = cluster_n > 1 ? 32 : 8;
    if (want < lo) want = lo;
    if (want > 1024) want = 1024;
    if (threads && want > threads) want = threads;
    // First fit, trying the preferred width, then wider, then narrower row groups.  The CTA size
    // that decides the per-thread capacity is the row group itself or the requested CTA size.
    int order[16];
    int n = 0;
    for (int t = want; t <= 1024; t <<= 1) order[n++] = t;
    for (int t = want >> 1; t >= lo; t >>= 1) order[n++] = t;
    for (int i = 0; i < n && tpr == 0; ++i) {
      const int t = order[i];
      if (threads && t > threads) continue;
      const int cta = threads ? threads : (t > 32 ? t : 32);
      if (ceil_div(cpc, t) <= max_k(caps, cta, vec)) tpr = t;
    }
    if (tpr == 0)
      return set_error(QB_ERR_UNSUPPORTED,
                       "%s: a row of %lld elements does not fit (vector width %d, cluster %d, threads %d)",
                       op, (long long)N, vec, cluster_n, threads);
  }
  if (cluster_n > 1) {
    if (tpr < 32) tpr = 32;
    threads = tpr;
  }
  int K = next_pow2(ceil_div(cpc, tpr));
  if (threads != 0 && cfg.threads_per_row != 0) {
    // An explicit row-group width too narrow for the registers is widened (the override is a
    // performance hint; results do not depend on it).
    while (K > max_k(caps, threads > tpr ? threads : tpr, vec) && tpr < 1024) {
      tpr <<= 1;
      if (threads < tpr) threads = tpr;
      K = next_pow2(ceil_div(cpc, tpr));
    }
  }
  if (threads == 0) {
    // Several rows per CTA for short rows, as long as the per-thread footprint allows the size.
    threads = tpr > 32 ? tpr : 32;
    while (threads < default_threads && K <= max_k(caps, threads * 2, vec)) threads <<= 1;
  }
  if (threads < tpr) threads = tpr;
  if (threads < 32) threads = 32;
  if (K > max_k(caps, threads, vec))
    return set_error(QB_ERR_UNSUPPORTED,
                     "%s: a row of %lld elements does not fit (vector width %d, cluster %d, threads %d, threads_per_row %d)",
                     op, (long long)N, vec, cluster_n, threads, tpr);
  out->vec = vec;
  out->tpr = tpr;
  out->threads = threads;
  out->rows_per_cta = threads / tpr;
  out->cluster_n = cluster_n;
  out->K = K;
  out->cols_per_cta = static_cast<int>(cpc * vec);
  return QB_OK;
}

// Number of CTAs of `kernel` that are resident on the whole device at once (cached per kernel and
// launch shape).  Persistent kernels use exactly this many CTAs: more would run as a second,
// partially filled wave.
int cached_occupancy(const void* kernel, int threads, size_t smem);
// Clusters of `cluster_n` CTAs of `kernel` that are resident on the device at once (cached).  A
// cluster must fit inside one GPC, so this is less than resident CTAs / cluster_n: on B200 with
// two 128-thread CTAs per SM, 32 clusters of 8 and 15 clusters of 16.  0 if the query fails.
int cached_max_clusters(const void* kernel, int threads, size_t smem, int cluster_n);
template <class Params>
int resident_clusters(void (*kernel)(Params), int threads, size_t smem, int cluster_n, int sm_count) {
  if (cluster_n > 1) {
    const int n = cached_max_clusters(reinterpret_cast<const void*>(kernel), threads, smem, cluster_n);
    if (n > 0) return n;
  }
  int per_sm = cached_occupancy(reinterpret_cast<const void*>(kernel), threads, smem);
  if (per_sm < 1) per_sm = 1;
  const int n = per_sm * sm_count / cluster_n;
  return n > 0 ? n : 1;
}
template <class Params>
int resident_ctas(void (*kernel)(Params), int threads, size_t smem, int sm_count) {
  int per_sm = cached_occupancy(reinterpret_cast<const void*>(kernel), threads, smem);
  if (per_sm < 1) per_sm = 1;
  return per_sm * sm_count;
}

// Raises the dynamic shared-memory limit (and allows non-portable cluster sizes) of `kernel` on
// the current device.  The attributes are set once per (kernel, device) and remembered, so the
// per-launch cost is one map lookup.  Returns a cudaError_t as int.
int ensure_kernel_attributes(const void* kernel, size_t smem, int cluster_n);

// Remembers (per host thread) which kernel function the last launch used; qb_last_kernel() turns
// it into a readable name on request.
void note_launch(const void* kernel);

// Launches `kernel` with an optional cluster dimension along x (grid.x must be a multiple of it).
template <class Params>
int launch_kernel(void (*kernel)(Params), dim3 grid, int threads, size_t smem, int cluster_n,
                  cudaStream_t stream, const Params& params, const char* name) {
  if (smem > 32 * 1024 || cluster_n > 8) {  // static + dynamic shared memory above 48 KB needs the opt-in
    const int e = ensure_kernel_attributes(reinterpret_cast<const void*>(kernel), smem, cluster_n);
    if (e != 0) {
      return set_error(QB_ERR_CUDA, "%s: cudaFuncSetAttribute(smem=%zu, cluster=%d): %s", name, smem,
                       cluster_n, cudaGetErrorString(static_cast<cudaError_t>(e)));
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (cluster_n > 1) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster_n;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  note_launch(reinterpret_cast<const void*>(kernel));
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, params);
  if (e != cudaSuccess) {
    return set_error(QB_ERR_CUDA, "%s: launch failed (grid %u x %u, block %d, cluster %d, smem %zu): %s",
                     name, grid.x, grid.y, threads, cluster_n, smem, cudaGetErrorString(e));
  }
  return QB_OK;
}

// Launch of a kernel that walks over `num_tiles` row tiles with a grid-stride loop: the grid is
// min(num_tiles, CTAs resident on the device) clusters (max_ctas > 0 overrides the cap), times
// grid_y independent slices (heads).
// per_sm_cap > 0 limits the CTAs per SM below what fits (cluster_n == 1 only).
template <class Params>
int launch_persistent(void (*kernel)(Params), int64_t num_tiles, int grid_y, int threads,
                      size_t smem, int cluster_n, int max_ctas, int sm_count, cudaStream_t stream,
                      const Params& params, const char* name, int per_sm_cap = 0) {
  int64_t cap = max_ctas > 0 ? max_ctas / cluster_n
                             : resident_clusters(kernel, threads, smem, cluster_n, sm_count);
  if (max_ctas <= 0 && per_sm_cap > 0 && cluster_n == 1 && cap > (int64_t)per_sm_cap * sm_count)
    cap = (int64_t)per_sm_cap * sm_count;
  if (grid_y > 1 && max_ctas <= 0) cap = (cap + grid_y - 1) / grid_y;
  if (cap < 1) cap = 1;
  int64_t clusters = num_tiles < cap ? num_tiles : cap;
  if (clusters < 1) clusters = 1;
  dim3 grid(static_cast<unsigned>(clusters * cluster_n), static_cast<unsigned>(grid_y), 1);
  return launch_kernel(kernel, grid, threads, smem, cluster_n, stream, params, name);
}

// ---------------------------------------------------------------------------------------------
// bulk-copy shared-memory ring (ring.cuh): host-side geometry
// ---------------------------------------------------------------------------------------------
// Device counter of ring waits that timed out on the current device (nullptr + error on failure).
unsigned int* ring_timeout_counter();

struct RingPlan {
  int cluster_n = 0;     // CTAs sharing a row
  int ns = 0;            // ring slots
  int cols_per_cta = 0;  // columns owned by one CTA (multiple of vec)
  int chunks_per_row = 0;  // slots one CTA's slice of a row occupies
  size_t smem = 0;       // dynamic shared memory: control block + slots
};

// A row of N elements (esz bytes each, vec elements per 16-byte chunk) with n_in streamed inputs is
// staged in slots of ch_bytes per input.  Picks the smallest power-of-two cluster (<= 16, or the
// one the caller asks for) whose per-CTA slice fits the ring, and as many slots as shared memory
// holds (at most max_slots).  Returns false if no cluster size fits.
inline bool plan_ring(int64_t N, int vec, int esz, int n_in, int ch_bytes, int ctl_bytes,
                      int max_smem_optin, int max_slots, int force_cluster, RingPlan* out) {
  const int64_t slot_bytes = (int64_t)n_in * ch_bytes;
  int64_t ns_max = ((int64_t)max_smem_optin - ctl_bytes) / slot_bytes;
  if (ns_max > max_slots) ns_max = max_slots;
  if (ns_max < 1) return false;
  const int64_t chunks = N / vec;
  for (int c = force_cluster > 0 ? force_cluster : 1; c <= 16; c <<= 1) {
    int cl = c;
    // every CTA of the cluster owns at least one chunk
    while (cl > 1 && (int64_t)(cl - 1) * ceil_div(chunks, cl) >= chunks) cl >>= 1;
    const int64_t cpc = ceil_div(chunks, cl);
    const int64_t r = ceil_div(cpc * vec * esz, ch_bytes);
    if (r <= ns_max) {
      out->cluster_n = cl;
      out->ns = static_cast<int>(ns_max);
      out->cols_per_cta = static_cast<int>(cpc * vec);
      out->chunks_per_row = static_cast<int>(r);
      out->smem = static_cast<size_t>(ctl_bytes) + static_cast<size_t>(ns_max * slot_bytes);
      return true;
    }
    if (force_cluster > 0) break;
  }
  return false;
}

}  // namespace qb
