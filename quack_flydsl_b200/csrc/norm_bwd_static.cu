// qb_norm_bwd_static: RMSNorm / LayerNorm backward (stage 1 + stage 2) for callers that cannot
// provide the fp32 partial-sum workspace because they are not allowed to allocate device memory.
//
// Who needs this: host code that runs after a "no more allocations" point -- an inference or
// training loop whose device memory is owned and frozen by a surrounding framework or memory
// pool, a plugin that is handed input and output buffers only, or a latency-critical loop that
// must avoid cudaMalloc / cudaFree because those calls synchronise the whole device.  The other
// entry points expect such a caller to bring its own dw_partial / db_partial buffers; this one
// keeps them inside the library instead.
//
// The workspace is a fixed, file-scope __device__ array of QB_STATIC_SCRATCH_BYTES (16 MiB).  It is
// part of the loaded module: every GPU that loads the library carries it until the process exits.
// All calls on a device share it and it keeps the last call's contents.  Nothing in it has to
// start at zero (stage 1 overwrites every partial slice it later reads), but two calls that
// overlap on the same GPU -- different streams, or different host threads -- would write the
// same slices: callers must order them.
#include <mutex>

#include "host_common.h"

namespace qb {

constexpr size_t kStaticScratchFloats = QB_STATIC_SCRATCH_BYTES / sizeof(float);

// In host code this name is only a handle for the runtime (a host-side shadow), never a device
// address: the device address is obtained once per device with cudaGetSymbolAddress below.
static __device__ __align__(256) float g_static_scratch[kStaticScratchFloats];

static constexpr int kMaxDevicesStatic = 64;
static float* g_scratch_ptr[kMaxDevicesStatic];
static std::mutex g_scratch_mutex;

// Device address of the scratch array on the current device.  The first call on a device performs
// the symbol lookup (with that device current) and caches the result.
static int static_scratch(float** out) {
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return set_error(QB_ERR_CUDA, "norm_bwd_static: cudaGetDevice: %s", cudaGetErrorString(e));
  if (device < 0 || device >= kMaxDevicesStatic)
    return set_error(QB_ERR_UNSUPPORTED, "norm_bwd_static: device ordinal %d out of range", device);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[device] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess)
      return set_error(QB_ERR_CUDA, "norm_bwd_static: cudaGetSymbolAddress on device %d: %s", device,
                       cudaGetErrorString(e));
    if (p == nullptr)
      return set_error(QB_ERR_CUDA, "norm_bwd_static: the workspace has no address on device %d", device);
    g_scratch_ptr[device] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[device];
  return QB_OK;
}

}  // namespace qb

using namespace qb;

extern "C" int qb_norm_bwd_static(const qb_norm_bwd_static_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "norm_bwd_static: null argument block");
  qb_norm_bwd_args a = args->bwd;  // copy: the workspace fields are filled in below
  if (a.N <= 0 || a.H <= 0 || a.M < 0)
    return set_error(QB_ERR_INVALID, "norm_bwd_static: bad sizes M=%lld H=%lld N=%lld",
                     (long long)a.M, (long long)a.H, (long long)a.N);
  const bool want_dw = args->dw != nullptr;
  const bool want_db = args->db != nullptr;
  if ((want_dw || want_db) && !is_float_dtype(args->param_dtype))
    return set_error(QB_ERR_INVALID, "norm_bwd_static: unsupported parameter dtype code");
  if (want_dw && a.weight == nullptr)
    return set_error(QB_ERR_INVALID, "norm_bwd_static: dw was requested but there is no weight");
  const int nbuf = (want_dw ? 1 : 0) + (want_db ? 1 : 0);
  const int64_t slice = a.H * a.N;  // floats of one partial slice of one buffer
  // Size limit: at least QB_STATIC_MIN_PARTIALS slices of every requested buffer must fit.
  if (nbuf > 0 && slice * nbuf * QB_STATIC_MIN_PARTIALS > (int64_t)kStaticScratchFloats)
    return set_error(QB_ERR_UNSUPPORTED,
                     "norm_bwd_static: H*N = %lld floats per slice with %d gradient buffer(s) exceeds "
                     "the built-in workspace (limit: H*N*buffers <= %lld)",
                     (long long)slice, nbuf,
                     (long long)(kStaticScratchFloats / QB_STATIC_MIN_PARTIALS));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (a.M == 0) {
    // an empty batch: the parameter gradients are zero and the workspace is not touched
    const size_t bytes = (size_t)slice * host_dtype_bytes(args->param_dtype);
    if (want_dw && cudaMemsetAsync(args->dw, 0, bytes, st) != cudaSuccess)
      return set_error(QB_ERR_CUDA, "norm_bwd_static: memset failed");
    if (want_db && cudaMemsetAsync(args->db, 0, bytes, st) != cudaSuccess)
      return set_error(QB_ERR_CUDA, "norm_bwd_static: memset failed");
    return QB_OK;
  }
  float* scratch = nullptr;
  if (int rc = static_scratch(&scratch)) return rc;

  // One partial slice per persistent CTA, as many as the stock heuristic wants, capped by what fits.
  int P = qb_norm_bwd_num_partials(a.N, a.x_dtype, a.is_layernorm, -1);
  if (P <= 0) return P < 0 ? P : set_error(QB_ERR_CUDA, "norm_bwd_static: no launch plan");
  if (a.H > 1) P = static_cast<int>((P + a.H / 2) / a.H) > 0 ? static_cast<int>((P + a.H / 2) / a.H) : 1;
  if (nbuf > 0) {
    const int64_t fit = (int64_t)kStaticScratchFloats / (slice * nbuf);
    if (P > fit) P = static_cast<int>(fit);
  }
  a.num_partials = P;
  a.dw_partial = want_dw ? scratch : nullptr;
  a.db_partial = want_db ? scratch + (want_dw ? (int64_t)P * slice : 0) : nullptr;
  if (int rc = qb_norm_bwd(&a, stream)) return rc;
  for (int which = 0; which < 2; ++which) {
    void* out = which == 0 ? args->dw : args->db;
    const float* part = which == 0 ? a.dw_partial : a.db_partial;
    if (out == nullptr) continue;
    qb_colsum_args c = {};
    c.partial = part;
    c.out = out;
    c.out_f32 = nullptr;
    c.P = P;
    c.cols = slice;
    c.out_dtype = args->param_dtype;
    if (int rc = qb_colsum(&c, stream)) return rc;
  }
  return QB_OK;
}
