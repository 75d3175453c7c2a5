// rstd[m] = rsqrt(sum_n x[m, n] * scale + eps) over a (M, N) matrix of partial sums of squares.
//
// Follows quack/rms_final_reduce.py:27-135 (RmsFinalReduce): the second kernel of a GEMM + RMSNorm
// pipeline whose GEMM epilogue leaves one partial sum of squares per output tile column.  N is
// the number of such tiles (1 ... a few hundred), so rows are short: a group of `tpr` lanes of
// one warp (tpr <= 32) owns a row, loops over its chunks and folds with shuffles -- no shared
// memory, no barrier.  Several rows share a warp when rows are shorter than a warp's reach.
#include "common.cuh"
#include "host_common.h"

namespace qb {

struct RmsFinalParams {
  qb_rms_final_reduce_args a;
  int tpr;  // lanes per row (power of two, <= 32)
  int vec;  // elements per access (power of two, <= 16 bytes)
};

template <int VEC>
__global__ void __launch_bounds__(256) rms_final_reduce_kernel(const RmsFinalParams p) {
  const qb_rms_final_reduce_args& a = p.a;
  const int t = threadIdx.x & (p.tpr - 1);
  const int rows_per_cta = blockDim.x / p.tpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * rows_per_cta + threadIdx.x / p.tpr;
  const int nchunks = static_cast<int>(a.N / VEC);
  float acc = 0.0f;
  if (row < a.M) {
    const int64_t base = row * a.x_row_stride;
    for (int c = t; c < nchunks; c += p.tpr) {
      float v[VEC];
      load_chunk<kDynDT, VEC, true>(v, a.x, base + static_cast<int64_t>(c) * VEC, a.x_dtype, true);
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc += v[i];
    }
  }
  // All 32 lanes take part in the shuffles; groups of tpr lanes fold independently.
  for (int off = p.tpr >> 1; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (row < a.M && t == 0) a.rstd[row] = rsqrtf(fmaf(acc, a.scale, a.eps));
}

}  // namespace qb

using namespace qb;

extern "C" int qb_rms_final_reduce(const qb_rms_final_reduce_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "rms_final_reduce: null argument block");
  const qb_rms_final_reduce_args& a = *args;
  if (a.x == nullptr || a.rstd == nullptr)
    return set_error(QB_ERR_INVALID, "rms_final_reduce: x and rstd are required");
  if (a.M < 0 || a.N <= 0 || a.N > (1 << 30))
    return set_error(QB_ERR_INVALID, "rms_final_reduce: bad sizes M=%lld N=%lld", (long long)a.M,
                     (long long)a.N);
  if (!is_float_dtype(a.x_dtype))
    return set_error(QB_ERR_INVALID, "rms_final_reduce: unsupported dtype code");
  if (a.M == 0) return QB_OK;
  if (current_device_facts() == nullptr) return QB_ERR_CUDA;
  VecWidth vw;
  vw.limit_elems(a.N);
  vw.add_tensor(a.x, a.x_dtype, a.x_row_stride);
  RmsFinalParams p;
  p.a = a;
  p.vec = vw.vec;
  const int64_t chunks = a.N / vw.vec;
  int tpr = 1;
  while (tpr < 32 && tpr < chunks) tpr <<= 1;
  p.tpr = tpr;
  const int threads = 256;
  const int rows_per_cta = threads / tpr;
  const int64_t ctas = ceil_div(a.M, rows_per_cta);
  if (ctas > 0x7fffffffLL) return set_error(QB_ERR_UNSUPPORTED, "rms_final_reduce: too many rows");
  dim3 grid(static_cast<unsigned>(ctas), 1, 1);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (vw.vec) {
    case 8: return launch_kernel(rms_final_reduce_kernel<8>, grid, threads, 0, 1, st, p, "rms_final_reduce");
    case 4: return launch_kernel(rms_final_reduce_kernel<4>, grid, threads, 0, 1, st, p, "rms_final_reduce");
    case 2: return launch_kernel(rms_final_reduce_kernel<2>, grid, threads, 0, 1, st, p, "rms_final_reduce");
    default: return launch_kernel(rms_final_reduce_kernel<1>, grid, threads, 0, 1, st, p, "rms_final_reduce");
  }
}
