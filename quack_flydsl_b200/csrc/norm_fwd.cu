// RMSNorm / LayerNorm forward for sm_100a.
//
// One row is read from HBM exactly once into fp32 registers (128-bit coalesced loads issued back to
// back), reduced thread -> warp -> CTA -> cluster, normalised from registers and written once.
// Behaviour follows the reference kernel quack/rmsnorm.py:150-362 (RMSNorm.kernel; LayerNorm
// branch :263-311) and its host stub quack/rmsnorm.py:108-148.
#include "common.cuh"
#include "host_common.h"

namespace qb {

struct NormFwdParams {
  qb_norm_fwd_args a;
  int tpr;            // threads per row
  int rows_per_cta;   // rows of one CTA tile
  int cluster_n;      // CTAs sharing a row
  int cols_per_cta;   // columns owned by one CTA of the cluster (multiple of VEC)
  int64_t num_tiles;  // ceil(M / rows_per_cta)
};

// DT: dtype shared by x / residual / out / residual_out, or kDynDT (per-tensor run-time dtypes).
// VEC: elements per chunk; K: chunks per thread; LN: LayerNorm instead of RMSNorm.
template <int DT, int VEC, int K, bool LN>
__global__ void __launch_bounds__((K * VEC > 16) ? 512 : 1024)
norm_fwd_kernel(const NormFwdParams p) {
  __shared__ ReduceScratch scratch;
  const qb_norm_fwd_args& a = p.a;
  const RowGeom g = make_geom(p.tpr, p.cluster_n);
  if (p.cluster_n > 1) cluster_arrive();  // completed by cluster_wait() before the first exchange

  const int N = static_cast<int>(a.N);
  const int h = blockIdx.y;
  const int col0 = static_cast<int>(g.crank) * p.cols_per_cta;
  const int ncols = min(p.cols_per_cta, N - col0);  // columns this CTA owns (may be <= 0)
  const float inv_n = 1.0f / static_cast<float>(N);

  // Column of chunk k of this thread and whether it exists.
  int col[K];
  bool cok[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int local = (k * p.tpr + g.t) * VEC;
    cok[k] = local < ncols;
    col[k] = col0 + local;
  }

  // Weight and bias: kept in registers across row tiles when the per-thread slice is small,
  // otherwise re-read (L1/L2 hits) after each row's reduction.
  constexpr bool kHoistW = (K * VEC <= 8);
  const bool has_w = a.weight != nullptr;
  const bool has_b = a.bias != nullptr;
  const int64_t wrow = static_cast<int64_t>(h) * N;
  float wr[kHoistW ? K : 1][VEC];
  float br[kHoistW ? K : 1][VEC];
  if constexpr (kHoistW) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if (has_w) {
        load_chunk<kDynDT, VEC, false>(wr[k], a.weight, wrow + col[k], a.weight_dtype, cok[k]);
#pragma unroll
        for (int i = 0; i < VEC; ++i) wr[k][i] += a.weight_offset;
      } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) wr[k][i] = 1.0f;
      }
      if (has_b) {
        load_chunk<kDynDT, VEC, false>(br[k], a.bias, wrow + col[k], a.bias_dtype, cok[k]);
      } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) br[k][i] = 0.0f;
      }
    }
  }

  const int64_t tile_stride = gridDim.x / p.cluster_n;
  int parity = 0;
  bool first = true;
  for (int64_t tile = blockIdx.x / p.cluster_n; tile < p.num_tiles; tile += tile_stride) {
    const int64_t m = tile * p.rows_per_cta + g.r;
    const bool row_ok = m < a.M;
    const int64_t row = m * a.H + h;

    // ---- load the row (all loads issued before the first use) ----
    float v[K][VEC];
    {
      uint32_t rx[K][RawWords<DT, VEC>::value];
#pragma unroll
      for (int k = 0; k < K; ++k)
        load_chunk_raw<DT, VEC>(rx[k], a.x, row * a.x_row_stride + col[k], a.x_dtype,
                                row_ok && cok[k]);
      if (a.residual != nullptr) {
        uint32_t rr[K][RawWords<DT, VEC>::value];
#pragma unroll
        for (int k = 0; k < K; ++k)
          load_chunk_raw<DT, VEC>(rr[k], a.residual, row * a.residual_row_stride + col[k],
                                  a.residual_dtype, row_ok && cok[k]);
#pragma unroll
        for (int k = 0; k < K; ++k) {
          float t[VEC];
          unpack_chunk<DT, VEC>(v[k], rx[k], a.x_dtype);
          unpack_chunk<DT, VEC>(t, rr[k], a.residual_dtype);
#pragma unroll
          for (int i = 0; i < VEC; ++i) v[k][i] += t[i];
        }
      } else {
#pragma unroll
        for (int k = 0; k < K; ++k) unpack_chunk<DT, VEC>(v[k], rx[k], a.x_dtype);
      }
    }
    if (a.residual_out != nullptr) {
#pragma unroll
      for (int k = 0; k < K; ++k)
        if (row_ok && cok[k])
          store_chunk<DT, VEC>(a.residual_out, row * a.residual_out_row_stride + col[k], v[k],
                               a.residual_out_dtype);
    }

    if (first && p.cluster_n > 1) cluster_wait();
    first = false;

    // ---- statistics ----
    float mean = 0.0f;
    float rstd;
    if constexpr (LN) {
      float s = 0.0f;
#pragma unroll
      for (int k = 0; k < K; ++k)
#pragma unroll
        for (int i = 0; i < VEC; ++i) s += v[k][i];
      mean = row_reduce<SumOp>(make_float2(s, 0.f), g, scratch, 0, parity).x * inv_n;
      float q = 0.0f;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        // Lanes outside the row must stay zero after centering or they would add mean^2 each.
        if (cok[k]) {
#pragma unroll
          for (int i = 0; i < VEC; ++i) {
            v[k][i] -= mean;
            q = fmaf(v[k][i], v[k][i], q);
          }
        }
      }
      const float var = row_reduce<SumOp>(make_float2(q, 0.f), g, scratch, 1, parity).x * inv_n;
      rstd = rsqrtf(var + a.eps);
    } else {
      float q = 0.0f;
#pragma unroll
      for (int k = 0; k < K; ++k)
#pragma unroll
        for (int i = 0; i < VEC; ++i) q = fmaf(v[k][i], v[k][i], q);
      const float ms = row_reduce<SumOp>(make_float2(q, 0.f), g, scratch, 0, parity).x * inv_n;
      rstd = rsqrtf(ms + a.eps);
    }
    parity ^= 1;

    if (row_ok && g.t == 0 && g.crank == 0) {
      if (a.rstd != nullptr) a.rstd[row] = rstd;
      if (LN && a.mean != nullptr) a.mean[row] = mean;
    }

    // ---- normalise and store ----
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float w[VEC], b[VEC];
      if constexpr (kHoistW) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) { w[i] = wr[k][i]; b[i] = br[k][i]; }
      } else {
        if (has_w) {
          load_chunk<kDynDT, VEC, false>(w, a.weight, wrow + col[k], a.weight_dtype, cok[k]);
#pragma unroll
          for (int i = 0; i < VEC; ++i) w[i] += a.weight_offset;
        } else {
#pragma unroll
          for (int i = 0; i < VEC; ++i) w[i] = 1.0f;
        }
        if (has_b) {
          load_chunk<kDynDT, VEC, false>(b, a.bias, wrow + col[k], a.bias_dtype, cok[k]);
        } else {
#pragma unroll
          for (int i = 0; i < VEC; ++i) b[i] = 0.0f;
        }
      }
      float y[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) y[i] = fmaf(v[k][i] * rstd, w[i], b[i]);
      if (row_ok && cok[k])
        store_chunk<DT, VEC>(a.out, row * a.out_row_stride + col[k], y, a.out_dtype);
    }
  }
  // A CTA that never entered the loop still owes the wait matching its arrive.
  if (first && p.cluster_n > 1) cluster_wait();
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
template <int DT, int VEC, int K>
static int launch_norm_fwd_k(const NormFwdParams& p, dim3 grid, int threads, cudaStream_t st) {
  if (p.a.is_layernorm)
    return launch_kernel(norm_fwd_kernel<DT, VEC, K, true>, grid, threads, 0, p.cluster_n, st, p,
                         "layernorm_fwd");
  return launch_kernel(norm_fwd_kernel<DT, VEC, K, false>, grid, threads, 0, p.cluster_n, st, p,
                       "rmsnorm_fwd");
}

template <int DT, int VEC>
static int launch_norm_fwd_v(const NormFwdParams& p, int K, dim3 grid, int threads,
                             cudaStream_t st) {
  switch (K) {
    case 1: return launch_norm_fwd_k<DT, VEC, 1>(p, grid, threads, st);
    case 2: return launch_norm_fwd_k<DT, VEC, 2>(p, grid, threads, st);
    case 4: return launch_norm_fwd_k<DT, VEC, 4>(p, grid, threads, st);
    case 8: return launch_norm_fwd_k<DT, VEC, 8>(p, grid, threads, st);
    case 16:
      if constexpr (VEC <= 4) return launch_norm_fwd_k<DT, VEC, 16>(p, grid, threads, st);
  }
  return set_error(QB_ERR_UNSUPPORTED, "norm_fwd: no kernel for %d chunks of %d per thread", K, VEC);
}

}  // namespace qb

using namespace qb;

extern "C" int qb_norm_fwd(const qb_norm_fwd_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "norm_fwd: null argument block");
  const qb_norm_fwd_args& a = *args;
  if (a.x == nullptr || a.out == nullptr)
    return set_error(QB_ERR_INVALID, "norm_fwd: x and out are required");
  if (a.M < 0 || a.N <= 0 || a.H <= 0)
    return set_error(QB_ERR_INVALID, "norm_fwd: bad sizes M=%lld H=%lld N=%lld", (long long)a.M,
                     (long long)a.H, (long long)a.N);
  if (!is_float_dtype(a.x_dtype) || !is_float_dtype(a.out_dtype) ||
      (a.weight && !is_float_dtype(a.weight_dtype)) || (a.bias && !is_float_dtype(a.bias_dtype)) ||
      (a.residual && !is_float_dtype(a.residual_dtype)) ||
      (a.residual_out && !is_float_dtype(a.residual_out_dtype)))
    return set_error(QB_ERR_INVALID, "norm_fwd: unsupported dtype code");
  if (a.N > (1 << 30)) return set_error(QB_ERR_UNSUPPORTED, "norm_fwd: N too large");
  if (a.H > 65535) return set_error(QB_ERR_UNSUPPORTED, "norm_fwd: H > 65535");
  if (a.M == 0) return QB_OK;
  const DeviceFacts* dev = current_device_facts();
  if (dev == nullptr) return QB_ERR_CUDA;

  // Vector width all tensors can be accessed with.
  VecWidth vw;
  vw.limit_elems(a.N);
  vw.add_tensor(a.x, a.x_dtype, a.x_row_stride);
  vw.add_tensor(a.out, a.out_dtype, a.out_row_stride);
  vw.add_tensor(a.residual, a.residual_dtype, a.residual_row_stride);
  vw.add_tensor(a.residual_out, a.residual_out_dtype, a.residual_out_row_stride);
  vw.add_param(a.weight, a.weight_dtype);
  vw.add_param(a.bias, a.bias_dtype);
  const int vec = vw.vec;

  // Uniform fast path: every streamed tensor has the same dtype and full 16-byte chunks.
  bool uniform = a.out_dtype == a.x_dtype && (!a.residual || a.residual_dtype == a.x_dtype) &&
                 (!a.residual_out || a.residual_out_dtype == a.x_dtype);
  if (vec != 16 / host_dtype_bytes(a.x_dtype)) uniform = false;

  // The kernel holds the row as fp32 registers: up to 64 values per thread in CTAs of <= 512
  // threads (32 on the generic mixed-dtype path, whose raw staging registers are wider) and 16
  // in CTAs of 1024 threads.
  RowPlan plan;
  const ElemCaps caps = {uniform ? 64 : 32, uniform ? 64 : 32, 16};
  const int64_t pref = (uniform && vec == 8) ? 16384 : 8192;
  if (int rc = plan_rows("norm_fwd", a.N, vec, caps, pref, 4, 256, a.cfg, &plan)) return rc;
  const int K = plan.K;
  const int threads = plan.threads;

  NormFwdParams p;
  p.a = a;
  p.tpr = plan.tpr;
  p.rows_per_cta = plan.rows_per_cta;
  p.cluster_n = plan.cluster_n;
  p.cols_per_cta = plan.cols_per_cta;
  p.num_tiles = ceil_div(a.M, p.rows_per_cta);
  const int64_t max_ctas = a.cfg.max_ctas > 0
                               ? a.cfg.max_ctas
                               : (int64_t)dev->sm_count * (2048 / threads) * 2;
  int64_t clusters = p.num_tiles;
  if (clusters > max_ctas / plan.cluster_n) clusters = max_ctas / plan.cluster_n;
  if (clusters < 1) clusters = 1;
  dim3 grid(static_cast<unsigned>(clusters * plan.cluster_n), static_cast<unsigned>(a.H), 1);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  if (uniform) {
    switch (a.x_dtype) {
      case QB_BF16: return launch_norm_fwd_v<QB_BF16, 8>(p, K, grid, threads, st);
      case QB_F16: return launch_norm_fwd_v<QB_F16, 8>(p, K, grid, threads, st);
      default: return launch_norm_fwd_v<QB_F32, 4>(p, K, grid, threads, st);
    }
  }
  switch (vec) {
    case 8: return launch_norm_fwd_v<kDynDT, 8>(p, K, grid, threads, st);
    case 4: return launch_norm_fwd_v<kDynDT, 4>(p, K, grid, threads, st);
    case 2: return launch_norm_fwd_v<kDynDT, 2>(p, K, grid, threads, st);
    default: return launch_norm_fwd_v<kDynDT, 1>(p, K, grid, threads, st);
  }
}
