// RMSNorm / LayerNorm backward for sm_100a: persistent stage-1 kernel and the deterministic
// stage-2 column sum.
//
// Stage 1 follows quack/rmsnorm.py:723-1205 (RMSNormBackward.kernel): a fixed grid of P CTAs (or
// clusters) walks the rows with stride P, keeps fp32 dw / db accumulators for its columns in
// registers for the whole launch and finally writes them as row p of the [P, N] partial buffers.
// x, dout (and dresidual_out) of the next rows are prefetched into shared memory with cp.async
// through a multi-stage ring; every thread reads back only the bytes it copied itself, so the
// ring needs no barriers.  Stage 2 replaces the reference's `dw_partial.sum(dim=0)`
// (quack/rmsnorm.py:1398-1399) by a fixed-order tree, so dw / db are bit-reproducible.
#include <type_traits>

#include "common.cuh"
#include "host_common.h"
#include "norm_bwd_ring.h"

namespace qb {

struct NormBwdParams {
  qb_norm_bwd_args a;
  int tpr;
  int rows_per_cta;
  int cluster_n;
  int cols_per_cta;
  int64_t num_tiles;
  int stages;  // shared-memory ring depth (>= 1)
  int n_in;    // streamed inputs per row: 2 (x, dout) or 3 (+ dresidual_out)
  unsigned int* timeouts;  // device counter of cluster-exchange waits that gave up
};

constexpr int kMaxStages = 8;

__device__ __forceinline__ void cp_async_wait_dyn(int n) {
  switch (n) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    case 3: cp_async_wait<3>(); break;
    case 4: cp_async_wait<4>(); break;
    case 5: cp_async_wait<5>(); break;
    case 6: cp_async_wait<6>(); break;
    default: cp_async_wait<7>(); break;
  }
}

// DT: dtype shared by x / dout / dx (/ dresidual_out / dresidual) or kDynDT.
// LN: LayerNorm (mean subtraction, second row statistic).  DB: accumulate db.
//
// Per row, with xc = x - mean (mean = 0 for RMSNorm), t = dout * w, S1 = sum(xc * t), S2 = sum(t):
//   dx = t * a + xc * b + c      a = rstd, b = -rstd^3 * S1 / N, c = -rstd * S2 / N (0 for RMSNorm)
//   dw += (dout * xc) * rstd     db += dout
// which is (wdy - xhat * mean(xhat * wdy) - mean(wdy)) * rstd with the row constants pulled out.
//
// TPR != 0 fixes the geometry at compile time (TPR threads per row, 128 threads per CTA): the
// chunk strides then become immediate offsets of the loads and stores.  This kernel is
// instruction-issue-bound, and the run-time strides cost LayerNorm backward 6 % (measured, bf16
// N = 4096).  TPR == 0 takes both from the launch.
// CL: the row may be shared by the CTAs of a cluster (p.cluster_n > 1).  Single-CTA rows get an
// instantiation of their own without the cluster exchange: this kernel sits at the 255-register
// limit, and the exchange code pushed the LayerNorm + db variant into spills (N = 16384:
// 5.3 -> 3.8 TB/s) when both lived in one kernel.
template <int DT, int VEC, int K, bool LN, bool DB, int TPR = 0, bool CL = false>
__global__ void __launch_bounds__((K * VEC <= 8) ? 1024 : ((K * VEC <= 16) ? 512 : 256))
norm_bwd_kernel(const NormBwdParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ ReduceScratch scratch;
  const qb_norm_bwd_args& a = p.a;
  const int ptpr = TPR ? TPR : p.tpr;
  const int cn = CL ? p.cluster_n : 1;
  const RowGeom g = make_geom(ptpr, cn);
  reduce_init(scratch, cn);
  if (cn > 1) cluster_arrive();

  constexpr int kSlot = RawWords<DT, VEC>::value * 4;  // bytes of one staged chunk
  const int N = static_cast<int>(a.N);
  const int h = blockIdx.y;
  const int nthreads = TPR ? 128 : static_cast<int>(blockDim.x);
  const int col0 = static_cast<int>(g.crank) * p.cols_per_cta;
  const int ncols = min(p.cols_per_cta, N - col0);
  const float inv_n = 1.0f / static_cast<float>(N);
  const bool has_dres_out = a.dresidual_out != nullptr;

  // Chunk k of this thread starts at column colbase + k * cstride and exists iff k < nk.
  const int colbase = col0 + g.t * VEC;
  const int cstride = ptpr * VEC;
  const int nchunks = ncols > 0 ? ncols / VEC : 0;
  const int nk = nchunks > g.t ? min(K, (nchunks - g.t + ptpr - 1) / ptpr) : 0;

  // Weight (+ offset) for this thread's columns, fp32, held for the whole launch.
  float w[K][VEC];
  const int64_t wrow = static_cast<int64_t>(h) * N;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    if (a.weight != nullptr) {
      load_chunk<kDynDT, VEC, false>(w[k], a.weight, wrow + colbase + k * cstride, a.weight_dtype,
                                     k < nk);
#pragma unroll
      for (int i = 0; i < VEC; ++i) w[k][i] += a.weight_offset;
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) w[k][i] = 1.0f;
    }
  }
  float dw[K][VEC];
  float db[DB ? K : 1][VEC];
#pragma unroll
  for (int k = 0; k < K; ++k)
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      dw[k][i] = 0.0f;
      if constexpr (DB) db[k][i] = 0.0f;
    }

  // Byte strides between this thread's chunks, per tensor (32-bit).
  const int esz_x = elem_bytes<DT>(a.x_dtype), esz_dy = elem_bytes<DT>(a.dout_dtype),
            esz_dro = elem_bytes<DT>(a.dresidual_out_dtype), esz_dx = elem_bytes<DT>(a.dx_dtype),
            esz_dr = elem_bytes<DT>(a.dresidual_dtype);
  const int step_x = cstride * esz_x, step_dy = cstride * esz_dy, step_dro = cstride * esz_dro,
            step_dx = cstride * esz_dx, step_dr = cstride * esz_dr;

  // Shared-memory ring: stage s, input j, chunk k, thread tid -> one slot of kSlot bytes.
  const int64_t P = gridDim.x / cn;
  const int64_t pidx = blockIdx.x / cn;
  const int chunk_bytes = nthreads * kSlot;           // between chunks k and k + 1
  const int in_bytes = K * chunk_bytes;               // one input of one stage
  const int stage_bytes = p.n_in * in_bytes;          // one stage
  unsigned char* const my_slot0 = smem_raw + threadIdx.x * kSlot;
  auto issue_tile = [&](int64_t tile, int stage) {
    if (tile < p.num_tiles) {
      const int64_t m = tile * p.rows_per_cta + g.r;
      if (m < a.M) {
        const int64_t row = m * a.H + h;
        unsigned char* sx = my_slot0 + stage * stage_bytes;
        const char* xp = reinterpret_cast<const char*>(a.x) + (row * a.x_row_stride + colbase) * esz_x;
        const char* dp = reinterpret_cast<const char*>(a.dout) + (row * a.dout_row_stride + colbase) * esz_dy;
        const char* rp = has_dres_out ? reinterpret_cast<const char*>(a.dresidual_out) +
                                            (row * a.dresidual_out_row_stride + colbase) * esz_dro
                                      : nullptr;
#pragma unroll
        for (int k = 0; k < K; ++k) {
          if (k < nk) {
            stage_chunk_p<DT, VEC>(sx + k * chunk_bytes, xp + k * step_x, a.x_dtype);
            stage_chunk_p<DT, VEC>(sx + in_bytes + k * chunk_bytes, dp + k * step_dy, a.dout_dtype);
            if (has_dres_out)
              stage_chunk_p<DT, VEC>(sx + 2 * in_bytes + k * chunk_bytes, rp + k * step_dro,
                                     a.dresidual_out_dtype);
          }
        }
      }
    }
    cp_async_commit();  // one group per tile slot, possibly empty
  };

  const int S = p.stages;
  // Chunk slots beyond this thread's last chunk (rows whose length is not K full rounds of the
  // row's threads, e.g. N = 6144 with 8 slots of 128 threads) are never copied into.  They are
  // zeroed once, so that the straight-line passes can run over all K slots: a zero dout chunk
  // adds nothing to any sum or accumulator, and only the dx store is predicated.
  if constexpr (DT != kDynDT) {
    for (int s = 0; s < S; ++s)
      for (int j = 0; j < p.n_in; ++j)
#pragma unroll
        for (int k = 0; k < K; ++k)
          if (k >= nk)
            *reinterpret_cast<uint4*>(my_slot0 + s * stage_bytes + j * in_bytes + k * chunk_bytes) =
                make_uint4(0u, 0u, 0u, 0u);
  }
  for (int s = 0; s < S - 1; ++s) issue_tile(pidx + s * P, s);

  // Row statistics of the first tile; the next tile's are fetched one iteration ahead.
  float rstd_nx = 0.0f, mean_nx = 0.0f;
  {
    const int64_t m = pidx * p.rows_per_cta + g.r;
    if (pidx < p.num_tiles && m < a.M) {
      rstd_nx = a.rstd[m * a.H + h];
      if constexpr (LN) mean_nx = a.mean[m * a.H + h];
    }
  }

  int rit = 0;
  bool first = true;
  int it = 0;
  for (int64_t tile = pidx; tile < p.num_tiles; tile += P, ++it) {
    issue_tile(tile + static_cast<int64_t>(S - 1) * P, (it + S - 1) % S);
    const int stage = it % S;
    const int64_t m = tile * p.rows_per_cta + g.r;
    const int nkr = m < a.M ? nk : 0;  // chunks of this thread that exist in this tile
    const int64_t row = m * a.H + h;
    const unsigned char* sx = my_slot0 + stage * stage_bytes;  // x slots; dout at + in_bytes
    char* dxp = reinterpret_cast<char*>(a.dx) + (row * a.dx_row_stride + colbase) * esz_dx;
    const float rstd = rstd_nx;
    const float neg_mean = -mean_nx;
    {
      const int64_t mn = (tile + P) * p.rows_per_cta + g.r;
      if (tile + P < p.num_tiles && mn < a.M) {
        rstd_nx = a.rstd[mn * a.H + h];
        if constexpr (LN) mean_nx = a.mean[mn * a.H + h];
      }
    }
    cp_async_wait_dyn(S - 1);  // this tile's group has landed; S-1 younger groups may be in flight

    // Both passes exist in a general form and in a straight-line form without per-chunk branches
    // for rows without a residual-gradient stream: mode 2 when all K chunks of this thread exist,
    // mode 1 when some are padding (zeroed slots, only the dx store is predicated).  The row
    // reduction between the passes stays outside of the per-thread choice: it contains a barrier.
    const bool plain = !has_dres_out && a.dresidual == nullptr;
    const int mode = !plain ? 0 : (nkr == K ? 2 : ((DT != kDynDT && m < a.M) ? 1 : 0));

    // ---- pass 1: S1 = sum(xc * t), S2 = sum(t) ----
    float s1v[VEC], s2v[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) { s1v[i] = 0.0f; s2v[i] = 0.0f; }
    auto pass1 = [&](auto full_tag) {
      constexpr int MODE = decltype(full_tag)::value;
      constexpr bool FULL = MODE != 0;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        if (FULL || k < nkr) {
          float x[VEC], dy[VEC], t[VEC];
          load_chunk_smem<DT, VEC>(x, sx + k * chunk_bytes, a.x_dtype);
          load_chunk_smem<DT, VEC>(dy, sx + in_bytes + k * chunk_bytes, a.dout_dtype);
          if constexpr (LN) vadd_s<VEC>(x, x, neg_mean);
          vmul<VEC>(t, dy, w[k]);
          vfma<VEC>(s1v, x, t, s1v);
          if constexpr (LN) vadd<VEC>(s2v, s2v, t);
        }
      }
    };
    if (mode != 0) pass1(std::integral_constant<int, 2>{}); else pass1(std::integral_constant<int, 0>{});
    const float s1 = hsum<VEC>(s1v);
    const float s2 = LN ? hsum<VEC>(s2v) : 0.0f;
    if (first && cn > 1) cluster_wait();
    first = false;
    const float2 red = row_reduce<SumOp, false, CL, !(LN && DB && TPR == 0)>(make_float2(s1, s2), g, scratch, 0, rit, p.timeouts);
    ++rit;
    const float ca = rstd;
    const float cb = -rstd * rstd * rstd * red.x * inv_n;
    const float cc = LN ? -rstd * red.y * inv_n : 0.0f;

    // ---- pass 2: dx, dresidual, dw / db accumulation ----
    auto pass2 = [&](auto full_tag) {
      constexpr int MODE = decltype(full_tag)::value;
      constexpr bool FULL = MODE != 0;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        if (FULL || k < nkr) {
          float x[VEC], dy[VEC], t[VEC], dx[VEC];
          load_chunk_smem<DT, VEC>(x, sx + k * chunk_bytes, a.x_dtype);
          load_chunk_smem<DT, VEC>(dy, sx + in_bytes + k * chunk_bytes, a.dout_dtype);
          if constexpr (LN) vadd_s<VEC>(x, x, neg_mean);
          vmul<VEC>(t, dy, w[k]);
          vfma_ss<VEC>(dx, t, ca, cc);       // t * a + c
          vfma_s<VEC>(dx, x, cb, dx);        // + xc * b
          vmul<VEC>(t, dy, x);               // dout * xc
          vfma_s<VEC>(dw[k], t, ca, dw[k]);  // dw += (dout * xc) * rstd
          if constexpr (DB) vadd<VEC>(db[k], db[k], dy);
          if constexpr (!FULL) {
            if (has_dres_out) {
              float dr[VEC];
              load_chunk_smem<DT, VEC>(dr, sx + 2 * in_bytes + k * chunk_bytes,
                                       a.dresidual_out_dtype);
              vadd<VEC>(dx, dx, dr);
            }
          }
          if (MODE != 1 || k < nk) store_chunk_p<DT, VEC>(dxp + k * step_dx, dx, a.dx_dtype);
          if constexpr (!FULL) {
            if (a.dresidual != nullptr)
              store_chunk_p<DT, VEC>(reinterpret_cast<char*>(a.dresidual) +
                                         (row * a.dresidual_row_stride + colbase) * esz_dr +
                                         k * step_dr,
                                     dx, a.dresidual_dtype);
          }
        }
      }
    };
    if (mode == 2) pass2(std::integral_constant<int, 2>{});
    else if (mode == 1) pass2(std::integral_constant<int, 1>{});
    else pass2(std::integral_constant<int, 0>{});
  }
  if (first && cn > 1) cluster_wait();
  cp_async_wait<0>();

  // ---- epilogue: this CTA's partial sums -> row pidx of the [P, H, N] workspaces ----
  const int64_t prow = (pidx * a.H + h) * static_cast<int64_t>(N);
  if (p.rows_per_cta == 1) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if (k < nk) {
        const int c = colbase + k * cstride;
        if (a.dw_partial != nullptr)
          store_chunk<QB_F32, VEC>(a.dw_partial, prow + c, dw[k], QB_F32);
        if constexpr (DB) {
          if (a.db_partial != nullptr)
            store_chunk<QB_F32, VEC>(a.db_partial, prow + c, db[k], QB_F32);
        }
      }
    }
  } else {
    // Several rows per CTA tile: fold the row groups in fixed order through shared memory
    // (the staging ring is idle now).  Layout [rows_per_cta][tpr * K * VEC] fp32.
    float* fold = reinterpret_cast<float*>(smem_raw);
    const int width = ptpr * K * VEC;
    for (int which = 0; which < (DB ? 2 : 1); ++which) {
      float* dst = which == 0 ? a.dw_partial : a.db_partial;
      __syncthreads();
      if (dst != nullptr) {
#pragma unroll
        for (int k = 0; k < K; ++k)
#pragma unroll
          for (int i = 0; i < VEC; ++i) {
            float val = dw[k][i];
            if constexpr (DB) val = which == 0 ? dw[k][i] : db[k][i];
            fold[g.r * width + (k * ptpr + g.t) * VEC + i] = val;
          }
      }
      __syncthreads();
      if (dst != nullptr) {
        for (int c = threadIdx.x; c < width; c += nthreads) {
          if (c < ncols) {
            float acc = 0.0f;
            for (int r = 0; r < p.rows_per_cta; ++r) acc += fold[r * width + c];
            dst[prow + col0 + c] = acc;
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// stage 2: out[c] = sum_p partial[p, c], fixed order, cast to the parameter dtype
// ---------------------------------------------------------------------------------------------
struct ColsumParams {
  qb_colsum_args a;
};

// Block (32, 8): 32 consecutive columns x 8 interleaved slices of P.  Each thread adds its
// partial rows p = ty, ty + 8, ... in increasing order; the 8 slices are then folded in slice
// order by the ty == 0 threads.  The summation order depends only on P, never on timing.
__global__ void __launch_bounds__(256) colsum_kernel(const ColsumParams p) {
  __shared__ float part[8][33];
  const qb_colsum_args& a = p.a;
  const int tx = threadIdx.x & 31;
  const int ty = threadIdx.x >> 5;
  const int64_t c = static_cast<int64_t>(blockIdx.x) * 32 + tx;
  float acc = 0.0f;
  if (c < a.cols) {
    for (int64_t r = ty; r < a.P; r += 8) acc += a.partial[r * a.cols + c];
  }
  part[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && c < a.cols) {
    float s = part[0][tx];
#pragma unroll
    for (int j = 1; j < 8; ++j) s += part[j][tx];
    if (a.out_f32 != nullptr) a.out_f32[c] = s;
    if (a.out != nullptr) {
      if (a.out_dtype == QB_F32) reinterpret_cast<float*>(a.out)[c] = s;
      else if (a.out_dtype == QB_BF16) reinterpret_cast<__nv_bfloat16*>(a.out)[c] = __float2bfloat16_rn(s);
      else reinterpret_cast<__half*>(a.out)[c] = __float2half_rn(s);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
template <int DT, int VEC, int K, int TPR, bool CL>
static int launch_norm_bwd_c(const NormBwdParams& p, dim3 grid, int threads, size_t smem,
                             cudaStream_t st) {
  const bool ln = p.a.is_layernorm != 0;
  const bool db = p.a.db_partial != nullptr;
  if constexpr (DT == kDynDT) {
    // The generic path always carries db accumulators (written only when requested).
    if (ln) return launch_kernel(norm_bwd_kernel<DT, VEC, K, true, true, TPR, CL>, grid, threads, smem,
                                 p.cluster_n, st, p, "layernorm_bwd");
    return launch_kernel(norm_bwd_kernel<DT, VEC, K, false, true, TPR, CL>, grid, threads, smem,
                         p.cluster_n, st, p, "rmsnorm_bwd");
  } else {
    if (ln && db) return launch_kernel(norm_bwd_kernel<DT, VEC, K, true, true, TPR, CL>, grid, threads,
                                       smem, p.cluster_n, st, p, "layernorm_bwd");
    if (ln) return launch_kernel(norm_bwd_kernel<DT, VEC, K, true, false, TPR, CL>, grid, threads, smem,
                                 p.cluster_n, st, p, "layernorm_bwd");
    if (db) return launch_kernel(norm_bwd_kernel<DT, VEC, K, false, true, TPR, CL>, grid, threads, smem,
                                 p.cluster_n, st, p, "rmsnorm_bwd");
    return launch_kernel(norm_bwd_kernel<DT, VEC, K, false, false, TPR, CL>, grid, threads, smem,
                         p.cluster_n, st, p, "rmsnorm_bwd");
  }
}

template <int DT, int VEC, int K, int TPR>
static int launch_norm_bwd_t(const NormBwdParams& p, dim3 grid, int threads, size_t smem,
                             cudaStream_t st) {
  if (p.cluster_n > 1) return launch_norm_bwd_c<DT, VEC, K, TPR, true>(p, grid, threads, smem, st);
  return launch_norm_bwd_c<DT, VEC, K, TPR, false>(p, grid, threads, smem, st);
}

template <int DT, int VEC, int K>
static int launch_norm_bwd_k(const NormBwdParams& p, dim3 grid, int threads, size_t smem,
                             cudaStream_t st) {
  // Compile-time geometry for the shapes the heuristics pick for the common hidden sizes
  // (8 chunks per thread, CTAs of 128 threads, 64 or 128 threads per row).
  if constexpr (DT != kDynDT && K == 8) {
    if (threads == 128 && p.tpr == 64) return launch_norm_bwd_t<DT, VEC, K, 64>(p, grid, threads, smem, st);
    if (threads == 128 && p.tpr == 128) return launch_norm_bwd_t<DT, VEC, K, 128>(p, grid, threads, smem, st);
  }
  return launch_norm_bwd_t<DT, VEC, K, 0>(p, grid, threads, smem, st);
}

template <int DT, int VEC>
static int launch_norm_bwd_v(const NormBwdParams& p, int K, dim3 grid, int threads, size_t smem,
                             cudaStream_t st) {
  // Rows whose chunk count is 3, 5, 6 or 7 times the threads of a row (16-bit hidden sizes such
  // as 3072, 5120, 7168) would fill only part of the power-of-two tile: every thread would carry
  // zeroed padding chunks through both passes.  Kernels with exactly that many chunks per thread
  // serve them (single-CTA rows, uniform 16-bit dtypes).  Measured, RMSNorm backward bf16, 512 MiB
  // per tensor: N = 5120 4.40 -> 5.21 TB/s, 10240 3.95 -> 5.11, 2560 4.39 -> 5.13, 3072 5.10 -> 5.45,
  // 1536 5.19 -> 5.96; dx is bit-identical to the padded kernel's.
  if constexpr (DT != kDynDT && VEC == 8) {
    const int64_t nchunks = p.cols_per_cta / VEC;
    if (p.cluster_n == 1 && !(p.a.cfg.flags & 1) && p.a.N == p.cols_per_cta && nchunks % p.tpr == 0) {
      const int64_t ku = nchunks / p.tpr;
      if (K == 4 && ku == 3) return launch_norm_bwd_c<DT, VEC, 3, 0, false>(p, grid, threads, smem, st);
      if (K == 8 && ku == 5) return launch_norm_bwd_c<DT, VEC, 5, 0, false>(p, grid, threads, smem, st);
      if (K == 8 && ku == 6) return launch_norm_bwd_c<DT, VEC, 6, 0, false>(p, grid, threads, smem, st);
      // (7 of 8: only where the 8-chunk kernel has no compile-time geometry -- with it, N = 7168
      // runs 5.73 against 5.55 TB/s; without, N = 14336 5.05 against 5.58)
      const bool has_static_geometry = threads == 128 && (p.tpr == 64 || p.tpr == 128);
      if (K == 8 && ku == 7 && !has_static_geometry)
        return launch_norm_bwd_c<DT, VEC, 7, 0, false>(p, grid, threads, smem, st);
    }
  }
  switch (K) {
    case 1: return launch_norm_bwd_k<DT, VEC, 1>(p, grid, threads, smem, st);
    case 2: return launch_norm_bwd_k<DT, VEC, 2>(p, grid, threads, smem, st);
    case 4: return launch_norm_bwd_k<DT, VEC, 4>(p, grid, threads, smem, st);
    case 8:
      if constexpr (DT != kDynDT) return launch_norm_bwd_k<DT, VEC, 8>(p, grid, threads, smem, st);
  }
  return set_error(QB_ERR_UNSUPPORTED, "norm_bwd: no kernel for %d chunks of %d per thread", K, VEC);
}

struct NormBwdPlan {
  RowPlan rows;
  bool uniform;
  int stages;
  int n_in;
  size_t smem;
};

// Shared launch planning of qb_norm_bwd and qb_norm_bwd_num_partials.
static int plan_norm_bwd(int64_t N, int vec, bool uniform, int x_dtype, bool has_dres_out,
                         const qb_launch_cfg& cfg, const DeviceFacts* dev, NormBwdPlan* out) {
  // Registers per thread: weight + dw (+ db) accumulators + two chunks in flight.
  // (The generic mixed-dtype kernels exist for at most 4 chunks per thread.)
  const int dyn = 4 * vec;
  const ElemCaps caps = uniform ? ElemCaps{vec == 8 ? 64 : 32, 16, 8}
                                : ElemCaps{dyn, dyn < 16 ? dyn : 16, dyn < 8 ? dyn : 8};
  // One CTA of 256 threads carries rows up to 64 elements per thread (16384 for 16-bit dtypes,
  // 8192 for fp32) before a cluster is used: measured N = 16384 bf16 5.0 -> 5.9 TB/s, N = 12288
  // 3.8 -> 4.6 TB/s against a cluster of two CTAs.
  // Longer rows: clusters of two such CTAs up to twice that length, then (more, smaller CTAs
  // hide the cluster barrier better) CTAs of 128 threads.
  const int64_t wide = vec == 8 ? 16384 : 8192;
  const int64_t pref = uniform ? (N <= 2 * wide ? wide : wide / 2) : 2048;
  if (int rc = plan_rows("norm_bwd", N, vec, caps, pref, 8, 128, cfg, &out->rows)) return rc;
  out->uniform = uniform;
  out->n_in = has_dres_out ? 3 : 2;
  const int slot = uniform ? 16 : 4 * vec;
  const size_t stage_bytes = (size_t)out->n_in * out->rows.K * out->rows.threads * slot;
  // Ring depth: as deep as shared memory allows (leaving room for a second CTA on the SM when
  // the stage is small), at most 4 by default.
  const size_t budget = (size_t)dev->max_smem_optin - 8192;  // static reduction scratch + margin
  int stages = cfg.stages > 0 ? cfg.stages : 2;  // two CTAs per SM beat a deeper ring
  if (stages > kMaxStages) stages = kMaxStages;
  while (stages > 1 && stage_bytes * stages > budget) --stages;
  if (stage_bytes * stages > budget)
    return set_error(QB_ERR_UNSUPPORTED, "norm_bwd: one stage of %zu bytes exceeds shared memory",
                     stage_bytes);
  out->stages = stages;
  out->smem = stage_bytes * stages;
  (void)x_dtype;
  return QB_OK;
}

static int default_num_partials(const NormBwdPlan& plan, const DeviceFacts* dev) {
  // CTAs that fit one SM, by threads and by shared memory.
  // (the kernels use about 250 registers per thread: two CTAs of 128 threads or one of 256)
  int per_sm = plan.rows.threads <= 128 ? 2 : 1;
  const size_t smem_per_sm = 228 * 1024;
  const int by_smem = static_cast<int>(smem_per_sm / (plan.smem + 2048));
  if (per_sm > by_smem) per_sm = by_smem;
  if (per_sm < 1) per_sm = 1;
  int clusters = dev->sm_count * per_sm / plan.rows.cluster_n;
  if (plan.rows.cluster_n > 1) {
    // A cluster has to fit into one GPC, so fewer clusters are resident than CTAs / cluster size
    // (B200: 32 clusters of 8, 15 of 16 at two CTAs per SM).  One cluster too many runs as a
    // second wave and nearly doubles the time, so ask the occupancy calculator.  All stage-1
    // instantiations have the same footprint class; the plainest one stands for them.
    const void* rep = plan.rows.vec == 4
                          ? reinterpret_cast<const void*>(norm_bwd_kernel<QB_F32, 4, 8, false, false, 0, true>)
                          : reinterpret_cast<const void*>(norm_bwd_kernel<QB_BF16, 8, 8, false, false, 0, true>);
    const int n = cached_max_clusters(rep, plan.rows.threads, plan.smem, plan.rows.cluster_n);
    if (n > 0 && n < clusters) clusters = n;
  }
  if (clusters < 1) clusters = 1;
  return clusters;
}

}  // namespace qb

using namespace qb;

extern "C" int qb_norm_bwd_num_partials(int64_t N, int32_t x_dtype, int32_t is_layernorm,
                                        int32_t device) {
  clear_error();
  (void)is_layernorm;
  (void)device;
  if (N <= 0 || !is_float_dtype(x_dtype)) return set_error(QB_ERR_INVALID, "num_partials: bad arguments");
  const DeviceFacts* dev = current_device_facts();
  if (dev == nullptr) return QB_ERR_CUDA;
  VecWidth vw;
  vw.limit_elems(N);
  while (vw.vec * host_dtype_bytes(x_dtype) > 16) vw.vec >>= 1;
  const bool uniform = vw.vec == 16 / host_dtype_bytes(x_dtype);
  // Shapes the bulk-copy ring kernel serves want one slice per resident cluster of that kernel.
  if (uniform) {
    const int n = norm_bwd_ring_num_partials(N, x_dtype, dev);
    if (n > 0) return n;
  }
  NormBwdPlan plan;
  qb_launch_cfg cfg = {};
  if (int rc = plan_norm_bwd(N, vw.vec, uniform, x_dtype, false, cfg, dev, &plan)) return rc;
  return default_num_partials(plan, dev);
}

extern "C" int qb_norm_bwd(const qb_norm_bwd_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "norm_bwd: null argument block");
  const qb_norm_bwd_args& a = *args;
  if (a.x == nullptr || a.dout == nullptr || a.rstd == nullptr || a.dx == nullptr)
    return set_error(QB_ERR_INVALID, "norm_bwd: x, dout, rstd and dx are required");
  if ((a.mean != nullptr) != (a.is_layernorm != 0))
    return set_error(QB_ERR_INVALID, "norm_bwd: mean is required iff is_layernorm");
  if (a.M < 0 || a.N <= 0 || a.H <= 0 || a.N > (1 << 30) || a.H > 65535)
    return set_error(QB_ERR_INVALID, "norm_bwd: bad sizes M=%lld H=%lld N=%lld", (long long)a.M,
                     (long long)a.H, (long long)a.N);
  if (!is_float_dtype(a.x_dtype) || !is_float_dtype(a.dout_dtype) || !is_float_dtype(a.dx_dtype) ||
      (a.weight && !is_float_dtype(a.weight_dtype)) ||
      (a.dresidual_out && !is_float_dtype(a.dresidual_out_dtype)) ||
      (a.dresidual && !is_float_dtype(a.dresidual_dtype)))
    return set_error(QB_ERR_INVALID, "norm_bwd: unsupported dtype code");
  if ((a.dw_partial != nullptr || a.db_partial != nullptr) && a.num_partials <= 0)
    return set_error(QB_ERR_INVALID, "norm_bwd: num_partials must be positive");
  const DeviceFacts* dev = current_device_facts();
  if (dev == nullptr) return QB_ERR_CUDA;

  VecWidth vw;
  vw.limit_elems(a.N);
  vw.add_tensor(a.x, a.x_dtype, a.x_row_stride);
  vw.add_tensor(a.dout, a.dout_dtype, a.dout_row_stride);
  vw.add_tensor(a.dx, a.dx_dtype, a.dx_row_stride);
  vw.add_tensor(a.dresidual_out, a.dresidual_out_dtype, a.dresidual_out_row_stride);
  vw.add_tensor(a.dresidual, a.dresidual_dtype, a.dresidual_row_stride);
  vw.add_param(a.weight, a.weight_dtype);
  vw.add_param(a.dw_partial, QB_F32);
  vw.add_param(a.db_partial, QB_F32);
  const int vec = vw.vec;
  bool uniform = a.dout_dtype == a.x_dtype && a.dx_dtype == a.x_dtype &&
                 (!a.dresidual_out || a.dresidual_out_dtype == a.x_dtype) &&
                 (!a.dresidual || a.dresidual_dtype == a.x_dtype);
  if (vec != 16 / host_dtype_bytes(a.x_dtype)) uniform = false;

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // Rows of three 16-byte chunks per thread (N = 6144, 12288, 24576, ... for 16-bit dtypes):
  // staged by bulk copies into a shared-memory ring with the whole CTA on one row (see
  // norm_bwd_ring.cu for the measurements).  Taken when the caller pinned no launch geometry and
  // the number of partial slices does not exceed the clusters resident at once.
  if (uniform && a.M > 0 && !(a.cfg.flags & QB_FLAG_NO_RING) && a.cfg.num_threads == 0 &&
      a.cfg.threads_per_row == 0 && a.cfg.cluster_n == 0 && a.cfg.stages == 0) {
    int64_t want = (a.dw_partial != nullptr || a.db_partial != nullptr)
                       ? a.num_partials
                       : (a.cfg.max_ctas > 0 ? a.cfg.max_ctas : 0);
    if (want == 0) {
      want = norm_bwd_ring_num_partials(a.N, a.x_dtype, dev);
    }
    if (want > 0) {
      const int rr = launch_norm_bwd_ring(a, want, dev, st);
      if (rr != QB_ERR_UNSUPPORTED) return rr;
      clear_error();
    }
  }

  NormBwdPlan plan;
  if (int rc = plan_norm_bwd(a.N, vec, uniform, a.x_dtype, a.dresidual_out != nullptr, a.cfg, dev,
                             &plan))
    return rc;

  NormBwdParams p;
  p.a = a;
  p.tpr = plan.rows.tpr;
  p.rows_per_cta = plan.rows.rows_per_cta;
  p.cluster_n = plan.rows.cluster_n;
  p.timeouts = nullptr;
  if (p.cluster_n > 1) {
    p.timeouts = ring_timeout_counter();
    if (p.timeouts == nullptr) return QB_ERR_CUDA;
  }
  p.cols_per_cta = plan.rows.cols_per_cta;
  p.num_tiles = ceil_div(a.M, p.rows_per_cta);
  p.stages = plan.stages;
  p.n_in = plan.n_in;
  // The grid is fixed by the workspace: one CTA (cluster) per partial-sum slice.
  int64_t clusters = (a.dw_partial != nullptr || a.db_partial != nullptr)
                         ? a.num_partials
                         : (a.cfg.max_ctas > 0 ? a.cfg.max_ctas / plan.rows.cluster_n
                                               : default_num_partials(plan, dev));
  if (clusters < 1) clusters = 1;
  if (clusters * plan.rows.cluster_n > 0x7fffffffLL)
    return set_error(QB_ERR_INVALID, "norm_bwd: num_partials too large");
  dim3 grid(static_cast<unsigned>(clusters * plan.rows.cluster_n), static_cast<unsigned>(a.H), 1);
  // The fold of multi-row CTAs reuses the ring: make sure it is large enough.
  size_t smem = plan.smem;
  const size_t fold_bytes =
      p.rows_per_cta > 1 ? (size_t)plan.rows.threads * plan.rows.K * vec * 4 : 0;
  if (smem < fold_bytes) smem = fold_bytes;

  if (uniform) {
    switch (a.x_dtype) {
      case QB_BF16: return launch_norm_bwd_v<QB_BF16, 8>(p, plan.rows.K, grid, plan.rows.threads, smem, st);
      case QB_F16: return launch_norm_bwd_v<QB_F16, 8>(p, plan.rows.K, grid, plan.rows.threads, smem, st);
      default: return launch_norm_bwd_v<QB_F32, 4>(p, plan.rows.K, grid, plan.rows.threads, smem, st);
    }
  }
  switch (vec) {
    case 8: return launch_norm_bwd_v<kDynDT, 8>(p, plan.rows.K, grid, plan.rows.threads, smem, st);
    case 4: return launch_norm_bwd_v<kDynDT, 4>(p, plan.rows.K, grid, plan.rows.threads, smem, st);
    case 2: return launch_norm_bwd_v<kDynDT, 2>(p, plan.rows.K, grid, plan.rows.threads, smem, st);
    default: return launch_norm_bwd_v<kDynDT, 1>(p, plan.rows.K, grid, plan.rows.threads, smem, st);
  }
}

extern "C" int qb_colsum(const qb_colsum_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "colsum: null argument block");
  const qb_colsum_args& a = *args;
  if (a.partial == nullptr || (a.out == nullptr && a.out_f32 == nullptr))
    return set_error(QB_ERR_INVALID, "colsum: partial and an output are required");
  if (a.P < 0 || a.cols < 0) return set_error(QB_ERR_INVALID, "colsum: bad sizes");
  if (a.out != nullptr && !is_float_dtype(a.out_dtype))
    return set_error(QB_ERR_INVALID, "colsum: unsupported dtype code");
  if (a.cols == 0) return QB_OK;
  ColsumParams p;
  p.a = a;
  dim3 grid(static_cast<unsigned>(ceil_div(a.cols, 32)), 1, 1);
  return launch_kernel(colsum_kernel, grid, 256, 0, 1, reinterpret_cast<cudaStream_t>(stream), p,
                       "colsum");
}
