// RMSNorm / LayerNorm forward for sm_100a.
//
// One row is read from HBM exactly once (128-bit coalesced loads issued back to back), reduced
// thread -> warp -> CTA -> cluster, normalised from registers and written once.  Behaviour follows
// the reference kernel quack/rmsnorm.py:150-362 (RMSNorm.kernel; LayerNorm branch :263-311) and
// its host stub quack/rmsnorm.py:108-148.
//
// What bounds these kernels is the number of bytes a resident thread keeps in flight, so the row
// is held in as few registers as possible: with a residual the fp32 sum x + residual (both packed
// inputs are in flight at once), without one the still-packed 16-bit input words, which are
// unpacked again by each pass over the row.  Weight (+ offset) and bias are converted to fp32 and
// copied once per CTA into shared memory (indexed by column, shared by all row groups of the
// CTA, one barrier); the CTA then walks over row tiles.
#include <type_traits>

#include "common.cuh"
#include "norm_fwd.h"

namespace qb {


// DT: dtype shared by x / residual / out / residual_out, or kDynDT (per-tensor run-time dtypes).
// VEC: elements per chunk; K: chunks per thread; LN: LayerNorm instead of RMSNorm;
// RAW: keep the packed input words instead of fp32 values (no residual, static 16-bit DT only).
template <int DT, int VEC, int K, bool LN, bool RAW, int STAGED>
__global__ void __launch_bounds__(RAW ? (K * VEC > 32 ? 256 : (K * VEC > 16 ? 512 : 1024))
                                      : (K * VEC > 32 ? 256 : (K * VEC > 16 ? 512 : 1024)),
                                  (K * VEC > 32) ? 2 : 1)
norm_fwd_kernel(const NormFwdParams p) {
  extern __shared__ __align__(16) unsigned char smem_params[];
  __shared__ ReduceScratch scratch;
  const qb_norm_fwd_args& a = p.a;
  const RowGeom g = make_geom(p.tpr, p.cluster_n);
  reduce_init(scratch, p.cluster_n);
  if (p.cluster_n > 1) cluster_arrive();  // completed by cluster_wait() before the first exchange

  const int N = static_cast<int>(a.N);
  const int h = blockIdx.y;
  const int nthreads = blockDim.x;
  const int col0 = static_cast<int>(g.crank) * p.cols_per_cta;
  const int ncols = min(p.cols_per_cta, N - col0);  // columns this CTA owns (may be <= 0)
  const float inv_n = 1.0f / static_cast<float>(N);

  // Chunk k of this thread starts at column colbase + k * cstride and exists iff k < nk.
  const int colbase = col0 + g.t * VEC;
  const int cstride = p.tpr * VEC;
  const int nchunks = ncols > 0 ? ncols / VEC : 0;
  const int nk = nchunks > g.t ? min(K, (nchunks - g.t + p.tpr - 1) / p.tpr) : 0;

  // Byte strides between this thread's chunks, per tensor (32-bit).
  const int esz_x = elem_bytes<DT>(a.x_dtype);
  const int esz_r = elem_bytes<DT>(a.residual_dtype);
  const int esz_o = elem_bytes<DT>(a.out_dtype);
  const int esz_ro = elem_bytes<DT>(a.residual_out_dtype);
  const int step_x = cstride * esz_x, step_r = cstride * esz_r, step_o = cstride * esz_o,
            step_ro = cstride * esz_ro;

  // Stage this CTA's column slice of (weight + weight_offset) and of the bias in shared memory as
  // fp32 (ones when there is no weight), chunk c at slot c, so that the per-row epilogue needs no
  // dtype dispatch and no global loads.  Slices too large for a useful
  // occupancy are read from global memory (L1/L2) instead.
  const bool has_w = a.weight != nullptr;
  const bool has_b = a.bias != nullptr;
  constexpr bool staged = STAGED != 0;
  constexpr bool packed_params = STAGED == 2;  // staged in their own 16-bit dtype, 16 bytes per chunk
  const int64_t wrow = static_cast<int64_t>(h) * N;
  // Slots exist for all tpr * K chunk positions of the tile geometry (the epilogue reads the
  // slots of padding chunks too, it only does not store their results).
  const int slice_chunks = p.tpr * K;
  // Layout of a staged slice: for 8-element chunks two planes of 4 floats per chunk, so that the
  // 16-byte reads of neighbouring threads are contiguous (no bank conflicts).
  const int plane = slice_chunks * 4;
  auto param_index = [&](int c, int i) -> int {
    if constexpr (VEC == 8) return (i >> 2) * plane + c * 4 + (i & 3);
    else return c * VEC + i;
  };
  auto load_param = [&](float (&o)[VEC], const float* base, int c) {
    if constexpr (VEC == 8) {
      uint32_t lo[4], hi[4];
      lds_raw<16>(lo, base + c * 4);
      lds_raw<16>(hi, base + plane + c * 4);
#pragma unroll
      for (int i = 0; i < 4; ++i) { o[i] = __uint_as_float(lo[i]); o[4 + i] = __uint_as_float(hi[i]); }
    } else {
      load_chunk_smem<QB_F32, VEC>(o, base + c * VEC, QB_F32);
    }
  };
  float* w_smem = reinterpret_cast<float*>(smem_params);
  float* b_smem = w_smem + static_cast<size_t>(slice_chunks) * VEC;
  if constexpr (packed_params) {
    // weight and bias share one 16-bit dtype: copy the chunks as they are (slot c = 16 bytes)
    static_assert(!packed_params || VEC == 8, "packed parameter staging uses 8-element chunks");
    uint4* w16 = reinterpret_cast<uint4*>(smem_params);
    uint4* b16 = w16 + slice_chunks;
    for (int c = threadIdx.x; c < nchunks; c += nthreads) {
      uint32_t raw[4];
      if (has_w) {
        ldg_cached<16>(raw, reinterpret_cast<const char*>(a.weight) + (wrow + col0 + c * VEC) * 2);
        w16[c] = make_uint4(raw[0], raw[1], raw[2], raw[3]);
      }
      if (has_b) {
        ldg_cached<16>(raw, reinterpret_cast<const char*>(a.bias) + (wrow + col0 + c * VEC) * 2);
        b16[c] = make_uint4(raw[0], raw[1], raw[2], raw[3]);
      }
    }
    __syncthreads();
  } else if constexpr (staged) {
    for (int c = threadIdx.x; c < nchunks; c += nthreads) {
      float pv[VEC];
      if (has_w) load_chunk<kDynDT, VEC, false>(pv, a.weight, wrow + col0 + c * VEC, a.weight_dtype);
#pragma unroll
      for (int i = 0; i < VEC; ++i)
        w_smem[param_index(c, i)] = has_w ? pv[i] + a.weight_offset : 1.0f;
      if (has_b) {  // the bias slice exists only when there is a bias
        load_chunk<kDynDT, VEC, false>(pv, a.bias, wrow + col0 + c * VEC, a.bias_dtype);
#pragma unroll
        for (int i = 0; i < VEC; ++i) b_smem[param_index(c, i)] = pv[i];
      }
    }
    __syncthreads();
  }
  const int chunk0 = g.t;  // chunk k of this thread is slice chunk chunk0 + k * tpr

  // Rows of one CTA may take different branches around a row reduction only if that reduction
  // neither shuffles across rows (rows narrower than a warp) nor uses the CTA-wide barrier for a
  // row group (see row_group_sync).
  const bool ln_fast = LN && p.tpr >= 32 && (p.tpr == 32 || p.tpr == nthreads || nthreads <= 15 * p.tpr);
  const int64_t tile_stride = gridDim.x / p.cluster_n;
  int rit = 0;
  bool first = true;
  for (int64_t tile = blockIdx.x / p.cluster_n; tile < p.num_tiles; tile += tile_stride) {
    const int64_t m = tile * p.rows_per_cta + g.r;
    const bool row_ok = m < a.M;
    const int64_t row = m * a.H + h;
    const int nkr = row_ok ? nk : 0;  // chunks of this thread that exist in this tile
    const char* xp = reinterpret_cast<const char*>(a.x) + (row * a.x_row_stride + colbase) * esz_x;
    char* op = reinterpret_cast<char*>(a.out) + (row * a.out_row_stride + colbase) * esz_o;

    // ---- load the row (all loads issued before the first use) ----
    constexpr int kRawWords = RawWords<DT, VEC>::value;
    uint32_t rx[RAW ? K : 1][kRawWords];
    float v[RAW ? 1 : K][VEC];
    // (Predicated loads also for full rows: the unpredicated form of load_row_raw, which gains
    // 5 % in the softmax forward, measured 3 % / 7 % slower here for RMSNorm / LayerNorm.)
    if constexpr (RAW) {
#pragma unroll
      for (int k = 0; k < K; ++k)
        load_chunk_raw_p<DT, VEC>(rx[k], xp + k * step_x, a.x_dtype, k < nkr);
    } else {
      uint32_t tx[K][kRawWords];
#pragma unroll
      for (int k = 0; k < K; ++k)
        load_chunk_raw_p<DT, VEC>(tx[k], xp + k * step_x, a.x_dtype, k < nkr);
      if (a.residual != nullptr) {
        const char* rp = reinterpret_cast<const char*>(a.residual) +
                         (row * a.residual_row_stride + colbase) * esz_r;
        uint32_t tr[K][kRawWords];
#pragma unroll
        for (int k = 0; k < K; ++k)
          load_chunk_raw_p<DT, VEC>(tr[k], rp + k * step_r, a.residual_dtype, k < nkr);
#pragma unroll
        for (int k = 0; k < K; ++k) {
          float t[VEC];
          unpack_chunk<DT, VEC>(v[k], tx[k], a.x_dtype);
          unpack_chunk<DT, VEC>(t, tr[k], a.residual_dtype);
          vadd<VEC>(v[k], v[k], t);
        }
      } else {
#pragma unroll
        for (int k = 0; k < K; ++k) unpack_chunk<DT, VEC>(v[k], tx[k], a.x_dtype);
      }
      if (a.residual_out != nullptr) {
        char* rop = reinterpret_cast<char*>(a.residual_out) +
                    (row * a.residual_out_row_stride + colbase) * esz_ro;
#pragma unroll
        for (int k = 0; k < K; ++k)
          if (k < nkr) store_chunk_p<DT, VEC>(rop + k * step_ro, v[k], a.residual_out_dtype);
      }
    }

    if (first && p.cluster_n > 1) cluster_wait();
    first = false;

    // ---- statistics (branch-free: chunks that do not exist were loaded as zeros) ----
    float mean = 0.0f;
    float rstd;
    if constexpr (LN) {
      // Sum and sum of squares in ONE pass over the registers and one reduction.  var = E[x^2] -
      // mean^2 loses (1 + mean^2 / var) ulps to cancellation, so it is only kept while the mean is
      // small against the spread (mean^2 <= 4 var: below 1e-6 relative); any other row -- and any
      // row with a NaN or infinity -- takes the centred second pass.  The choice is the same for
      // all threads of a row; it may differ between the rows of a CTA only where the reduction
      // does not synchronise threads of different rows (ln_fast), otherwise the rows of a warp
      // or of the CTA decide together.
      float sv[VEC], qv[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) { sv[i] = 0.0f; qv[i] = 0.0f; }
#pragma unroll
      for (int k = 0; k < K; ++k) {
        if constexpr (RAW) {
          float t[VEC];
          unpack_chunk<DT, VEC>(t, rx[k], a.x_dtype);
          vadd<VEC>(sv, sv, t);
          vfma<VEC>(qv, t, t, qv);
        } else {
          vadd<VEC>(sv, sv, v[k]);
          vfma<VEC>(qv, v[k], v[k], qv);
        }
      }
      const float2 sq =
          row_reduce<SumOp, true>(make_float2(hsum<VEC>(sv), hsum<VEC>(qv)), g, scratch, 0, rit, p.timeouts);
      mean = sq.x * inv_n;
      float var = fmaf(-mean, mean, sq.y * inv_n);
      bool exact = !(mean * mean <= 4.0f * var);
      if (!ln_fast) {
        // rows narrower than a warp (shuffle-only reductions): one choice per warp; row groups on
        // the CTA-wide barrier: one choice per CTA
        exact = (p.tpr < 32) ? (__any_sync(0xffffffffu, exact) != 0) : (__syncthreads_or(exact) != 0);
      }
      if (exact) {
        // sum (x - mean)^2; padding chunks hold zeros and get offset 0 instead of -mean
#pragma unroll
        for (int i = 0; i < VEC; ++i) qv[i] = 0.0f;
#pragma unroll
        for (int k = 0; k < K; ++k) {
          float d[VEC];
          const float off = (k < nk) ? -mean : 0.0f;
          if constexpr (RAW) {
            float t[VEC];
            forget_values(rx[k]);
            unpack_chunk<DT, VEC>(t, rx[k], a.x_dtype);
            vadd_s<VEC>(d, t, off);
          } else {
            vadd_s<VEC>(d, v[k], off);
          }
          vfma<VEC>(qv, d, d, qv);
        }
        var = row_reduce<SumOp, true>(make_float2(hsum<VEC>(qv), 0.f), g, scratch, 1, rit, p.timeouts).x * inv_n;
      }
      rstd = rsqrtf(var + a.eps);
    } else {
      float qv[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) qv[i] = 0.0f;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        if constexpr (RAW) {
          float t[VEC];
          unpack_chunk<DT, VEC>(t, rx[k], a.x_dtype);
          vfma<VEC>(qv, t, t, qv);
        } else {
          vfma<VEC>(qv, v[k], v[k], qv);
        }
      }
      const float ms =
          row_reduce<SumOp, true>(make_float2(hsum<VEC>(qv), 0.f), g, scratch, 0, rit, p.timeouts).x * inv_n;
      rstd = rsqrtf(ms + a.eps);
    }
    ++rit;

    if (row_ok && g.t == 0 && g.crank == 0) {
      if (a.rstd != nullptr) a.rstd[row] = rstd;
      if (LN && a.mean != nullptr) a.mean[row] = mean;
    }

    // ---- normalise and store: y = (x * ra + rb) * w + b with ra = rstd, rb = -mean * rstd ----
    const float ra = rstd;
    const float rb = -mean * rstd;
    if constexpr (staged) {
#pragma unroll
      for (int k = 0; k < K; ++k) {
        float w[VEC], b[VEC], y[VEC], xc[VEC];
        if constexpr (packed_params) {
          const uint4* w16 = reinterpret_cast<const uint4*>(smem_params);
          const uint4* b16 = w16 + slice_chunks;
          const bool pbf16 = (has_w ? a.weight_dtype : a.bias_dtype) == QB_BF16;
          uint32_t raw[4];
          if (has_w) {
            lds_raw<16>(raw, w16 + chunk0 + k * p.tpr);
            unpack16<VEC>(w, raw, pbf16);
            vadd_s<VEC>(w, w, a.weight_offset);
          } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) w[i] = 1.0f;
          }
          if (has_b) {
            lds_raw<16>(raw, b16 + chunk0 + k * p.tpr);
            unpack16<VEC>(b, raw, pbf16);
          } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) b[i] = 0.0f;
          }
        } else {
          load_param(w, w_smem, chunk0 + k * p.tpr);
          if (has_b) {
            load_param(b, b_smem, chunk0 + k * p.tpr);
          } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) b[i] = 0.0f;
          }
        }
        if constexpr (RAW) {
          forget_values(rx[k]);
          unpack_chunk<DT, VEC>(xc, rx[k], a.x_dtype);
          vfma_ss<VEC>(xc, xc, ra, rb);
        } else {
          vfma_ss<VEC>(xc, v[k], ra, rb);
        }
        vfma<VEC>(y, xc, w, b);
        if (k < nkr) store_chunk_p<DT, VEC>(op + k * step_o, y, a.out_dtype);
      }
    } else {
#pragma unroll
      for (int k = 0; k < K; ++k) {
        if (k < nkr) {
          float w[VEC], b[VEC], y[VEC], xc[VEC];
          const int c = colbase + k * cstride;
          if (has_w) {
            load_chunk<kDynDT, VEC, false>(w, a.weight, wrow + c, a.weight_dtype);
            vadd_s<VEC>(w, w, a.weight_offset);
          } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) w[i] = 1.0f;
          }
          if (has_b) {
            load_chunk<kDynDT, VEC, false>(b, a.bias, wrow + c, a.bias_dtype);
          } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) b[i] = 0.0f;
          }
          if constexpr (RAW) {
            forget_values(rx[k]);
            unpack_chunk<DT, VEC>(xc, rx[k], a.x_dtype);
            vfma_ss<VEC>(xc, xc, ra, rb);
          } else {
            vfma_ss<VEC>(xc, v[k], ra, rb);
          }
          vfma<VEC>(y, xc, w, b);
          store_chunk_p<DT, VEC>(op + k * step_o, y, a.out_dtype);
        }
      }
    }
  }
  // A CTA that never entered the loop still owes the wait matching its arrive.
  if (first && p.cluster_n > 1) cluster_wait();
}

struct FwdGrid {
  int max_ctas;    // override of the persistent-grid cap (0 = resident CTAs)
  int sm_count;
  int per_sm_cap;  // CTAs per SM beyond which more rows in flight cost bandwidth (0 = no cap)
};

template <int DT, int VEC, int K, bool RAW, bool LN>
static int launch_norm_fwd_s(const NormFwdParams& p, FwdGrid grid, int threads, size_t smem,
                             cudaStream_t st) {
  const int heads = static_cast<int>(p.a.H);
  const char* name = LN ? "layernorm_fwd" : "rmsnorm_fwd";
  if constexpr (VEC == 8) {
    if (p.stage_params == 2)
      return launch_persistent(norm_fwd_kernel<DT, VEC, K, LN, RAW, 2>, p.num_tiles, heads, threads,
                               smem, p.cluster_n, grid.max_ctas, grid.sm_count, st, p, name,
                               grid.per_sm_cap);
  }
  if (p.stage_params)
    return launch_persistent(norm_fwd_kernel<DT, VEC, K, LN, RAW, 1>, p.num_tiles, heads,
                             threads, smem, p.cluster_n, grid.max_ctas, grid.sm_count, st, p, name,
                             grid.per_sm_cap);
  return launch_persistent(norm_fwd_kernel<DT, VEC, K, LN, RAW, 0>, p.num_tiles, heads, threads,
                           smem, p.cluster_n, grid.max_ctas, grid.sm_count, st, p, name,
                           grid.per_sm_cap);
}

template <int DT, int VEC, int K, bool RAW>
static int launch_norm_fwd_k(const NormFwdParams& p, FwdGrid grid, int threads, size_t smem,
                             cudaStream_t st) {
  if (p.a.is_layernorm) return launch_norm_fwd_s<DT, VEC, K, RAW, true>(p, grid, threads, smem, st);
  return launch_norm_fwd_s<DT, VEC, K, RAW, false>(p, grid, threads, smem, st);
}

template <int DT, int VEC, bool RAW>
static int launch_norm_fwd_v(const NormFwdParams& p, int K, FwdGrid grid, int threads, size_t smem,
                             cudaStream_t st) {
  switch (K) {
    case 1: return launch_norm_fwd_k<DT, VEC, 1, RAW>(p, grid, threads, smem, st);
    case 2: return launch_norm_fwd_k<DT, VEC, 2, RAW>(p, grid, threads, smem, st);
    case 4: return launch_norm_fwd_k<DT, VEC, 4, RAW>(p, grid, threads, smem, st);
    case 8: return launch_norm_fwd_k<DT, VEC, 8, RAW>(p, grid, threads, smem, st);
    case 16:
      if constexpr (VEC <= 4 || RAW)
        return launch_norm_fwd_k<DT, VEC, 16, RAW>(p, grid, threads, smem, st);
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
  // Packed-register mode: 16-bit rows without a residual.
  const bool raw = uniform && a.residual == nullptr && a.residual_out == nullptr &&
                   a.x_dtype != QB_F32 && !(a.cfg.flags & 1);

  NormFwdParams p;
  p.timeouts = nullptr;
  p.a = a;
  p.flags = a.cfg.flags;
  // Long rows with at least one row per SM: the streamed two-pass kernel with the row parked in
  // L2.  Measured on B200 (bf16, 1 GiB per tensor) it overtakes the register / cluster kernels
  // from 64 KB per row (48 KB for LayerNorm, 128 KB with a residual, where two tensors are
  // streamed); flag bit 4
  // forces it for any row, flag bit 1 disables it.
  const int64_t row_bytes = a.N * host_dtype_bytes(a.x_dtype);
  const bool long_row =
      row_bytes >= (a.residual != nullptr ? (128 << 10) : (a.is_layernorm ? (48 << 10) : (64 << 10)));
  // The streamed kernel writes residual_out in its first pass and reads x / residual again in the
  // second one, so residual_out must not overlap either input (the register kernels allow that).
  // `out` is written in the second pass only, element by element by the thread that read the same
  // element, so an out that IS an input (same address, same stride) is safe; a shifted overlap is
  // not.
  auto overlaps = [&](const void* o, int64_t o_stride, const void* in, int64_t in_stride,
                      bool exact_alias_ok) {
    if (o == nullptr || in == nullptr) return false;
    if (exact_alias_ok && o == in && o_stride == in_stride) return false;
    const int eb = host_dtype_bytes(a.x_dtype);
    const char* o0 = static_cast<const char*>(o);
    const char* o1 = o0 + ((a.M - 1) * o_stride + a.N) * eb;
    const char* i0 = static_cast<const char*>(in);
    const char* i1 = i0 + ((a.M - 1) * in_stride + a.N) * eb;
    return o0 < i1 && i0 < o1;
  };
  const bool aliased =
      overlaps(a.residual_out, a.residual_out_row_stride, a.x, a.x_row_stride, false) ||
      overlaps(a.residual_out, a.residual_out_row_stride, a.residual, a.residual_row_stride, false) ||
      overlaps(a.out, a.out_row_stride, a.x, a.x_row_stride, true) ||
      overlaps(a.out, a.out_row_stride, a.residual, a.residual_row_stride, true);
  // Per-thread capacity in row elements: fp32-held rows 64 (<= 512 threads) / 16 (1024 threads);
  // packed 16-bit rows twice that; the generic mixed-dtype path (wider staging registers) 32.
  RowPlan plan;
  const ElemCaps caps = raw ? ElemCaps{128, 32, 16, 16}
                            : (uniform ? ElemCaps{64, 32, 16} : ElemCaps{32, 32, 16});
  const int64_t pref = raw ? 32768 : ((uniform && vec == 8) ? 16384 : 8192);
  // Packed rows: 16 chunks per thread (one warp per 4096-element row), CTAs of 256 threads from
  // 6144 elements on (measured: RMSNorm N = 8192 6.0 -> 6.5 TB/s, N = 12288 5.1 -> 6.2,
  // LayerNorm N = 6144 4.2 -> 5.0); fp32-held rows 8 chunks per thread.
  // (Exception, re-measured with the grid rule below: a packed RMSNorm row of exactly 8192 elements
  // runs 6.08 TB/s as one 128-thread CTA of 8 chunks per thread against 5.57 TB/s the other way;
  // LayerNorm, with its second pass over the registers, keeps 16 chunks: 5.88 against 4.40 TB/s.)
  const bool one_cta_row = raw && !a.is_layernorm && a.N * host_dtype_bytes(a.x_dtype) == 16384;
  int k_target = (raw && !one_cta_row) ? 16 : 8;
  int default_threads = raw && a.N >= 6144 && !one_cta_row ? 256 : 128;
  // RMSNorm rows of 2 - 8 KB (16-bit hidden sizes 1024 ... 4096): half the chunks per thread and
  // twice the threads per row.  Measured (bf16, 512 MiB per tensor, with residual / without):
  // N = 4096 6.06 -> 6.39 / 5.63 -> 6.16 TB/s, N = 2048 5.82 -> 6.39 / 5.60 -> 6.08,
  // N = 1024 5.97 -> 6.07 / 5.79 -> 6.12.
  // Only rows that fill such a tile exactly (N = 3072 would leave a quarter of it empty: -2 %).
  const int64_t row_bytes_x = a.N * host_dtype_bytes(a.x_dtype);
  if (!a.is_layernorm && uniform && vec == 8 && row_bytes_x >= 2048 && row_bytes_x <= 8192) {
    const int kt = raw ? 8 : 4;
    const int64_t chunks = a.N / vec;
    const int64_t tpr_c = chunks / kt;
    if (chunks % kt == 0 && (tpr_c & (tpr_c - 1)) == 0) {
      k_target = kt;
      if (raw && row_bytes_x >= 6144) default_threads = 256;
    }
  }
  // RMSNorm rows that split evenly over a cluster stay on the register kernel: with the st.async
  // exchange it beats the two-pass kernel at every long row measured (bf16, 512 MiB per tensor,
  // without / with residual: N = 65536 5.36 / 6.04 against 4.91 / 5.65 TB/s, N = 131072 5.13 /
  // 5.75 against 4.17 / 5.00, N = 262144 4.78 / 5.12 against 3.48 / 4.70).  Rows that would leave
  // more than an eighth of the cluster's register tile empty (N = 40960: 4.55 against 5.13) and
  // LayerNorm (whose parameters are not staged in the cluster kernel: 2.9 against 4.5) take the
  // two-pass kernel.
  bool prefer_cluster = false;
  if (!a.is_layernorm && long_row && !(a.cfg.flags & 16)) {
    RowPlan probe;
    if (plan_rows("norm_fwd", a.N, vec, caps, pref, k_target, default_threads, qb_launch_cfg{}, &probe) == QB_OK) {
      const int64_t tile = static_cast<int64_t>(probe.cluster_n) * probe.tpr * probe.K * vec;
      prefer_cluster = tile > 0 && (tile - a.N) * 8 <= tile;
    }
    clear_error();
  }
  if (uniform && a.H == 1 && a.cfg.cluster_n == 0 && !(a.cfg.flags & 2) && a.M >= dev->sm_count &&
      !aliased && !prefer_cluster && (long_row || (a.cfg.flags & 16))) {
    // CTA sizes that exist: 256 and 512 threads (a caller's hint is rounded to one of them).
    const int t = a.cfg.num_threads > 0 ? (a.cfg.num_threads > 256 ? 512 : 256)
                                        : (a.residual != nullptr ? 512 : 256);
    p.tpr = t;
    p.rows_per_cta = 1;
    p.cluster_n = 1;
    p.cols_per_cta = static_cast<int>(a.N);
    p.num_tiles = a.M;
    p.stage_params = 0;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    return launch_norm_fwd_stream_any(p, t, dev, st);
  }
  if (int rc = plan_rows("norm_fwd", a.N, vec, caps, pref, k_target, default_threads, a.cfg, &plan))
    return rc;
  const int K = plan.K;
  const int threads = plan.threads;

  p.tpr = plan.tpr;
  p.rows_per_cta = plan.rows_per_cta;
  p.cluster_n = plan.cluster_n;
  if (p.cluster_n > 1) {
    p.timeouts = ring_timeout_counter();
    if (p.timeouts == nullptr) return QB_ERR_CUDA;
  }
  p.cols_per_cta = plan.cols_per_cta;
  p.num_tiles = ceil_div(a.M, p.rows_per_cta);
  // fp32 (weight + offset) and bias slices of this CTA's columns (ones / zeros when absent), if
  // small enough to leave room for several CTAs per SM.
  size_t smem = static_cast<size_t>(plan.tpr) * plan.K * vec * 4 * (a.bias ? 2 : 1);
  p.stage_params = smem <= 64 * 1024;
  if (!p.stage_params) {
    // Too large as fp32: 16-bit weight and bias of one dtype are staged as they are (half the
    // bytes, unpacked in the epilogue) while that fits.
    const size_t packed = static_cast<size_t>(plan.tpr) * plan.K * 16 * (a.bias ? 2 : 1);
    const int pdt = a.weight ? a.weight_dtype : a.bias_dtype;
    const bool same = (a.weight == nullptr || a.bias == nullptr || a.weight_dtype == a.bias_dtype);
    if (vec == 8 && (a.weight || a.bias) && pdt != QB_F32 && same && packed <= 64 * 1024) {
      p.stage_params = 2;
      smem = packed;
    } else {
      smem = 0;
    }
  }
  // Persistent grid: exactly the CTAs that are resident at once, each walking over row tiles (so
  // weight / bias are staged once per CTA, not once per row).
  // CTAs per SM.  Measured on B200 (bf16): CTAs whose tile holds 32 KB of input rows run best three
  // to an SM (96 KB of rows in flight), not four -- RMSNorm with a residual at N = 8192: 2 / 3 / 4
  // CTAs per SM 5.82 / 6.41 / 5.99 TB/s; LayerNorm at N = 4096 (4 rows per CTA): 5.18 / 6.08 /
  // 5.90 TB/s -- so the persistent grid of such kernels is capped at 96 KB per SM.  Larger tiles
  // (64 KB: two CTAs per SM) keep everything that fits.
  const int64_t tile_bytes = static_cast<int64_t>(plan.rows_per_cta) * plan.cols_per_cta *
                             host_dtype_bytes(a.x_dtype) * (a.residual != nullptr ? 2 : 1);
  const int per_sm_cap =
      (tile_bytes > 0 && tile_bytes <= (32 << 10)) ? static_cast<int>((96 << 10) / tile_bytes) : 0;
  const FwdGrid grid = {a.cfg.max_ctas, dev->sm_count, a.H == 1 ? per_sm_cap : 0};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  if (uniform) {
    if (raw) {
      if (a.x_dtype == QB_BF16)
        return launch_norm_fwd_v<QB_BF16, 8, true>(p, K, grid, threads, smem, st);
      return launch_norm_fwd_v<QB_F16, 8, true>(p, K, grid, threads, smem, st);
    }
    switch (a.x_dtype) {
      case QB_BF16: return launch_norm_fwd_v<QB_BF16, 8, false>(p, K, grid, threads, smem, st);
      case QB_F16: return launch_norm_fwd_v<QB_F16, 8, false>(p, K, grid, threads, smem, st);
      default: return launch_norm_fwd_v<QB_F32, 4, false>(p, K, grid, threads, smem, st);
    }
  }
  switch (vec) {
    case 8: return launch_norm_fwd_v<kDynDT, 8, false>(p, K, grid, threads, smem, st);
    case 4: return launch_norm_fwd_v<kDynDT, 4, false>(p, K, grid, threads, smem, st);
    case 2: return launch_norm_fwd_v<kDynDT, 2, false>(p, K, grid, threads, smem, st);
    default: return launch_norm_fwd_v<kDynDT, 1, false>(p, K, grid, threads, smem, st);
  }
}
