// Cross-entropy forward / backward and the vocabulary-sharded combine, for sm_100a.
//
// Forward follows quack/cross_entropy.py:113-265 (CrossEntropy.kernel): per row an online
// (max, sum-exp) pair (quack/reduce.py:227-324), lse = max + log(sum), loss = w[t] * (lse - x[t])
// and exactly 0 for ignored rows.  The row is streamed through registers once (no need to keep
// it), so any row length runs in one CTA; a cluster splits long rows only when there are too few
// rows to fill the GPU.  Backward follows quack/cross_entropy.py:463-546
// (CrossEntropyBackward.kernel): a purely elementwise 2-D grid.
// Loads in this file use the default L2 policy instead of the evict-first "streaming" one:
// measured on B200, evict-first loads lose 1-3 % here whenever L2 still holds lines that other
// kernels left with the default policy (they are never displaced by evict-first traffic), while
// default-policy loads run at the same speed in either state.  Stores stay evict-first.
#define QB_LDG_MOD ""
#include <type_traits>

#include "common.cuh"
#include "host_common.h"

namespace qb {

struct CeFwdParams {
  qb_ce_fwd_args a;
  int tpr, rows_per_cta, cluster_n, cols_per_cta;
  int64_t num_tiles;
  int flags;  // qb_launch_cfg.flags
  unsigned int* timeouts;  // device counter of cluster-exchange waits that gave up
};

// A target names a class only if it is not ignore_index and lies inside [0, num_classes) (no upper
// bound when num_classes is 0); anything else makes the row an ignored one.
__device__ __forceinline__ bool target_ignored(int64_t tgt, int64_t ignore_index, int64_t num_classes) {
  return tgt == ignore_index || tgt < 0 || (num_classes > 0 && tgt >= num_classes);
}

constexpr int kCeUnroll = 4;  // chunks in flight per thread and loop iteration

template <int DT, int VEC>
__global__ void __launch_bounds__(512) ce_fwd_kernel(const CeFwdParams p) {
  __shared__ ReduceScratch scratch;
  const qb_ce_fwd_args& a = p.a;
  const RowGeom g = make_geom(p.tpr, p.cluster_n);
  reduce_init(scratch, p.cluster_n);
  if (p.cluster_n > 1) cluster_arrive();
  const int N = static_cast<int>(a.N);
  const int col0 = static_cast<int>(g.crank) * p.cols_per_cta;
  const int ncols = min(p.cols_per_cta, N - col0);
  const int nchunks = ncols > 0 ? ncols / VEC : 0;

  const int64_t tile_stride = gridDim.x / p.cluster_n;
  int rit = 0;
  bool first = true;
  for (int64_t tile = blockIdx.x / p.cluster_n; tile < p.num_tiles; tile += tile_stride) {
    const int64_t row = tile * p.rows_per_cta + g.r;
    const bool row_ok = row < a.M;
    const int64_t xrow = row * a.x_row_stride + col0;

    // Running maximum m and s = sum 2^(x*log2e + off.hi) over this thread's elements.
    float m = neg_inf();
    float s = 0.0f;
    ExpOffset off = exp_offset(m);
    int c = g.t;
    if constexpr (DT != kDynDT) {
      // Blocks of kCeUnroll chunks that lie completely inside the row: unpredicated loads through
      // one byte pointer, the block's maximum first (packed for 16-bit dtypes) and one re-basing
      // check per block instead of one per chunk.
      constexpr int kEsz = DT == QB_F32 ? 4 : 2;
      const int step = p.tpr * VEC * kEsz;
      const char* xp = reinterpret_cast<const char*>(a.x) + (xrow + static_cast<int64_t>(c) * VEC) * kEsz;
      for (; row_ok && c + (kCeUnroll - 1) * p.tpr < nchunks; c += p.tpr * kCeUnroll, xp += step * kCeUnroll) {
        uint32_t raw[kCeUnroll][RawWords<DT, VEC>::value];
#pragma unroll
        for (int u = 0; u < kCeUnroll; ++u) ldg_stream_full<VEC * kEsz>(raw[u], xp + u * step);
        float cm;
        if constexpr (DT == QB_F32) {
          cm = __uint_as_float(raw[0][0]);
#pragma unroll
          for (int u = 0; u < kCeUnroll; ++u)
#pragma unroll
            for (int i = 0; i < VEC; ++i) cm = fmaxf(cm, __uint_as_float(raw[u][i]));
        } else {
          cm = packed_max16<DT, VEC>(raw[0]);
#pragma unroll
          for (int u = 1; u < kCeUnroll; ++u) cm = fmaxf(cm, packed_max16<DT, VEC>(raw[u]));
        }
        if (cm > m) {
          const ExpOffset nw = exp_offset(cm);
          s *= fast_exp2(nw.hi - off.hi);
          m = cm;
          off = nw;
        }
#pragma unroll
        for (int u = 0; u < kCeUnroll; ++u) {
          float v[VEC];
          unpack_chunk<DT, VEC>(v, raw[u], DT);
#pragma unroll
          for (int i = 0; i < VEC; ++i) s += fast_exp2(fmaf(v[i], kLog2e, off.hi));
        }
      }
    }
    for (; c < nchunks; c += p.tpr * kCeUnroll) {
      uint32_t raw[kCeUnroll][RawWords<DT, VEC>::value];
#pragma unroll
      for (int u = 0; u < kCeUnroll; ++u) {
        const int cu = c + u * p.tpr;
        load_chunk_raw<DT, VEC>(raw[u], a.x, xrow + static_cast<int64_t>(cu) * VEC, a.x_dtype,
                                row_ok && cu < nchunks);
      }
#pragma unroll
      for (int u = 0; u < kCeUnroll; ++u) {
        const int cu = c + u * p.tpr;
        if (row_ok && cu < nchunks) {
          float v[VEC];
          unpack_chunk<DT, VEC>(v, raw[u], a.x_dtype);
          float cm = v[0];
#pragma unroll
          for (int i = 1; i < VEC; ++i) cm = fmaxf(cm, v[i]);
          if (cm > m) {
            // Re-base the partial sum on the new maximum: exact difference of the two offsets.
            const ExpOffset nw = exp_offset(cm);
            s *= fast_exp2(nw.hi - off.hi);
            m = cm;
            off = nw;
          }
#pragma unroll
          for (int i = 0; i < VEC; ++i) s += fast_exp2(fmaf(v[i], kLog2e, off.hi));
        }
      }
    }
    s *= fast_exp2(off.lo);  // now s == sum exp(x - m)

    if (first && p.cluster_n > 1) cluster_wait();
    first = false;
    const float2 ms = row_reduce<MaxSumExpOp>(make_float2(m, s), g, scratch, 0, rit, p.timeouts);
    ++rit;

    if (row_ok && g.t == 0 && g.crank == 0) {
      const int64_t tgt = load_index(a.target, row, a.target_dtype);
      const bool ignored = target_ignored(tgt, a.ignore_index, a.num_classes);
      const int64_t local = tgt - a.col_offset;
      const bool owned = !ignored && local >= 0 && local < a.N;
      float tl = 0.0f;
      if (!ignored) {
        if (a.target_logit != nullptr) {
          tl = a.target_logit_ndim == 2
                   ? load_scalar(a.target_logit, row * a.target_logit_row_stride + tgt,
                                 a.target_logit_dtype)
                   : load_scalar(a.target_logit, row, a.target_logit_dtype);
        } else if (owned) {
          tl = load_scalar(a.x, row * a.x_row_stride + local, a.x_dtype);
        }
      }
      const float log_s = logf(ms.y);
      if (a.lse != nullptr) a.lse[row] = ms.x + log_s;
      if (a.loss != nullptr) {
        float wt = 1.0f;
        if (a.weight != nullptr && !ignored) wt = load_scalar(a.weight, tgt, a.weight_dtype);
        // (max - target logit) + log(sum) loses less than (max + log(sum)) - target logit.
        a.loss[row] = ignored ? 0.0f : wt * ((ms.x - tl) + log_s);
      }
      if (a.row_max != nullptr) a.row_max[row] = ms.x;
      if (a.row_sumexp != nullptr) a.row_sumexp[row] = ms.y;
      if (a.row_tgt != nullptr) a.row_tgt[row] = tl;
    }
  }
  if (first && p.cluster_n > 1) cluster_wait();
}

// ---------------------------------------------------------------------------------------------
// forward with dx in one launch: loss, lse and dx = w[t] * (softmax(x) - onehot)
// ---------------------------------------------------------------------------------------------
// The reference's forward kernel keeps the row in shared memory and writes dx from there
// (quack/cross_entropy.py:240-265).  Vocabulary rows (64 ... 512 KB) do not fit, so here one CTA
// streams its row twice: pass 1 (online log-sum-exp, as in ce_fwd_kernel) leaves the row in L2,
// pass 2 re-reads it from L2 newest lines first and writes dx.  DRAM sees one read and one write
// per logit, as in the reference.  dx may alias x: every chunk is read and written by the same
// thread, and everything pass 1 needs from the row is read before pass 2 starts.
// T threads share the row (T == blockDim.x), U chunks in flight per thread; blocks of T * U
// chunks, all but possibly the last one full.
template <int DT, int U, int T>
__global__ void __launch_bounds__(T, (T >= 1024) ? 1 : (1024 / T)) ce_fwd_dx_kernel(const CeFwdParams p) {
  static_assert(DT == QB_F32 || DT == QB_F16 || DT == QB_BF16, "concrete dtype required");
  constexpr int VEC = DT == QB_F32 ? 4 : 8;
  constexpr int kStep = T * 16;
  constexpr int kBlockBytes = U * kStep;
  __shared__ ReduceScratch scratch;
  const qb_ce_fwd_args& a = p.a;
  const RowGeom g = make_geom(T, 1);
  const int N = static_cast<int>(a.N);
  const int nchunks = N / VEC;
  const int nfull = nchunks / (T * U);
  const bool tail = nfull * (T * U) < nchunks;
  const int tail_c0 = nfull * (T * U) + g.t;
  const uint64_t keep = l2_policy((p.flags & 4) ? 2 : 0);
  const uint64_t drop = l2_policy((p.flags & 8) ? 2 : 1);
  int rit = 0;
  for (int64_t row = blockIdx.x; row < a.M; row += gridDim.x) {
    const char* xin = reinterpret_cast<const char*>(a.x) + (row * a.x_row_stride * (16 / VEC) + g.t * 16);
    char* dxo = reinterpret_cast<char*>(a.dx) + (row * a.dx_row_stride * (16 / VEC) + g.t * 16);

    // Row scalars (same address for all threads: broadcast loads), read before this row's dx
    // is written because dx may alias x.
    const int64_t tgt = load_index(a.target, row, a.target_dtype);
    const bool ignored = target_ignored(tgt, a.ignore_index, a.num_classes);
    const int64_t local = tgt - a.col_offset;
    const bool owned = !ignored && local >= 0 && local < a.N;
    float gscale = 0.0f;  // w[target], 0 for ignored rows
    if (!ignored) gscale = a.weight != nullptr ? load_scalar(a.weight, tgt, a.weight_dtype) : 1.0f;
    const int tcol = owned ? static_cast<int>(local) : -1;
    float tl = 0.0f;
    if (g.t == 0 && !ignored) {
      if (a.target_logit != nullptr) {
        tl = a.target_logit_ndim == 2
                 ? load_scalar(a.target_logit, row * a.target_logit_row_stride + tgt,
                               a.target_logit_dtype)
                 : load_scalar(a.target_logit, row, a.target_logit_dtype);
      } else if (owned) {
        tl = load_scalar(a.x, row * a.x_row_stride + local, a.x_dtype);
      }
    }

    // ---- pass 1 ----
    float m = neg_inf(), s = 0.0f;
    ExpOffset off = exp_offset(m);
    // The block's chunks live at row scope: the block pass 1 reads last is the one pass 2 starts
    // with, so it stays in registers across the row reduction instead of being read again.
    uint32_t r[U][4];
    auto pass1 = [&](auto full_tag, const char* q, int c0) {
      constexpr bool FULL = decltype(full_tag)::value;
#pragma unroll
      for (int u = 0; u < U; ++u) ldg16_hint<!FULL>(r[u], q + u * kStep, c0 + u * T < nchunks, keep);
      float cm = neg_inf();
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (FULL || c0 + u * T < nchunks) {
          if constexpr (DT == QB_F32) {
#pragma unroll
            for (int i = 0; i < VEC; ++i) cm = fmaxf(cm, __uint_as_float(r[u][i]));
          } else {
            cm = fmaxf(cm, packed_max16<DT, VEC>(r[u]));
          }
        }
      }
      if (cm > m) {
        const ExpOffset nw = exp_offset(cm);
        s *= fast_exp2(nw.hi - off.hi);
        m = cm;
        off = nw;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (FULL || c0 + u * T < nchunks) {
          float v[VEC];
          unpack_chunk<DT, VEC>(v, r[u], DT);
#pragma unroll
          for (int i = 0; i < VEC; ++i) s += fast_exp2(fmaf(v[i], kLog2e, off.hi));
        }
      }
    };
    {
      const char* q = xin;
      for (int b = 0; b < nfull; ++b, q += kBlockBytes) pass1(std::true_type{}, q, 0);
      if (tail) pass1(std::false_type{}, q, tail_c0);
    }
    s *= fast_exp2(off.lo);
    const float2 ms = row_reduce<MaxSumExpOp>(make_float2(m, s), g, scratch, 0, rit, p.timeouts);
    ++rit;
    const float log_s = logf(ms.y);
    const float lse = ms.x + log_s;
    if (g.t == 0) {
      if (a.lse != nullptr) a.lse[row] = lse;
      if (a.loss != nullptr) a.loss[row] = ignored ? 0.0f : gscale * ((ms.x - tl) + log_s);
      if (a.row_max != nullptr) a.row_max[row] = ms.x;
      if (a.row_sumexp != nullptr) a.row_sumexp[row] = ms.y;
      if (a.row_tgt != nullptr) a.row_tgt[row] = tl;
    }

    // ---- pass 2: dx, newest lines first ----
    off = exp_offset(lse);
    const float pscale = fast_exp2(off.lo) * gscale;
    auto pass2 = [&](auto full_tag, auto resident_tag, const char* q, char* qo, int c0) {
      constexpr bool FULL = decltype(full_tag)::value;
      constexpr bool RESIDENT = decltype(resident_tag)::value;  // the chunks are still in r
      if constexpr (!RESIDENT) {
#pragma unroll
        for (int u = 0; u < U; ++u) ldg16_hint<!FULL>(r[u], q + u * kStep, c0 + u * T < nchunks, drop);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float v[VEC], d[VEC];
        unpack_chunk<DT, VEC>(v, r[u], DT);
#pragma unroll
        for (int i = 0; i < VEC; ++i) d[i] = fast_exp2(fmaf(v[i], kLog2e, off.hi)) * pscale;
        const unsigned rel = static_cast<unsigned>(tcol - (c0 + u * T) * VEC);
        if (rel < static_cast<unsigned>(VEC)) {
#pragma unroll
          for (int i = 0; i < VEC; ++i)
            if (rel == static_cast<unsigned>(i)) d[i] -= gscale;
        }
        if (FULL || c0 + u * T < nchunks) store_chunk_p<DT, VEC>(qo + u * kStep, d, DT);
      }
    };
    {
      const int64_t end = static_cast<int64_t>(nfull) * kBlockBytes;
      if (tail) pass2(std::false_type{}, std::true_type{}, xin + end, dxo + end, tail_c0);
      const char* q = xin + end;
      char* qo = dxo + end;
      for (int b = nfull - 1; b >= 0; --b) {
        q -= kBlockBytes;
        qo -= kBlockBytes;
        if (!tail && b == nfull - 1) pass2(std::true_type{}, std::true_type{}, q, qo, b * (T * U) + g.t);
        else pass2(std::true_type{}, std::false_type{}, q, qo, b * (T * U) + g.t);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// backward: dx = (exp(x - lse) - onehot) * dloss * w[target]
// ---------------------------------------------------------------------------------------------
struct CeBwdParams {
  qb_ce_bwd_args a;
  int tpr, rows_per_cta;
  int cols_per_block;  // tpr * kCeBwdUnroll * VEC
  int64_t num_tiles;
};

constexpr int kCeBwdUnroll = 8;  // chunks per thread and column block

template <int DT, int VEC>
__global__ void __launch_bounds__(512) ce_bwd_kernel(const CeBwdParams p) {
  const qb_ce_bwd_args& a = p.a;
  const int t = threadIdx.x & (p.tpr - 1);
  const int r = threadIdx.x / p.tpr;
  const int N = static_cast<int>(a.N);
  const int colbase = blockIdx.y * p.cols_per_block + t * VEC;
  const int cstride = p.tpr * VEC;
  // chunks of this thread inside the row: u < nu
  const int nu = colbase < N ? min(kCeBwdUnroll, (N - colbase + cstride - 1) / cstride) : 0;
  for (int64_t tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
    const int64_t row = tile * p.rows_per_cta + r;
    const bool row_ok = row < a.M;
    const int nur = row_ok ? nu : 0;
    uint32_t raw[kCeBwdUnroll][RawWords<DT, VEC>::value];
    const int esz_x = elem_bytes<DT>(a.x_dtype), esz_dx = elem_bytes<DT>(a.dx_dtype);
    const char* xp = reinterpret_cast<const char*>(a.x) + (row * a.x_row_stride + colbase) * esz_x;
    char* dxp = reinterpret_cast<char*>(a.dx) + (row * a.dx_row_stride + colbase) * esz_dx;
    const int step_x = cstride * esz_x, step_dx = cstride * esz_dx;
#pragma unroll
    for (int u = 0; u < kCeBwdUnroll; ++u)
      load_chunk_raw_p<DT, VEC>(raw[u], xp + u * step_x, a.x_dtype, u < nur);
    // Row scalars (the same addresses for every thread of the row group: broadcast loads).
    float gscale = 0.0f;  // dloss * w[target], 0 for ignored rows
    float lse = 0.0f;
    int tcol = -1;  // local column of the target, -1 if none inside this shard
    if (row_ok) {
      const int64_t tgt = load_index(a.target, row, a.target_dtype);
      lse = a.lse[row];
      if (!target_ignored(tgt, a.ignore_index, a.num_classes)) {
        gscale = a.dloss != nullptr ? a.dloss[row * a.dloss_stride] : 1.0f;
        if (a.weight != nullptr) gscale *= load_scalar(a.weight, tgt, a.weight_dtype);
        const int64_t local = tgt - a.col_offset;
        if (local >= 0 && local < a.N) tcol = static_cast<int>(local);
      }
    }
    // exp(x - lse) = 2^(x*log2e + hi) * 2^lo; the row-constant 2^lo is folded into the scale.
    const ExpOffset off = exp_offset(lse);
    const float pscale = fast_exp2(off.lo) * gscale;
#pragma unroll
    for (int u = 0; u < kCeBwdUnroll; ++u) {
      if (u < nur) {
        const int c = colbase + u * cstride;
        float v[VEC], d[VEC];
        unpack_chunk<DT, VEC>(v, raw[u], a.x_dtype);
#pragma unroll
        for (int i = 0; i < VEC; ++i) d[i] = fast_exp2(fmaf(v[i], kLog2e, off.hi)) * pscale;
        // one-hot term: at most one element of one chunk of the row
        const unsigned rel = static_cast<unsigned>(tcol - c);
        if (rel < static_cast<unsigned>(VEC)) {
#pragma unroll
          for (int i = 0; i < VEC; ++i)
            if (rel == static_cast<unsigned>(i)) d[i] -= gscale;
        }
        store_chunk_p<DT, VEC>(dxp + u * step_dx, d, a.dx_dtype);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// vocabulary-sharded combine: fixed shard order, one thread per row
// ---------------------------------------------------------------------------------------------
struct CeCombineParams {
  qb_ce_combine_args a;
};

__global__ void __launch_bounds__(256) ce_combine_kernel(const CeCombineParams p) {
  const qb_ce_combine_args& a = p.a;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= a.M) return;
  float m = neg_inf();
  for (int64_t g = 0; g < a.G; ++g) m = fmaxf(m, a.stats[(g * 3 + 0) * a.M + row]);
  float s = 0.0f;
  float t = 0.0f;
  for (int64_t g = 0; g < a.G; ++g) {
    const float mg = a.stats[(g * 3 + 0) * a.M + row];
    const float sg = a.stats[(g * 3 + 1) * a.M + row];
    if (mg != neg_inf()) s += sg * exp2f((mg - m) * kLog2e);
    t += a.stats[(g * 3 + 2) * a.M + row];
  }
  const float log_s = logf(s);
  if (a.lse != nullptr) a.lse[row] = m + log_s;
  if (a.loss != nullptr) {
    const int64_t tgt = load_index(a.target, row, a.target_dtype);
    const bool ignored = target_ignored(tgt, a.ignore_index, a.num_classes);
    float wt = 1.0f;
    if (a.weight != nullptr && !ignored) wt = load_scalar(a.weight, tgt, a.weight_dtype);
    a.loss[row] = ignored ? 0.0f : wt * ((m - t) + log_s);
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
template <class Params, template <int, int> class Launcher>
static int dispatch_dt_vec(bool uniform, int dt, int vec, const Params& p, dim3 grid, int threads,
                           int cluster_n, cudaStream_t st) {
  if (uniform) {
    switch (dt) {
      case QB_BF16: return Launcher<QB_BF16, 8>::run(p, grid, threads, cluster_n, st);
      case QB_F16: return Launcher<QB_F16, 8>::run(p, grid, threads, cluster_n, st);
      default: return Launcher<QB_F32, 4>::run(p, grid, threads, cluster_n, st);
    }
  }
  switch (vec) {
    case 8: return Launcher<kDynDT, 8>::run(p, grid, threads, cluster_n, st);
    case 4: return Launcher<kDynDT, 4>::run(p, grid, threads, cluster_n, st);
    case 2: return Launcher<kDynDT, 2>::run(p, grid, threads, cluster_n, st);
    default: return Launcher<kDynDT, 1>::run(p, grid, threads, cluster_n, st);
  }
}

template <int DT, int VEC>
struct CeFwdLauncher {
  static int run(const CeFwdParams& p, dim3 grid, int threads, int cluster_n, cudaStream_t st) {
    return launch_kernel(ce_fwd_kernel<DT, VEC>, grid, threads, 0, cluster_n, st, p, "ce_fwd");
  }
};
template <int DT, int VEC>
struct CeBwdLauncher {
  static int run(const CeBwdParams& p, dim3 grid, int threads, int cluster_n, cudaStream_t st) {
    return launch_kernel(ce_bwd_kernel<DT, VEC>, grid, threads, 0, cluster_n, st, p, "ce_bwd");
  }
};

static int run_ce_bwd(const qb_ce_bwd_args& a, cudaStream_t st) {
  const DeviceFacts* dev = current_device_facts();
  if (dev == nullptr) return QB_ERR_CUDA;
  VecWidth vw;
  vw.limit_elems(a.N);
  vw.add_tensor(a.x, a.x_dtype, a.x_row_stride);
  vw.add_tensor(a.dx, a.dx_dtype, a.dx_row_stride);
  const int vec = vw.vec;
  const bool uniform = a.x_dtype == a.dx_dtype && vec == 16 / host_dtype_bytes(a.x_dtype);
  int threads = a.cfg.num_threads > 0 ? a.cfg.num_threads : 256;
  if (!is_pow2(threads) || threads < 32 || threads > 512)
    return set_error(QB_ERR_INVALID, "ce_bwd: bad num_threads %d", threads);
  const int64_t chunks = a.N / vec;
  int tpr = next_pow2(ceil_div(chunks, kCeBwdUnroll));
  if (tpr < 8) tpr = 8;
  if (tpr > threads) tpr = threads;
  CeBwdParams p;
  p.a = a;
  p.tpr = tpr;
  p.rows_per_cta = threads / tpr;
  p.cols_per_block = tpr * kCeBwdUnroll * vec;
  p.num_tiles = ceil_div(a.M, p.rows_per_cta);
  const int64_t col_blocks = ceil_div(a.N, p.cols_per_block);
  if (col_blocks > 65535) return set_error(QB_ERR_UNSUPPORTED, "ce_bwd: N too large");
  int64_t gx = p.num_tiles;
  const int64_t cap = a.cfg.max_ctas > 0 ? a.cfg.max_ctas : (int64_t)1 << 30;
  if (gx * col_blocks > cap) gx = cap / col_blocks > 0 ? cap / col_blocks : 1;
  if (gx > 0x7fffffffLL) gx = 0x7fffffffLL;
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(col_blocks), 1);
  return dispatch_dt_vec<CeBwdParams, CeBwdLauncher>(uniform, a.x_dtype, vec, p, grid, threads, 1,
                                                     st);
}

template <int DT, int T>
static int launch_ce_fwd_dx_t(const CeFwdParams& p, const DeviceFacts* dev, cudaStream_t st) {
  auto kernel = ce_fwd_dx_kernel<DT, 8, T>;
  const int occ = cached_occupancy(reinterpret_cast<const void*>(kernel), T, 0);
  int64_t ctas = static_cast<int64_t>(dev->sm_count) * (occ > 0 ? occ : 1);
  if (p.a.cfg.max_ctas > 0) ctas = p.a.cfg.max_ctas;
  if (ctas > p.a.M) ctas = p.a.M;
  // Evict-last marking in pass 1 only while the rows in flight fit comfortably in L2.
  CeFwdParams q = p;
  if (ctas * p.a.N * host_dtype_bytes(p.a.x_dtype) > (48LL << 20)) q.flags |= 4;
  dim3 grid(static_cast<unsigned>(ctas), 1, 1);
  return launch_kernel(kernel, grid, T, 0, 1, st, q, "ce_fwd (with dx)");
}

template <int DT>
static int launch_ce_fwd_dx(const CeFwdParams& p, int threads, const DeviceFacts* dev,
                            cudaStream_t st) {
  switch (threads) {
    case 256: return launch_ce_fwd_dx_t<DT, 256>(p, dev, st);
    case 512: return launch_ce_fwd_dx_t<DT, 512>(p, dev, st);
    case 1024: return launch_ce_fwd_dx_t<DT, 1024>(p, dev, st);
    default: return set_error(QB_ERR_INVALID, "ce_fwd (with dx): num_threads must be 256, 512 or 1024");
  }
}

}  // namespace qb

using namespace qb;

extern "C" int qb_ce_bwd(const qb_ce_bwd_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "ce_bwd: null argument block");
  const qb_ce_bwd_args& a = *args;
  if (a.x == nullptr || a.target == nullptr || a.lse == nullptr || a.dx == nullptr)
    return set_error(QB_ERR_INVALID, "ce_bwd: x, target, lse and dx are required");
  if (a.M < 0 || a.N <= 0 || a.N > (1 << 30))
    return set_error(QB_ERR_INVALID, "ce_bwd: bad sizes M=%lld N=%lld", (long long)a.M,
                     (long long)a.N);
  if (!is_float_dtype(a.x_dtype) || !is_float_dtype(a.dx_dtype) ||
      (a.weight && !is_float_dtype(a.weight_dtype)) ||
      (a.target_dtype != QB_I32 && a.target_dtype != QB_I64))
    return set_error(QB_ERR_INVALID, "ce_bwd: unsupported dtype code");
  if (a.M == 0) return QB_OK;
  return run_ce_bwd(a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int qb_ce_fwd(const qb_ce_fwd_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "ce_fwd: null argument block");
  const qb_ce_fwd_args& a = *args;
  if (a.x == nullptr || a.target == nullptr)
    return set_error(QB_ERR_INVALID, "ce_fwd: x and target are required");
  const bool sharded = a.row_max != nullptr || a.row_sumexp != nullptr || a.row_tgt != nullptr;
  if (a.loss == nullptr && !sharded)
    return set_error(QB_ERR_INVALID, "ce_fwd: loss is required unless the row_* outputs are given");
  if (a.dx != nullptr && a.lse == nullptr)
    return set_error(QB_ERR_INVALID, "ce_fwd: dx requires the lse output");
  if (a.M < 0 || a.N <= 0 || a.N > (1 << 30))
    return set_error(QB_ERR_INVALID, "ce_fwd: bad sizes M=%lld N=%lld", (long long)a.M,
                     (long long)a.N);
  if (!is_float_dtype(a.x_dtype) || (a.weight && !is_float_dtype(a.weight_dtype)) ||
      (a.target_logit && !is_float_dtype(a.target_logit_dtype)) ||
      (a.target_dtype != QB_I32 && a.target_dtype != QB_I64) ||
      (a.target_logit && a.target_logit_ndim != 1 && a.target_logit_ndim != 2))
    return set_error(QB_ERR_INVALID, "ce_fwd: unsupported dtype code or target_logit rank");
  if (a.M == 0) return QB_OK;
  const DeviceFacts* dev = current_device_facts();
  if (dev == nullptr) return QB_ERR_CUDA;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  VecWidth vw;
  vw.limit_elems(a.N);
  vw.add_tensor(a.x, a.x_dtype, a.x_row_stride);
  const int vec = vw.vec;
  const bool uniform = vec == 16 / host_dtype_bytes(a.x_dtype);
  if (a.dx != nullptr) {
    // Vocabulary-sized rows with enough rows to give every SM one: loss, lse and dx in one
    // launch that streams each row twice (the second time from L2).
    VecWidth vd = vw;
    vd.add_tensor(a.dx, a.x_dtype, a.dx_row_stride);
    const int64_t row_bytes = a.N * host_dtype_bytes(a.x_dtype);
    if (vd.vec == 16 / host_dtype_bytes(a.x_dtype) && a.cfg.cluster_n == 0 &&
        !(a.cfg.flags & 2) && a.M >= dev->sm_count && row_bytes >= (64 << 10)) {
      CeFwdParams p;
      p.timeouts = nullptr;
      p.a = a;
      p.tpr = 0;
      p.rows_per_cta = 1;
      p.cluster_n = 1;
      p.cols_per_cta = static_cast<int>(a.N);
      p.num_tiles = a.M;
      p.flags = a.cfg.flags;
      const int t = a.cfg.num_threads > 0
                        ? a.cfg.num_threads
                        : (row_bytes <= (96 << 10) ? 256 : (row_bytes <= (192 << 10) ? 512 : 1024));
      switch (a.x_dtype) {
        case QB_BF16: return launch_ce_fwd_dx<QB_BF16>(p, t, dev, st);
        case QB_F16: return launch_ce_fwd_dx<QB_F16>(p, t, dev, st);
        default: return launch_ce_fwd_dx<QB_F32>(p, t, dev, st);
      }
    }
  }
  int threads = a.cfg.num_threads > 0 ? a.cfg.num_threads : 128;
  if (!is_pow2(threads) || threads < 32 || threads > 512)
    return set_error(QB_ERR_INVALID, "ce_fwd: bad num_threads %d", threads);
  const int64_t chunks = a.N / vec;
  // Threads per row: about 64 chunks (16 loop trips of kCeUnroll) per thread, i.e. as few threads
  // per row as keeps 128 of them busy -- short rows then need no shared-memory exchange at all
  // and a CTA carries many rows.  Measured on B200 (bf16): N = 4096 3.3 -> 6.2 TB/s with 8
  // instead of 128 threads per row; the best width doubles with every doubling of N.
  int tpr = a.cfg.threads_per_row > 0 ? a.cfg.threads_per_row
                                      : next_pow2(ceil_div(chunks, 16 * kCeUnroll));
  if (!is_pow2(tpr)) return set_error(QB_ERR_INVALID, "ce_fwd: bad threads_per_row %d", tpr);
  if (tpr < 8) tpr = 8;
  if (tpr > threads) tpr = threads;
  int cluster_n = a.cfg.cluster_n;
  if (cluster_n < 0 || (cluster_n && !is_pow2(cluster_n)) || cluster_n > kMaxCluster)
    return set_error(QB_ERR_INVALID, "ce_fwd: bad cluster_n %d", cluster_n);
  if (cluster_n == 0) {
    // Split rows over a cluster only when whole-row CTAs would leave SMs idle.
    cluster_n = 1;
    if (tpr == threads) {
      while (cluster_n < 8 && a.M * cluster_n * 2 <= 2 * (int64_t)dev->sm_count &&
             chunks / (cluster_n * 2) >= (int64_t)threads * kCeUnroll)
        cluster_n <<= 1;
    }
  }
  if (cluster_n > 1) {
    tpr = threads;  // one row per CTA tile when a cluster shares the row
    while (cluster_n > 1 && (int64_t)(cluster_n - 1) * ceil_div(chunks, cluster_n) >= chunks)
      cluster_n >>= 1;
  }
  CeFwdParams p;
  p.a = a;
  p.tpr = tpr;
  p.rows_per_cta = threads / tpr;
  p.cluster_n = cluster_n;
  p.timeouts = nullptr;
  if (cluster_n > 1) {
    p.timeouts = ring_timeout_counter();
    if (p.timeouts == nullptr) return QB_ERR_CUDA;
  }
  p.cols_per_cta = static_cast<int>(ceil_div(chunks, cluster_n) * vec);
  p.num_tiles = ceil_div(a.M, p.rows_per_cta);
  p.flags = a.cfg.flags;
  const int64_t max_ctas =
      a.cfg.max_ctas > 0 ? a.cfg.max_ctas
                         : (cluster_n == 1 ? (int64_t)0x7fffffff
                                           : (int64_t)dev->sm_count * (2048 / threads) * 2);
  int64_t clusters = p.num_tiles;
  if (clusters > max_ctas / cluster_n) clusters = max_ctas / cluster_n;
  if (clusters < 1) clusters = 1;
  dim3 grid(static_cast<unsigned>(clusters * cluster_n), 1, 1);
  if (int rc = dispatch_dt_vec<CeFwdParams, CeFwdLauncher>(uniform, a.x_dtype, vec, p, grid,
                                                           threads, cluster_n, st))
    return rc;
  if (a.dx == nullptr) return QB_OK;

  // Gradient w.r.t. the logits from the lse just written: dx = w[t] * (softmax - onehot).
  qb_ce_bwd_args b = {};
  b.x = a.x;
  b.target = a.target;
  b.dloss = nullptr;  // upstream gradient 1
  b.lse = a.lse;
  b.weight = a.weight;
  b.dx = a.dx;
  b.M = a.M;
  b.N = a.N;
  b.x_row_stride = a.x_row_stride;
  b.dx_row_stride = a.dx_row_stride;
  b.dloss_stride = 0;
  b.col_offset = a.col_offset;
  b.ignore_index = a.ignore_index;
  b.num_classes = a.num_classes;
  b.x_dtype = a.x_dtype;
  b.dx_dtype = a.x_dtype;
  b.target_dtype = a.target_dtype;
  b.weight_dtype = a.weight_dtype;
  return run_ce_bwd(b, st);
}

extern "C" int qb_ce_combine(const qb_ce_combine_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "ce_combine: null argument block");
  const qb_ce_combine_args& a = *args;
  if (a.stats == nullptr || a.target == nullptr || (a.loss == nullptr && a.lse == nullptr))
    return set_error(QB_ERR_INVALID, "ce_combine: stats, target and an output are required");
  if (a.G <= 0 || a.M < 0) return set_error(QB_ERR_INVALID, "ce_combine: bad sizes");
  if ((a.target_dtype != QB_I32 && a.target_dtype != QB_I64) ||
      (a.weight && !is_float_dtype(a.weight_dtype)))
    return set_error(QB_ERR_INVALID, "ce_combine: unsupported dtype code");
  if (a.M == 0) return QB_OK;
  CeCombineParams p;
  p.a = a;
  dim3 grid(static_cast<unsigned>(ceil_div(a.M, 256)), 1, 1);
  return launch_kernel(ce_combine_kernel, grid, 256, 0, 1, reinterpret_cast<cudaStream_t>(stream),
                       p, "ce_combine");
}
