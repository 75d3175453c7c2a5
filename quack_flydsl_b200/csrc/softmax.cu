// Softmax forward and backward over the last dimension, for sm_100a.
//
// Forward follows quack/softmax.py:87-176 (Softmax.kernel, online (max, sum-exp) pair combined in
// one exchange, quack/reduce.py:227-324); backward follows quack/softmax.py:275-353
// (SoftmaxBackward.kernel).  A row is read once, kept in registers, and written once; rows longer
// than one CTA's register capacity are split over a thread-block cluster whose CTAs exchange
// their partials through distributed shared memory.
// Loads in this file use the default L2 policy instead of the evict-first "streaming" one:
// measured on B200, evict-first loads lose 1-3 % here whenever L2 still holds lines that other
// kernels left with the default policy (they are never displaced by evict-first traffic), while
// default-policy loads run at the same speed in either state.  Stores stay evict-first.
#define QB_LDG_MOD ""
#include <type_traits>

#include "common.cuh"
#include "host_common.h"
#include "softmax.h"

namespace qb {

// RAW (16-bit inputs): the row stays packed in registers (twice the bytes in flight per register)
// and is unpacked by each pass; the exponential is then evaluated twice per element (once for the
// sum, once for the output).  Otherwise the exponentials are kept as fp32 registers.
// TPR != 0 fixes the threads per row at compile time, which turns the chunk strides into
// immediate offsets (the kernel is close to instruction-issue-bound: +4.6 % at N = 4096, bf16).
template <int DT, int VEC, int K, bool RAW, int TPR = 0>
__global__ void __launch_bounds__(RAW ? (K * VEC > 64 ? 256 : (K * VEC > 32 ? 512 : 1024))
                                      : (K * VEC > 16 ? 512 : 1024))
softmax_fwd_kernel(const SoftmaxParams p) {
  __shared__ ReduceScratch scratch;
  const int ptpr = TPR ? TPR : p.tpr;
  const RowGeom g = make_geom(ptpr, p.cluster_n);
  reduce_init(scratch, p.cluster_n);
  if (p.cluster_n > 1) cluster_arrive();
  const int col0 = static_cast<int>(g.crank) * p.cols_per_cta;
  const int ncols = min(p.cols_per_cta, p.N - col0);
  const int colbase = col0 + g.t * VEC;
  const int cstride = ptpr * VEC;
  const int nchunks = ncols > 0 ? ncols / VEC : 0;
  const int nk = nchunks > g.t ? min(K, (nchunks - g.t + ptpr - 1) / ptpr) : 0;
  const int64_t tile_stride = gridDim.x / p.cluster_n;
  int rit = 0;
  bool first = true;
  for (int64_t tile = blockIdx.x / p.cluster_n; tile < p.num_tiles; tile += tile_stride) {
    const int64_t row = tile * p.rows_per_cta + g.r;
    const bool row_ok = row < p.M;
    const int nkr = row_ok ? nk : 0;  // chunks of this thread that exist in this tile
    constexpr int kRawWords = RawWords<DT, VEC>::value;
    uint32_t rx[K][kRawWords];
    const int esz_i = elem_bytes<DT>(p.dt0), esz_o = elem_bytes<DT>(p.dto);
    const char* xp = reinterpret_cast<const char*>(p.in0) + (row * p.ld0 + colbase) * esz_i;
    char* op = reinterpret_cast<char*>(p.out) + (row * p.ldo + colbase) * esz_o;
    const int step_i = cstride * esz_i, step_o = cstride * esz_o;
    load_row_raw<DT, VEC, K>(rx, xp, step_i, p.dt0, nkr);

    // Thread-local maximum over the chunks that exist.
    float m_t = neg_inf();
    float v[RAW ? 1 : K][VEC];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if constexpr (RAW) {
        if (k < nkr) m_t = fmaxf(m_t, packed_max16<DT, VEC>(rx[k]));
      } else {
        unpack_chunk<DT, VEC>(v[k], rx[k], p.dt0);
        if (k < nkr) {
#pragma unroll
          for (int i = 0; i < VEC; ++i) m_t = fmaxf(m_t, v[k][i]);
        } else {
#pragma unroll
          for (int i = 0; i < VEC; ++i) v[k][i] = neg_inf();
        }
      }
    }
    // e_i = exp(x_i - m_t) = 2^(x_i * log2e + off.hi) * 2^off.lo
    const ExpOffset off = exp_offset(m_t);
    float s_t = 0.0f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if constexpr (RAW) {
        if (k < nkr) {
          float t[VEC];
          unpack_chunk<DT, VEC>(t, rx[k], p.dt0);
#pragma unroll
          for (int i = 0; i < VEC; ++i) s_t += fast_exp2(fmaf(t[i], kLog2e, off.hi));
        }
      } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          v[k][i] = fast_exp2(fmaf(v[k][i], kLog2e, off.hi));
          s_t += v[k][i];
        }
      }
    }
    const float corr = fast_exp2(off.lo);
    s_t *= corr;
    if (first && p.cluster_n > 1) cluster_wait();
    first = false;
    const float2 ms = row_reduce<MaxSumExpOp>(make_float2(m_t, s_t), g, scratch, 0, rit, p.timeouts);
    ++rit;
    // y_i = e_i * exp(m_t - m) / s
    const float scale = (m_t == neg_inf())
                            ? 0.0f
                            : corr * fast_exp2((m_t - ms.x) * kLog2e) * (1.0f / ms.y);
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if (k < nkr) {
        float y[VEC];
        if constexpr (RAW) {
          float t[VEC];
          forget_values(rx[k]);
          unpack_chunk<DT, VEC>(t, rx[k], p.dt0);
#pragma unroll
          for (int i = 0; i < VEC; ++i) y[i] = fast_exp2(fmaf(t[i], kLog2e, off.hi)) * scale;
        } else {
#pragma unroll
          for (int i = 0; i < VEC; ++i) y[i] = v[k][i] * scale;
        }
        store_chunk_p<DT, VEC>(op + k * step_o, y, p.dto);
      }
    }
  }
  if (first && p.cluster_n > 1) cluster_wait();
}

// dx = y * (dy - sum(dy * y)).  dy and y stay packed in registers; they are unpacked once for the
// dot product and once more for the output.
template <int DT, int VEC, int K>
__global__ void __launch_bounds__((K * VEC > 16) ? 512 : 1024)
softmax_bwd_kernel(const SoftmaxParams p) {
  __shared__ ReduceScratch scratch;
  const RowGeom g = make_geom(p.tpr, p.cluster_n);
  reduce_init(scratch, p.cluster_n);
  if (p.cluster_n > 1) cluster_arrive();
  const int col0 = static_cast<int>(g.crank) * p.cols_per_cta;
  const int ncols = min(p.cols_per_cta, p.N - col0);
  const int colbase = col0 + g.t * VEC;
  const int cstride = p.tpr * VEC;
  const int nchunks = ncols > 0 ? ncols / VEC : 0;
  const int nk = nchunks > g.t ? min(K, (nchunks - g.t + p.tpr - 1) / p.tpr) : 0;
  const int64_t tile_stride = gridDim.x / p.cluster_n;
  int rit = 0;
  bool first = true;
  for (int64_t tile = blockIdx.x / p.cluster_n; tile < p.num_tiles; tile += tile_stride) {
    const int64_t row = tile * p.rows_per_cta + g.r;
    const bool row_ok = row < p.M;
    uint32_t rdy[K][RawWords<DT, VEC>::value];
    uint32_t ry[K][RawWords<DT, VEC>::value];
    const int nkr = row_ok ? nk : 0;
    const int esz0 = elem_bytes<DT>(p.dt0), esz1 = elem_bytes<DT>(p.dt1), esz_o = elem_bytes<DT>(p.dto);
    const char* dyp = reinterpret_cast<const char*>(p.in0) + (row * p.ld0 + colbase) * esz0;
    const char* yp = reinterpret_cast<const char*>(p.in1) + (row * p.ld1 + colbase) * esz1;
    char* op = reinterpret_cast<char*>(p.out) + (row * p.ldo + colbase) * esz_o;
    const int step0 = cstride * esz0, step1 = cstride * esz1, step_o = cstride * esz_o;
    // (Predicated loads also for rows that fill the tile: the split into an unpredicated and a
    // predicated form, which helps the forward, cost this kernel 10-14 % on rows of three chunks
    // per thread -- N = 3072, 6144, 12288 -- and gained nothing on full tiles.)
#pragma unroll
    for (int k = 0; k < K; ++k) load_chunk_raw_p<DT, VEC>(rdy[k], dyp + k * step0, p.dt0, k < nkr);
#pragma unroll
    for (int k = 0; k < K; ++k) load_chunk_raw_p<DT, VEC>(ry[k], yp + k * step1, p.dt1, k < nkr);
    float dot = 0.0f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float dy[VEC], y[VEC];
      unpack_chunk<DT, VEC>(dy, rdy[k], p.dt0);
      unpack_chunk<DT, VEC>(y, ry[k], p.dt1);
#pragma unroll
      for (int i = 0; i < VEC; ++i) dot = fmaf(dy[i], y[i], dot);
    }
    if (first && p.cluster_n > 1) cluster_wait();
    first = false;
    dot = row_reduce<SumOp>(make_float2(dot, 0.f), g, scratch, 0, rit, p.timeouts).x;
    ++rit;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float dy[VEC], y[VEC], dx[VEC];
      forget_values(rdy[k]);
      forget_values(ry[k]);
      unpack_chunk<DT, VEC>(dy, rdy[k], p.dt0);
      unpack_chunk<DT, VEC>(y, ry[k], p.dt1);
#pragma unroll
      for (int i = 0; i < VEC; ++i) dx[i] = y[i] * (dy[i] - dot);
      if (k < nkr) store_chunk_p<DT, VEC>(op + k * step_o, dx, p.dto);
    }
  }
  if (first && p.cluster_n > 1) cluster_wait();
}

// ---------------------------------------------------------------------------------------------
// Long rows: two streamed passes per row with the row parked in L2 between them
// ---------------------------------------------------------------------------------------------
// A row that does not fit one CTA's registers is not split over a cluster here.  One CTA owns the
// whole row and reads it twice: pass 1 streams it for the row statistic (online (max, sum-exp)
// forward, sum(dy * y) backward) with an L2 evict-last policy, pass 2 streams it again -- in
// reverse order, most recently touched lines first -- with an evict-first policy, computes the
// result and writes it.  The grid is sized so that the rows in flight (resident CTAs x row bytes)
// cover only a fraction of L2, which makes the second read an L2 hit: DRAM still sees one read
// and one write per element, and no CTA ever waits on another one.
// DT is one of the three concrete dtypes (all tensors share it, full 16-byte chunks); T threads
// share one row (T == blockDim.x); U = chunks in flight per thread and input.  A row is walked in
// blocks of T * U chunks; all blocks but possibly the last are full and take straight-line code
// with compile-time address offsets.
template <int DT, bool BWD, int U, int T>
__global__ void __launch_bounds__(T, (T >= 1024) ? 1 : (1024 / T)) softmax_stream_kernel(const SoftmaxParams p) {
  static_assert(DT == QB_F32 || DT == QB_F16 || DT == QB_BF16, "concrete dtype required");
  constexpr int VEC = DT == QB_F32 ? 4 : 8;
  constexpr int kStep = T * 16;           // bytes between a thread's chunks u and u + 1
  constexpr int kBlockBytes = U * kStep;  // bytes of one block of the row
  __shared__ ReduceScratch scratch;
  const RowGeom g = make_geom(T, 1);
  const int nchunks = p.N / VEC;
  const int nfull = nchunks / (T * U);           // full blocks
  const bool tail = nfull * (T * U) < nchunks;   // one more, partial, block
  const int tail_c0 = nfull * (T * U) + g.t;     // this thread's first chunk of the partial block
  const uint64_t keep = l2_policy((p.flags & 4) ? 2 : 0);
  const uint64_t drop = l2_policy((p.flags & 8) ? 2 : 1);
  int rit = 0;
  for (int64_t row = blockIdx.x; row < p.M; row += gridDim.x) {
    const char* in0 = reinterpret_cast<const char*>(p.in0) + (row * p.ld0 * (16 / VEC) + g.t * 16);
    const char* in1 = BWD ? reinterpret_cast<const char*>(p.in1) + (row * p.ld1 * (16 / VEC) + g.t * 16)
                          : nullptr;
    char* out = reinterpret_cast<char*>(p.out) + (row * p.ldo * (16 / VEC) + g.t * 16);

    float m = neg_inf(), s = 0.0f;  // forward: running max and sum 2^(x*log2e + off.hi)
    ExpOffset off = exp_offset(m);
    float sv[BWD ? VEC : 1];        // backward: partial sums of dy * y
#pragma unroll
    for (int i = 0; i < (BWD ? VEC : 1); ++i) sv[i] = 0.0f;

    // The block's chunks live at row scope: the block pass 1 reads last is the one pass 2 starts
    // with, so it is kept in registers across the row reduction instead of being read again
    // (rows of two blocks, e.g. N = 131072 with 1024 threads: a quarter less L2 traffic and one
    // load latency less per row).
    uint32_t r0[U][4];
    uint32_t r1[BWD ? U : 1][4];

    // ---- pass 1 ----
    auto pass1 = [&](auto full_tag, const char* q0, const char* q1, int c0) {
      constexpr bool FULL = decltype(full_tag)::value;
#pragma unroll
      for (int u = 0; u < U; ++u) ldg16_hint<!FULL>(r0[u], q0 + u * kStep, c0 + u * T < nchunks, keep);
      if constexpr (BWD) {
#pragma unroll
        for (int u = 0; u < U; ++u) ldg16_hint<!FULL>(r1[u], q1 + u * kStep, c0 + u * T < nchunks, keep);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          float v[VEC], y[VEC];
          unpack_chunk<DT, VEC>(v, r0[u], DT);
          unpack_chunk<DT, VEC>(y, r1[u], DT);  // padding chunks are zeros: they add nothing
          if constexpr (BWD) vfma<VEC>(sv, v, y, sv);
        }
      } else {
        // maximum of the whole block first, one re-basing of the partial sum per block
        float cm = neg_inf();
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (FULL || c0 + u * T < nchunks) {
            if constexpr (DT == QB_F32) {
#pragma unroll
              for (int i = 0; i < VEC; ++i) cm = fmaxf(cm, __uint_as_float(r0[u][i]));
            } else {
              cm = fmaxf(cm, packed_max16<DT, VEC>(r0[u]));
            }
          }
        }
        if (cm > m) {
          const ExpOffset nw = exp_offset(cm);
          s *= fast_exp2(nw.hi - off.hi);
          m = cm;
          off = nw;
        }
        // (One scalar accumulator: packed partial sums need eight more registers, which this
        // kernel, held to 64 by its 1024-thread CTAs, does not have -- measured 3 % slower.)
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (FULL || c0 + u * T < nchunks) {
            float v[VEC];
            unpack_chunk<DT, VEC>(v, r0[u], DT);
#pragma unroll
            for (int i = 0; i < VEC; ++i) s += fast_exp2(fmaf(v[i], kLog2e, off.hi));
          }
        }
      }
    };
    {
      const char* q0 = in0;
      const char* q1 = in1;
      for (int b = 0; b < nfull; ++b, q0 += kBlockBytes, q1 += kBlockBytes)
        pass1(std::true_type{}, q0, q1, 0);
      if (tail) pass1(std::false_type{}, q0, q1, tail_c0);
    }

    float scale = 0.0f, dot = 0.0f;
    if constexpr (BWD) {
      dot = row_reduce<SumOp>(make_float2(hsum<(BWD ? VEC : 1)>(sv), 0.f), g, scratch, 0, rit, p.timeouts).x;
    } else {
      s *= fast_exp2(off.lo);
      const float2 ms = row_reduce<MaxSumExpOp>(make_float2(m, s), g, scratch, 0, rit, p.timeouts);
      off = exp_offset(ms.x);
      scale = ms.x == neg_inf() ? 0.0f : fast_exp2(off.lo) * (1.0f / ms.y);
    }
    ++rit;

    // ---- pass 2: newest lines first ----
    auto pass2 = [&](auto full_tag, auto resident_tag, const char* q0, const char* q1, char* qo, int c0) {
      constexpr bool FULL = decltype(full_tag)::value;
      constexpr bool RESIDENT = decltype(resident_tag)::value;  // the chunks are still in r0 / r1
      if constexpr (!RESIDENT) {
#pragma unroll
        for (int u = 0; u < U; ++u) ldg16_hint<!FULL>(r0[u], q0 + u * kStep, c0 + u * T < nchunks, drop);
        if constexpr (BWD) {
#pragma unroll
          for (int u = 0; u < U; ++u) ldg16_hint<!FULL>(r1[u], q1 + u * kStep, c0 + u * T < nchunks, drop);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float v[VEC], o[VEC];
        unpack_chunk<DT, VEC>(v, r0[u], DT);
        if constexpr (BWD) {
          float y[VEC];
          unpack_chunk<DT, VEC>(y, r1[u], DT);
#pragma unroll
          for (int i = 0; i < VEC; ++i) o[i] = y[i] * (v[i] - dot);
        } else {
          // (Folding the normaliser into the exponent and packed fp32x2 arithmetic were tried
          // here: 2 % slower at N = 65536 / 131072, the kernel sits at its 64-register limit.)
#pragma unroll
          for (int i = 0; i < VEC; ++i) o[i] = fast_exp2(fmaf(v[i], kLog2e, off.hi)) * scale;
        }
        if (FULL || c0 + u * T < nchunks) store_chunk_p<DT, VEC>(qo + u * kStep, o, DT);
      }
    };
    {
      const int64_t end = static_cast<int64_t>(nfull) * kBlockBytes;
      if (tail) pass2(std::false_type{}, std::true_type{}, in0 + end, in1 + end, out + end, tail_c0);
      const char* q0 = in0 + end;
      const char* q1 = in1 + end;
      char* qo = out + end;
      for (int b = nfull - 1; b >= 0; --b) {
        q0 -= kBlockBytes;
        q1 -= kBlockBytes;
        qo -= kBlockBytes;
        if (!tail && b == nfull - 1) pass2(std::true_type{}, std::true_type{}, q0, q1, qo, 0);
        else pass2(std::true_type{}, std::false_type{}, q0, q1, qo, 0);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
template <int DT, int VEC, bool BWD, bool RAW>
static int launch_softmax_v(const SoftmaxParams& p, int K, dim3 grid, int threads,
                            cudaStream_t st) {
  const char* name = BWD ? "softmax_bwd" : "softmax_fwd";
#define QB_CASE(KK)                                                                              \
  case KK:                                                                                       \
    if constexpr (BWD)                                                                           \
      return launch_kernel(softmax_bwd_kernel<DT, VEC, KK>, grid, threads, 0, p.cluster_n, st,   \
                           p, name);                                                             \
    else                                                                                         \
      return launch_kernel(softmax_fwd_kernel<DT, VEC, KK, RAW>, grid, threads, 0, p.cluster_n,  \
                           st, p, name);
  switch (K) {
    QB_CASE(1)
    QB_CASE(2)
    QB_CASE(4)
    QB_CASE(8)
    case 16:
      if constexpr (VEC <= 4 || (RAW && !BWD)) {
        if constexpr (BWD)
          return launch_kernel(softmax_bwd_kernel<DT, VEC, 16>, grid, threads, 0, p.cluster_n, st,
                               p, name);
        else {
          // compile-time geometry for the shapes the heuristics pick at N = 4096, 8192 and 16384
          if constexpr (RAW) {
            if (p.tpr == 32) return launch_kernel(softmax_fwd_kernel<DT, VEC, 16, RAW, 32>, grid, threads,
                                                  0, p.cluster_n, st, p, name);
            if (p.tpr == 64) return launch_kernel(softmax_fwd_kernel<DT, VEC, 16, RAW, 64>, grid, threads,
                                                  0, p.cluster_n, st, p, name);
            if (p.tpr == 128) return launch_kernel(softmax_fwd_kernel<DT, VEC, 16, RAW, 128>, grid,
                                                   threads, 0, p.cluster_n, st, p, name);
          }
          return launch_kernel(softmax_fwd_kernel<DT, VEC, 16, RAW>, grid, threads, 0,
                               p.cluster_n, st, p, name);
        }
      }
  }
#undef QB_CASE
  return set_error(QB_ERR_UNSUPPORTED, "%s: no kernel for %d chunks of %d per thread", name, K, VEC);
}

template <int DT, bool BWD, int U, int T>
static int launch_softmax_stream_t(const SoftmaxParams& p, const qb_launch_cfg& cfg,
                                   const DeviceFacts* dev, cudaStream_t st) {
  auto kernel = softmax_stream_kernel<DT, BWD, U, T>;
  const int occ = cached_occupancy(reinterpret_cast<const void*>(kernel), T, 0);
  // Rows in flight (one per resident CTA) are what has to stay in L2 between the two passes.
  int64_t ctas = static_cast<int64_t>(dev->sm_count) * (occ > 0 ? occ : 1);
  if (cfg.max_ctas > 0) ctas = cfg.max_ctas;
  if (ctas > p.M) ctas = p.M;
  dim3 grid(static_cast<unsigned>(ctas), 1, 1);
  // Pass 1 marks the row evict-last only while all rows in flight fit comfortably in L2; beyond
  // that (measured: 76 MB in flight) the plain policy keeps more of the second pass in L2.
  SoftmaxParams q = p;
  const int64_t in_flight = ctas * static_cast<int64_t>(p.N) * host_dtype_bytes(p.dt0) * (BWD ? 2 : 1);
  if (in_flight > (48LL << 20)) q.flags |= 4;
  return launch_kernel(kernel, grid, T, 0, 1, st, q,
                       BWD ? "softmax_bwd (streamed)" : "softmax_fwd (streamed)");
}

template <int DT, bool BWD, int U>
static int launch_softmax_stream_u(const SoftmaxParams& p, const qb_launch_cfg& cfg,
                                   const DeviceFacts* dev, int threads, cudaStream_t st) {
  switch (threads) {
    case 256: return launch_softmax_stream_t<DT, BWD, U, 256>(p, cfg, dev, st);
    case 512: return launch_softmax_stream_t<DT, BWD, U, 512>(p, cfg, dev, st);
    case 1024: return launch_softmax_stream_t<DT, BWD, U, 1024>(p, cfg, dev, st);
    default:
      return set_error(QB_ERR_INVALID, "softmax (streamed): num_threads must be 256, 512 or 1024");
  }
}

template <bool BWD>
static int launch_softmax_stream(SoftmaxParams& p, const qb_launch_cfg& cfg, const DeviceFacts* dev,
                                 cudaStream_t st) {
  // Measured on B200 (bf16, 1 GiB per tensor): the best CTA size walks a row in about two blocks
  // of its chunks in flight -- forward 256 threads up to 48K elements, 512 up to 96K, else 1024
  // (8 chunks in flight per thread); backward 512 threads up to 48K elements, else 1024 (2 chunks
  // per thread and input).
  const int64_t row_bytes = static_cast<int64_t>(p.N) * host_dtype_bytes(p.dt0);
  int threads = cfg.num_threads;
  if (threads <= 0) {
    if (BWD) threads = row_bytes <= (96 << 10) ? 512 : 1024;
    else threads = row_bytes <= (96 << 10) ? 256 : (row_bytes <= (192 << 10) ? 512 : 1024);
  }
  p.tpr = threads;
  p.rows_per_cta = 1;
  p.cluster_n = 1;
  p.cols_per_cta = p.N;
  p.num_tiles = p.M;
  p.flags = cfg.flags;
  // cfg.stages selects the chunks in flight per thread and input (default 8 forward, 2 backward).
  const int u = cfg.stages > 0 ? cfg.stages : (BWD ? 2 : 8);
#define QB_STREAM(DT)                                                                         \
  if (u == (BWD ? 4 : 8)) return launch_softmax_stream_u<DT, BWD, (BWD ? 4 : 8)>(p, cfg, dev, threads, st); \
  if (u == (BWD ? 2 : 4)) return launch_softmax_stream_u<DT, BWD, (BWD ? 2 : 4)>(p, cfg, dev, threads, st); \
  return set_error(QB_ERR_INVALID, "softmax (streamed): unsupported chunks in flight %d", u);
  switch (p.dt0) {
    case QB_BF16: QB_STREAM(QB_BF16)
    case QB_F16: QB_STREAM(QB_F16)
    default: QB_STREAM(QB_F32)
  }
#undef QB_STREAM
}

template <bool BWD>
static int softmax_dispatch(SoftmaxParams& p, bool uniform, int vec, const qb_launch_cfg& cfg,
                            cudaStream_t st) {
  const DeviceFacts* dev = current_device_facts();
  if (dev == nullptr) return QB_ERR_CUDA;
  RowPlan plan;
  // Packed 16-bit rows (forward RAW mode, backward always): 128 elements per thread up to 256
  // threads, 64 up to 512, 32 at 1024; fp32-held rows half of that.
  const bool raw = uniform && p.dt0 != QB_F32 && !(cfg.flags & 1);
  const bool packed = raw || (BWD && uniform);
  ElemCaps caps = packed ? ElemCaps{BWD ? 64 : 128, 64, BWD ? 16 : 32, BWD ? 8 : 16}
                         : (uniform ? ElemCaps{64, 64, 16} : ElemCaps{32, 32, 16});
  const int64_t pref = (packed && !BWD) ? 32768 : ((uniform && vec == 8) ? 16384 : 8192);
  // Rows too long for one CTA's registers take the streamed two-pass kernel with the row parked
  // in L2, unless the caller pinned a cluster size, set flag bit 1, or there are fewer rows than
  // SMs (then splitting rows over clusters keeps more SMs busy).  The question "too long for one
  // CTA" is put to the heuristic plan, whatever thread count the caller may have pinned.
  const int k_target = BWD ? 4 : (packed ? 16 : 8);
  const char* opname = BWD ? "softmax_bwd" : "softmax_fwd";
  if (uniform && cfg.cluster_n == 0 && !(cfg.flags & 2) && p.M >= dev->sm_count) {
    RowPlan probe;
    const int rc = plan_rows(opname, p.N, vec, caps, pref, k_target, 128, qb_launch_cfg{}, &probe);
    if (rc != QB_OK || probe.cluster_n > 1) {
      clear_error();
      // Long rows.  Backward: the row is split over a thread-block cluster whose CTAs keep their
      // slices in registers and exchange the row's dot product through distributed shared memory
      // (softmax_cluster.cu; faster than the alternatives at every row length measured, see
      // there); rows beyond its capacity fall through to the shared-memory ring and then to the
      // two-pass L2 kernel.  Forward: the two-pass L2 kernel (bf16, 2 GiB per tensor, N = 65536 /
      // 131072: 5.86 / 5.70 TB/s against 5.42 / 5.21 for the cluster kernel and 5.63 / 5.63 for
      // the ring: the forward pass is bound by instruction issue and the special function unit,
      // and the L2 kernel pays its per-row latency once per 128 KB instead of once per 32 KB).
      // Flags pick one kernel explicitly.
      const bool only_stream = (cfg.flags & QB_FLAG_NO_RING) != 0;
      const bool want_cluster = !only_stream && ((cfg.flags & QB_FLAG_CLUSTER_REGS) || (BWD && !(cfg.flags & QB_FLAG_RING)));
      const bool want_ring = !only_stream && (BWD || (cfg.flags & QB_FLAG_RING));
      if (want_cluster) {
        const int rc2 = launch_softmax_cluster<BWD>(p, cfg, dev, st);
        if (rc2 != QB_ERR_UNSUPPORTED) return rc2;
        clear_error();
      }
      if (want_ring) {
        const int rr = launch_softmax_ring<BWD>(p, cfg, dev, st);
        if (rr != QB_ERR_UNSUPPORTED) return rr;
        clear_error();
      }
      return launch_softmax_stream<BWD>(p, cfg, dev, st);
    }
  }
  if (int rc = plan_rows(opname, p.N, vec, caps, pref, k_target, 128, cfg, &plan)) return rc;
  p.tpr = plan.tpr;
  p.rows_per_cta = plan.rows_per_cta;
  p.cluster_n = plan.cluster_n;
  if (p.cluster_n > 1) {
    p.timeouts = ring_timeout_counter();
    if (p.timeouts == nullptr) return QB_ERR_CUDA;
  }
  p.cols_per_cta = plan.cols_per_cta;
  p.num_tiles = ceil_div(p.M, p.rows_per_cta);
  // Rows owned by a single CTA: one tile per CTA (nothing to amortise, and the hardware block
  // scheduler balances best).  Rows split over a cluster: a bounded grid whose clusters walk over
  // rows, so that the cluster start-up handshake is paid once per CTA.
  const int64_t max_ctas =
      cfg.max_ctas > 0 ? cfg.max_ctas
                       : (plan.cluster_n == 1 ? (int64_t)0x7fffffff
                                              : (int64_t)dev->sm_count * (2048 / plan.threads) * 2);
  int64_t clusters = p.num_tiles;
  if (clusters > max_ctas / plan.cluster_n) clusters = max_ctas / plan.cluster_n;
  if (clusters < 1) clusters = 1;
  dim3 grid(static_cast<unsigned>(clusters * plan.cluster_n), 1, 1);
  if (uniform) {
    switch (p.dt0) {
      case QB_BF16:
        if (raw || BWD) return launch_softmax_v<QB_BF16, 8, BWD, true>(p, plan.K, grid, plan.threads, st);
        return launch_softmax_v<QB_BF16, 8, BWD, false>(p, plan.K, grid, plan.threads, st);
      case QB_F16:
        if (raw || BWD) return launch_softmax_v<QB_F16, 8, BWD, true>(p, plan.K, grid, plan.threads, st);
        return launch_softmax_v<QB_F16, 8, BWD, false>(p, plan.K, grid, plan.threads, st);
      default: return launch_softmax_v<QB_F32, 4, BWD, false>(p, plan.K, grid, plan.threads, st);
    }
  }
  switch (vec) {
    case 8: return launch_softmax_v<kDynDT, 8, BWD, false>(p, plan.K, grid, plan.threads, st);
    case 4: return launch_softmax_v<kDynDT, 4, BWD, false>(p, plan.K, grid, plan.threads, st);
    case 2: return launch_softmax_v<kDynDT, 2, BWD, false>(p, plan.K, grid, plan.threads, st);
    default: return launch_softmax_v<kDynDT, 1, BWD, false>(p, plan.K, grid, plan.threads, st);
  }
}

}  // namespace qb

using namespace qb;

extern "C" int qb_softmax_fwd(const qb_softmax_fwd_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "softmax_fwd: null argument block");
  const qb_softmax_fwd_args& a = *args;
  if (a.x == nullptr || a.out == nullptr)
    return set_error(QB_ERR_INVALID, "softmax_fwd: x and out are required");
  if (a.M < 0 || a.N <= 0 || a.N > (1 << 30))
    return set_error(QB_ERR_INVALID, "softmax_fwd: bad sizes M=%lld N=%lld", (long long)a.M,
                     (long long)a.N);
  if (!is_float_dtype(a.x_dtype) || !is_float_dtype(a.out_dtype))
    return set_error(QB_ERR_INVALID, "softmax_fwd: unsupported dtype code");
  if (a.M == 0) return QB_OK;
  VecWidth vw;
  vw.limit_elems(a.N);
  vw.add_tensor(a.x, a.x_dtype, a.x_row_stride);
  vw.add_tensor(a.out, a.out_dtype, a.out_row_stride);
  const bool uniform = a.x_dtype == a.out_dtype && vw.vec == 16 / host_dtype_bytes(a.x_dtype);
  SoftmaxParams p = {};
  p.in0 = a.x;
  p.out = a.out;
  p.M = a.M;
  p.N = static_cast<int>(a.N);
  p.ld0 = a.x_row_stride;
  p.ldo = a.out_row_stride;
  p.dt0 = a.x_dtype;
  p.dto = a.out_dtype;
  return softmax_dispatch<false>(p, uniform, vw.vec, a.cfg, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int qb_softmax_bwd(const qb_softmax_bwd_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "softmax_bwd: null argument block");
  const qb_softmax_bwd_args& a = *args;
  if (a.dy == nullptr || a.y == nullptr || a.dx == nullptr)
    return set_error(QB_ERR_INVALID, "softmax_bwd: dy, y and dx are required");
  if (a.M < 0 || a.N <= 0 || a.N > (1 << 30))
    return set_error(QB_ERR_INVALID, "softmax_bwd: bad sizes M=%lld N=%lld", (long long)a.M,
                     (long long)a.N);
  if (!is_float_dtype(a.dy_dtype) || !is_float_dtype(a.y_dtype) || !is_float_dtype(a.dx_dtype))
    return set_error(QB_ERR_INVALID, "softmax_bwd: unsupported dtype code");
  if (a.M == 0) return QB_OK;
  VecWidth vw;
  vw.limit_elems(a.N);
  vw.add_tensor(a.dy, a.dy_dtype, a.dy_row_stride);
  vw.add_tensor(a.y, a.y_dtype, a.y_row_stride);
  vw.add_tensor(a.dx, a.dx_dtype, a.dx_row_stride);
  const bool uniform = a.dy_dtype == a.y_dtype && a.dy_dtype == a.dx_dtype &&
                       vw.vec == 16 / host_dtype_bytes(a.dy_dtype);
  SoftmaxParams p = {};
  p.in0 = a.dy;
  p.in1 = a.y;
  p.out = a.dx;
  p.M = a.M;
  p.N = static_cast<int>(a.N);
  p.ld0 = a.dy_row_stride;
  p.ld1 = a.y_row_stride;
  p.ldo = a.dx_row_stride;
  p.dt0 = a.dy_dtype;
  p.dt1 = a.y_dtype;
  p.dto = a.dx_dtype;
  return softmax_dispatch<true>(p, uniform, vw.vec, a.cfg, reinterpret_cast<cudaStream_t>(stream));
}
