// Softmax forward / backward for long rows on sm_100a: the row is split over the CTAs of a
// thread-block cluster, every CTA keeps its slice packed in registers, HBM sees exactly one read
// and one write per element, and the per-row statistic travels through distributed shared memory.
//
// This is the layout the reference uses for N >= 32K (quack/softmax.py:53-64 picks the cluster
// size, quack/reduce.py:70-118,227-324 exchanges the partials through mbarriers), with a software
// pipeline over rows added: a persistent cluster owns rows j, j + C, j + 2C, ... and the loads of
// the next row (NB == 2) or the next two rows (NB == 3) are already in flight while the current
// row is reduced, exchanged and written.  With NB == 3 the cluster barrier is split: the partials
// of row j + 1 are pushed and the barrier is arrived at before row j is written, and only waited
// for after it, so the barrier's latency is covered by the stores of the previous row.
//
// The partials travel by st.async: a store into a peer's shared memory that counts its bytes on an
// mbarrier of that peer (the reference's store_shared_remote + mbarrier pair, quack/utils.py:27-58).
// barrier.cluster is not used inside the row loop: its arrive has release semantics, which makes
// the thread wait for its global loads in flight -- exactly the prefetched rows (measured: 4.0
// instead of 5.9 TB/s at N = 65536).  Every mbarrier wait is bounded (bounded_mbar_wait): a wait that
// does not succeed within about a second sets the CTA's abort flag and bumps the device-side counter the
// host reads, and the kernel runs to its end instead of hanging.
// Loads in this file use the default L2 policy instead of the evict-first "streaming" one:
// measured on B200, evict-first loads lose 1-3 % here whenever L2 still holds lines that other
// kernels left with the default policy (they are never displaced by evict-first traffic), while
// default-policy loads run at the same speed in either state.  Stores stay evict-first.
#define QB_LDG_MOD ""
#include <type_traits>

#include "ring.cuh"
#include "host_common.h"
#include "softmax.h"

namespace qb {

struct __align__(16) ClusterScratch {
  unsigned long long bar[2];        // counts the bytes of the cluster's partials, by row parity
  float2 cta_part[2][kMaxCluster];  // one partial per CTA of the cluster, by row parity
  float2 warp_part[2][kMaxWarps];   // per-warp partials of this CTA, by row parity
  int abort;                        // set once a wait of this CTA timed out
};

struct SoftmaxClusterParams {
  SoftmaxParams s;
  unsigned int* timeouts;  // device counter of timed-out waits
};

// DT: concrete dtype shared by all tensors (full 16-byte chunks).  K chunks per thread and input,
// T threads per CTA, NB register buffers (rows in flight + 1).
// Registers: the row buffers take NIN * NB * K * 4 of them; up to 32 leave room for everything
// else within 64 registers per thread (2048 threads per SM), more than that asks for 128.
template <bool BWD, int K, int T, int NB>
struct ClusterOcc {
  static constexpr int kDataRegs = (BWD ? 2 : 1) * NB * K * 4;
  static constexpr int kRegs = kDataRegs <= 32 ? 64 : 128;
  static constexpr int kMinBlocks = (65536 / (T * kRegs)) > 0 ? (65536 / (T * kRegs)) : 1;
};

template <int DT, bool BWD, int K, int T, int NB>
__global__ void __launch_bounds__(T, ClusterOcc<BWD, K, T, NB>::kMinBlocks)
softmax_cluster_kernel(const SoftmaxClusterParams q) {
  const SoftmaxParams& p = q.s;
  static_assert(DT == QB_F32 || DT == QB_F16 || DT == QB_BF16, "concrete dtype required");
  static_assert(NB >= 1 && NB <= 3, "one to three row buffers");
  constexpr int VEC = DT == QB_F32 ? 4 : 8;
  constexpr int ESZ = 16 / VEC;
  constexpr int W = T / 32;
  constexpr int kStep = T * 16;  // bytes between a thread's chunks k and k + 1
  __shared__ ClusterScratch sc;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cn = p.cluster_n;
  const uint32_t crank = cn > 1 ? cluster_cta_rank() : 0u;
  if (tid == 0) {
    mbar_init(smem_u32(&sc.bar[0]), 1);
    mbar_init(smem_u32(&sc.bar[1]), 1);
    sc.abort = 0;
    mbar_fence_init();
  }
  __syncthreads();
  // all CTAs of the cluster are running, with their barriers set up, before the first remote store
  if (cn > 1) cluster_arrive();

  const int col0 = static_cast<int>(crank) * p.cols_per_cta;
  const int ncols = max(0, min(p.cols_per_cta, p.N - col0));
  uint32_t okmask = 0;  // bit k: chunk k of this thread lies inside the row
#pragma unroll
  for (int k = 0; k < K; ++k)
    if ((k * T + tid) * VEC < ncols) okmask |= 1u << k;
  const bool all_ok = okmask == (1u << K) - 1u;

  const int64_t nclusters = gridDim.x / cn;
  const int64_t cid = blockIdx.x / cn;
  const int64_t nrows = cid < p.M ? (p.M - cid + nclusters - 1) / nclusters : 0;  // rows of this cluster
  const int64_t thread_off = static_cast<int64_t>(col0) + tid * VEC;

  uint32_t b0[NB][K][4];
  uint32_t b1[BWD ? NB : 1][K][4];

  auto issue = [&](uint32_t (&d0)[K][4], uint32_t (&d1)[K][4], int64_t j) {
    const bool live = j < nrows;
    const int64_t row = live ? cid + j * nclusters : 0;
    const char* s0 = reinterpret_cast<const char*>(p.in0) + (row * p.ld0 + thread_off) * ESZ;
#pragma unroll
    for (int k = 0; k < K; ++k) ldg_stream<16>(d0[k], s0 + k * kStep, live && ((okmask >> k) & 1u));
    if constexpr (BWD) {
      const char* s1 = reinterpret_cast<const char*>(p.in1) + (row * p.ld1 + thread_off) * ESZ;
#pragma unroll
      for (int k = 0; k < K; ++k) ldg_stream<16>(d1[k], s1 + k * kStep, live && ((okmask >> k) & 1u));
    }
  };

  // ---- per-row statistic of this thread's chunks, reduced over the CTA; result in warp 0 ----
  // forward: (max, sum of exp(x - max)); backward: (sum of dy * y, -)
  auto local_stat = [&](uint32_t (&d0)[K][4], uint32_t (&d1)[K][4], int par) -> float2 {
    float2 v;
    if constexpr (BWD) {
      float sv[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) sv[i] = 0.0f;
#pragma unroll
      for (int k = 0; k < K; ++k) {  // chunks outside the row were loaded as zeros
        float dy[VEC], y[VEC];
        unpack_chunk<DT, VEC>(dy, d0[k], DT);
        unpack_chunk<DT, VEC>(y, d1[k], DT);
        vfma<VEC>(sv, dy, y, sv);
      }
      float s = hsum<VEC>(sv);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      v = make_float2(s, 0.0f);
    } else {
      float m = neg_inf();
#pragma unroll
      for (int k = 0; k < K; ++k) {
        if (all_ok || ((okmask >> k) & 1u)) {
          if constexpr (DT == QB_F32) {
#pragma unroll
            for (int i = 0; i < VEC; ++i) m = fmaxf(m, __uint_as_float(d0[k][i]));
          } else {
            m = fmaxf(m, packed_max16<DT, VEC>(d0[k]));
          }
        }
      }
      // the warp's maximum first, so that the sum needs no re-basing afterwards
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const ExpOffset off = exp_offset(m);
      float sv[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) sv[i] = 0.0f;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        if (all_ok || ((okmask >> k) & 1u)) {
          float x[VEC], e[VEC];
          unpack_chunk<DT, VEC>(x, d0[k], DT);
          vfma_ss<VEC>(e, x, kLog2e, off.hi);
#pragma unroll
          for (int i = 0; i < VEC; ++i) e[i] = fast_exp2(e[i]);
          vadd<VEC>(sv, sv, e);
        }
      }
      float s = hsum<VEC>(sv) * fast_exp2(off.lo);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      v = make_float2(m, s);
    }
    // across the warps of the CTA: warp 0 folds the W partials
    if (lane == 0) sc.warp_part[par][warp] = v;
    __syncthreads();
    if (warp == 0) {
      float2 q = lane < W ? sc.warp_part[par][lane] : (BWD ? make_float2(0.f, 0.f) : make_float2(neg_inf(), 0.f));
      if constexpr (BWD) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) q.x += __shfl_xor_sync(0xffffffffu, q.x, o);
      } else {
        float mm = q.x;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
        float s = q.x == neg_inf() ? 0.0f : q.y * fast_exp2((q.x - mm) * kLog2e);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        q = make_float2(mm, s);
      }
      v = q;
    }
    return v;  // meaningful in warp 0
  };
  // warp 0 sends the CTA's partial to slot [crank] of every CTA of the cluster; row j uses the
  // buffers and the barrier of parity j & 1, in phase (j >> 1) & 1
  auto push = [&](float2 v, int par) {
    if (warp == 0) {
      if (cn > 1) {
        if (lane == 0) mbar_arrive_expect_tx_relaxed(smem_u32(&sc.bar[par]), static_cast<uint32_t>(cn) * 8u);
        if (lane < cn)
          st_async_f2(map_to_cta(smem_u32(&sc.cta_part[par][crank]), lane), v,
                      map_to_cta(smem_u32(&sc.bar[par]), lane));
      } else if (lane == 0) {
        sc.cta_part[par][0] = v;
      }
    }
    if (cn == 1) __syncthreads();
  };
  auto wait_row = [&](int64_t j) {
    if (cn > 1)
      bounded_mbar_wait(&sc.abort, smem_u32(&sc.bar[j & 1]), static_cast<uint32_t>(j >> 1) & 1u, q.timeouts);
  };
  // every thread folds the cluster's partials in rank order (bit-identical in all CTAs)
  auto fold = [&](int par) -> float2 {
    const float2* buf = sc.cta_part[par];
    if constexpr (BWD) {
      float s = buf[0].x;
      for (int c = 1; c < cn; ++c) s += buf[c].x;
      return make_float2(s, 0.0f);
    } else {
      float m = buf[0].x;
      for (int c = 1; c < cn; ++c) m = fmaxf(m, buf[c].x);
      float s = 0.0f;
      for (int c = 0; c < cn; ++c) {
        const float2 q = buf[c];
        s += q.x == neg_inf() ? 0.0f : q.y * fast_exp2((q.x - m) * kLog2e);
      }
      return make_float2(m, s);
    }
  };
  // result pass of one row
  auto result = [&](uint32_t (&d0)[K][4], uint32_t (&d1)[K][4], int64_t j, float2 st) {
    const int64_t row = cid + j * nclusters;
    char* o = reinterpret_cast<char*>(p.out) + (row * p.ldo + thread_off) * ESZ;
    float roff = 0.0f, rscale = 1.0f;
    if constexpr (!BWD) {
      const ExpOffset ro = exp_offset(st.x);
      if constexpr (DT == QB_F32) {
        roff = ro.hi;  // y = 2^(x*log2e + hi) * (2^lo / sum)
        rscale = st.x == neg_inf() ? 0.0f : fast_exp2(ro.lo) * (1.0f / st.y);
      } else {
        // 16-bit outputs: the normaliser goes into the exponent
        roff = st.x == neg_inf() ? 0.0f : ro.hi + (ro.lo - __log2f(st.y));
      }
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float a[VEC], r[VEC];
      forget_values(d0[k]);
      unpack_chunk<DT, VEC>(a, d0[k], DT);
      if constexpr (BWD) {
        float y[VEC];
        forget_values(d1[k]);
        unpack_chunk<DT, VEC>(y, d1[k], DT);
#pragma unroll
        for (int i = 0; i < VEC; ++i) r[i] = y[i] * (a[i] - st.x);
      } else {
        float e[VEC];
        vfma_ss<VEC>(e, a, kLog2e, roff);
        if constexpr (DT == QB_F32) {
#pragma unroll
          for (int i = 0; i < VEC; ++i) r[i] = fast_exp2(e[i]) * rscale;
        } else {
#pragma unroll
          for (int i = 0; i < VEC; ++i) r[i] = fast_exp2(e[i]);
        }
      }
      if (all_ok || ((okmask >> k) & 1u)) store_chunk_p<DT, VEC>(o + k * kStep, r, DT);
    }
  };

  // ---- prologue: the first NB - 1 rows are requested ----
#pragma unroll
  for (int s = 0; s < NB - 1; ++s) issue(b0[s], b1[BWD ? s : 0], s);
  if (cn > 1) cluster_wait();  // matches the arrive at the top
  if constexpr (NB == 3) {
    if (nrows > 0) {
      const float2 v = local_stat(b0[0], b1[0], 0);
      push(v, 0);
    }
  }
  for (int64_t j0 = 0; j0 < nrows; j0 += NB) {
#pragma unroll
    for (int s = 0; s < NB; ++s) {
      const int64_t j = j0 + s;
      if (j >= nrows) break;
      const int par = static_cast<int>(j & 1);
      issue(b0[(s + NB - 1) % NB], b1[BWD ? (s + NB - 1) % NB : 0], j + NB - 1);
      if constexpr (NB <= 2) {
        const float2 v = local_stat(b0[s], b1[BWD ? s : 0], par);
        push(v, par);
        wait_row(j);
        result(b0[s], b1[BWD ? s : 0], j, fold(par));
      } else {
        // statistic of row j + 1 before row j is written; its exchange completes meanwhile
        const bool more = j + 1 < nrows;
        float2 v = make_float2(0.f, 0.f);
        if (more) v = local_stat(b0[(s + 1) % NB], b1[BWD ? (s + 1) % NB : 0], par ^ 1);
        wait_row(j);
        const float2 st = fold(par);
        if (more) push(v, par ^ 1);
        result(b0[s], b1[BWD ? s : 0], j, st);
      }
    }
  }
}

template <int DT, bool BWD, int K, int T, int NB>
static int launch_softmax_cluster_t(SoftmaxParams p, const qb_launch_cfg& cfg, const DeviceFacts* dev,
                                    cudaStream_t st) {
  constexpr int VEC = DT == QB_F32 ? 4 : 8;
  const int64_t cap = static_cast<int64_t>(K) * T * VEC;  // elements one CTA holds
  // the smallest cluster that holds the row; any size up to 16 is allowed (beyond 8 the launch
  // opts in to non-portable cluster sizes), e.g. 5 CTAs for N = 40960
  int cn = static_cast<int>(ceil_div(static_cast<int64_t>(p.N), cap));
  if (cn > kMaxCluster) return QB_ERR_UNSUPPORTED;
  if (cfg.cluster_n > 0) {
    if (cfg.cluster_n < cn || cfg.cluster_n > kMaxCluster) return QB_ERR_UNSUPPORTED;
    cn = cfg.cluster_n;
  }
  // equal slices, whole chunks
  const int64_t chunks = p.N / VEC;
  const int64_t cpc = ceil_div(chunks, cn);
  p.cluster_n = cn;
  p.cols_per_cta = static_cast<int>(cpc * VEC);
  p.tpr = T;
  p.rows_per_cta = 1;
  p.num_tiles = p.M;
  unsigned int* timeouts = ring_timeout_counter();
  if (timeouts == nullptr) return QB_ERR_CUDA;
  SoftmaxClusterParams q;
  auto kernel = softmax_cluster_kernel<DT, BWD, K, T, NB>;
  int clusters = resident_clusters(kernel, T, 0, cn, dev->sm_count);
  if (cfg.max_ctas > 0) clusters = cfg.max_ctas / cn;
  if (clusters > p.M) clusters = static_cast<int>(p.M);
  if (clusters < 1) clusters = 1;
  dim3 grid(static_cast<unsigned>(clusters * cn), 1, 1);
  q.s = p;
  q.timeouts = timeouts;
  return launch_kernel(kernel, grid, T, 0, cn, st, q,
                       BWD ? "softmax_bwd (cluster)" : "softmax_fwd (cluster)");
}

template <int DT, bool BWD>
static int launch_softmax_cluster_dt(const SoftmaxParams& p, const qb_launch_cfg& cfg,
                                     const DeviceFacts* dev, cudaStream_t st) {
  // cfg.num_threads = threads per CTA (512 / 1024), cfg.stages = chunks per thread and input,
  // cfg.ctas_per_sm = register buffers (2 / 3).
  // Defaults, measured on B200 (bf16, 2 GiB per tensor, GB/s of algorithmic bytes, backward):
  // CTAs of 128 threads x 8 chunks without prefetch, four or more per SM, 6.7 / 6.7 / 6.3 TB/s at
  // N = 32768 / 65536 / 131072 (two-pass L2 kernel 6.3 / 6.5 / 5.7, shared-memory ring 6.1 / 5.7 /
  // 5.3); rows that need more than 16 such CTAs take CTAs of 1024 threads x 2 chunks with the
  // next row prefetched (N = 262144: 5.6 against 4.7 / 4.9).  Forward: 128 x 16.
  constexpr int VEC = DT == QB_F32 ? 4 : 8;
  int t = cfg.num_threads, k = cfg.stages, nb = cfg.ctas_per_sm;
  if (t <= 0 && k <= 0 && nb <= 0) {
    if (BWD) {
      if (static_cast<int64_t>(p.N) <= static_cast<int64_t>(kMaxCluster) * 128 * 8 * VEC) { t = 128; k = 8; nb = 1; }
      else { t = 1024; k = 2; nb = 2; }
    } else {
      t = 128; k = 16; nb = 1;
    }
  }
#define QB_CL_CASE(TT, KK, NN) \
  if (t == TT && k == KK && nb == NN) return launch_softmax_cluster_t<DT, BWD, KK, TT, NN>(p, cfg, dev, st);
  if constexpr (BWD) {
    QB_CL_CASE(128, 8, 1)
    QB_CL_CASE(256, 4, 1)
    QB_CL_CASE(512, 2, 2)
    QB_CL_CASE(1024, 2, 2)
    QB_CL_CASE(256, 4, 2)
    QB_CL_CASE(512, 4, 2)
    QB_CL_CASE(256, 2, 3)
    QB_CL_CASE(512, 2, 3)
    QB_CL_CASE(256, 4, 3)
  } else {
    QB_CL_CASE(128, 16, 1)
    QB_CL_CASE(256, 8, 1)
    QB_CL_CASE(128, 8, 2)
    QB_CL_CASE(512, 4, 1)
    QB_CL_CASE(512, 4, 2)
    QB_CL_CASE(1024, 4, 2)
    QB_CL_CASE(1024, 2, 2)
    QB_CL_CASE(512, 2, 3)
    QB_CL_CASE(512, 4, 3)
    QB_CL_CASE(256, 8, 2)
    QB_CL_CASE(256, 4, 3)
    QB_CL_CASE(256, 8, 3)
  }
#undef QB_CL_CASE
  return QB_ERR_UNSUPPORTED;
}

template <bool BWD>
int launch_softmax_cluster(const SoftmaxParams& p, const qb_launch_cfg& cfg, const DeviceFacts* dev,
                           cudaStream_t st) {
  switch (p.dt0) {
    case QB_BF16: return launch_softmax_cluster_dt<QB_BF16, BWD>(p, cfg, dev, st);
    case QB_F16: return launch_softmax_cluster_dt<QB_F16, BWD>(p, cfg, dev, st);
    default: return launch_softmax_cluster_dt<QB_F32, BWD>(p, cfg, dev, st);
  }
}

template int launch_softmax_cluster<false>(const SoftmaxParams&, const qb_launch_cfg&,
                                           const DeviceFacts*, cudaStream_t);
template int launch_softmax_cluster<true>(const SoftmaxParams&, const qb_launch_cfg&,
                                          const DeviceFacts*, cudaStream_t);

}  // namespace qb
