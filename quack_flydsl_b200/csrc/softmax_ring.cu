// Softmax forward / backward for long rows on sm_100a: the row is staged in shared memory by bulk
// asynchronous copies (ring.cuh) and read from there twice, so HBM sees one read and one write
// per element.  Rows longer than one CTA's shared memory are split over a thread-block cluster
// whose CTAs exchange their (max, sum-exp) / dot-product partials through distributed shared
// memory and mbarriers.
//
// Follows quack/softmax.py:87-176 (forward, online (max, sum-exp) pair) and :275-353 (backward);
// the cluster sizes the reference picks for N >= 32K (quack/softmax.py:53-64) are replaced by
// "smallest cluster whose slice fits the ring".
#include <type_traits>

#include "ring.cuh"
#include "softmax.h"

namespace qb {

struct SoftmaxRingParams {
  SoftmaxParams s;
  RingGeom g;
};

// DT: concrete dtype shared by all tensors (full 16-byte chunks).  T consumer threads plus one
// producer warp; every consumer thread owns U 16-byte chunks of each slot.
template <int DT, bool BWD, int T, int U>
__global__ void __launch_bounds__(T + 32, 1) softmax_ring_kernel(const SoftmaxRingParams q) {
  static_assert(DT == QB_F32 || DT == QB_F16 || DT == QB_BF16, "concrete dtype required");
  constexpr int VEC = DT == QB_F32 ? 4 : 8;
  constexpr int ESZ = 16 / VEC;
  constexpr int CH = T * U * 16;  // bytes of one input in one slot
  constexpr int NIN = BWD ? 2 : 1;
  constexpr int W = T / 32;
  extern __shared__ __align__(128) unsigned char smem[];
  RingCtl* ctl = reinterpret_cast<RingCtl*>(smem);
  unsigned char* ring = smem + kRingCtlBytes;
  const SoftmaxParams& p = q.s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ns = q.g.ns;
  const int cluster_n = q.g.cluster_n;
  const uint32_t crank = cluster_n > 1 ? cluster_cta_rank() : 0u;
  ring_init(ctl, ns, W, cluster_n);

  const int col0 = static_cast<int>(crank) * q.g.cols_per_cta;
  const int ncols = max(0, min(q.g.cols_per_cta, p.N - col0));
  const int SB = ncols * ESZ;           // bytes of this CTA's slice of a row, per input
  const int R = (SB + CH - 1) / CH;     // slots per row
  const int64_t nclusters = gridDim.x / cluster_n;
  const int64_t cid = blockIdx.x / cluster_n;

  if (warp == W) {
    // ---------------- producer warp (lane 0 issues) ----------------
    RingPos pos{0, 0u};
    int lap = 0;
    const uint64_t pol = l2_policy((p.flags & 4) ? 2 : ((p.flags & 8) ? 0 : 1));
    for (int64_t row = cid; row < p.M; row += nclusters) {
      const char* s0 = reinterpret_cast<const char*>(p.in0) + (row * p.ld0 + col0) * ESZ;
      const char* s1 = BWD ? reinterpret_cast<const char*>(p.in1) + (row * p.ld1 + col0) * ESZ : nullptr;
      for (int c = 0; c < R; ++c) {
        if (lane == 0) {
          ring_wait(ctl, smem_u32(&ctl->empty[pos.slot]), pos.phase ^ 1u, q.g.timeouts);
          const uint32_t bytes = static_cast<uint32_t>(min(CH, SB - c * CH));
          const uint32_t full = smem_u32(&ctl->full[pos.slot]);
          const uint32_t dst = smem_u32(ring + static_cast<size_t>(pos.slot) * (NIN * CH));
          mbar_arrive_expect_tx(full, bytes * NIN);
          bulk_g2s(dst, s0 + static_cast<size_t>(c) * CH, bytes, full, pol);
          if constexpr (BWD) bulk_g2s(dst + CH, s1 + static_cast<size_t>(c) * CH, bytes, full, pol);
        }
        __syncwarp();
        if (++pos.slot == ns) { pos.slot = 0; pos.phase ^= 1u; ++lap; }
      }
    }
    // Shared memory must outlive the copies in flight: wait (bounded, also when aborting) for the
    // last copy issued into every slot.
    if (lane == 0) {
      for (int s = 0; s < ns; ++s) {
        const bool this_lap = s < pos.slot;
        if (!this_lap && lap == 0) continue;  // never used
        const uint32_t ph = this_lap ? pos.phase : (pos.phase ^ 1u);
        const uint32_t bar = smem_u32(&ctl->full[s]);
        const unsigned long long t0 = global_timer_ns();
        while (!mbar_try_wait(bar, ph) && global_timer_ns() - t0 < kRingTimeoutNs) {}
      }
    }
    __syncwarp();
  } else {
    // ---------------- consumer warps ----------------
    // Per row: statistic pass over the row's slots, row reduction, result pass (which releases
    // the slots).  (Interleaving the result pass of row i with the statistic pass of row i + 1
    // was measured slower on B200, forward and backward.)
    RingPos p1{0, 0u};  // next slot of the statistic pass
    RingPos p2{0, 0u};  // next slot of the result pass
    // forward: running max m and VEC partial sums of 2^(x*log2e + off.hi) (packed fp32x2 adds);
    // backward: VEC partial sums of dy * y
    float m = neg_inf();
    float sv[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) sv[i] = 0.0f;
    ExpOffset off = exp_offset(m);

    // Statistic pass over one slot.  FULL: every chunk of the slot holds data.
    auto stat_slot = [&](auto full_tag, int c) {
      constexpr bool FULL = decltype(full_tag)::value;
      ring_wait(ctl, smem_u32(&ctl->full[p1.slot]), p1.phase, q.g.timeouts);
      const unsigned char* base = ring + static_cast<size_t>(p1.slot) * (NIN * CH) + tid * 16;
      const int valid = FULL ? CH : SB - c * CH;  // bytes of this slot that hold data
      uint32_t r0[U][4];
      uint32_t r1[BWD ? U : 1][4];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (FULL || (tid + u * T) * 16 < valid) {
          lds_raw<16>(r0[u], base + u * (T * 16));
          if constexpr (BWD) lds_raw<16>(r1[u], base + CH + u * (T * 16));
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) { r0[u][i] = 0u; if constexpr (BWD) r1[u][i] = 0u; }
        }
      }
      if constexpr (BWD) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          float v[VEC], y[VEC];
          unpack_chunk<DT, VEC>(v, r0[u], DT);
          unpack_chunk<DT, VEC>(y, r1[u], DT);  // padding chunks are zeros: they add nothing
          vfma<VEC>(sv, v, y, sv);
        }
      } else {
        // maximum of the thread's chunks of this slot first, one re-basing of the partial sum
        float cm = neg_inf();
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (FULL || (tid + u * T) * 16 < valid) {
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
          const float f = fast_exp2(nw.hi - off.hi);
#pragma unroll
          for (int i = 0; i < VEC; ++i) sv[i] *= f;
          m = cm;
          off = nw;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (FULL || (tid + u * T) * 16 < valid) {
            float v[VEC], e[VEC];
            unpack_chunk<DT, VEC>(v, r0[u], DT);
            vfma_ss<VEC>(e, v, kLog2e, off.hi);
#pragma unroll
            for (int i = 0; i < VEC; ++i) e[i] = fast_exp2(e[i]);
            vadd<VEC>(sv, sv, e);
          }
        }
      }
      p1.advance(ns);
    };
    // Row reduction; leaves what the result pass needs in (roff, rscale) / rdot.
    float roff = 0.0f, rscale = 0.0f, rdot = 0.0f;
    auto finish_stat = [&](int row_it) {
      if constexpr (BWD) {
        const float2 w = warp_reduce_f2<SumOp>(make_float2(hsum<VEC>(sv), 0.f));
        rdot = ring_row_reduce<SumOp>(w, ctl, row_it, warp, lane, W, cluster_n, crank, q.g.timeouts).x;
      } else {
        const float s = hsum<VEC>(sv) * fast_exp2(off.lo);
        const float2 w = warp_reduce_f2<MaxSumExpOp>(make_float2(m, s));
        const float2 ms = ring_row_reduce<MaxSumExpOp>(w, ctl, row_it, warp, lane, W, cluster_n, crank,
                                                       q.g.timeouts);
        const ExpOffset ro = exp_offset(ms.x);
        if constexpr (DT == QB_F32) {
          // y = 2^(x*log2e + hi) * (2^lo / sum)
          roff = ro.hi;
          rscale = ms.x == neg_inf() ? 0.0f : fast_exp2(ro.lo) * (1.0f / ms.y);
        } else {
          // 16-bit outputs: the normaliser goes into the exponent, y = 2^(x*log2e + hi + lo - log2(sum))
          roff = ms.x == neg_inf() ? 0.0f : ro.hi + (ro.lo - __log2f(ms.y));
          rscale = 1.0f;
        }
        m = neg_inf();
        off = exp_offset(m);
      }
#pragma unroll
      for (int i = 0; i < VEC; ++i) sv[i] = 0.0f;
    };
    // Result pass over one slot of the row whose output starts at `out`.
    auto result_slot = [&](auto full_tag, int c, char* out) {
      constexpr bool FULL = decltype(full_tag)::value;
      const unsigned char* base = ring + static_cast<size_t>(p2.slot) * (NIN * CH) + tid * 16;
      const int valid = FULL ? CH : SB - c * CH;
      uint32_t r0[U][4];
      uint32_t r1[BWD ? U : 1][4];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (FULL || (tid + u * T) * 16 < valid) {
          lds_raw<16>(r0[u], base + u * (T * 16));
          if constexpr (BWD) lds_raw<16>(r1[u], base + CH + u * (T * 16));
        }
      }
      char* o = out + static_cast<size_t>(c) * CH;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (FULL || (tid + u * T) * 16 < valid) {
          float v[VEC], r[VEC];
          unpack_chunk<DT, VEC>(v, r0[u], DT);
          if constexpr (BWD) {
            float y[VEC];
            unpack_chunk<DT, VEC>(y, r1[u], DT);
#pragma unroll
            for (int i = 0; i < VEC; ++i) r[i] = y[i] * (v[i] - rdot);
          } else {
            float e[VEC];
            vfma_ss<VEC>(e, v, kLog2e, roff);
            if constexpr (DT == QB_F32) {
#pragma unroll
              for (int i = 0; i < VEC; ++i) r[i] = fast_exp2(e[i]) * rscale;
            } else {
#pragma unroll
              for (int i = 0; i < VEC; ++i) r[i] = fast_exp2(e[i]);
            }
          }
          store_chunk_p<DT, VEC>(o + u * (T * 16), r, DT);
        }
      }
      // The slot may be refilled once every lane has read its chunks.  The stores above consumed
      // the loaded registers, so the reads have completed; no fence (it would wait for the stores).
      __syncwarp();
      if (lane == 0) mbar_arrive_relaxed(smem_u32(&ctl->empty[p2.slot]));
      p2.advance(ns);
    };
    auto slot_is_full = [&](int c) { return SB - c * CH >= CH; };

    int it = 0;
    auto stat_row = [&](int row_it) {
      for (int c = 0; c < R; ++c) {
        if (slot_is_full(c)) stat_slot(std::true_type{}, c); else stat_slot(std::false_type{}, c);
      }
      finish_stat(row_it);
    };
    for (int64_t row = cid; row < p.M; row += nclusters, ++it) {
      char* out = reinterpret_cast<char*>(p.out) + (row * p.ldo + col0) * ESZ + tid * 16;
      stat_row(it);
      for (int c = 0; c < R; ++c) {
        if (slot_is_full(c)) result_slot(std::true_type{}, c, out);
        else result_slot(std::false_type{}, c, out);
      }
    }
  }
  // No CTA of a cluster may exit while a peer can still store into its shared memory.
  if (cluster_n > 1) cluster_sync_all();
}

template <int DT, bool BWD, int T, int U>
static int launch_softmax_ring_t(const SoftmaxParams& p, const qb_launch_cfg& cfg,
                                 const DeviceFacts* dev, cudaStream_t st) {
  constexpr int VEC = DT == QB_F32 ? 4 : 8;
  constexpr int CH = T * U * 16;
  RingPlan plan;
  // Shared memory per CTA: everything the SM has, or half of it when two CTAs are to share an SM
  // (their passes then overlap: one CTA computes on its resident row while the other one stores).
  const int per_sm = cfg.ctas_per_sm == 2 ? 2 : 1;
  const int smem_cap = per_sm == 1 ? dev->max_smem_optin : (dev->max_smem_optin + 1024) / 2 - 1024;
  if (!plan_ring(p.N, VEC, 16 / VEC, BWD ? 2 : 1, CH, kRingCtlBytes, smem_cap, kRingMaxSlots,
                 cfg.cluster_n, &plan))
    return QB_ERR_UNSUPPORTED;
  if ((T / 32) * plan.cluster_n > kRingMaxPartials) return QB_ERR_UNSUPPORTED;
  unsigned int* timeouts = ring_timeout_counter();
  if (timeouts == nullptr) return QB_ERR_CUDA;
  auto kernel = softmax_ring_kernel<DT, BWD, T, U>;
  int clusters = resident_clusters(kernel, T + 32, plan.smem, plan.cluster_n, dev->sm_count);
  if (cfg.max_ctas > 0) clusters = cfg.max_ctas / plan.cluster_n;
  if (clusters > p.M) clusters = static_cast<int>(p.M);
  if (clusters < 1) clusters = 1;
  SoftmaxRingParams q;
  q.s = p;
  q.g.ns = plan.ns;
  q.g.cluster_n = plan.cluster_n;
  q.g.cols_per_cta = plan.cols_per_cta;
  q.g.timeouts = timeouts;
  dim3 grid(static_cast<unsigned>(clusters * plan.cluster_n), 1, 1);
  return launch_kernel(kernel, grid, T + 32, plan.smem, plan.cluster_n, st, q,
                       BWD ? "softmax_bwd (ring)" : "softmax_fwd (ring)");
}

template <int DT, bool BWD>
static int launch_softmax_ring_dt(const SoftmaxParams& p, const qb_launch_cfg& cfg,
                                  const DeviceFacts* dev, cudaStream_t st) {
  // cfg.num_threads = consumer threads (256 / 512 / 768), cfg.stages = 16-byte chunks per thread
  // and slot.  Measured on B200 (bf16, 2 and 4 GiB per tensor): backward 256 consumers x 4 chunks
  // (16 KB per input and slot: 6.65 TB/s at N = 65536, 6.08 at 131072, against 6.54 / 5.87 with
  // 512 x 2), forward 512 x 4 (32 KB slots: the forward pass is bound by instruction issue and
  // the special function unit, and larger slots amortise the per-slot bookkeeping).
  const int t = cfg.num_threads > 0 ? cfg.num_threads : (BWD ? 256 : 512);
  const int u = cfg.stages > 0 ? cfg.stages : 4;
#define QB_RING_CASE(TT, UU) \
  if (t == TT && u == UU) return launch_softmax_ring_t<DT, BWD, TT, UU>(p, cfg, dev, st);
  QB_RING_CASE(256, 4)
  QB_RING_CASE(256, 8)
  QB_RING_CASE(512, 2)
  QB_RING_CASE(512, 4)
  QB_RING_CASE(768, 2)
#undef QB_RING_CASE
  return QB_ERR_UNSUPPORTED;
}

template <bool BWD>
int launch_softmax_ring(const SoftmaxParams& p, const qb_launch_cfg& cfg, const DeviceFacts* dev,
                        cudaStream_t st) {
  switch (p.dt0) {
    case QB_BF16: return launch_softmax_ring_dt<QB_BF16, BWD>(p, cfg, dev, st);
    case QB_F16: return launch_softmax_ring_dt<QB_F16, BWD>(p, cfg, dev, st);
    default: return launch_softmax_ring_dt<QB_F32, BWD>(p, cfg, dev, st);
  }
}

template int launch_softmax_ring<false>(const SoftmaxParams&, const qb_launch_cfg&,
                                        const DeviceFacts*, cudaStream_t);
template int launch_softmax_ring<true>(const SoftmaxParams&, const qb_launch_cfg&,
                                       const DeviceFacts*, cudaStream_t);

}  // namespace qb
