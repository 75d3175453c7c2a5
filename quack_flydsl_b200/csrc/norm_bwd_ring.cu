// RMSNorm / LayerNorm backward, stage 1, with the rows staged by bulk asynchronous copies.
//
// Same mathematics and the same [P, N] partial-sum contract as norm_bwd_kernel (norm_bwd.cu,
// after quack/rmsnorm.py:723-1205); what differs is how the data reach the arithmetic.  Thread 0
// streams x and dout into a shared-memory ring with cp.async.bulk (the TMA path the reference's
// Blackwell heuristic turns on for this kernel, quack/rmsnorm_config.py:226-240,
// quack/rmsnorm.py:686-693,931-950); all 256 or 512 threads of the CTA share each row, so a
// thread owns few columns and the fp32 weight / dw / db registers shrink from 192 to 72 per
// thread.  The price of wide rows -- a reduction over 8 or 16 warps per row -- is one mbarrier
// exchange across the warps and, for long rows, across the CTAs of a cluster.
//
// Measured against norm_bwd_kernel on B200 (bf16, 512 MiB per tensor, LayerNorm / RMSNorm GB/s):
// N = 4096: 5417 / 5612 against 5687 / 6166; N = 8192: 5135 / 5492 against 5773 / 6235;
// N = 16384: 4972 / 5201 against 5416 / 5994 -- the cp.async kernel keeps those.  Rows of three
// 16-byte chunks per thread, which leave a quarter of the cp.async kernel's power-of-two tile
// empty, go the other way: N = 6144: 4939 / 4732 against 4293 / 4819; N = 12288: 4413 / 5203
// against 4091 / 4648; N = 24576: 4223 / 4940 against 3349 / 3687.  This kernel therefore serves
// exactly those: one dtype for x / dout / dx with full 16-byte chunks, no residual-gradient
// streams, H == 1, N = cluster_n * 3 * T * (16 / element size) with T = 512 (cluster_n 1, 2, 4)
// or T = 256 (cluster_n 1).
#include <type_traits>

#include "ring.cuh"
#include "norm_bwd_ring.h"

namespace qb {

struct NormBwdRingParams {
  qb_norm_bwd_args a;
  RingGeom g;
  int64_t num_steps;  // ceil(M / RPS)
};


// Sums NV values (NV a power of two <= 32) over the lanes of a warp with NV - 1 + log2(32 / NV)
// shuffles instead of 5 * NV: while more than one value is left, the two halves of the warp each
// keep one half of the values.  Afterwards every lane holds the warp total of value
// (lane >> (5 - log2 NV)) in v[0].
template <int NV>
__device__ __forceinline__ void warp_sum_values(float (&v)[NV], int lane) {
  int off = 16;
#pragma unroll
  for (int n = NV / 2; n >= 1; n >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < n; ++i) {
      const float send = upper ? v[i] : v[i + n];
      const float keep = upper ? v[i + n] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
    off >>= 1;
  }
  for (; off > 0; off >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
}

template <int NV>
struct Log2 {
  static constexpr int value = 1 + Log2<NV / 2>::value;
};
template <>
struct Log2<1> {
  static constexpr int value = 0;
};

// Reduces NV per-thread values over all consumer threads of all CTAs of the cluster.  Every
// thread returns the same totals (fixed summation order, bit-identical in every CTA).  buf is
// [2][W * cluster_n][NV] floats of shared memory, `it` the number of reductions done so far.
template <int NV>
__device__ __forceinline__ void ring_sum_values(float (&v)[NV], float* buf, RingCtl* ctl, int it,
                                                int warp, int lane, int consumer_warps,
                                                int cluster_n, uint32_t crank,
                                                unsigned int* timeouts) {
  constexpr int LG = Log2<NV>::value;
  warp_sum_values<NV>(v, lane);
  const int par = it & 1;
  const uint32_t phase = static_cast<uint32_t>(it >> 1) & 1u;
  const int nparts = consumer_warps * cluster_n;
  float* mine = buf + static_cast<size_t>(par) * nparts * NV;
  const uint32_t bar_local = smem_u32(&ctl->red[par]);
  // lane l publishes value (l % NV) to CTA c0 + l / NV
  const float val = __shfl_sync(0xffffffffu, v[0], (lane & (NV - 1)) << (5 - LG));
  const uint32_t dst_local =
      smem_u32(mine + (static_cast<int>(crank) * consumer_warps + warp) * NV + (lane & (NV - 1)));
  for (int c0 = 0; c0 < cluster_n; c0 += 32 / NV) {
    const int c = c0 + lane / NV;
    if (c < cluster_n)
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(map_to_cta(dst_local, c)), "f"(val)
                   : "memory");
  }
  __syncwarp();
  if (lane < cluster_n) mbar_arrive_remote(map_to_cta(bar_local, lane));
  ring_wait<true>(ctl, bar_local, phase, timeouts);
  // lane l folds value (l % NV) over the partials l / NV, l / NV + 32 / NV, ...
  float acc = 0.0f;
  for (int p = lane / NV; p < nparts; p += 32 / NV) acc += mine[p * NV + (lane & (NV - 1))];
#pragma unroll
  for (int o = 16; o >= NV; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] = __shfl_sync(0xffffffffu, acc, i);
}

// DT: dtype of x / dout / dx.  KC: 16-byte chunks per thread and row.  RPS: rows per ring slot.
// T: threads per CTA, all of which share each row (512: one CTA per SM; 256: two).
template <int DT, int KC, int RPS, bool LN, bool DB, int T>
__global__ void __launch_bounds__(T, 512 / T) norm_bwd_ring_kernel(const NormBwdRingParams q) {
  static_assert(DT == QB_F32 || DT == QB_F16 || DT == QB_BF16, "concrete dtype required");
  constexpr int W = T / 32;
  constexpr int VEC = DT == QB_F32 ? 4 : 8;
  constexpr int ESZ = 16 / VEC;
  constexpr int ROWB = KC * T * 16;       // bytes of this CTA's slice of one row
  constexpr int SLOTB = 2 * RPS * ROWB;   // x rows, then dout rows
  constexpr int NV = RPS * (LN ? 2 : 1);  // partial sums per slot
  extern __shared__ __align__(128) unsigned char smem[];
  RingCtl* ctl = reinterpret_cast<RingCtl*>(smem);
  const qb_norm_bwd_args& a = q.a;
  const int ns = q.g.ns;
  const int cluster_n = q.g.cluster_n;
  unsigned char* ring = smem + kRingCtlBytes;
  float* redbuf = reinterpret_cast<float*>(ring + static_cast<size_t>(ns) * SLOTB);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t crank = cluster_n > 1 ? cluster_cta_rank() : 0u;
  ring_init(ctl, ns, W, cluster_n);

  const int N = static_cast<int>(a.N);
  const int col0 = static_cast<int>(crank) * (KC * T * VEC);
  const int64_t nclusters = gridDim.x / cluster_n;
  const int64_t cid = blockIdx.x / cluster_n;

  // No producer warp here: after the row reduction of a step every warp has read the step's slot
  // (the reduction's barrier comes after the reads), so thread 0 refills that slot right there,
  // NS steps ahead, without any "slot is free" signalling -- and the CTA stays at 16 warps, which
  // leaves 128 registers per thread.
  auto issue_step = [&](int64_t step, int slot) {
    const int64_t row0 = step * RPS;
    const int nrows = static_cast<int>(min(static_cast<int64_t>(RPS), a.M - row0));
    const uint32_t full = smem_u32(&ctl->full[slot]);
    const uint32_t dst = smem_u32(ring + static_cast<size_t>(slot) * SLOTB);
    const uint64_t pol = l2_policy(1);  // evict first: every byte is read once
    mbar_arrive_expect_tx(full, static_cast<uint32_t>(nrows) * 2u * ROWB);
    for (int r = 0; r < nrows; ++r) {
      const char* xs = reinterpret_cast<const char*>(a.x) + ((row0 + r) * a.x_row_stride + col0) * ESZ;
      const char* ds = reinterpret_cast<const char*>(a.dout) + ((row0 + r) * a.dout_row_stride + col0) * ESZ;
      bulk_g2s(dst + r * ROWB, xs, ROWB, full, pol);
      bulk_g2s(dst + (RPS + r) * ROWB, ds, ROWB, full, pol);
    }
  };
  if (tid == 0) {
    for (int s = 0; s < ns; ++s) {
      const int64_t step = cid + s * nclusters;
      if (step < q.num_steps) issue_step(step, s);
    }
  }
  {
    // ---------------- consumer warps ----------------
    const float inv_n = 1.0f / static_cast<float>(N);
    float w[KC][VEC];
#pragma unroll
    for (int j = 0; j < KC; ++j) {
      if (a.weight != nullptr) {
        load_chunk<kDynDT, VEC, false>(w[j], a.weight, col0 + (j * T + tid) * VEC, a.weight_dtype);
#pragma unroll
        for (int i = 0; i < VEC; ++i) w[j][i] += a.weight_offset;
      } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) w[j][i] = 1.0f;
      }
    }
    float dw[KC][VEC];
    float db[DB ? KC : 1][VEC];
#pragma unroll
    for (int j = 0; j < KC; ++j)
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        dw[j][i] = 0.0f;
        if constexpr (DB) db[j][i] = 0.0f;
      }

    RingPos pos{0, 0u};
    int it = 0;
    for (int64_t step = cid; step < q.num_steps; step += nclusters, ++it) {
      const int64_t row0 = step * RPS;
      float rstd[RPS], nmean[RPS];
      bool ok[RPS];
#pragma unroll
      for (int r = 0; r < RPS; ++r) {
        ok[r] = row0 + r < a.M;
        rstd[r] = ok[r] ? a.rstd[row0 + r] : 0.0f;
        nmean[r] = (LN && ok[r]) ? -a.mean[row0 + r] : 0.0f;
      }
      ring_wait(ctl, smem_u32(&ctl->full[pos.slot]), pos.phase, q.g.timeouts);
      const unsigned char* base = ring + static_cast<size_t>(pos.slot) * SLOTB + tid * 16;
      uint32_t rx[RPS][KC][4], rdy[RPS][KC][4];
#pragma unroll
      for (int r = 0; r < RPS; ++r) {
#pragma unroll
        for (int j = 0; j < KC; ++j) {
          if (ok[r]) {
            lds_raw<16>(rx[r][j], base + r * ROWB + j * (T * 16));
            lds_raw<16>(rdy[r][j], base + (RPS + r) * ROWB + j * (T * 16));
          } else {  // a row past the end: zeros add nothing to any sum
#pragma unroll
            for (int i = 0; i < 4; ++i) { rx[r][j][i] = 0u; rdy[r][j][i] = 0u; }
          }
        }
      }
      // ---- pass 1: S1 = sum(xc * t), S2 = sum(t) with xc = x - mean, t = dout * w ----
      float part[NV];
#pragma unroll
      for (int r = 0; r < RPS; ++r) {
        float s1v[VEC], s2v[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) { s1v[i] = 0.0f; s2v[i] = 0.0f; }
#pragma unroll
        for (int j = 0; j < KC; ++j) {
          float x[VEC], dy[VEC], t[VEC];
          unpack_chunk<DT, VEC>(x, rx[r][j], DT);
          unpack_chunk<DT, VEC>(dy, rdy[r][j], DT);
          if constexpr (LN) vadd_s<VEC>(x, x, nmean[r]);
          vmul<VEC>(t, dy, w[j]);
          vfma<VEC>(s1v, x, t, s1v);
          if constexpr (LN) vadd<VEC>(s2v, s2v, t);
        }
        part[r] = hsum<VEC>(s1v);
        if constexpr (LN) part[RPS + r] = hsum<VEC>(s2v);
      }
      // The rows are in registers now (the sums above consumed every loaded word).
      ring_sum_values<NV>(part, redbuf, ctl, it, warp, lane, W, cluster_n, crank, q.g.timeouts);
      // Every warp of this CTA has passed its reads of the slot: refill it for the step NS ahead.
      if (tid == 0) {
        const int64_t ahead = step + static_cast<int64_t>(ns) * nclusters;
        if (ahead < q.num_steps) issue_step(ahead, pos.slot);
      }

      // ---- pass 2: dx = t * ca + xc * cb + cc; dw += dout * xc * rstd; db += dout ----
#pragma unroll
      for (int r = 0; r < RPS; ++r) {
        if (ok[r]) {
          const float ca = rstd[r];
          const float cb = -rstd[r] * rstd[r] * rstd[r] * part[r] * inv_n;
          const float cc = LN ? -rstd[r] * part[LN ? RPS + r : 0] * inv_n : 0.0f;
          char* dxp = reinterpret_cast<char*>(a.dx) +
                      ((row0 + r) * a.dx_row_stride + col0) * ESZ + tid * 16;
#pragma unroll
          for (int j = 0; j < KC; ++j) {
            float x[VEC], dy[VEC], t[VEC], dx[VEC];
            forget_values(rx[r][j]);
            forget_values(rdy[r][j]);
            unpack_chunk<DT, VEC>(x, rx[r][j], DT);
            unpack_chunk<DT, VEC>(dy, rdy[r][j], DT);
            if constexpr (LN) vadd_s<VEC>(x, x, nmean[r]);
            vmul<VEC>(t, dy, w[j]);
            vfma_ss<VEC>(dx, t, ca, cc);
            vfma_s<VEC>(dx, x, cb, dx);
            store_chunk_p<DT, VEC>(dxp + j * (T * 16), dx, DT);
            vmul<VEC>(t, dy, x);
            vfma_s<VEC>(dw[j], t, ca, dw[j]);
            if constexpr (DB) vadd<VEC>(db[j], db[j], dy);
          }
        }
      }
      pos.advance(ns);
    }

    // ---- epilogue: this cluster's partial sums -> row cid of the [P, N] workspaces ----
    const int64_t prow = cid * static_cast<int64_t>(N);
#pragma unroll
    for (int j = 0; j < KC; ++j) {
      const int c = col0 + (j * T + tid) * VEC;
      if (a.dw_partial != nullptr) store_chunk<QB_F32, VEC>(a.dw_partial, prow + c, dw[j], QB_F32);
      if constexpr (DB) {
        if (a.db_partial != nullptr) store_chunk<QB_F32, VEC>(a.db_partial, prow + c, db[j], QB_F32);
      }
    }
  }
  // Only after a timed-out wait can copies still be in flight here: shared memory must outlive
  // them, so wait (bounded) for the last copy issued into every slot.
  if (tid == 0 && *reinterpret_cast<volatile int*>(&ctl->abort) != 0) {
    const int64_t mine = q.num_steps > cid ? (q.num_steps - cid + nclusters - 1) / nclusters : 0;
    for (int s = 0; s < ns; ++s) {
      if (mine <= s) continue;
      const uint32_t ph = static_cast<uint32_t>((mine - s + ns - 1) / ns - 1) & 1u;
      const uint32_t bar = smem_u32(&ctl->full[s]);
      const unsigned long long t0 = global_timer_ns();
      while (!mbar_try_wait(bar, ph) && global_timer_ns() - t0 < kRingTimeoutNs) {}
    }
  }
  if (cluster_n > 1) cluster_sync_all();
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
template <int KC>
struct RowsPerSlot {  // rows per ring slot: about 48 KB of x + dout per slot
  static constexpr int value = KC == 1 ? 4 : (KC == 2 ? 2 : 1);
};

struct NbrPlan {
  int threads;    // 256 (two CTAs per SM) or 512 (one)
  int cluster_n, kc, ns;
  size_t smem;
};

// Geometry of the ring kernel for a row of N elements with `threads` per CTA, or false if it
// does not apply.  The same geometry serves every variant (with or without db, RMSNorm or
// LayerNorm), so the number of partial-sum slices does not depend on them.
static bool plan_norm_bwd_ring(int64_t N, int x_dtype, int threads, int max_smem_optin, NbrPlan* out) {
  const int vec = 16 / host_dtype_bytes(x_dtype);
  const int per_sm = 512 / threads;
  const int64_t unit = static_cast<int64_t>(threads) * vec * 3;  // columns of one CTA: KC = 3
  if (N % unit != 0) return false;
  const int64_t c = N / unit;
  if (!is_pow2(c) || c > (threads == 512 ? 4 : 1)) return false;
  const int smem_cap = per_sm == 1 ? max_smem_optin : (max_smem_optin + 1024) / per_sm - 1024;
  const size_t slot = static_cast<size_t>(2) * 3 * threads * 16;  // one row: x and dout
  const size_t red = static_cast<size_t>(2) * (threads / 32) * c * 8 * sizeof(float);
  int ns = static_cast<int>((static_cast<size_t>(smem_cap) - kRingCtlBytes - red) / slot);
  if (ns > 4) ns = 4;
  if (ns < 2) return false;
  out->threads = threads;
  out->cluster_n = static_cast<int>(c);
  out->kc = 3;
  out->ns = ns;
  out->smem = kRingCtlBytes + static_cast<size_t>(ns) * slot + red;
  return true;
}

template <int DT, int KC, bool LN, bool DB, int T>
static int launch_nbr(const qb_norm_bwd_args& a, const NbrPlan& plan, int64_t clusters,
                      cudaStream_t st) {
  constexpr int RPS = RowsPerSlot<KC>::value;
  unsigned int* timeouts = ring_timeout_counter();
  if (timeouts == nullptr) return QB_ERR_CUDA;
  NormBwdRingParams q;
  q.a = a;
  q.g.ns = plan.ns;
  q.g.cluster_n = plan.cluster_n;
  q.g.cols_per_cta = plan.kc * T * (DT == QB_F32 ? 4 : 8);
  q.g.timeouts = timeouts;
  q.num_steps = ceil_div(a.M, RPS);
  dim3 grid(static_cast<unsigned>(clusters * plan.cluster_n), 1, 1);
  return launch_kernel(norm_bwd_ring_kernel<DT, KC, RPS, LN, DB, T>, grid, T, plan.smem,
                       plan.cluster_n, st, q, LN ? "layernorm_bwd (ring)" : "rmsnorm_bwd (ring)");
}

template <int DT, int KC, int T>
static int launch_nbr_k(const qb_norm_bwd_args& a, const NbrPlan& plan, int64_t clusters,
                        cudaStream_t st) {
  const bool ln = a.is_layernorm != 0;
  const bool db = a.db_partial != nullptr;
  if (ln && db) return launch_nbr<DT, KC, true, true, T>(a, plan, clusters, st);
  if (ln) return launch_nbr<DT, KC, true, false, T>(a, plan, clusters, st);
  if (db) return launch_nbr<DT, KC, false, true, T>(a, plan, clusters, st);
  return launch_nbr<DT, KC, false, false, T>(a, plan, clusters, st);
}

template <int DT, int T>
static int launch_nbr_dt(const qb_norm_bwd_args& a, const NbrPlan& plan, int64_t clusters,
                         cudaStream_t st) {
  if (plan.kc == 3) return launch_nbr_k<DT, 3, T>(a, plan, clusters, st);
  return QB_ERR_UNSUPPORTED;
}

static int nbr_resident_clusters(const NbrPlan& plan, const DeviceFacts* dev) {
  const int per_sm = 512 / plan.threads;
  if (plan.cluster_n == 1) return dev->sm_count * per_sm;  // shared memory and threads
  // every instantiation has the same footprint class; the plainest one stands for them
  const void* rep = plan.threads == 512
      ? reinterpret_cast<const void*>(norm_bwd_ring_kernel<QB_BF16, 3, 1, false, false, 512>)
      : reinterpret_cast<const void*>(norm_bwd_ring_kernel<QB_BF16, 3, 1, false, false, 256>);
  const int n = cached_max_clusters(rep, plan.threads, plan.smem, plan.cluster_n);
  return n > 0 ? n : dev->sm_count * per_sm / plan.cluster_n;
}

// 512 threads (one CTA per SM; clusters of up to 4 for long rows) where the row fits that way,
// else 256 threads (two CTAs per SM).
static bool plan_norm_bwd_ring_any(int64_t N, int x_dtype, int max_smem_optin, NbrPlan* out) {
  return plan_norm_bwd_ring(N, x_dtype, 512, max_smem_optin, out) ||
         plan_norm_bwd_ring(N, x_dtype, 256, max_smem_optin, out);
}

int norm_bwd_ring_num_partials(int64_t N, int x_dtype, const DeviceFacts* dev) {
  NbrPlan plan;
  if (!plan_norm_bwd_ring_any(N, x_dtype, dev->max_smem_optin, &plan)) return 0;
  return nbr_resident_clusters(plan, dev);
}

int launch_norm_bwd_ring(const qb_norm_bwd_args& a, int64_t clusters, const DeviceFacts* dev,
                         cudaStream_t st) {
  if (a.H != 1 || a.dresidual_out != nullptr || a.dresidual != nullptr) return QB_ERR_UNSUPPORTED;
  if (a.dout_dtype != a.x_dtype || a.dx_dtype != a.x_dtype) return QB_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(a.dw_partial) | reinterpret_cast<uintptr_t>(a.db_partial)) % 16 != 0)
    return QB_ERR_UNSUPPORTED;
  NbrPlan plan;
  if (!plan_norm_bwd_ring_any(a.N, a.x_dtype, dev->max_smem_optin, &plan))
    return QB_ERR_UNSUPPORTED;
  // More partial slices than resident clusters would run as a second wave.
  if (clusters > nbr_resident_clusters(plan, dev)) return QB_ERR_UNSUPPORTED;
#define QB_NBR(DT)                                                                  \
  return plan.threads == 512 ? launch_nbr_dt<DT, 512>(a, plan, clusters, st)        \
                             : launch_nbr_dt<DT, 256>(a, plan, clusters, st);
  switch (a.x_dtype) {
    case QB_BF16: QB_NBR(QB_BF16)
    case QB_F16: QB_NBR(QB_F16)
    default: QB_NBR(QB_F32)
  }
#undef QB_NBR
}

}  // namespace qb
