// Bulk-copy row ring for sm_100a: rows are staged in shared memory by the bulk asynchronous copy
// engine (cp.async.bulk, the 1-D form of TMA) and consumed from there twice -- once for the row
// statistic, once for the result -- so HBM sees exactly one read per element whatever the row
// length, and the next row is already being fetched while the current one is computed on.
//
// Role in the reference: the TMA load path of the backward norm kernel and its producer /
// consumer pipeline (quack/rmsnorm.py:686-693,931-950, quack/pipeline.py:400-535) and the
// mbarrier-based cluster reduction (quack/reduce.py:70-118, quack/utils.py:27-58).  The design is
// different: a CTA owns a ring of NS slots; slot g % NS holds chunk g of the CTA's stream of row
// slices (one chunk = CH bytes of each streamed input).  A dedicated producer warp waits for a
// slot to be released (empty barrier), announces the byte count on the slot's full barrier and
// issues the copies; the consumer warps wait on the full barrier, make two passes over the R
// chunks of a row and release each slot in the second pass.  With NS >= R the whole row is
// resident; with NS > R the head of the next row is loaded during the current row.
//
// Every wait is bounded: a wait that has not succeeded after kRingTimeoutNs sets the CTA's abort
// flag and bumps a device-side counter the host can read; from then on every wait of the CTA
// returns at once, so a kernel that lost a signal runs to its end (with wrong results for the
// affected rows) instead of hanging.  Copies only read this GPU's global memory, and each copy
// has exactly one destination: the shared memory of the CTA that issued it.
#pragma once

#include "common.cuh"

namespace qb {

constexpr int kRingMaxSlots = 32;
constexpr int kRingMaxPartials = 256;  // consumer warps x cluster size

// Arrive without a release fence.  For the "slot may be refilled" signal of a consumer warp: what
// must come first are the warp's shared-memory READS of the slot, and those have completed once an
// instruction that uses the loaded registers has been issued before this one.  (The default
// release form also waits for the warp's global stores in flight, which stalls a kernel that
// streams its results out.)
__device__ __forceinline__ void mbar_arrive_relaxed(uint32_t bar) {
  asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// Arrive (release at cluster scope) on a barrier of any CTA of the cluster; `bar_cluster` is a
// shared::cluster address from map_to_cta.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
               : "memory");
}
__device__ __forceinline__ void st_cluster_f2(uint32_t addr_cluster, float2 v) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr_cluster), "f"(v.x), "f"(v.y)
               : "memory");
}

// Bulk copy global -> this CTA's shared memory; completion is counted in bytes on `bar`.
// src and dst 16-byte aligned, bytes a multiple of 16.  `policy` is an L2 cache policy.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// Control block of a ring, at the start of the kernel's dynamic shared memory.
struct __align__(16) RingCtl {
  unsigned long long full[kRingMaxSlots];
  unsigned long long empty[kRingMaxSlots];
  unsigned long long red[2];                // row-reduction barriers, by row parity
  float2 red_buf[2][kRingMaxPartials];      // partials of all warps of all CTAs of the cluster
  int abort;                                // set once a wait of this CTA timed out
  int pad[3];
};
constexpr int kRingCtlBytes = (sizeof(RingCtl) + 127) / 128 * 128;

// Bounded wait.  CLUSTER: acquire at cluster scope.  Returns false if the CTA is aborting.
template <bool CLUSTER = false>
__device__ __forceinline__ bool ring_wait(RingCtl* ctl, uint32_t bar, uint32_t parity,
                                          unsigned int* timeouts) {
  if ((CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) != 0) return true;
  volatile int* ab = &ctl->abort;
  if (*ab) return false;
  const unsigned long long t0 = global_timer_ns();
  for (;;) {
    // try_wait itself suspends the thread for a while; the clock and the abort flag are looked
    // at once per 32 attempts
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if ((CLUSTER ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) != 0) return true;
    if (*ab) return false;
    if (global_timer_ns() - t0 > kRingTimeoutNs) {
      *ab = 1;
      if (timeouts != nullptr) atomicAdd(timeouts, 1u);
      return false;
    }
  }
}

// Position in the ring: slot index and the phase bit of that slot's barriers.
struct RingPos {
  int slot;
  uint32_t phase;
  __device__ __forceinline__ void advance(int ns) {
    if (++slot == ns) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// Initialises the barriers (one thread), publishes them to the CTA and, for clusters, to the
// other CTAs.  W = consumer warps per CTA.  Must be executed by every thread of the CTA.
__device__ __forceinline__ void ring_init(RingCtl* ctl, int ns, int consumer_warps, int cluster_n) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1);
      mbar_init(smem_u32(&ctl->empty[s]), consumer_warps);
    }
    mbar_init(smem_u32(&ctl->red[0]), consumer_warps * cluster_n);
    mbar_init(smem_u32(&ctl->red[1]), consumer_warps * cluster_n);
    ctl->abort = 0;
    mbar_fence_init();
  }
  __syncthreads();
  if (cluster_n > 1) cluster_sync_all();
}

// Row reduction over the consumer warps of all CTAs of the cluster through mbarriers: every warp
// stores its partial into slot [crank * W + warp] of every CTA's buffer and arrives on that CTA's
// barrier; every consumer thread then waits on its own CTA's barrier and folds all slots in one
// fixed order, so all threads of all CTAs obtain bit-identical results.  `it` counts the rows
// this CTA has reduced so far (buffers and barriers alternate by its parity).  Called by consumer
// threads only; `v` must already be reduced within the warp.
template <class Op>
__device__ __forceinline__ float2 ring_row_reduce(float2 v, RingCtl* ctl, int it, int warp, int lane,
                                                  int consumer_warps, int cluster_n, uint32_t crank,
                                                  unsigned int* timeouts) {
  const int par = it & 1;
  const uint32_t phase = static_cast<uint32_t>(it >> 1) & 1u;
  const uint32_t slot_local = smem_u32(&ctl->red_buf[par][crank * consumer_warps + warp]);
  const uint32_t bar_local = smem_u32(&ctl->red[par]);
  if (lane < cluster_n) {
    st_cluster_f2(map_to_cta(slot_local, lane), v);
    mbar_arrive_remote(map_to_cta(bar_local, lane));
  }
  ring_wait<true>(ctl, bar_local, phase, timeouts);
  const int nslots = consumer_warps * cluster_n;
  const float2* buf = ctl->red_buf[par];
  float2 acc = Op::identity();
  for (int i = lane; i < nslots; i += 32) acc = Op::combine(acc, buf[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = Op::combine(acc, shfl_xor_f2(acc, o));
  return acc;
}

template <class Op>
__device__ __forceinline__ float2 warp_reduce_f2(float2 v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = Op::combine(v, shfl_xor_f2(v, o));
  return v;
}

// Geometry of a ring launch, computed on the host.
struct RingGeom {
  int ns;             // slots
  int cluster_n;      // CTAs sharing a row
  int cols_per_cta;   // columns (elements) owned by one CTA, multiple of the 16-byte chunk
  unsigned int* timeouts;  // device counter of timed-out waits
};

}  // namespace qb
