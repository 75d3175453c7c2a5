// Shared between the translation units of the softmax path: launch parameters and the entry of
// the shared-memory ring kernels for long rows.
#ifndef QB_SOFTMAX_H_
#define QB_SOFTMAX_H_

#include "host_common.h"

namespace qb {

struct SoftmaxParams {
  const void* in0;  // fwd: x        bwd: dy
  const void* in1;  // fwd: unused   bwd: y
  void* out;        // fwd: y        bwd: dx
  int64_t M;
  int N;
  int64_t ld0, ld1, ldo;
  int dt0, dt1, dto;
  int tpr, rows_per_cta, cluster_n, cols_per_cta;
  int64_t num_tiles;
  int flags;  // qb_launch_cfg.flags
  unsigned int* timeouts;  // device counter of cluster-exchange waits that gave up
};

// Long rows through the bulk-copy shared-memory ring (softmax_ring.cu).  Returns QB_OK after the
// launch, QB_ERR_UNSUPPORTED (without touching the error string's meaning for the caller) when the
// row cannot be served by the ring so that the caller can fall back to another kernel.
template <bool BWD>
int launch_softmax_ring(const SoftmaxParams& p, const qb_launch_cfg& cfg, const DeviceFacts* dev,
                        cudaStream_t st);

// Long rows split over a thread-block cluster with the slices held in registers and the next
// rows' loads in flight (softmax_cluster.cu).  Same return convention as launch_softmax_ring.
template <bool BWD>
int launch_softmax_cluster(const SoftmaxParams& p, const qb_launch_cfg& cfg, const DeviceFacts* dev,
                           cudaStream_t st);

}  // namespace qb

#endif  // QB_SOFTMAX_H_
