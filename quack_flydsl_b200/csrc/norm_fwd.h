// Shared between the two translation units of the norm forward path: the launch parameters and
// the entry of the streamed long-row kernels.
#ifndef QB_NORM_FWD_H_
#define QB_NORM_FWD_H_

#include "host_common.h"

namespace qb {

struct NormFwdParams {
  qb_norm_fwd_args a;
  int tpr;            // threads per row
  int rows_per_cta;   // rows of one CTA tile
  int cluster_n;      // CTAs sharing a row
  int cols_per_cta;   // columns owned by one CTA of the cluster (multiple of VEC)
  int64_t num_tiles;  // ceil(M / rows_per_cta)
  int stage_params;   // weight / bias slices are staged in shared memory
  int flags;          // qb_launch_cfg.flags
  unsigned int* timeouts;  // device counter of cluster-exchange waits that gave up
};

// Launches the streamed two-pass kernel for p (uniform dtype, one row per CTA of `threads`).
int launch_norm_fwd_stream_any(const NormFwdParams& p, int threads, const DeviceFacts* dev,
                               cudaStream_t st);

}  // namespace qb

#endif  // QB_NORM_FWD_H_
