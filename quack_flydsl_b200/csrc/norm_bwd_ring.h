// Entry points of the bulk-copy ring variant of the norm backward (norm_bwd_ring.cu), used by the
// dispatcher in norm_bwd.cu.
#ifndef QB_NORM_BWD_RING_H_
#define QB_NORM_BWD_RING_H_

#include "host_common.h"

namespace qb {

// Launches the ring kernel with `clusters` partial-sum slices.  The caller has already verified
// that x / dout / dx share one dtype and are addressable in full 16-byte chunks.  Returns
// QB_ERR_UNSUPPORTED (leaving the error string alone) when the shape is not served, so that the
// caller can use norm_bwd_kernel instead.
int launch_norm_bwd_ring(const qb_norm_bwd_args& a, int64_t clusters, const DeviceFacts* dev,
                         cudaStream_t st);

// Partial-sum slices the ring kernel wants for a row length (one cluster per slice, all resident
// at once), or 0 if the ring kernel does not serve the shape.
int norm_bwd_ring_num_partials(int64_t N, int x_dtype, const DeviceFacts* dev);

}  // namespace qb

#endif  // QB_NORM_BWD_RING_H_
