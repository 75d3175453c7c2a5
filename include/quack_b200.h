/*
 * quack_b200.h -- C ABI of libquack_b200.so: row-reduction kernels for NVIDIA B200 (sm_100a).
 *
 * Every entry point takes a pointer to a plain-old-data argument block (raw device pointers,
 * sizes, strides in ELEMENTS, dtype codes, scalars) and the CUDA stream to launch on.  The
 * library never allocates or frees device memory, never synchronises the host and keeps no
 * mutable state between calls apart from per-device, per-kernel attribute caches.  All outputs
 * and workspaces are allocated and owned by the caller.  A call returns QB_OK (0) once the
 * kernels are enqueued, or a negative qb_status; qb_last_error() then returns a thread-local,
 * human readable message.  No entry point aborts the process.
 *
 * The entry points replace the TVM-FFI packed functions that the reference (QuACK 0.6.1) builds
 * with cute.compile(..., "--enable-tvm-ffi") and calls from its torch.library op bodies; the
 * reference interface each one stands in for is cited at its declaration (paths are relative to
 * the reference project).
 */
#ifndef QUACK_B200_H_
#define QUACK_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QB_ABI_VERSION 3

/* element types of streamed tensors */
enum qb_dtype { QB_F32 = 0, QB_F16 = 1, QB_BF16 = 2 };
/* integer types of class-index tensors */
enum qb_itype { QB_I32 = 0, QB_I64 = 1 };

enum qb_status {
  QB_OK = 0,
  QB_ERR_INVALID = -1,     /* malformed arguments (null pointer, bad dtype, bad size) */
  QB_ERR_UNSUPPORTED = -2, /* legal request the kernels cannot serve (e.g. row too long) */
  QB_ERR_CUDA = -3         /* the CUDA runtime reported an error while launching */
};

/* Opaque CUDA stream handle (cudaStream_t). */
typedef struct CUstream_st* qb_stream_t;

/*
 * Optional launch overrides; all-zero selects the built-in sm_100a heuristics.  Plays the role of
 * the reference's RmsNormFwdConfig / RmsNormBwdConfig (quack/rmsnorm_config.py:16-26,94-107).
 */
typedef struct qb_launch_cfg {
  int32_t num_threads;     /* threads per CTA (power of two, 32..1024) */
  int32_t threads_per_row; /* threads cooperating on one row inside a CTA (power of two) */
  int32_t cluster_n;       /* CTAs of a thread-block cluster that share one row (1,2,4,8,16) */
  int32_t max_ctas;        /* cap on the grid (persistent kernels); 0 = heuristic */
  int32_t stages;          /* shared-memory prefetch stages (norm backward); chunks in flight per
                              thread and input (streamed softmax: 4 / 8 forward, 2 / 4 backward);
                              0 = heuristic */
  int32_t flags;           /* kernel-selection bits for tuning builds; 0 = heuristic (see the
                              QB_FLAG_* constants below) */
  int32_t ctas_per_sm;     /* shared-memory ring kernels: CTAs that share one SM (1 or 2); softmax
                              cluster-register kernel: row buffers per thread (1 = no prefetch, 2, 3);
                              0 = heuristic */
  int32_t reserved;
} qb_launch_cfg;

/* qb_launch_cfg.flags: which of several equivalent kernels serves a call.  Results do not depend
 * on them; they exist so that a tuning build can compare the alternatives. */
#define QB_FLAG_NO_PACKED 1    /* keep rows as fp32 registers where the packed 16-bit mode applies */
#define QB_FLAG_NO_TWO_PASS 2  /* long rows: never the two-pass kernels, always registers + clusters */
#define QB_FLAG_L2_PLAIN_1 4   /* two-pass kernels that re-read from L2: plain L2 policy, pass 1 */
#define QB_FLAG_L2_PLAIN_2 8   /* ... and pass 2 */
#define QB_FLAG_FORCE_TWO_PASS 16 /* two-pass kernel for any row length */
#define QB_FLAG_NO_RING 32     /* long rows: the two-pass kernel that re-reads the row from L2 */
#define QB_FLAG_RING 64        /* softmax, long rows: the shared-memory ring kernel */
#define QB_FLAG_CLUSTER_REGS 128 /* softmax, long rows: register-resident slices over a cluster */

/* Device facts the host side needs for workspace sizing. */
typedef struct qb_device_info {
  int32_t device;
  int32_t sm_count;
  int32_t cc_major;
  int32_t cc_minor;
  int32_t max_smem_optin; /* bytes */
  int32_t max_cluster;    /* largest cluster_n the library will use */
  int32_t reserved[2];
} qb_device_info;

/*
 * RMSNorm / LayerNorm forward.
 * Replaces the compiled RMSNorm kernel called by quack::_rmsnorm_fwd (quack/rmsnorm.py:365-423,
 * kernel quack/rmsnorm.py:150-362).
 *   h = x (+ residual)                      (fp32)
 *   residual_out = h                        (if residual_out != NULL)
 *   RMSNorm:   rstd = rsqrt(mean(h^2) + eps);            out = h * rstd * (w + weight_offset) + b
 *   LayerNorm: mean = mean(h); rstd = rsqrt(var(h)+eps); out = (h - mean) * rstd * (w + off) + b
 * x/out/residual/residual_out are (M*H, N) matrices with unit column stride and the given row
 * strides; weight/bias are (H, N) contiguous (H = 1 for the ordinary per-feature case) and may be
 * NULL; rstd/mean are (M*H) fp32 and may be NULL.  Row r uses head r % H.
 */
typedef struct qb_norm_fwd_args {
  const void* x;
  const void* weight;
  const void* bias;
  const void* residual;
  void* out;
  void* residual_out;
  float* rstd;
  float* mean;
  int64_t M;
  int64_t H;
  int64_t N;
  int64_t x_row_stride;
  int64_t residual_row_stride;
  int64_t out_row_stride;
  int64_t residual_out_row_stride;
  int32_t x_dtype;
  int32_t weight_dtype;
  int32_t bias_dtype;
  int32_t residual_dtype;
  int32_t out_dtype;
  int32_t residual_out_dtype;
  int32_t is_layernorm;
  float eps;
  float weight_offset;
  int32_t pad0;
  qb_launch_cfg cfg;
} qb_norm_fwd_args;

int qb_norm_fwd(const qb_norm_fwd_args* args, qb_stream_t stream);

/*
 * RMSNorm / LayerNorm backward, stage 1 (persistent kernel).
 * Replaces the compiled RMSNormBackward kernel called by quack::_rmsnorm_bwd
 * (quack/rmsnorm.py:1208-1286, kernel quack/rmsnorm.py:723-1205).
 *   xhat = (x - mean) * rstd   (mean = 0 for RMSNorm)
 *   wdy  = dout * (w + weight_offset)
 *   dx   = (wdy - xhat * mean(xhat*wdy) [- mean(wdy) for LayerNorm]) * rstd (+ dresidual_out)
 *   dresidual = dx                      (written only if dresidual != NULL; own dtype)
 *   dw_partial[p, h, :] = sum over the rows CTA p handled of dout * xhat   (fp32)
 *   db_partial[p, h, :] = sum over the rows CTA p handled of dout          (fp32)
 * num_partials (P) is the first dimension of dw_partial / db_partial and fixes the number of
 * row-owning CTAs (times cluster_n CTAs each); every one of the P*H slices is fully written even
 * if its CTA handled no row, so the workspaces need no initialisation.
 */
typedef struct qb_norm_bwd_args {
  const void* x;
  const void* weight;
  const void* dout;
  const float* rstd;
  const float* mean; /* required iff is_layernorm */
  const void* dresidual_out;
  void* dx;
  void* dresidual;
  float* dw_partial;
  float* db_partial;
  int64_t M;
  int64_t H;
  int64_t N;
  int64_t x_row_stride;
  int64_t dout_row_stride;
  int64_t dresidual_out_row_stride;
  int64_t dx_row_stride;
  int64_t dresidual_row_stride;
  int32_t num_partials;
  int32_t x_dtype;
  int32_t weight_dtype;
  int32_t dout_dtype;
  int32_t dresidual_out_dtype;
  int32_t dx_dtype;
  int32_t dresidual_dtype;
  int32_t is_layernorm;
  float weight_offset;
  int32_t pad0;
  qb_launch_cfg cfg;
} qb_norm_bwd_args;

int qb_norm_bwd(const qb_norm_bwd_args* args, qb_stream_t stream);

/*
 * Number of partial-sum slices (P) the backward heuristics want for a row length, i.e. the first
 * dimension of dw_partial.  Replaces get_sm_count (quack/rmsnorm_config.py:265-293).
 */
int qb_norm_bwd_num_partials(int64_t N, int32_t x_dtype, int32_t is_layernorm, int32_t device);

/*
 * Norm backward, stage 2: deterministic fixed-order reduction of the fp32 partials over P and
 * cast to the parameter dtype.  Replaces `dw_partial.sum(dim=0).to(weight.dtype)`
 * (quack/rmsnorm.py:1398-1399, 1719-1720).  partial is (P, cols) fp32 contiguous; out is (cols).
 * If out_f32 != NULL the fp32 sum is also stored there (used before a cross-GPU all-reduce so
 * that every rank rounds the same global sum).  Either output may be NULL.
 */
typedef struct qb_colsum_args {
  const float* partial;
  void* out;
  float* out_f32;
  int64_t P;
  int64_t cols;
  int32_t out_dtype;
  int32_t pad0;
} qb_colsum_args;

int qb_colsum(const qb_colsum_args* args, qb_stream_t stream);

/*
 * Stage 2 fused with the cross-GPU sum: out[c] = sum over ranks of sum_p partial[p, c], for the
 * row-sharded norm backward on the GPUs of one node (one process per GPU).  One launch replaces
 * qb_colsum + an all-reduce of the fp32 vector: every block stores its column sums into its slot
 * of every rank's exchange buffer (plain stores to peer-mapped memory), raises a flag there,
 * waits -- with a time limit -- for the same block's flags from all ranks and adds the slots in
 * rank order, so all ranks obtain bit-identical gradients.  Up to two partial buffers of the same
 * shape (dw and db) are reduced by the same launch.  No counterpart in the reference, which has
 * no multi-GPU path for these operators (its dw / db reduction is quack/rmsnorm.py:1398-1399).
 *
 * Exchange buffers: every rank calls qb_peer_buffer_create (cudaMalloc + zero fill + CUDA IPC
 * handle; the only entry point of this library that allocates device memory), the
 * QB_PEER_HANDLE_BYTES handles are exchanged by the caller (e.g. torch.distributed
 * all_gather_object), and every rank maps the others' buffers with qb_peer_buffer_open.
 * peers[r] is rank r's buffer as seen from the calling process (peers[rank] the local one).
 * cap_cols (a multiple of 32, the same on all ranks) bounds cols * num_buffers; at most 32768
 * columns are exchanged per launch (all blocks must be resident together), more returns
 * QB_ERR_UNSUPPORTED.  seq is the caller's step counter: 1 for the first call on a set of
 * buffers, then incremented by exactly one per call, the same on every rank.  Calls on one set of
 * buffers must not overlap.  status (optional, device memory) counts the waits that gave up after
 * two seconds; it stays 0 in a healthy job.
 */
#define QB_MAX_PEERS 8
#define QB_PEER_HANDLE_BYTES 64

typedef struct qb_colsum_allreduce_args {
  const float* partial0; /* [P, cols] fp32 */
  const float* partial1; /* second buffer of the same shape, or NULL */
  void* out0;            /* [cols] in out_dtype, or NULL */
  void* out1;
  float* out0_f32;       /* [cols] fp32, or NULL */
  float* out1_f32;
  void* peers[QB_MAX_PEERS];
  uint32_t* status;
  int64_t P;
  int64_t cols;
  int64_t cap_cols;
  int32_t num_buffers;   /* 1 or 2 */
  int32_t out_dtype;
  int32_t world;
  int32_t rank;
  uint32_t seq;
  int32_t pad0;
} qb_colsum_allreduce_args;

int qb_colsum_allreduce(const qb_colsum_allreduce_args* args, qb_stream_t stream);

/*
 * Vocabulary-sharded cross-entropy: exchange of the per-row (max, sum-exp, target logit) between
 * the GPUs of one node fused with their fold into (loss, lse) -- one launch instead of an
 * all-gather of the (3, M) fp32 block followed by qb_ce_combine, same arithmetic and shard order
 * as qb_ce_combine.  stats is this rank's (3, M) block; the exchange buffers, peers, seq and status
 * are those of qb_colsum_allreduce (one step counter per set of buffers, shared by both entry
 * points); needs 3 * M <= cap_cols and at most 262144 rows per launch.  No counterpart in the
 * reference (single-GPU analogue: the lse_partial mode, quack/cross_entropy.py:676-694).
 */
typedef struct qb_ce_combine_exchange_args {
  const float* stats;  /* (3, M) fp32 of this rank */
  const void* target;
  const void* weight;  /* optional */
  float* loss;
  float* lse;
  void* peers[QB_MAX_PEERS];
  uint32_t* status;
  int64_t M;
  int64_t cap_cols;
  int64_t ignore_index;
  int64_t num_classes;
  int32_t target_dtype;
  int32_t weight_dtype;
  int32_t world;
  int32_t rank;
  uint32_t seq;
  int32_t pad0;
} qb_ce_combine_exchange_args;

int qb_ce_combine_exchange(const qb_ce_combine_exchange_args* args, qb_stream_t stream);
/* Bytes of one rank's exchange buffer for `world` ranks and cap_cols columns (-1: bad arguments). */
int64_t qb_peer_buffer_bytes(int32_t world, int64_t cap_cols);
int qb_peer_buffer_create(int32_t world, int64_t cap_cols, void** local, unsigned char* handle);
int qb_peer_buffer_open(const unsigned char* handle, void** peer);
int qb_peer_buffer_close(void* peer);
int qb_peer_buffer_destroy(void* local);

/*
 * Softmax forward over the last dimension of an (M, N) matrix.
 * Replaces the compiled Softmax kernel called by quack::_softmax_fwd (quack/softmax.py:193-207,
 * kernel quack/softmax.py:87-176).
 */
typedef struct qb_softmax_fwd_args {
  const void* x;
  void* out;
  int64_t M;
  int64_t N;
  int64_t x_row_stride;
  int64_t out_row_stride;
  int32_t x_dtype;
  int32_t out_dtype;
  qb_launch_cfg cfg;
} qb_softmax_fwd_args;

int qb_softmax_fwd(const qb_softmax_fwd_args* args, qb_stream_t stream);

/*
 * Softmax backward: dx = y * (dy - sum(dy * y)).
 * Replaces the compiled SoftmaxBackward kernel called by quack::_softmax_backward
 * (quack/softmax.py:373-391, kernel quack/softmax.py:275-353).
 */
typedef struct qb_softmax_bwd_args {
  const void* dy;
  const void* y;
  void* dx;
  int64_t M;
  int64_t N;
  int64_t dy_row_stride;
  int64_t y_row_stride;
  int64_t dx_row_stride;
  int32_t dy_dtype;
  int32_t y_dtype;
  int32_t dx_dtype;
  int32_t pad0;
  qb_launch_cfg cfg;
} qb_softmax_bwd_args;

int qb_softmax_bwd(const qb_softmax_bwd_args* args, qb_stream_t stream);

/*
 * Cross-entropy forward (optionally also the gradient w.r.t. the logits).
 * Replaces the compiled CrossEntropy kernel called by quack::cross_entropy_fwd_out
 * (quack/cross_entropy.py:312-364, kernel quack/cross_entropy.py:113-265).
 *   lse[r]  = log(sum_j exp(x[r, j]))
 *   loss[r] = w[t] * (lse[r] - tl[r])          or exactly 0 if t == ignore_index
 *     where t = target[r] and tl[r] = x[r, t], or target_logit[r, t] / target_logit[r] if given
 *   dx[r,:] = w[t] * (softmax(x[r,:]) - onehot(t))   or exactly 0 if t == ignore_index
 * Sharded use (vocabulary split over GPUs): if row_max / row_sumexp / row_tgt are given the
 * kernel stores, per row, max_j x, sum_j exp(x - max) and the raw target logit (0 when the
 * target column is outside [col_offset, col_offset + N) or ignored), and loss / lse may be NULL.
 * target holds GLOBAL class ids; col_offset is the id of this shard's first column.
 * A target that is negative (other than ignore_index) or >= num_classes (when given) names no
 * class: the row is treated like an ignored one instead of reading weight / target_logit out of
 * bounds.
 * dx may alias x (in-place).
 */
typedef struct qb_ce_fwd_args {
  const void* x;
  const void* target;
  const void* target_logit; /* optional */
  const void* weight;       /* optional per-class weights, indexed by global class id */
  float* loss;              /* optional when the row_* outputs are given */
  float* lse;               /* optional */
  void* dx;                 /* optional */
  float* row_max;           /* optional (sharded) */
  float* row_sumexp;        /* optional (sharded) */
  float* row_tgt;           /* optional (sharded) */
  int64_t M;
  int64_t N;
  int64_t x_row_stride;
  int64_t dx_row_stride;
  int64_t target_logit_row_stride; /* elements; used when target_logit_ndim == 2 */
  int64_t col_offset;
  int64_t ignore_index;
  int64_t num_classes; /* classes a target may name (length of weight, columns of a 2-D
                          target_logit); 0 = no upper bound known */
  int32_t x_dtype;
  int32_t target_dtype; /* qb_itype */
  int32_t target_logit_dtype;
  int32_t target_logit_ndim; /* 1 or 2 */
  int32_t weight_dtype;
  int32_t pad0;
  qb_launch_cfg cfg;
} qb_ce_fwd_args;

int qb_ce_fwd(const qb_ce_fwd_args* args, qb_stream_t stream);

/*
 * Cross-entropy backward from a saved log-sum-exp.
 * Replaces the compiled CrossEntropyBackward kernel called by quack::cross_entropy_bwd_out
 * (quack/cross_entropy.py:574-628, kernel quack/cross_entropy.py:463-546).
 *   dx[r, j] = (exp(x[r, j] - lse[r]) - [col_offset + j == target[r]]) * dloss[r] * w[target[r]]
 * and exactly 0 for rows whose target equals ignore_index.  dloss is read with an element stride
 * (0 is allowed: one broadcast value).  dx may alias x.
 */
typedef struct qb_ce_bwd_args {
  const void* x;
  const void* target;
  const float* dloss;
  const float* lse;
  const void* weight; /* optional */
  void* dx;
  int64_t M;
  int64_t N;
  int64_t x_row_stride;
  int64_t dx_row_stride;
  int64_t dloss_stride;
  int64_t col_offset;
  int64_t ignore_index;
  int64_t num_classes; /* as in qb_ce_fwd_args */
  int32_t x_dtype;
  int32_t dx_dtype;
  int32_t target_dtype;
  int32_t weight_dtype;
  qb_launch_cfg cfg;
} qb_ce_bwd_args;

int qb_ce_bwd(const qb_ce_bwd_args* args, qb_stream_t stream);

/*
 * Vocabulary-sharded cross-entropy, combine step.  The reference has no multi-GPU path; its
 * single-GPU analogue is the lse_partial mode of CrossEntropyFunction
 * (quack/cross_entropy.py:676-694).  stats is (G, 3, M) fp32: for each shard g the per-row
 * max, sum-exp (relative to that max) and raw target logit, gathered in rank order.  Computes, in
 * fixed shard order, m = max_g m_g, s = sum_g s_g * exp(m_g - m), t = sum_g t_g,
 * lse = m + log(s), loss = w[target] * (lse - t), or exactly 0 for ignored rows.
 */
typedef struct qb_ce_combine_args {
  const float* stats;
  const void* target;
  const void* weight; /* optional */
  float* loss;
  float* lse;
  int64_t G;
  int64_t M;
  int64_t ignore_index;
  int64_t num_classes; /* as in qb_ce_fwd_args */
  int32_t target_dtype;
  int32_t weight_dtype;
} qb_ce_combine_args;

int qb_ce_combine(const qb_ce_combine_args* args, qb_stream_t stream);

/*
 * rstd[m] = rsqrt(sum_n x[m, n] * scale + eps) for an (M, N) matrix of partial sums of squares
 * (fp32 / fp16 / bf16, unit column stride): the finalising step of a GEMM + RMSNorm pipeline.
 * Replaces the compiled RmsFinalReduce kernel called by quack::rms_final_reduce_out
 * (quack/rms_final_reduce.py:138-153, kernel :27-135).
 */
typedef struct qb_rms_final_reduce_args {
  const void* x;
  float* rstd; /* (M) fp32 */
  int64_t M;
  int64_t N;
  int64_t x_row_stride;
  float scale;
  float eps;
  int32_t x_dtype;
  int32_t pad0;
} qb_rms_final_reduce_args;

int qb_rms_final_reduce(const qb_rms_final_reduce_args* args, qb_stream_t stream);

/*
 * Top-k over the last dimension of an (M, N) matrix, largest first, optionally followed by a
 * softmax over the k selected values.
 * Replaces the compiled TopK kernel called by quack::_topk_fwd (quack/topk.py:234-254, kernel
 * quack/topk.py:26-233).  N must be a power of two <= 4096 and k <= 128 (the reference's
 * contract); values (M, k) has x's dtype, indices (M, k) is int32; both contiguous.  Equal values
 * come out in order of increasing column.
 */
typedef struct qb_topk_fwd_args {
  const void* x;
  void* values;
  int32_t* indices;
  int64_t M;
  int64_t N;
  int64_t k;
  int64_t x_row_stride;
  int32_t x_dtype;
  int32_t softmax; /* 0 / 1 */
} qb_topk_fwd_args;

int qb_topk_fwd(const qb_topk_fwd_args* args, qb_stream_t stream);

/*
 * Top-k backward: every row of dx (M, N) is written completely -- zeros, then
 *   dx[r, indices[r, j]] = dvalues[r, j]                                        (softmax == 0)
 *   dx[r, indices[r, j]] = values[r, j] * (dvalues[r, j] - sum_i dvalues[r, i] * values[r, i])
 * where values is the forward's (softmaxed) output.  Replaces the compiled TopKBackward kernel
 * called by quack::_topk_bwd (quack/topk.py:461-491, kernel quack/topk.py:275-460).  dvalues,
 * values and indices are (M, k) contiguous; dx has unit column stride.
 */
typedef struct qb_topk_bwd_args {
  const void* dvalues;
  const void* values; /* required iff softmax */
  const int32_t* indices;
  void* dx;
  int64_t M;
  int64_t N;
  int64_t k;
  int64_t dx_row_stride;
  int32_t dvalues_dtype;
  int32_t values_dtype;
  int32_t dx_dtype;
  int32_t softmax;
} qb_topk_bwd_args;

int qb_topk_bwd(const qb_topk_bwd_args* args, qb_stream_t stream);

/*
 * Norm backward without a caller-provided workspace.  No counterpart in the reference (there the
 * caller always allocates dw_partial / db_partial with torch, quack/rmsnorm.py:1368-1379); added
 * for hosts that may not allocate device memory: code running after an application's "memory is
 * frozen" point, plugins that only receive input / output buffers, loops that cannot afford the
 * device-wide synchronisation of cudaMalloc / cudaFree.
 *
 * Runs stage 1 (qb_norm_bwd) and stage 2 (qb_colsum) with the fp32 partial sums kept in a
 * QB_STATIC_SCRATCH_BYTES array that is part of the library image on every GPU.  bwd.dw_partial,
 * bwd.db_partial and bwd.num_partials are ignored.  dw / db receive the finished (H, N) parameter
 * gradients in param_dtype; pass NULL for a gradient that is not wanted (db == NULL: no bias).
 * Limit: H * N * (number of requested gradients) <= QB_STATIC_SCRATCH_BYTES / 4 /
 * QB_STATIC_MIN_PARTIALS floats (65536 with the defaults, e.g. N = 32768 with dw and db);
 * larger rows return QB_ERR_UNSUPPORTED.  The call allocates nothing.  Its first call on a device
 * looks up the array's device address (cudaGetSymbolAddress) and should therefore be made once
 * during start-up, before any stream capture.  All calls on a GPU share the array, which keeps
 * the previous call's contents: calls that may overlap on the same GPU (other streams, other
 * threads) race and must be ordered by the caller.
 */
#define QB_STATIC_SCRATCH_BYTES (16u << 20)
#define QB_STATIC_MIN_PARTIALS 64

typedef struct qb_norm_bwd_static_args {
  qb_norm_bwd_args bwd;
  void* dw;
  void* db;
  int32_t param_dtype;
  int32_t pad0;
} qb_norm_bwd_static_args;

int qb_norm_bwd_static(const qb_norm_bwd_static_args* args, qb_stream_t stream);

/*
 * Health counter of the shared-memory ring kernels (long rows).  Every wait inside those kernels
 * is bounded; a wait that gave up lets its kernel run to the end with wrong results for the rows
 * concerned and increments a per-device counter.  Stores the current device's count (0 in a
 * healthy process) into *count.  Synchronises the device (it is a diagnostic, not a hot-path
 * call).  No counterpart in the reference, whose pipelines wait without a limit
 * (quack/pipeline.py:400-535).
 */
int qb_ring_timeouts(uint32_t* count);

/* Fills *info for a CUDA device ordinal (-1 = current device). */
int qb_query_device(int32_t device, qb_device_info* info);

/* Message of the last failing call made by this thread ("" if none). */
const char* qb_last_error(void);

/*
 * Name of the device kernel (template arguments included, e.g.
 * "void qb::norm_fwd_kernel<2, 8, 8, false, false, 1>(qb::NormFwdParams)") that the last entry
 * point called by this host thread launched last; "" if none.  Lets a benchmark or a profile
 * summary state which instantiation served a shape.  No counterpart in the reference, where the
 * kernel is whatever the JIT compiled for the call.
 */
const char* qb_last_kernel(void);

/* ABI self-description: QB_ABI_VERSION the library was built with. */
int qb_abi_version(void);

/*
 * sizeof() of an argument block as compiled into the library, so a foreign-language binding can
 * verify its struct layout before the first call.  which: 0 launch_cfg, 1 norm_fwd, 2 norm_bwd,
 * 3 colsum, 4 softmax_fwd, 5 softmax_bwd, 6 ce_fwd, 7 ce_bwd, 8 ce_combine, 9 device_info,
 * 10 norm_bwd_static, 11 rms_final_reduce, 12 topk_fwd, 13 topk_bwd, 14 colsum_allreduce,
 * 15 ce_combine_exchange.
 * Returns -1 for an unknown code.
 */
int qb_sizeof_args(int32_t which);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* QUACK_B200_H_ */
