// Stage 2 of the norm backward fused with the cross-GPU sum of the parameter gradients.
//
// Rows shard over the GPUs of one node; every GPU reduces dw / db over its own rows into the
// [P, cols] fp32 partial buffers (stage 1), and the column sums then have to be added over the
// ranks.  As two steps that is qb_colsum followed by an NCCL all-reduce of a 32 KiB vector, whose
// cost is pure latency (about 16 us per step on NVLink, against 9 us for the column sum itself).
// Here one kernel does both: every block sums its 32 columns over P in the fixed order of
// colsum_kernel, stores the 32 fp32 results into its own slot of EVERY rank's exchange buffer with
// plain stores to peer-mapped memory, raises a per-block flag on every rank, waits for the flags
// of the same block from all ranks and adds the G slots in rank order.  All ranks add the same
// values in the same order, so the gradients are bit-identical on every GPU and from run to run.
//
// The exchange buffer is allocated once per communicator with cudaMalloc and shared through CUDA
// IPC handles (qb_peer_buffer_*); nothing is bound to an NVLink multicast object and no load ever
// reads another GPU's memory -- the only remote accesses are plain stores.  Flags carry a step
// number that only grows, slots and flags alternate by the step's parity, and every wait is
// bounded: a block that has not seen a peer's flag after kPeerTimeoutNs adds 1 to the status word
// and carries on with whatever the slots hold, so a missing peer costs wrong numbers for that
// call, which the host can detect, but never a hung GPU.
//
// No counterpart in the reference, which has no multi-GPU path for these operators.
#include <string.h>

#include "common.cuh"
#include "host_common.h"

namespace qb {

constexpr unsigned long long kPeerTimeoutNs = 2000000000ull;  // 2 s

struct PeerReduceParams {
  qb_colsum_allreduce_args a;
};

__device__ __forceinline__ unsigned long long peer_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float ld_relaxed_sys_f32(const float* p) {
  float v;
  asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

// Layout of one rank's exchange buffer, in 4-byte words:
//   data  [2 parities][world][cap_cols]   fp32
//   flags [2 parities][world][cap_blocks] uint32      cap_blocks = cap_cols / 32
// Block (32, 8) as in colsum_kernel; grid = ceil(total_cols / 32) where the columns of the (up to
// two) partial buffers are laid side by side.
__global__ void __launch_bounds__(256) colsum_allreduce_kernel(const PeerReduceParams p) {
  __shared__ float part[8][33];
  const qb_colsum_allreduce_args& a = p.a;
  const int tx = threadIdx.x & 31;
  const int ty = threadIdx.x >> 5;
  const int64_t total = a.cols * a.num_buffers;
  const int64_t c = static_cast<int64_t>(blockIdx.x) * 32 + tx;  // column of [dw | db]
  const bool live = c < total;
  const int which = live && c >= a.cols ? 1 : 0;
  const int64_t cc = live ? c - which * a.cols : 0;
  const float* partial = which ? a.partial1 : a.partial0;
  float acc = 0.0f;
  if (live) {
    for (int64_t r = ty; r < a.P; r += 8) acc += partial[r * a.cols + cc];
  }
  part[ty][tx] = acc;
  __syncthreads();
  if (ty != 0) return;
  float s = part[0][tx];
#pragma unroll
  for (int j = 1; j < 8; ++j) s += part[j][tx];

  const int G = a.world;
  const uint32_t par = a.seq & 1u;
  const int64_t cap_cols = a.cap_cols;
  const int64_t cap_blocks = cap_cols / 32;
  const int64_t data_words = 2 * static_cast<int64_t>(G) * cap_cols;
  // my slot in rank r's buffer, and the flag that announces it
  if (live) {
    for (int r = 0; r < G; ++r) {
      float* data = reinterpret_cast<float*>(a.peers[r]);
      data[(static_cast<int64_t>(par) * G + a.rank) * cap_cols + c] = s;
    }
  }
  __threadfence_system();
  __syncwarp();
  if (tx < G) {
    uint32_t* flags = reinterpret_cast<uint32_t*>(a.peers[tx]) + data_words;
    st_release_sys_u32(&flags[(static_cast<int64_t>(par) * G + a.rank) * cap_blocks + blockIdx.x], a.seq);
  }
  // wait for every rank's flag of this block in my own buffer
  if (tx < G) {
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(a.peers[a.rank]) + data_words;
    const uint32_t* f = &flags[(static_cast<int64_t>(par) * G + tx) * cap_blocks + blockIdx.x];
    // (a flag at or beyond this step: steps only grow, and a peer can be at most one step ahead)
    auto reached = [&](uint32_t v) { return static_cast<int32_t>(v - a.seq) >= 0; };
    if (!reached(ld_acquire_sys_u32(f))) {
      const unsigned long long t0 = peer_timer_ns();
      bool ok = false;
      while (!ok) {
#pragma unroll 1
        for (int i = 0; i < 64 && !ok; ++i) {
          ok = reached(ld_acquire_sys_u32(f));
          if (!ok) __nanosleep(64);
        }
        if (!ok && peer_timer_ns() - t0 > kPeerTimeoutNs) {
          if (a.status != nullptr) atomicAdd(a.status, 1u);
          break;
        }
      }
    }
  }
  __syncwarp();
  if (!live) return;
  const float* mine = reinterpret_cast<const float*>(a.peers[a.rank]);
  float tot = 0.0f;
  for (int r = 0; r < G; ++r)
    tot += ld_relaxed_sys_f32(&mine[(static_cast<int64_t>(par) * G + r) * cap_cols + c]);
  float* o32 = which ? a.out1_f32 : a.out0_f32;
  void* o = which ? a.out1 : a.out0;
  if (o32 != nullptr) o32[cc] = tot;
  if (o != nullptr) {
    if (a.out_dtype == QB_F32) reinterpret_cast<float*>(o)[cc] = tot;
    else if (a.out_dtype == QB_BF16) reinterpret_cast<__nv_bfloat16*>(o)[cc] = __float2bfloat16_rn(tot);
    else reinterpret_cast<__half*>(o)[cc] = __float2half_rn(tot);
  }
}

// ---------------------------------------------------------------------------------------------
// Vocabulary-sharded cross-entropy: exchange of the per-row statistics fused with their fold
// ---------------------------------------------------------------------------------------------
// Every rank holds (max, sum-exp, target logit) of its column slice for all M rows.  One block of
// 256 threads owns 256 rows: it stores their three statistics into its slot of every rank's
// exchange buffer, raises its flag there, waits (bounded) for the same block's flags from all
// ranks and folds the G shards in rank order exactly as ce_combine_kernel does.  Replaces an
// all-gather of the (3, M) block followed by ce_combine.  Slot of rank r, parity par:
// data[(par * G + r) * cap_cols + k * M + row], k = 0 (max), 1 (sum-exp), 2 (target logit).
struct CeExchangeParams {
  qb_ce_combine_exchange_args a;
};

__device__ __forceinline__ bool peer_wait_flag(const uint32_t* f, uint32_t seq, uint32_t* status) {
  auto reached = [&](uint32_t v) { return static_cast<int32_t>(v - seq) >= 0; };
  if (reached(ld_acquire_sys_u32(f))) return true;
  const unsigned long long t0 = peer_timer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i) {
      if (reached(ld_acquire_sys_u32(f))) return true;
      __nanosleep(64);
    }
    if (peer_timer_ns() - t0 > kPeerTimeoutNs) {
      if (status != nullptr) atomicAdd(status, 1u);
      return false;
    }
  }
}

__global__ void __launch_bounds__(256) ce_combine_exchange_kernel(const CeExchangeParams p) {
  const qb_ce_combine_exchange_args& a = p.a;
  const int tid = threadIdx.x;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 256 + tid;
  const bool live = row < a.M;
  const int G = a.world;
  const uint32_t par = a.seq & 1u;
  const int64_t cap_cols = a.cap_cols;
  const int64_t cap_blocks = cap_cols / 32;
  const int64_t data_words = 2 * static_cast<int64_t>(G) * cap_cols;
  const int64_t slot = (static_cast<int64_t>(par) * G + a.rank) * cap_cols;
  if (live) {
    const float m = a.stats[row], s = a.stats[a.M + row], t = a.stats[2 * a.M + row];
    for (int r = 0; r < G; ++r) {
      float* data = reinterpret_cast<float*>(a.peers[r]) + slot;
      data[row] = m;
      data[a.M + row] = s;
      data[2 * a.M + row] = t;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (tid < G) {
    uint32_t* flags = reinterpret_cast<uint32_t*>(a.peers[tid]) + data_words;
    st_release_sys_u32(&flags[(static_cast<int64_t>(par) * G + a.rank) * cap_blocks + blockIdx.x], a.seq);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(a.peers[a.rank]) + data_words;
    peer_wait_flag(&mine[(static_cast<int64_t>(par) * G + tid) * cap_blocks + blockIdx.x], a.seq, a.status);
  }
  __syncthreads();
  if (!live) return;
  const float* mine = reinterpret_cast<const float*>(a.peers[a.rank]);
  float m = neg_inf();
  for (int g = 0; g < G; ++g)
    m = fmaxf(m, ld_relaxed_sys_f32(&mine[(static_cast<int64_t>(par) * G + g) * cap_cols + row]));
  float s = 0.0f, t = 0.0f;
  for (int g = 0; g < G; ++g) {
    const float* sl = mine + (static_cast<int64_t>(par) * G + g) * cap_cols;
    const float mg = ld_relaxed_sys_f32(&sl[row]);
    const float sg = ld_relaxed_sys_f32(&sl[a.M + row]);
    if (mg != neg_inf()) s += sg * exp2f((mg - m) * kLog2e);
    t += ld_relaxed_sys_f32(&sl[2 * a.M + row]);
  }
  const float log_s = logf(s);
  if (a.lse != nullptr) a.lse[row] = m + log_s;
  if (a.loss != nullptr) {
    const int64_t tgt = load_index(a.target, row, a.target_dtype);
    const bool ignored = tgt == a.ignore_index || tgt < 0 || (a.num_classes > 0 && tgt >= a.num_classes);
    float wt = 1.0f;
    if (a.weight != nullptr && !ignored) wt = load_scalar(a.weight, tgt, a.weight_dtype);
    a.loss[row] = ignored ? 0.0f : wt * ((m - t) + log_s);
  }
}

}  // namespace qb

using namespace qb;

extern "C" int qb_ce_combine_exchange(const qb_ce_combine_exchange_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "ce_combine_exchange: null argument block");
  const qb_ce_combine_exchange_args& a = *args;
  if (a.stats == nullptr || (a.loss == nullptr && a.lse == nullptr))
    return set_error(QB_ERR_INVALID, "ce_combine_exchange: stats and an output are required");
  if (a.loss != nullptr && a.target == nullptr)
    return set_error(QB_ERR_INVALID, "ce_combine_exchange: the loss needs the targets");
  if (a.M < 0) return set_error(QB_ERR_INVALID, "ce_combine_exchange: bad sizes");
  if (a.world < 1 || a.world > QB_MAX_PEERS || a.rank < 0 || a.rank >= a.world)
    return set_error(QB_ERR_INVALID, "ce_combine_exchange: bad rank %d of %d", a.rank, a.world);
  if (a.seq == 0) return set_error(QB_ERR_INVALID, "ce_combine_exchange: step numbers start at 1");
  const int64_t blocks = ceil_div(a.M, 256);
  if (a.cap_cols <= 0 || a.cap_cols % 32 != 0 || 3 * a.M > a.cap_cols || blocks > a.cap_cols / 32)
    return set_error(QB_ERR_UNSUPPORTED, "ce_combine_exchange: %lld rows exceed the exchange buffer (%lld words)",
                     (long long)a.M, (long long)a.cap_cols);
  if (blocks > 1024)  // all blocks wait for their peers: they have to be resident together
    return set_error(QB_ERR_UNSUPPORTED, "ce_combine_exchange: more than 262144 rows per launch");
  for (int r = 0; r < a.world; ++r)
    if (a.peers[r] == nullptr) return set_error(QB_ERR_INVALID, "ce_combine_exchange: peer %d is not mapped", r);
  if (a.loss != nullptr && a.target_dtype != QB_I32 && a.target_dtype != QB_I64)
    return set_error(QB_ERR_INVALID, "ce_combine_exchange: unsupported target dtype");
  if (a.M == 0) return QB_OK;
  CeExchangeParams p;
  p.a = a;
  dim3 grid(static_cast<unsigned>(blocks), 1, 1);
  return launch_kernel(ce_combine_exchange_kernel, grid, 256, 0, 1, reinterpret_cast<cudaStream_t>(stream), p,
                       "ce_combine_exchange");
}

extern "C" int64_t qb_peer_buffer_bytes(int32_t world, int64_t cap_cols) {
  if (world <= 0 || world > QB_MAX_PEERS || cap_cols <= 0 || cap_cols % 32 != 0) return -1;
  return (2 * static_cast<int64_t>(world) * cap_cols + 2 * static_cast<int64_t>(world) * (cap_cols / 32)) * 4;
}

extern "C" int qb_peer_buffer_create(int32_t world, int64_t cap_cols, void** local, unsigned char* handle) {
  clear_error();
  const int64_t bytes = qb_peer_buffer_bytes(world, cap_cols);
  if (bytes <= 0 || local == nullptr || handle == nullptr)
    return set_error(QB_ERR_INVALID, "peer_buffer_create: bad arguments");
  void* ptr = nullptr;
  cudaError_t e = cudaMalloc(&ptr, static_cast<size_t>(bytes));
  if (e != cudaSuccess) return set_error(QB_ERR_CUDA, "peer_buffer_create: cudaMalloc: %s", cudaGetErrorString(e));
  e = cudaMemset(ptr, 0, static_cast<size_t>(bytes));  // flags start below every step number (>= 1)
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) {
    cudaFree(ptr);
    return set_error(QB_ERR_CUDA, "peer_buffer_create: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == QB_PEER_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *local = ptr;
  return QB_OK;
}

extern "C" int qb_peer_buffer_open(const unsigned char* handle, void** peer) {
  clear_error();
  if (handle == nullptr || peer == nullptr) return set_error(QB_ERR_INVALID, "peer_buffer_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* ptr = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(QB_ERR_CUDA, "peer_buffer_open: %s", cudaGetErrorString(e));
  *peer = ptr;
  return QB_OK;
}

extern "C" int qb_peer_buffer_close(void* peer) {
  clear_error();
  if (peer == nullptr) return QB_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(peer);
  if (e != cudaSuccess) return set_error(QB_ERR_CUDA, "peer_buffer_close: %s", cudaGetErrorString(e));
  return QB_OK;
}

extern "C" int qb_peer_buffer_destroy(void* local) {
  clear_error();
  if (local == nullptr) return QB_OK;
  const cudaError_t e = cudaFree(local);
  if (e != cudaSuccess) return set_error(QB_ERR_CUDA, "peer_buffer_destroy: %s", cudaGetErrorString(e));
  return QB_OK;
}

extern "C" int qb_colsum_allreduce(const qb_colsum_allreduce_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "colsum_allreduce: null argument block");
  const qb_colsum_allreduce_args& a = *args;
  if (a.num_buffers < 1 || a.num_buffers > 2 || a.partial0 == nullptr ||
      (a.num_buffers == 2 && a.partial1 == nullptr))
    return set_error(QB_ERR_INVALID, "colsum_allreduce: one or two partial buffers are required");
  if (a.P < 0 || a.cols <= 0) return set_error(QB_ERR_INVALID, "colsum_allreduce: bad sizes");
  if (a.world < 1 || a.world > QB_MAX_PEERS || a.rank < 0 || a.rank >= a.world)
    return set_error(QB_ERR_INVALID, "colsum_allreduce: bad rank %d of %d", a.rank, a.world);
  if (a.seq == 0) return set_error(QB_ERR_INVALID, "colsum_allreduce: step numbers start at 1");
  if (a.cap_cols <= 0 || a.cap_cols % 32 != 0 || a.cols * a.num_buffers > a.cap_cols)
    return set_error(QB_ERR_UNSUPPORTED, "colsum_allreduce: %lld columns exceed the exchange buffer (%lld)",
                     (long long)(a.cols * a.num_buffers), (long long)a.cap_cols);
  // every block waits for its peers' blocks, so all blocks of a launch have to be resident at
  // once: 1024 blocks of 256 threads fit any sm_100 part with room to spare
  if (a.cols * a.num_buffers > 32768)
    return set_error(QB_ERR_UNSUPPORTED, "colsum_allreduce: more than 32768 columns per launch");
  for (int r = 0; r < a.world; ++r)
    if (a.peers[r] == nullptr) return set_error(QB_ERR_INVALID, "colsum_allreduce: peer %d is not mapped", r);
  if ((a.out0 != nullptr || a.out1 != nullptr) && !is_float_dtype(a.out_dtype))
    return set_error(QB_ERR_INVALID, "colsum_allreduce: unsupported dtype code");
  PeerReduceParams p;
  p.a = a;
  dim3 grid(static_cast<unsigned>(ceil_div(a.cols * a.num_buffers, 32)), 1, 1);
  return launch_kernel(colsum_allreduce_kernel, grid, 256, 0, 1, reinterpret_cast<cudaStream_t>(stream), p,
                       "colsum_allreduce");
}
