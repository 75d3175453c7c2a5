// Top-k over the last dimension (optionally followed by a softmax over the k values), forward and
// backward, for sm_100a.
//
// Follows quack/topk.py:26-233 (TopK, forward), :275-460 (TopKBackward) and the bitonic networks
// of quack/sort/.  Contract of the forward: N and k powers of two, N <= 4096, k <= 128; values
// come back sorted in descending order with their int32 column indices.
//
// Forward design.  Every element becomes one integer key whose unsigned order is "larger value
// first, then smaller column": the order-preserving image of the value's bits in the high half,
// the complemented column in the low half (32-bit keys for 16-bit dtypes, 64-bit keys for fp32).
// Sorting keys therefore sorts (value, column) pairs exactly -- no mantissa bits are given up for
// the index -- and a compare-exchange is one max and one min.
//   * Register kernel: TPR <= 32 lanes share a row, each holding E >= k keys.  A lane sorts its
//     keys with a fully unrolled bitonic network, keeps the best K, and log2(TPR) shuffle rounds
//     merge the lanes' lists (max of my list and the partner's reversed list is a bitonic sequence
//     holding the best K of both; log2 K more compare-exchange stages sort it).  All lanes end up
//     with the same list.
//   * Shared-memory kernel: one CTA per row, the whole row of keys in shared memory, plain bitonic
//     sort.  Serves what does not fit the register budget (fp32 rows of more than 2048 elements or
//     k = 128).
// The backward writes every row of dx completely: zeros, then the k gradients scattered to their
// columns (through the softmax Jacobian if the forward applied one).
#include <type_traits>

#include "common.cuh"
#include "host_common.h"

namespace qb {

struct TopkFwdParams {
  qb_topk_fwd_args a;
  int k;
};

// ---- keys ----
__device__ __forceinline__ uint32_t ordered16(uint32_t b) {  // b: 16 value bits
  return (b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u);
}
__device__ __forceinline__ uint32_t unordered16(uint32_t o) {
  return (o & 0x8000u) ? (o ^ 0x8000u) : (~o & 0xffffu);
}
__device__ __forceinline__ uint32_t ordered32(uint32_t b) {
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ uint32_t unordered32(uint32_t o) {
  return (o & 0x80000000u) ? (o ^ 0x80000000u) : ~o;
}

template <class KT>
struct Key;
template <>
struct Key<uint32_t> {  // 16-bit dtypes
  static __device__ __forceinline__ uint32_t make(uint32_t bits, int col) {
    return (ordered16(bits) << 16) | (0xffffu - static_cast<uint32_t>(col));
  }
  static __device__ __forceinline__ uint32_t value_bits(uint32_t k) { return unordered16(k >> 16); }
  static __device__ __forceinline__ int column(uint32_t k) { return static_cast<int>(0xffffu - (k & 0xffffu)); }
  static __device__ __forceinline__ uint32_t shfl_xor(uint32_t k, int m) {
    return __shfl_xor_sync(0xffffffffu, k, m);
  }
};
template <>
struct Key<unsigned long long> {  // fp32
  static __device__ __forceinline__ unsigned long long make(uint32_t bits, int col) {
    return (static_cast<unsigned long long>(ordered32(bits)) << 32) |
           (0xffffffffu - static_cast<uint32_t>(col));
  }
  static __device__ __forceinline__ uint32_t value_bits(unsigned long long k) {
    return unordered32(static_cast<uint32_t>(k >> 32));
  }
  static __device__ __forceinline__ int column(unsigned long long k) {
    return static_cast<int>(0xffffffffu - static_cast<uint32_t>(k));
  }
  static __device__ __forceinline__ unsigned long long shfl_xor(unsigned long long k, int m) {
    return __shfl_xor_sync(0xffffffffu, k, m);
  }
};

// descending compare-exchange: afterwards a >= b
template <class KT>
__device__ __forceinline__ void cex(KT& a, KT& b) {
  const KT hi = a > b ? a : b;
  const KT lo = a > b ? b : a;
  a = hi;
  b = lo;
}

// Sorts v[0..E) in descending order (bitonic network, compile-time indices).
template <class KT, int E>
__device__ __forceinline__ void sort_desc(KT (&v)[E]) {
#pragma unroll
  for (int size = 2; size <= E; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          if ((i & size) == 0) cex(v[i], v[j]);  // descending block
          else cex(v[j], v[i]);                  // ascending block
        }
      }
    }
  }
}
// Sorts a bitonic sequence v[0..K) in descending order.
template <class KT, int K>
__device__ __forceinline__ void merge_desc(KT (&v)[K]) {
#pragma unroll
  for (int stride = K >> 1; stride > 0; stride >>= 1) {
#pragma unroll
    for (int i = 0; i < K; ++i)
      if ((i & stride) == 0) cex(v[i], v[i + stride]);
  }
}

__device__ __forceinline__ float bits_to_float(uint32_t bits, int dt) {
  if (dt == QB_F32) return __uint_as_float(bits);
  if (dt == QB_BF16) return __uint_as_float(bits << 16);
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
}
__device__ __forceinline__ void store_value(void* base, int64_t idx, float v, int dt) {
  if (dt == QB_F32) reinterpret_cast<float*>(base)[idx] = v;
  else if (dt == QB_BF16) reinterpret_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
  else reinterpret_cast<__half*>(base)[idx] = __float2half_rn(v);
}

// Writes the first k entries of a sorted key list: lane t of the row group writes entries
// t, t + TPR, ...  With softmax the k values are replaced by their softmax (fp32 arithmetic).
template <class KT, int K>
__device__ __forceinline__ void emit_topk(const KT (&v)[K], const qb_topk_fwd_args& a, int64_t row,
                                          int k, int t, int tpr) {
  float scale = 1.0f, off = 0.0f;
  if (a.softmax) {
    // values are sorted: the first one is the maximum
    const float m = bits_to_float(Key<KT>::value_bits(v[0]), a.x_dtype);
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < K; ++j)
      if (j < k) s += fast_exp2((bits_to_float(Key<KT>::value_bits(v[j]), a.x_dtype) - m) * kLog2e);
    scale = 1.0f / s;
    off = m;
  }
#pragma unroll
  for (int j = 0; j < K; ++j) {
    if (j < k && (j & (tpr - 1)) == t) {
      const float x = bits_to_float(Key<KT>::value_bits(v[j]), a.x_dtype);
      const float y = a.softmax ? fast_exp2((x - off) * kLog2e) * scale : x;
      store_value(a.values, row * k + j, y, a.x_dtype);
      a.indices[row * k + j] = Key<KT>::column(v[j]);
    }
  }
}

// KT: key type.  E: keys per lane (power of two).  K: list length kept per lane (k <= K <= E).
// TPR: lanes per row (power of two <= 32).
template <class KT, int E, int K, int TPR>
__global__ void __launch_bounds__(128) topk_reg_kernel(const TopkFwdParams p) {
  const qb_topk_fwd_args& a = p.a;
  constexpr int ROWS = 128 / TPR;
  const int t = threadIdx.x & (TPR - 1);
  const int64_t row = static_cast<int64_t>(blockIdx.x) * ROWS + threadIdx.x / TPR;
  const bool row_ok = row < a.M;  // lanes of rows past the end still take part in the shuffles
  constexpr bool WIDE = std::is_same<KT, unsigned long long>::value;
  constexpr int VEC = WIDE ? 4 : 8;            // elements per 16-byte chunk
  constexpr int CH = E >= VEC ? E / VEC : 1;   // 16-byte chunks per lane
  KT v[E];
  const char* xrow = reinterpret_cast<const char*>(a.x) + (row_ok ? row : 0) * a.x_row_stride * (WIDE ? 4 : 2);
  if constexpr (E >= VEC) {
    // chunk c of the row goes to lane c % TPR: coalesced 16-byte loads
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int chunk = c * TPR + t;
      uint32_t w[4];
      ldg_cached<16>(w, xrow + chunk * 16, row_ok);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const uint32_t bits = WIDE ? w[i] : ((i & 1) ? (w[i >> 1] >> 16) : (w[i >> 1] & 0xffffu));
        v[c * VEC + i] = Key<KT>::make(bits, chunk * VEC + i);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const int col = t * E + i;
      uint32_t bits = 0;
      if (row_ok) {
        if (WIDE) bits = reinterpret_cast<const uint32_t*>(xrow)[col];
        else bits = reinterpret_cast<const unsigned short*>(xrow)[col];
      }
      v[i] = Key<KT>::make(bits, col);
    }
  }
  sort_desc<KT, E>(v);
  KT top[K];
#pragma unroll
  for (int i = 0; i < K; ++i) top[i] = v[i];
  // merge the lanes' lists: after the round with mask m, groups of 2m lanes agree
#pragma unroll
  for (int m = 1; m < TPR; m <<= 1) {
    KT other[K];
#pragma unroll
    for (int i = 0; i < K; ++i) other[i] = Key<KT>::shfl_xor(top[K - 1 - i], m);
#pragma unroll
    for (int i = 0; i < K; ++i) top[i] = top[i] > other[i] ? top[i] : other[i];
    merge_desc<KT, K>(top);
  }
  if (row_ok) emit_topk<KT, K>(top, a, row, p.k, t, TPR);
}

// One CTA per row, keys in shared memory, plain bitonic sort; then the first k keys are written.
template <class KT>
__global__ void __launch_bounds__(512) topk_smem_kernel(const TopkFwdParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  KT* keys = reinterpret_cast<KT*>(smem_raw);
  const qb_topk_fwd_args& a = p.a;
  constexpr bool WIDE = std::is_same<KT, unsigned long long>::value;
  const int N = static_cast<int>(a.N);
  const int64_t row = blockIdx.x;
  const char* xrow = reinterpret_cast<const char*>(a.x) + row * a.x_row_stride * (WIDE ? 4 : 2);
  for (int c = threadIdx.x; c < N; c += blockDim.x) {
    const uint32_t bits = WIDE ? reinterpret_cast<const uint32_t*>(xrow)[c]
                               : reinterpret_cast<const unsigned short*>(xrow)[c];
    keys[c] = Key<KT>::make(bits, c);
  }
  for (int size = 2; size <= N; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int q = threadIdx.x; q < N / 2; q += blockDim.x) {
        const int i = ((q & ~(stride - 1)) << 1) | (q & (stride - 1));  // index with bit `stride` clear
        const int j = i | stride;
        KT x = keys[i], y = keys[j];
        const bool desc = (i & size) == 0;
        if ((x < y) == desc) { keys[i] = y; keys[j] = x; }
      }
    }
  }
  __syncthreads();
  // softmax over the first k values (one warp), then the stores
  float off = 0.0f, scale = 1.0f;
  if (a.softmax) {
    off = bits_to_float(Key<KT>::value_bits(keys[0]), a.x_dtype);
    float s = 0.0f;
    for (int j = threadIdx.x & 31; j < p.k; j += 32)
      s += fast_exp2((bits_to_float(Key<KT>::value_bits(keys[j]), a.x_dtype) - off) * kLog2e);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    scale = 1.0f / s;
  }
  for (int j = threadIdx.x; j < p.k; j += blockDim.x) {
    const float x = bits_to_float(Key<KT>::value_bits(keys[j]), a.x_dtype);
    const float y = a.softmax ? fast_exp2((x - off) * kLog2e) * scale : x;
    store_value(a.values, row * p.k + j, y, a.x_dtype);
    a.indices[row * p.k + j] = Key<KT>::column(keys[j]);
  }
}

// ---------------------------------------------------------------------------------------------
// backward: dx = scatter(indices, g), g = dvalues or values * (dvalues - sum(dvalues * values))
// ---------------------------------------------------------------------------------------------
struct TopkBwdParams {
  qb_topk_bwd_args a;
};

// One warp per row: zero the row (16-byte stores where the row allows), then scatter.
__global__ void __launch_bounds__(256) topk_bwd_kernel(const TopkBwdParams p) {
  const qb_topk_bwd_args& a = p.a;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= a.M) return;
  const int esz = a.dx_dtype == QB_F32 ? 4 : 2;
  char* drow = reinterpret_cast<char*>(a.dx) + row * a.dx_row_stride * esz;
  const int64_t row_bytes = a.N * esz;
  const uint32_t zero[4] = {0u, 0u, 0u, 0u};
  if ((reinterpret_cast<uintptr_t>(drow) & 15) == 0 && (row_bytes & 15) == 0) {
    for (int64_t b = lane * 16; b < row_bytes; b += 32 * 16) stg_stream<16>(drow + b, zero);
  } else {
    for (int64_t c = lane; c < a.N; c += 32) store_value(a.dx, row * a.dx_row_stride + c, 0.0f, a.dx_dtype);
  }
  float dot = 0.0f;
  if (a.softmax) {
    for (int j = lane; j < a.k; j += 32)
      dot += load_scalar(a.dvalues, row * a.k + j, a.dvalues_dtype) *
             load_scalar(a.values, row * a.k + j, a.values_dtype);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  }
  __syncwarp();  // the zeros of every lane come before the scattered values
  for (int j = lane; j < a.k; j += 32) {
    float g = load_scalar(a.dvalues, row * a.k + j, a.dvalues_dtype);
    if (a.softmax) g = load_scalar(a.values, row * a.k + j, a.values_dtype) * (g - dot);
    const int col = a.indices[row * a.k + j];
    if (col >= 0 && col < a.N) store_value(a.dx, row * a.dx_row_stride + col, g, a.dx_dtype);
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
template <class KT, int E, int K, int TPR>
static int launch_topk_reg_one(const TopkFwdParams& p, cudaStream_t st) {
  constexpr int rows = 128 / TPR;
  dim3 grid(static_cast<unsigned>(ceil_div(p.a.M, rows)), 1, 1);
  return launch_kernel(topk_reg_kernel<KT, E, K, TPR>, grid, 128, 0, 1, st, p, "topk_fwd");
}

// Full warps per row (N >= 32 k): E = N / 32 keys per lane, list length K = the smallest of E,
// E / 2, E / 4 that holds k (shorter requests keep E / 4 and write their first k).
template <class KT, int E>
static int launch_topk_warp(const TopkFwdParams& p, cudaStream_t st) {
  if constexpr (E >= 4) {
    if (p.k <= E / 4) return launch_topk_reg_one<KT, E, E / 4, 32>(p, st);
  }
  if constexpr (E >= 2) {
    if (p.k <= E / 2) return launch_topk_reg_one<KT, E, E / 2, 32>(p, st);
  }
  return launch_topk_reg_one<KT, E, E, 32>(p, st);
}

// Fewer than 32 lanes per row (N < 32 k): every lane holds E = next_pow2(k) keys.  Instantiated
// for k <= 32; the rare wider lists on short rows (N < 32 k with k = 64 or 128) take the
// shared-memory kernel.
template <class KT, int E>
static int launch_topk_sub(const TopkFwdParams& p, int tpr, cudaStream_t st) {
  if constexpr (E > 32) return QB_ERR_UNSUPPORTED;
  else switch (tpr) {
    case 1: return launch_topk_reg_one<KT, E, E, 1>(p, st);
    case 2: return launch_topk_reg_one<KT, E, E, 2>(p, st);
    case 4: return launch_topk_reg_one<KT, E, E, 4>(p, st);
    case 8: return launch_topk_reg_one<KT, E, E, 8>(p, st);
    case 16: return launch_topk_reg_one<KT, E, E, 16>(p, st);
  }
  return QB_ERR_UNSUPPORTED;
}

template <class KT>
static int launch_topk_reg(const TopkFwdParams& p, int e, int tpr, cudaStream_t st) {
  constexpr bool WIDE = std::is_same<KT, unsigned long long>::value;
#define QB_E(EE)                                                   \
  case EE:                                                         \
    return tpr == 32 ? launch_topk_warp<KT, EE>(p, st) : launch_topk_sub<KT, EE>(p, tpr, st);
  switch (e) {
    QB_E(1) QB_E(2) QB_E(4) QB_E(8) QB_E(16) QB_E(32) QB_E(64)
    case 128:
      if constexpr (!WIDE)
        return tpr == 32 ? launch_topk_warp<KT, 128>(p, st) : launch_topk_sub<KT, 128>(p, tpr, st);
  }
#undef QB_E
  return QB_ERR_UNSUPPORTED;
}

}  // namespace qb

using namespace qb;

extern "C" int qb_topk_fwd(const qb_topk_fwd_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "topk_fwd: null argument block");
  const qb_topk_fwd_args& a = *args;
  if (a.x == nullptr || a.values == nullptr || a.indices == nullptr)
    return set_error(QB_ERR_INVALID, "topk_fwd: x, values and indices are required");
  if (!is_float_dtype(a.x_dtype)) return set_error(QB_ERR_INVALID, "topk_fwd: unsupported dtype code");
  if (a.M < 0 || a.N <= 0 || a.k <= 0 || a.k > a.N)
    return set_error(QB_ERR_INVALID, "topk_fwd: bad sizes M=%lld N=%lld k=%lld", (long long)a.M,
                     (long long)a.N, (long long)a.k);
  if (!is_pow2(a.N) || a.N > 4096 || a.k > 128)
    return set_error(QB_ERR_UNSUPPORTED,
                     "topk_fwd: N must be a power of two <= 4096 and k <= 128 (got N=%lld, k=%lld)",
                     (long long)a.N, (long long)a.k);
  if (a.M == 0) return QB_OK;
  const bool wide = a.x_dtype == QB_F32;
  const int esz = wide ? 4 : 2;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  TopkFwdParams p;
  p.a = a;
  p.k = static_cast<int>(a.k);
  // Register kernel: E = max(next_pow2(k), N / 32) keys per lane on TPR = N / E lanes, while the
  // keys fit the register budget (128 32-bit registers) and the rows can be read in 16-byte chunks.
  const int kp = next_pow2(a.k);
  int e = static_cast<int>(a.N / 32);
  if (e < kp) e = kp;
  const int tpr = static_cast<int>(a.N / e);
  const bool aligned = (reinterpret_cast<uintptr_t>(a.x) % 16) == 0 && (a.x_row_stride * esz) % 16 == 0;
  if (e * (wide ? 2 : 1) <= 128 && tpr >= 1 && (aligned || e < 16 / esz)) {
    const int rc = wide ? launch_topk_reg<unsigned long long>(p, e, tpr, st)
                        : launch_topk_reg<uint32_t>(p, e, tpr, st);
    if (rc != QB_ERR_UNSUPPORTED) return rc;
    clear_error();
  }
  const int threads = a.N / 2 >= 512 ? 512 : (a.N / 2 >= 32 ? static_cast<int>(a.N / 2) : 32);
  dim3 grid(static_cast<unsigned>(a.M), 1, 1);
  const size_t smem = static_cast<size_t>(a.N) * (wide ? 8 : 4);
  if (wide) return launch_kernel(topk_smem_kernel<unsigned long long>, grid, threads, smem, 1, st, p, "topk_fwd");
  return launch_kernel(topk_smem_kernel<uint32_t>, grid, threads, smem, 1, st, p, "topk_fwd");
}

extern "C" int qb_topk_bwd(const qb_topk_bwd_args* args, qb_stream_t stream) {
  clear_error();
  if (args == nullptr) return set_error(QB_ERR_INVALID, "topk_bwd: null argument block");
  const qb_topk_bwd_args& a = *args;
  if (a.dvalues == nullptr || a.indices == nullptr || a.dx == nullptr)
    return set_error(QB_ERR_INVALID, "topk_bwd: dvalues, indices and dx are required");
  if (a.softmax && a.values == nullptr)
    return set_error(QB_ERR_INVALID, "topk_bwd: the softmax backward needs the forward's values");
  if (!is_float_dtype(a.dvalues_dtype) || !is_float_dtype(a.dx_dtype) ||
      (a.values && !is_float_dtype(a.values_dtype)))
    return set_error(QB_ERR_INVALID, "topk_bwd: unsupported dtype code");
  if (a.M < 0 || a.N <= 0 || a.k <= 0 || a.k > a.N)
    return set_error(QB_ERR_INVALID, "topk_bwd: bad sizes M=%lld N=%lld k=%lld", (long long)a.M,
                     (long long)a.N, (long long)a.k);
  if (a.M == 0) return QB_OK;
  TopkBwdParams p;
  p.a = a;
  dim3 grid(static_cast<unsigned>(ceil_div(a.M, 8)), 1, 1);
  return launch_kernel(topk_bwd_kernel, grid, 256, 0, 1, reinterpret_cast<cudaStream_t>(stream), p,
                       "topk_bwd");
}
