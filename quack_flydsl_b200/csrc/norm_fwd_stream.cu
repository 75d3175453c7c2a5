// RMSNorm / LayerNorm forward for long rows (sm_100a): the streamed two-pass kernels.
// A translation unit of its own so that it compiles in parallel with the register kernels.
#include <type_traits>

#include "common.cuh"
#include "norm_fwd.h"

namespace qb {

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
// ---------------------------------------------------------------------------------------------
// Long rows: two streamed passes per row with the row parked in L2 between them
// ---------------------------------------------------------------------------------------------
// One CTA owns a whole row, however long, and reads it twice: pass 1 streams it from HBM for the
// row statistics (and writes residual_out), pass 2 re-reads it -- newest lines first, from L2 --
// normalises and writes the output.  HBM sees each element once in each direction, no CTA waits
// for another one, and nothing depends on the row fitting into registers.  LayerNorm statistics
// are one-pass but not the naive sum of squares: every block of a thread's chunks yields its own
// (mean, sum of squared deviations), merged pairwise (Chan et al.), then across threads by two
// row reductions -- as robust against a large common offset as the two-pass register kernel.
// DT: the dtype of x / residual / out / residual_out (16-byte chunks); RES: a residual is added;
// T threads per CTA (== blockDim.x); WSAME: weight and bias have dtype DT too (else run-time dtypes).
template <int DT, bool LN, bool RES, int T, bool WSAME>
__global__ void __launch_bounds__(T, 512 / T) norm_fwd_stream_kernel(const NormFwdParams p) {
  static_assert(DT == QB_F32 || DT == QB_F16 || DT == QB_BF16, "concrete dtype required");
  constexpr int VEC = DT == QB_F32 ? 4 : 8;
  // 512 threads per SM with up to 128 registers each: 12 chunks (192 bytes) in flight per thread.
  constexpr int U1 = RES ? 6 : 12;  // chunks in flight per thread and input, pass 1
  constexpr int U2 = (WSAME ? 4 : 2);  // pass 2: x, weight and bias chunks all in flight
  constexpr int kStep = T * 16;
  __shared__ ReduceScratch scratch;
  const qb_norm_fwd_args& a = p.a;
  const RowGeom g = make_geom(T, 1);
  const int N = static_cast<int>(a.N);
  const int nchunks = N / VEC;
  const float inv_n = 1.0f / static_cast<float>(N);
  const uint64_t keep = l2_policy((p.flags & 4) ? 2 : 0);
  const uint64_t drop = l2_policy((p.flags & 8) ? 2 : 1);
  const bool has_w = a.weight != nullptr, has_b = a.bias != nullptr;
  int rit = 0;
  for (int64_t row = blockIdx.x; row < a.M; row += gridDim.x) {
    const char* xin = reinterpret_cast<const char*>(a.x) + (row * a.x_row_stride * (16 / VEC) + g.t * 16);
    const char* rin = RES ? reinterpret_cast<const char*>(a.residual) +
                                (row * a.residual_row_stride * (16 / VEC) + g.t * 16)
                          : nullptr;
    char* out = reinterpret_cast<char*>(a.out) + (row * a.out_row_stride * (16 / VEC) + g.t * 16);
    char* rout = a.residual_out != nullptr
                     ? reinterpret_cast<char*>(a.residual_out) +
                           (row * a.residual_out_row_stride * (16 / VEC) + g.t * 16)
                     : nullptr;

    // ---- pass 1: statistics (and residual_out) ----
    // The block stays packed in registers; every use unpacks (and adds the residual) again.
    float ssq = 0.0f, ssq2 = 0.0f;                 // RMSNorm: sum of squares (two chains)
    float cnt = 0.0f, mu = 0.0f, m2 = 0.0f;        // LayerNorm: running count, mean, sum sq. dev.
    auto pass1 = [&](auto full_tag, int c0) {
      constexpr bool FULL = decltype(full_tag)::value;
      uint32_t rx[U1][4];
      uint32_t rr[RES ? U1 : 1][4];
      const int64_t off = static_cast<int64_t>(c0 - g.t) * 16;
#pragma unroll
      for (int u = 0; u < U1; ++u) ldg16_hint<!FULL>(rx[u], xin + off + u * kStep, c0 + u * T < nchunks, keep);
      if constexpr (RES) {
#pragma unroll
        for (int u = 0; u < U1; ++u) ldg16_hint<!FULL>(rr[u], rin + off + u * kStep, c0 + u * T < nchunks, keep);
      }
      auto value = [&](float (&h)[VEC], int u) {
        unpack_chunk<DT, VEC>(h, rx[u], DT);
        if constexpr (RES) {
          float r[VEC];
          unpack_chunk<DT, VEC>(r, rr[u], DT);
          vadd<VEC>(h, h, r);
        }
      };
      float bsum = 0.0f, bsum2 = 0.0f;
      int nb = 0;
#pragma unroll
      for (int u = 0; u < U1; ++u) {
        float h[VEC];
        value(h, u);
        const bool here = FULL || c0 + u * T < nchunks;
        if (rout != nullptr && here) store_chunk_p<DT, VEC>(rout + off + u * kStep, h, DT);
        if constexpr (LN) {
          if (here) {
#pragma unroll
            for (int i = 0; i < VEC; i += 2) { bsum += h[i]; bsum2 += h[i + 1]; }
            nb += VEC;
          }
        } else {
#pragma unroll
          for (int i = 0; i < VEC; i += 2) {  // padding chunks are zeros
            ssq = fmaf(h[i], h[i], ssq);
            ssq2 = fmaf(h[i + 1], h[i + 1], ssq2);
          }
        }
      }
      if constexpr (LN) {
        if (nb > 0) {
          const float fnb = static_cast<float>(nb);
          const float bmean = (bsum + bsum2) / fnb;
          float bm2 = 0.0f, bm2b = 0.0f;
#pragma unroll
          for (int u = 0; u < U1; ++u) {
            if (FULL || c0 + u * T < nchunks) {
              float d[VEC];
              forget_values(rx[u]);
              if constexpr (RES) forget_values(rr[u]);
              value(d, u);
#pragma unroll
              for (int i = 0; i < VEC; i += 2) {
                const float e0 = d[i] - bmean, e1 = d[i + 1] - bmean;
                bm2 = fmaf(e0, e0, bm2);
                bm2b = fmaf(e1, e1, bm2b);
              }
            }
          }
          const float tot = cnt + fnb;
          const float delta = bmean - mu;
          mu += delta * (fnb / tot);
          m2 += (bm2 + bm2b) + delta * delta * (cnt * fnb / tot);
          cnt = tot;
        }
      }
    };
    {
      const int nfull = nchunks / (T * U1);
      for (int b = 0; b < nfull; ++b) pass1(std::true_type{}, b * (T * U1) + g.t);
      if (nfull * (T * U1) < nchunks) pass1(std::false_type{}, nfull * (T * U1) + g.t);
    }
    float rstd, mean = 0.0f;
    if constexpr (LN) {
      // mean = sum(cnt_t * mu_t) / N;  M2 = sum(m2_t + cnt_t * (mu_t - mean)^2)
      const float2 r1 = row_reduce<SumOp>(make_float2(cnt * mu, 0.0f), g, scratch, 0, rit);
      mean = r1.x * inv_n;
      const float dm = mu - mean;
      const float2 r2 = row_reduce<SumOp>(make_float2(m2 + cnt * dm * dm, 0.0f), g, scratch, 1, rit);
      rstd = rsqrtf(r2.x * inv_n + a.eps);
    } else {
      const float2 r1 = row_reduce<SumOp>(make_float2(ssq + ssq2, 0.0f), g, scratch, 0, rit);
      rstd = rsqrtf(r1.x * inv_n + a.eps);
    }
    ++rit;
    if (g.t == 0) {
      if (a.rstd != nullptr) a.rstd[row] = rstd;
      if (LN && a.mean != nullptr) a.mean[row] = mean;
    }
    const float shift = -mean * rstd;

    // ---- pass 2: y = ((x [+ res]) * rstd - mean * rstd) * (w + offset) + b ----
    auto pass2 = [&](auto full_tag, int c0) {
      constexpr bool FULL = decltype(full_tag)::value;
      constexpr int WDT = WSAME ? DT : kDynDT;
      constexpr int kW = RawWords<WDT, VEC>::value;
      uint32_t rx[U2][4];
      uint32_t rr[RES ? U2 : 1][4];
      uint32_t rw[U2][kW], rb[U2][kW];
      const int64_t off = static_cast<int64_t>(c0 - g.t) * 16;
#pragma unroll
      for (int u = 0; u < U2; ++u) ldg16_hint<!FULL>(rx[u], xin + off + u * kStep, c0 + u * T < nchunks, drop);
      if constexpr (RES) {
#pragma unroll
        for (int u = 0; u < U2; ++u) ldg16_hint<!FULL>(rr[u], rin + off + u * kStep, c0 + u * T < nchunks, drop);
      }
      // weight / bias chunks of these columns (L1 / L2 resident), all issued before the first use
#pragma unroll
      for (int u = 0; u < U2; ++u) {
        const bool here = FULL || c0 + u * T < nchunks;
        const int64_t col = static_cast<int64_t>(c0 + u * T) * VEC;
        if (has_w) load_chunk_raw<WDT, VEC, false>(rw[u], a.weight, col, a.weight_dtype, here);
        if (has_b) load_chunk_raw<WDT, VEC, false>(rb[u], a.bias, col, a.bias_dtype, here);
      }
#pragma unroll
      for (int u = 0; u < U2; ++u) {
        float h[VEC], y[VEC];
        unpack_chunk<DT, VEC>(h, rx[u], DT);
        if constexpr (RES) {
          float r[VEC];
          unpack_chunk<DT, VEC>(r, rr[u], DT);
          vadd<VEC>(h, h, r);
        }
        vfma_ss<VEC>(y, h, rstd, shift);
        if (has_w) {
          float we[VEC];
          unpack_chunk<WDT, VEC>(we, rw[u], a.weight_dtype);
          vadd_s<VEC>(we, we, a.weight_offset);
          if (has_b) {
            float bb[VEC];
            unpack_chunk<WDT, VEC>(bb, rb[u], a.bias_dtype);
            vfma<VEC>(y, y, we, bb);
          } else {
            vmul<VEC>(y, y, we);
          }
        } else if (has_b) {
          float bb[VEC];
          unpack_chunk<WDT, VEC>(bb, rb[u], a.bias_dtype);
          vadd<VEC>(y, y, bb);
        }
        if (FULL || c0 + u * T < nchunks) store_chunk_p<DT, VEC>(out + off + u * kStep, y, DT);
      }
    };
    {
      const int nfull = nchunks / (T * U2);
      if (nfull * (T * U2) < nchunks) pass2(std::false_type{}, nfull * (T * U2) + g.t);
      for (int b = nfull - 1; b >= 0; --b) pass2(std::true_type{}, b * (T * U2) + g.t);
    }
  }
}

template <int DT, bool LN, bool RES, int T, bool WSAME>
static int launch_norm_fwd_stream_w(const NormFwdParams& p, const DeviceFacts* dev, cudaStream_t st) {
  auto kernel = norm_fwd_stream_kernel<DT, LN, RES, T, WSAME>;
  const int occ = cached_occupancy(reinterpret_cast<const void*>(kernel), T, 0);
  int64_t ctas = static_cast<int64_t>(dev->sm_count) * (occ > 0 ? occ : 1);
  if (p.a.cfg.max_ctas > 0) ctas = p.a.cfg.max_ctas;
  if (ctas > p.a.M) ctas = p.a.M;
  // Evict-last marking in pass 1 only while the rows in flight fit comfortably in L2.
  NormFwdParams q = p;
  const int64_t in_flight = ctas * p.a.N * host_dtype_bytes(p.a.x_dtype) * (RES ? 2 : 1);
  if (in_flight > (48LL << 20)) q.flags |= 4;
  dim3 grid(static_cast<unsigned>(ctas), 1, 1);
  return launch_kernel(kernel, grid, T, 0, 1, st, q, LN ? "layernorm_fwd (streamed)" : "rmsnorm_fwd (streamed)");
}

template <int DT, bool LN, bool RES, int T>
static int launch_norm_fwd_stream_t(const NormFwdParams& p, const DeviceFacts* dev, cudaStream_t st) {
  // weight and bias in the dtype of x (or absent): typed 16-byte parameter loads
  const bool wsame = (p.a.weight == nullptr || p.a.weight_dtype == DT) &&
                     (p.a.bias == nullptr || p.a.bias_dtype == DT);
  if (wsame) return launch_norm_fwd_stream_w<DT, LN, RES, T, true>(p, dev, st);
  return launch_norm_fwd_stream_w<DT, LN, RES, T, false>(p, dev, st);
}

template <int DT, bool LN, bool RES>
static int launch_norm_fwd_stream_r(const NormFwdParams& p, int threads, const DeviceFacts* dev,
                                    cudaStream_t st) {
  switch (threads) {
    case 256: return launch_norm_fwd_stream_t<DT, LN, RES, 256>(p, dev, st);
    case 512: return launch_norm_fwd_stream_t<DT, LN, RES, 512>(p, dev, st);
    default:
      return set_error(QB_ERR_INVALID, "norm_fwd (streamed): num_threads must be 256 or 512");
  }
}

template <int DT>
static int launch_norm_fwd_stream(const NormFwdParams& p, int threads, const DeviceFacts* dev,
                                  cudaStream_t st) {
  const bool ln = p.a.is_layernorm != 0, res = p.a.residual != nullptr;
  if (ln) return res ? launch_norm_fwd_stream_r<DT, true, true>(p, threads, dev, st)
                     : launch_norm_fwd_stream_r<DT, true, false>(p, threads, dev, st);
  return res ? launch_norm_fwd_stream_r<DT, false, true>(p, threads, dev, st)
             : launch_norm_fwd_stream_r<DT, false, false>(p, threads, dev, st);
}

int launch_norm_fwd_stream_any(const NormFwdParams& p, int threads, const DeviceFacts* dev,
                               cudaStream_t st) {
  switch (p.a.x_dtype) {
    case QB_BF16: return launch_norm_fwd_stream<QB_BF16>(p, threads, dev, st);
    case QB_F16: return launch_norm_fwd_stream<QB_F16>(p, threads, dev, st);
    default: return launch_norm_fwd_stream<QB_F32>(p, threads, dev, st);
  }
}

}  // namespace qb
