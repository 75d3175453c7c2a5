// Device-side building blocks shared by the row-reduction kernels: dtype-generic vector
// loads/stores (<= 128 bit, streaming cache hints), cp.async staging, warp / block / cluster
// reductions through shuffles, shared memory and distributed shared memory, and fast math.
//
// Role in the reference: quack/reduce.py:20-324 (warp_reduce, block_reduce, cluster_reduce,
// row_reduce, online_softmax_reduce), quack/reduction_base.py:12-94 (tile geometry, reduction
// buffers, cluster init), quack/utils.py:27-58 (remote shared-memory store) and
// quack/copy_utils.py:226-315 (vectorised predicated copies).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "quack_b200.h"

namespace qb {

constexpr int kDynDT = -1;  // template dtype code: read the dtype at run time
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__host__ __device__ __forceinline__ int dtype_bytes(int dt) { return dt == QB_F32 ? 4 : 2; }

// ---------------------------------------------------------------------------------------------
// math
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }

// exp2 offset for a running maximum m, split so that 2^(x*log2e + hi) * 2^lo == exp(x - m)
// up to the rounding of one fused multiply-add.
struct ExpOffset {
  float hi, lo;
};
__device__ __forceinline__ ExpOffset exp_offset(float m) {
  ExpOffset o;
  if (m == neg_inf()) {
    o.hi = 0.0f;
    o.lo = 0.0f;
  } else {
    o.hi = -m * kLog2e;
    o.lo = fmaf(-m, kLog2e, -o.hi);
  }
  return o;
}


// ---------------------------------------------------------------------------------------------
// raw global / shared memory access of 2, 4, 8 or 16 bytes
// ---------------------------------------------------------------------------------------------
// Cache policy of the streaming accesses.  Every large tensor on this path is read once and
// written once, so the default is the evict-first "cache streaming" policy.  The loads are
// ordinary coherent loads (no .nc), so a kernel may overwrite its own input in place.
#ifndef QB_LDG_MOD
#define QB_LDG_MOD ".cs"
#endif
#ifndef QB_STG_MOD
#define QB_STG_MOD ".cs"
#endif

// Predicated streaming load of BYTES bytes; the words read as zero when pred is false and the
// address is then not dereferenced.  Written in PTX so that a row's loads form straight-line
// code (no branch per chunk) and can all be in flight together.
template <int BYTES>
__device__ __forceinline__ void ldg_stream(uint32_t* w, const void* p,
                                           bool pred = true) {
  const uint32_t pr = pred ? 1u : 0u;
  if constexpr (BYTES == 16) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t"
        "mov.u32 %0, 0;\n\tmov.u32 %1, 0;\n\tmov.u32 %2, 0;\n\tmov.u32 %3, 0;\n\t"
        "@q ld.global" QB_LDG_MOD ".v4.u32 {%0, %1, %2, %3}, [%4];\n\t}"
        : "=&r"(w[0]), "=&r"(w[1]), "=&r"(w[2]), "=&r"(w[3])
        : "l"(p), "r"(pr)
        : "memory");
  } else if constexpr (BYTES == 8) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %3, 0;\n\t"
        "mov.u32 %0, 0;\n\tmov.u32 %1, 0;\n\t"
        "@q ld.global" QB_LDG_MOD ".v2.u32 {%0, %1}, [%2];\n\t}"
        : "=&r"(w[0]), "=&r"(w[1])
        : "l"(p), "r"(pr)
        : "memory");
  } else if constexpr (BYTES == 4) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t"
        "mov.u32 %0, 0;\n\t"
        "@q ld.global" QB_LDG_MOD ".u32 %0, [%1];\n\t}"
        : "=&r"(w[0])
        : "l"(p), "r"(pr)
        : "memory");
  } else {
    static_assert(BYTES == 2, "unsupported access width");
    asm volatile(
        "{\n\t.reg .pred q;\n\t.reg .b16 h;\n\tsetp.ne.b32 q, %2, 0;\n\t"
        "mov.b16 h, 0;\n\t"
        "@q ld.global" QB_LDG_MOD ".u16 h, [%1];\n\t"
        "cvt.u32.u16 %0, h;\n\t}"
        : "=&r"(w[0])
        : "l"(p), "r"(pr)
        : "memory");
  }
}

// L2 cache policies for kernels that read a row twice (kind 0: evict last, 1: evict first,
// 2: evict normal), and a 16-byte load that carries one.  PRED: predicated with zero fill, else
// unconditional.
__device__ __forceinline__ uint64_t l2_policy(int kind) {
  uint64_t pol;
  if (kind == 0) asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  else if (kind == 1) asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  else asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
template <bool PRED>
__device__ __forceinline__ void ldg16_hint(uint32_t* w, const void* ptr, bool pred, uint64_t pol) {
  if constexpr (PRED) {
    const uint32_t pr = pred ? 1u : 0u;
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t"
        "mov.u32 %0, 0;\n\tmov.u32 %1, 0;\n\tmov.u32 %2, 0;\n\tmov.u32 %3, 0;\n\t"
        "@q ld.global.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %6;\n\t}"
        : "=&r"(w[0]), "=&r"(w[1]), "=&r"(w[2]), "=&r"(w[3])
        : "l"(ptr), "r"(pr), "l"(pol)
        : "memory");
  } else {
    asm volatile("ld.global.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                 : "l"(ptr), "l"(pol)
                 : "memory");
  }
}

// Predicated cached load (read-only path, default policy) for the small tensors that every CTA
// re-reads: weight and bias.
template <int BYTES>
__device__ __forceinline__ void ldg_cached(uint32_t* w, const void* p,
                                           bool pred = true) {
  const uint32_t pr = pred ? 1u : 0u;
  if constexpr (BYTES == 16) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t"
        "mov.u32 %0, 0;\n\tmov.u32 %1, 0;\n\tmov.u32 %2, 0;\n\tmov.u32 %3, 0;\n\t"
        "@q ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];\n\t}"
        : "=&r"(w[0]), "=&r"(w[1]), "=&r"(w[2]), "=&r"(w[3])
        : "l"(p), "r"(pr));
  } else if constexpr (BYTES == 8) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %3, 0;\n\t"
        "mov.u32 %0, 0;\n\tmov.u32 %1, 0;\n\t"
        "@q ld.global.nc.v2.u32 {%0, %1}, [%2];\n\t}"
        : "=&r"(w[0]), "=&r"(w[1])
        : "l"(p), "r"(pr));
  } else if constexpr (BYTES == 4) {
    asm volatile(
        "{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t"
        "mov.u32 %0, 0;\n\t"
        "@q ld.global.nc.u32 %0, [%1];\n\t}"
        : "=&r"(w[0])
        : "l"(p), "r"(pr));
  } else {
    static_assert(BYTES == 2, "unsupported access width");
    asm volatile(
        "{\n\t.reg .pred q;\n\t.reg .b16 h;\n\tsetp.ne.b32 q, %2, 0;\n\t"
        "mov.b16 h, 0;\n\t"
        "@q ld.global.nc.u16 h, [%1];\n\t"
        "cvt.u32.u16 %0, h;\n\t}"
        : "=&r"(w[0])
        : "l"(p), "r"(pr));
  }
}

// Unpredicated form of ldg_stream: no zero fill (four moves) and no predicate set-up per load.
// For the common case that every chunk of a thread's row exists.
template <int BYTES>
__device__ __forceinline__ void ldg_stream_full(uint32_t* w, const void* p) {
  if constexpr (BYTES == 16) {
    asm volatile("ld.global" QB_LDG_MOD ".v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                 : "l"(p)
                 : "memory");
  } else if constexpr (BYTES == 8) {
    asm volatile("ld.global" QB_LDG_MOD ".v2.u32 {%0, %1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "l"(p) : "memory");
  } else {
    ldg_stream<BYTES>(w, p, true);
  }
}

template <int BYTES>
__device__ __forceinline__ void stg_stream(void* p, const uint32_t* w) {
  if constexpr (BYTES == 16) {
    asm volatile("st.global" QB_STG_MOD ".v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(w[0]),
                 "r"(w[1]), "r"(w[2]), "r"(w[3])
                 : "memory");
  } else if constexpr (BYTES == 8) {
    asm volatile("st.global" QB_STG_MOD ".v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(w[0]), "r"(w[1])
                 : "memory");
  } else if constexpr (BYTES == 4) {
    asm volatile("st.global" QB_STG_MOD ".u32 [%0], %1;" ::"l"(p), "r"(w[0]) : "memory");
  } else {
    static_assert(BYTES == 2, "unsupported access width");
    asm volatile("{\n\t.reg .b16 h;\n\tcvt.u16.u32 h, %1;\n\tst.global" QB_STG_MOD
                 ".u16 [%0], h;\n\t}" ::"l"(p), "r"(w[0])
                 : "memory");
  }
}

template <int BYTES>
__device__ __forceinline__ void lds_raw(uint32_t* w, const void* p) {
  if constexpr (BYTES == 16) {
    uint4 v = *reinterpret_cast<const uint4*>(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (BYTES == 8) {
    uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x; w[1] = v.y;
  } else if constexpr (BYTES == 4) {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  } else {
    static_assert(BYTES == 2, "unsupported access width");
    w[0] = *reinterpret_cast<const unsigned short*>(p);
  }
}

// Asynchronous global -> shared copy (LDGSTS).  4/8/16 bytes go through cp.async; a 2-byte
// element (scalar path of a 16-bit tensor) has no cp.async form and is copied synchronously.
// A thread only ever reads back bytes it copied itself, so cp.async.wait_group is the only
// synchronisation needed.
template <int BYTES>
__device__ __forceinline__ void cp_async_g2s(void* smem_dst, const void* gmem_src) {
  if constexpr (BYTES == 2) {
    uint32_t w[1];
    ldg_stream<2>(w, gmem_src);
    *reinterpret_cast<unsigned short*>(smem_dst) = static_cast<unsigned short>(w[0]);
  } else {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    if constexpr (BYTES == 16) {
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem_src) : "memory");
    } else if constexpr (BYTES == 8) {
      asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(gmem_src) : "memory");
    } else {
      static_assert(BYTES == 4, "unsupported access width");
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem_src) : "memory");
    }
  }
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------------------------
// dtype conversion of packed words
// ---------------------------------------------------------------------------------------------
// Number of 32-bit words a chunk of VEC elements occupies for dtype code DT (kDynDT: worst case).
template <int DT, int VEC>
struct RawWords {
  static constexpr int value = (DT == QB_F32 || DT == kDynDT) ? VEC : (VEC + 1) / 2;
};

template <int VEC>
__device__ __forceinline__ void unpack16(float (&v)[VEC], const uint32_t* w, bool is_bf16) {
  if constexpr (VEC == 1) {
    const unsigned short u = static_cast<unsigned short>(w[0]);
    v[0] = is_bf16 ? __uint_as_float(static_cast<uint32_t>(u) << 16)
                   : __half2float(__ushort_as_half(u));
  } else {
    if (is_bf16) {
#pragma unroll
      for (int i = 0; i < VEC / 2; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    } else {
#pragma unroll
      for (int i = 0; i < VEC / 2; ++i) {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
        const float2 f = __half22float2(h);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    }
  }
}

template <int VEC>
__device__ __forceinline__ void pack16(uint32_t* w, const float (&v)[VEC], bool is_bf16) {
  if constexpr (VEC == 1) {
    w[0] = is_bf16 ? static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v[0])))
                   : static_cast<uint32_t>(__half_as_ushort(__float2half_rn(v[0])));
  } else {
    if (is_bf16) {
#pragma unroll
      for (int i = 0; i < VEC / 2; ++i) {
        const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&b);
      }
    } else {
#pragma unroll
      for (int i = 0; i < VEC / 2; ++i) {
        const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
  }
}

// Makes the compiler forget what it knows about the raw words of a chunk (no instruction is
// emitted).  Kernels that keep a row packed and unpack it once per pass call this before each
// repeated unpack: otherwise common-subexpression elimination keeps the unpacked fp32 values of
// the first pass alive in registers, which defeats the purpose of keeping the row packed.
template <int WORDS>
__device__ __forceinline__ void forget_values(uint32_t (&w)[WORDS]) {
#pragma unroll
  for (int i = 0; i < WORDS; ++i) asm volatile("" : "+r"(w[i]));
}

// Unpack a raw chunk (as loaded from memory) to fp32.  DT is the compile-time dtype or kDynDT,
// in which case the run-time code dt decides (a kernel-uniform branch).
template <int DT, int VEC>
__device__ __forceinline__ void unpack_chunk(float (&v)[VEC], const uint32_t* w, int dt) {
  const int d = (DT == kDynDT) ? dt : DT;
  if (d == QB_F32) {
#pragma unroll
    for (int i = 0; i < VEC; ++i) v[i] = __uint_as_float(w[i]);
  } else {
    unpack16<VEC>(v, w, d == QB_BF16);
  }
}

// Maximum of the VEC packed 16-bit elements of a raw chunk (exact: the maximum of bf16 / fp16
// values is one of them), without unpacking every element.
template <int DT, int VEC>
__device__ __forceinline__ float packed_max16(const uint32_t* w) {
  static_assert(VEC >= 2 && (DT == QB_BF16 || DT == QB_F16), "packed 16-bit chunks only");
  if constexpr (DT == QB_BF16) {
    __nv_bfloat162 m = *reinterpret_cast<const __nv_bfloat162*>(&w[0]);
#pragma unroll
    for (int i = 1; i < VEC / 2; ++i) m = __hmax2(m, *reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    return fmaxf(__low2float(m), __high2float(m));
  } else {
    __half2 m = *reinterpret_cast<const __half2*>(&w[0]);
#pragma unroll
    for (int i = 1; i < VEC / 2; ++i) m = __hmax2(m, *reinterpret_cast<const __half2*>(&w[i]));
    return fmaxf(__low2float(m), __high2float(m));
  }
}

// The packed fp32x2 instructions of sm_100 (fma.rn.f32x2 ...) are used for the element-wise
// arithmetic.  Measured on B200 (LayerNorm forward and RMSNorm backward, bf16) they remove about
// 11 % of the executed warp instructions and 5 % of the run time compared with scalar fp32.
#ifndef QB_USE_F32X2
#define QB_USE_F32X2 1
#endif
// Element-wise helpers on VEC-wide register arrays (optionally through the packed fp32x2
// instructions, see QB_USE_F32X2).
template <int VEC>
__device__ __forceinline__ void vmul(float (&o)[VEC], const float (&a)[VEC], const float (&b)[VEC]) {
  if constexpr (VEC >= 2 && QB_USE_F32X2) {
#pragma unroll
    for (int i = 0; i < VEC; i += 2) {
      const float2 r = __fmul2_rn(make_float2(a[i], a[i + 1]), make_float2(b[i], b[i + 1]));
      o[i] = r.x; o[i + 1] = r.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) o[i] = a[i] * b[i];
  }
}
// o = a * b + c
template <int VEC>
__device__ __forceinline__ void vfma(float (&o)[VEC], const float (&a)[VEC], const float (&b)[VEC],
                                     const float (&c)[VEC]) {
  if constexpr (VEC >= 2 && QB_USE_F32X2) {
#pragma unroll
    for (int i = 0; i < VEC; i += 2) {
      const float2 r = __ffma2_rn(make_float2(a[i], a[i + 1]), make_float2(b[i], b[i + 1]),
                                  make_float2(c[i], c[i + 1]));
      o[i] = r.x; o[i + 1] = r.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) o[i] = fmaf(a[i], b[i], c[i]);
  }
}
// o = a * s + c with a scalar s
template <int VEC>
__device__ __forceinline__ void vfma_s(float (&o)[VEC], const float (&a)[VEC], float s,
                                       const float (&c)[VEC]) {
  if constexpr (VEC >= 2 && QB_USE_F32X2) {
    const float2 s2 = make_float2(s, s);
#pragma unroll
    for (int i = 0; i < VEC; i += 2) {
      const float2 r = __ffma2_rn(make_float2(a[i], a[i + 1]), s2, make_float2(c[i], c[i + 1]));
      o[i] = r.x; o[i + 1] = r.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) o[i] = fmaf(a[i], s, c[i]);
  }
}
// o = a * s + t with scalars s, t
template <int VEC>
__device__ __forceinline__ void vfma_ss(float (&o)[VEC], const float (&a)[VEC], float s, float t) {
  if constexpr (VEC >= 2 && QB_USE_F32X2) {
    const float2 s2 = make_float2(s, s), t2 = make_float2(t, t);
#pragma unroll
    for (int i = 0; i < VEC; i += 2) {
      const float2 r = __ffma2_rn(make_float2(a[i], a[i + 1]), s2, t2);
      o[i] = r.x; o[i + 1] = r.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) o[i] = fmaf(a[i], s, t);
  }
}
template <int VEC>
__device__ __forceinline__ void vadd(float (&o)[VEC], const float (&a)[VEC], const float (&b)[VEC]) {
  if constexpr (VEC >= 2 && QB_USE_F32X2) {
#pragma unroll
    for (int i = 0; i < VEC; i += 2) {
      const float2 r = __fadd2_rn(make_float2(a[i], a[i + 1]), make_float2(b[i], b[i + 1]));
      o[i] = r.x; o[i + 1] = r.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) o[i] = a[i] + b[i];
  }
}
template <int VEC>
__device__ __forceinline__ void vadd_s(float (&o)[VEC], const float (&a)[VEC], float s) {
  if constexpr (VEC >= 2 && QB_USE_F32X2) {
    const float2 s2 = make_float2(s, s);
#pragma unroll
    for (int i = 0; i < VEC; i += 2) {
      const float2 r = __fadd2_rn(make_float2(a[i], a[i + 1]), s2);
      o[i] = r.x; o[i + 1] = r.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) o[i] = a[i] + s;
  }
}

// o = a + b elementwise sum of all lanes (horizontal), used at the end of a pass
template <int VEC>
__device__ __forceinline__ float hsum(const float (&a)[VEC]) {
  float s = a[0];
#pragma unroll
  for (int i = 1; i < VEC; ++i) s += a[i];
  return s;
}

// ---------------------------------------------------------------------------------------------
// chunk = VEC consecutive elements (<= 16 bytes for the widest tensor of the launch)
// ---------------------------------------------------------------------------------------------
// Raw (still packed) load of the VEC elements starting at element index idx of a tensor with base
// pointer `base`; if pred is false nothing is read and the words are zero.  Kernels issue the raw
// loads of all chunks of all tensors first and unpack afterwards, so that every load of a row is
// in flight before the first use.
template <int DT, int VEC, bool STREAM = true>
__device__ __forceinline__ void load_chunk_raw(uint32_t (&w)[RawWords<DT, VEC>::value],
                                               const void* base, int64_t idx, int dt,
                                               bool pred = true) {
  const int d = (DT == kDynDT) ? dt : DT;
  if (d == QB_F32) {
    if constexpr (DT == QB_F32 || DT == kDynDT) {
      const char* p = reinterpret_cast<const char*>(base) + idx * 4;
      if constexpr (VEC == 8) {
        if constexpr (STREAM) { ldg_stream<16>(w, p, pred); ldg_stream<16>(w + 4, p + 16, pred); }
        else { ldg_cached<16>(w, p, pred); ldg_cached<16>(w + 4, p + 16, pred); }
      } else {
        if constexpr (STREAM) ldg_stream<VEC * 4>(w, p, pred); else ldg_cached<VEC * 4>(w, p, pred);
      }
    }
  } else {
    const char* p = reinterpret_cast<const char*>(base) + idx * 2;
    if constexpr (STREAM) ldg_stream<VEC * 2>(w, p, pred); else ldg_cached<VEC * 2>(w, p, pred);
  }
}

// Convenience: raw load + unpack of one chunk.
template <int DT, int VEC, bool STREAM = true>
__device__ __forceinline__ void load_chunk(float (&v)[VEC], const void* base, int64_t idx, int dt,
                                           bool pred = true) {
  uint32_t w[RawWords<DT, VEC>::value];
  load_chunk_raw<DT, VEC, STREAM>(w, base, idx, dt, pred);
  unpack_chunk<DT, VEC>(v, w, dt);
}

template <int DT, int VEC>
__device__ __forceinline__ void store_chunk(void* base, int64_t idx, const float (&v)[VEC],
                                            int dt) {
  const int d = (DT == kDynDT) ? dt : DT;
  if (d == QB_F32) {
    char* p = reinterpret_cast<char*>(base) + idx * 4;
    if constexpr (VEC == 8) {
      uint32_t a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) { a[i] = __float_as_uint(v[i]); b[i] = __float_as_uint(v[4 + i]); }
      stg_stream<16>(p, a);
      stg_stream<16>(p + 16, b);
    } else {
      uint32_t a[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) a[i] = __float_as_uint(v[i]);
      stg_stream<VEC * 4>(p, a);
    }
  } else {
    char* p = reinterpret_cast<char*>(base) + idx * 2;
    uint32_t a[(VEC + 1) / 2];
    pack16<VEC>(a, v, d == QB_BF16);
    stg_stream<VEC * 2>(p, a);
  }
}

// Asynchronous copy of one chunk into a shared-memory slot of 4*VEC bytes (slot size is the fp32
// worst case so the layout does not depend on the dtype); read back with load_chunk_smem.
template <int DT, int VEC>
__device__ __forceinline__ void stage_chunk(void* slot, const void* base, int64_t idx, int dt) {
  const int d = (DT == kDynDT) ? dt : DT;
  if (d == QB_F32) {
    const char* p = reinterpret_cast<const char*>(base) + idx * 4;
    if constexpr (VEC == 8) {
      cp_async_g2s<16>(slot, p);
      cp_async_g2s<16>(reinterpret_cast<char*>(slot) + 16, p + 16);
    } else {
      cp_async_g2s<VEC * 4>(slot, p);
    }
  } else {
    cp_async_g2s<VEC * 2>(slot, reinterpret_cast<const char*>(base) + idx * 2);
  }
}

template <int DT, int VEC>
__device__ __forceinline__ void load_chunk_smem(float (&v)[VEC], const void* slot, int dt) {
  const int d = (DT == kDynDT) ? dt : DT;
  if (d == QB_F32) {
    if constexpr (VEC == 8) {
      uint32_t a[4], b[4];
      lds_raw<16>(a, slot);
      lds_raw<16>(b, reinterpret_cast<const char*>(slot) + 16);
#pragma unroll
      for (int i = 0; i < 4; ++i) { v[i] = __uint_as_float(a[i]); v[4 + i] = __uint_as_float(b[i]); }
    } else {
      uint32_t a[VEC];
      lds_raw<VEC * 4>(a, slot);
#pragma unroll
      for (int i = 0; i < VEC; ++i) v[i] = __uint_as_float(a[i]);
    }
  } else {
    uint32_t a[(VEC + 1) / 2];
    lds_raw<VEC * 2>(a, slot);
    unpack16<VEC>(v, a, d == QB_BF16);
  }
}

// Pointer-based forms: `p` is the address of the chunk's first element.  Kernels compute one byte
// pointer per row tile and step it by a 32-bit chunk stride, which keeps the per-chunk address
// arithmetic to one or two integer instructions.
template <int DT>
__device__ __forceinline__ int elem_bytes(int dt) {
  return (DT == kDynDT) ? (dt == QB_F32 ? 4 : 2) : (DT == QB_F32 ? 4 : 2);
}

template <int DT, int VEC, bool STREAM = true>
__device__ __forceinline__ void load_chunk_raw_p(uint32_t (&w)[RawWords<DT, VEC>::value],
                                                 const void* ptr, int dt, bool pred = true) {
  const int d = (DT == kDynDT) ? dt : DT;
  const char* p = reinterpret_cast<const char*>(ptr);
  if (d == QB_F32) {
    if constexpr (DT == QB_F32 || DT == kDynDT) {
      if constexpr (VEC == 8) {
        if constexpr (STREAM) { ldg_stream<16>(w, p, pred); ldg_stream<16>(w + 4, p + 16, pred); }
        else { ldg_cached<16>(w, p, pred); ldg_cached<16>(w + 4, p + 16, pred); }
      } else {
        if constexpr (STREAM) ldg_stream<VEC * 4>(w, p, pred); else ldg_cached<VEC * 4>(w, p, pred);
      }
    }
  } else {
    if constexpr (STREAM) ldg_stream<VEC * 2>(w, p, pred); else ldg_cached<VEC * 2>(w, p, pred);
  }
}

// All K chunks of a thread's row slice: chunk k at `base + k * step` exists iff k < nkr.  When all
// of them exist (rows that fill the tile: the common hidden sizes) the loads are unpredicated,
// which saves the zero fill and the predicate set-up of every load (softmax forward, bf16,
// N = 4096: 5.6 -> 5.9 TB/s; the norm forward measured slower with it and keeps predicated loads).
template <int DT, int VEC, int K>
__device__ __forceinline__ void load_row_raw(uint32_t (&w)[K][RawWords<DT, VEC>::value], const char* base,
                                             int step, int dt, int nkr) {
  constexpr bool kOneLoad = DT == QB_BF16 || DT == QB_F16 || (DT == QB_F32 && VEC <= 4);
  if (kOneLoad && nkr == K) {
    constexpr int kBytes = (DT == QB_F32 ? 4 : 2) * VEC;
#pragma unroll
    for (int k = 0; k < K; ++k) ldg_stream_full<kBytes>(w[k], base + k * step);
  } else {
#pragma unroll
    for (int k = 0; k < K; ++k) load_chunk_raw_p<DT, VEC>(w[k], base + k * step, dt, k < nkr);
  }
}

template <int DT, int VEC>
__device__ __forceinline__ void store_chunk_p(void* ptr, const float (&v)[VEC], int dt) {
  const int d = (DT == kDynDT) ? dt : DT;
  char* p = reinterpret_cast<char*>(ptr);
  if (d == QB_F32) {
    if constexpr (VEC == 8) {
      uint32_t a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) { a[i] = __float_as_uint(v[i]); b[i] = __float_as_uint(v[4 + i]); }
      stg_stream<16>(p, a);
      stg_stream<16>(p + 16, b);
    } else {
      uint32_t a[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) a[i] = __float_as_uint(v[i]);
      stg_stream<VEC * 4>(p, a);
    }
  } else {
    uint32_t a[(VEC + 1) / 2];
    pack16<VEC>(a, v, d == QB_BF16);
    stg_stream<VEC * 2>(p, a);
  }
}

template <int DT, int VEC>
__device__ __forceinline__ void stage_chunk_p(void* slot, const void* ptr, int dt) {
  const int d = (DT == kDynDT) ? dt : DT;
  const char* p = reinterpret_cast<const char*>(ptr);
  if (d == QB_F32) {
    if constexpr (VEC == 8) {
      cp_async_g2s<16>(slot, p);
      cp_async_g2s<16>(reinterpret_cast<char*>(slot) + 16, p + 16);
    } else {
      cp_async_g2s<VEC * 4>(slot, p);
    }
  } else {
    cp_async_g2s<VEC * 2>(slot, p);
  }
}

// Scalar element load (row scalars, target logits, class weights).
__device__ __forceinline__ float load_scalar(const void* base, int64_t idx, int dt) {
  if (dt == QB_F32) return reinterpret_cast<const float*>(base)[idx];
  const unsigned short u = reinterpret_cast<const unsigned short*>(base)[idx];
  return dt == QB_BF16 ? __uint_as_float(static_cast<uint32_t>(u) << 16)
                       : __half2float(__ushort_as_half(u));
}

__device__ __forceinline__ int64_t load_index(const void* base, int64_t idx, int itype) {
  return itype == QB_I64 ? reinterpret_cast<const int64_t*>(base)[idx]
                         : static_cast<int64_t>(reinterpret_cast<const int32_t*>(base)[idx]);
}

// ---------------------------------------------------------------------------------------------
// thread-block cluster primitives (PTX; valid only in kernels launched with a cluster dimension)
// ---------------------------------------------------------------------------------------------
// mbarrier / st.async primitives (shared by the cluster reductions below and the bulk-copy ring)
// ---------------------------------------------------------------------------------------------
constexpr unsigned long long kRingTimeoutNs = 2000000000ull;  // 2 s per wait
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier primitives (shared::cta unless stated) ----
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ uint32_t mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok;
}
// Wait with cluster-scope acquire: pairs with mbar_arrive_remote of another CTA of the cluster.
__device__ __forceinline__ uint32_t mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok;
}
// Address of the local shared-memory location `local` in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
// st.async of 8 bytes into a peer CTA's shared memory; the bytes are counted on an mbarrier of that
// peer (the reference's store_shared_remote + mbarrier pair, quack/utils.py:27-58).
__device__ __forceinline__ void st_async_f2(uint32_t addr_cluster, float2 v, uint32_t bar_cluster) {
  asm volatile(
      "st.async.weak.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
          addr_cluster),
      "f"(v.x), "f"(v.y), "r"(bar_cluster)
      : "memory");
}
// Announces `bytes` on a local mbarrier and arrives on it, without a release fence (nothing this
// thread wrote has to be published by the arrival; the data comes with the st.async stores).
__device__ __forceinline__ void mbar_arrive_expect_tx_relaxed(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.relaxed.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  cluster_arrive();
  cluster_wait();
}
// Store 8 bytes into the shared memory of CTA `rank` of this cluster, at the address that
// corresponds to local shared-memory pointer `local`.
__device__ __forceinline__ void st_shared_cluster_f2(void* local, uint32_t rank, float2 v) {
  const uint32_t laddr = static_cast<uint32_t>(__cvta_generic_to_shared(local));
  uint32_t raddr;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(raddr) : "r"(laddr), "r"(rank));
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(raddr), "f"(v.x), "f"(v.y)
               : "memory");
}

// ---------------------------------------------------------------------------------------------
// row reductions: thread -> warp (shuffle) -> CTA (shared memory) -> cluster (DSMEM)
// ---------------------------------------------------------------------------------------------
// Values are float2 so one exchange serves a pair (LayerNorm backward's two sums, the
// (max, sum-exp) pair of the online softmax).
struct SumOp {
  __device__ static __forceinline__ float2 identity() { return make_float2(0.f, 0.f); }
  __device__ static __forceinline__ float2 combine(float2 a, float2 b) {
    return make_float2(a.x + b.x, a.y + b.y);
  }
};
// (running max m, sum of exp2((x - m) * log2e)); identity is (-inf, 0).
struct MaxSumExpOp {
  __device__ static __forceinline__ float2 identity() { return make_float2(neg_inf(), 0.f); }
  __device__ static __forceinline__ float2 combine(float2 a, float2 b) {
    const float m = fmaxf(a.x, b.x);
    // exp2(-inf - -inf) would be NaN: a side whose max is -inf contributes nothing.
    const float sa = (a.x == neg_inf()) ? 0.f : a.y * fast_exp2((a.x - m) * kLog2e);
    const float sb = (b.x == neg_inf()) ? 0.f : b.y * fast_exp2((b.x - m) * kLog2e);
    return make_float2(m, sa + sb);
  }
};
struct MaxOp {
  __device__ static __forceinline__ float2 identity() { return make_float2(neg_inf(), neg_inf()); }
  __device__ static __forceinline__ float2 combine(float2 a, float2 b) {
    return make_float2(fmaxf(a.x, b.x), fmaxf(a.y, b.y));
  }
};

constexpr int kMaxWarps = 32;
constexpr int kMaxCluster = 16;
constexpr int kClusterSlots = 128;  // warp partials of a whole cluster exchanged in one step
constexpr int kRedStages = 2;       // independent reductions per row tile
// Shared-memory scratch of the reductions.  Indexed [stage][parity] so that consecutive row tiles
// of a persistent CTA never overwrite a buffer a slower warp may still be reading.
struct __align__(16) ReduceScratch {
  float2 warp_part[kRedStages][2][kMaxWarps];
  float2 cta_part[kRedStages][2][kClusterSlots];
  unsigned long long bar[kRedStages][2];  // cluster exchange: counts the bytes of the partials
  int abort;                              // set once a wait of this CTA timed out
  // Kernels place their dynamic shared memory (staging rings, parameter slices) behind this
  // struct; its size is kept a multiple of 1 KB so that those buffers start on the same
  // boundary as before the barriers were added.
  char pad[1024 - kRedStages * 2 * 8 - 16];
};
static_assert(sizeof(ReduceScratch) % 1024 == 0, "keeps dynamic shared memory 1 KB aligned");

// Position of a thread in the row-tile geometry of its CTA.
struct RowGeom {
  int tpr;            // threads per row (power of two)
  int t;              // index of this thread within its row group
  int r;              // row of the CTA tile this thread works on
  int lane;           // lane in warp
  int warp_in_row;    // warp index within the row group (tpr >= 32), else 0
  int warps_per_row;  // tpr / 32 (>= 1 when tpr >= 32), else 1
  int warp_base;      // first slot of this row group in warp_part[]
  int cluster_n;
  uint32_t crank;
};

__device__ __forceinline__ RowGeom make_geom(int tpr, int cluster_n) {
  RowGeom g;
  const int tid = threadIdx.x;
  g.tpr = tpr;
  g.t = tid & (tpr - 1);
  g.r = tid / tpr;
  g.lane = tid & 31;
  g.warps_per_row = tpr >= 32 ? (tpr >> 5) : 1;
  g.warp_in_row = tpr >= 32 ? (g.t >> 5) : 0;
  g.warp_base = tpr >= 32 ? g.r * g.warps_per_row : 0;
  g.cluster_n = cluster_n;
  g.crank = cluster_n > 1 ? cluster_cta_rank() : 0u;
  return g;
}

// Sets up the cluster exchange of row_reduce.  Every thread of the CTA calls it once, before the
// kernel's barrier.cluster arrive / wait pair that precedes the first exchange (that pair
// publishes the initialised barriers to the other CTAs of the cluster).
__device__ __forceinline__ void reduce_init(ReduceScratch& s, int cluster_n) {
  if (cluster_n > 1) {
    if (threadIdx.x == 0) {
#pragma unroll
      for (int st = 0; st < kRedStages; ++st) {
        mbar_init(smem_u32(&s.bar[st][0]), 1);
        mbar_init(smem_u32(&s.bar[st][1]), 1);
      }
      s.abort = 0;
      mbar_fence_init();
    }
    __syncthreads();
  }
}

// Bounded wait on a local mbarrier: gives up after about a second (kReduceWaitCycles of the SM
// clock, a 32-bit counter: one register), sets the CTA's abort flag (every later wait of the CTA
// then returns at once) and bumps the device counter the host can read, so a lost signal costs
// wrong results for the rows concerned, never a hung GPU.
constexpr unsigned int kReduceWaitCycles = 0x70000000u;
__device__ __forceinline__ void bounded_mbar_wait(int* abort_flag, uint32_t bar, uint32_t parity,
                                                  unsigned int* timeouts) {
  if (mbar_try_wait(bar, parity) != 0) return;
  const unsigned int t0 = static_cast<unsigned int>(clock());
#pragma unroll 1
  for (;;) {
    if (mbar_try_wait(bar, parity) != 0) return;
    if (*reinterpret_cast<volatile int*>(abort_flag)) return;
    if (static_cast<unsigned int>(clock()) - t0 > kReduceWaitCycles) {
      *reinterpret_cast<volatile int*>(abort_flag) = 1;
      if (timeouts != nullptr) atomicAdd(timeouts, 1u);
      return;
    }
  }
}
__device__ __forceinline__ void reduce_wait(ReduceScratch& s, uint32_t bar, uint32_t parity,
                                            unsigned int* timeouts) {
  bounded_mbar_wait(&s.abort, bar, parity, timeouts);
}

__device__ __forceinline__ float2 shfl_xor_f2(float2 v, int mask) {
  return make_float2(__shfl_xor_sync(0xffffffffu, v.x, mask),
                     __shfl_xor_sync(0xffffffffu, v.y, mask));
}

// Reduces `v` over all threads that share a row (and over the cluster's CTAs).  Every thread of
// the row returns the same value.  Must be called by all threads of the CTA (and, with clusters,
// by all CTAs of the cluster) the same number of times with the same (stage, parity).
// Barrier among the threads that share a row.  ROWBAR: when a CTA carries several rows, each row
// group (whole warps) synchronises on a hardware barrier of its own (ids 1 ... 15) instead of
// the CTA-wide barrier 0.  Measured on B200: LayerNorm forward N = 8192 (4 rows of 2 warps per
// CTA) +15 %, but softmax backward N = 4096 -23 % and LayerNorm backward -6 %, so it is opt-in
// per kernel.
template <bool ROWBAR>
__device__ __forceinline__ void row_group_sync(const RowGeom& g) {
  if constexpr (ROWBAR) {
    // The choice is CTA-uniform: either every row group uses a named barrier of its own or every
    // thread takes barrier 0.  (A CTA with more than 15 row groups, e.g. 1024 threads at 64 per
    // row, must not mix the two: barrier 0 counts the whole CTA.)
    if (g.tpr >= 32 && g.tpr < static_cast<int>(blockDim.x) &&
        static_cast<int>(blockDim.x) <= 15 * g.tpr) {
      asm volatile("bar.sync %0, %1;" ::"r"(g.r + 1), "r"(g.tpr) : "memory");
      return;
    }
  }
  __syncthreads();
}

// `rit` counts the rows this CTA has reduced so far: buffers (and, for clusters, barriers) are
// double-buffered by its parity, and a barrier's phase is bit 1 of it.
// CL = false compiles the cluster paths out (for kernels instantiated separately for
// single-CTA rows: the exchange code costs registers that the norm backward does not have).
// ASYNC = false keeps the cluster exchange on plain remote stores published by barrier.cluster
// (fewer registers; see the note in the function).
template <class Op, bool ROWBAR = false, bool CL = true, bool ASYNC = true>
__device__ __forceinline__ float2 row_reduce(float2 v, const RowGeom& g, ReduceScratch& s,
                                             int stage, int rit, unsigned int* timeouts = nullptr) {
  const int parity = rit & 1;
  // 1. within the warp (or the sub-warp row group)
  if (g.tpr >= 32) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = Op::combine(v, shfl_xor_f2(v, o));
  } else {
    for (int o = g.tpr >> 1; o > 0; o >>= 1) v = Op::combine(v, shfl_xor_f2(v, o));
  }
  if (CL && g.cluster_n > 1) {
    // 2+3 (cluster): every warp pushes its partial into slot [crank * warps + warp] of every
    //    CTA's buffer through distributed shared memory, every thread waits until all partials
    //    have arrived in its own CTA's buffer, and every warp folds all slots in the same order,
    //    so all CTAs obtain bit-identical results.
    const int nslots = g.warps_per_row * g.cluster_n;
    if (nslots <= kClusterSlots) {
      // The partials travel by st.async and are counted on an mbarrier of the receiving CTA
      // instead of being published by barrier.cluster: that barrier's arrive has release
      // semantics, which stalls the thread until its global loads and stores in flight have
      // completed -- in a persistent kernel the previous row's stores and the next row's
      // prefetch (measured on the softmax backward: 5.6 -> 6.8 TB/s at N = 65536).  Buffer and
      // barrier [stage][parity] are reused every second row; a peer can only send row j + 2
      // after every warp of this CTA has sent row j + 1, hence after it has folded row j.
      float2* buf = s.cta_part[stage][parity];
      if constexpr (ASYNC) {
        const uint32_t phase = static_cast<uint32_t>(rit >> 1) & 1u;
        const uint32_t bar = smem_u32(&s.bar[stage][parity]);
        if (threadIdx.x == 0) mbar_arrive_expect_tx_relaxed(bar, static_cast<uint32_t>(nslots) * 8u);
        if (g.lane < g.cluster_n)
          st_async_f2(map_to_cta(smem_u32(&buf[g.crank * g.warps_per_row + g.warp_in_row]), g.lane), v,
                      map_to_cta(bar, g.lane));
        reduce_wait(s, bar, phase, timeouts);
      } else {
        // The exchange above costs about six registers more than this one.  The LayerNorm
        // backward with db accumulators and run-time geometry has none to spare (it spilled and
        // lost 20 %), so it stays on plain remote stores + one barrier.cluster round trip.
        if (g.lane < g.cluster_n)
          st_shared_cluster_f2(&buf[g.crank * g.warps_per_row + g.warp_in_row], g.lane, v);
        cluster_sync_all();
      }
      float2 acc = Op::identity();
      for (int i = g.lane; i < nslots; i += 32) acc = Op::combine(acc, buf[i]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc = Op::combine(acc, shfl_xor_f2(acc, o));
      return acc;
    }
  }
  // 2. across the warps of the row group
  if (g.warps_per_row > 1) {
    float2* buf = s.warp_part[stage][parity];
    if (g.lane == 0) buf[g.warp_base + g.warp_in_row] = v;
    row_group_sync<ROWBAR>(g);
    v = g.lane < g.warps_per_row ? buf[g.warp_base + g.lane] : Op::identity();
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = Op::combine(v, shfl_xor_f2(v, o));
  }
  // 3. across the CTAs of the cluster (only when the one-step exchange above does not fit):
  //    every CTA pushes its partial into slot [crank] of every CTA's buffer, a cluster barrier
  //    publishes the stores, and all CTAs fold the slots in rank order.
  if (CL && g.cluster_n > 1) {
    float2* buf = s.cta_part[stage][parity];
    if (threadIdx.x < g.cluster_n) st_shared_cluster_f2(&buf[g.crank], threadIdx.x, v);
    cluster_sync_all();
    float2 acc = buf[0];
    for (int c = 1; c < g.cluster_n; ++c) acc = Op::combine(acc, buf[c]);
    v = acc;
  }
  return v;
}

}  // namespace qb
