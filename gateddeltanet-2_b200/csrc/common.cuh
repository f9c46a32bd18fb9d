// Shared device helpers for the GDN2 sm_100a kernels: element I/O, the
// warp-level bf16 tensor-core fragment helpers, and launch/status plumbing.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/gdn2.h"

#define GDN2_DEV __device__ __forceinline__

namespace gdn2 {

constexpr int kChunk = 64;       // tokens per chunk (C)
constexpr int kSub = 16;         // rows of one anchored sub-block
constexpr float kLn2 = 0.69314718055994530942f;
constexpr float kRcpLn2 = 1.44269504088896340736f;
constexpr float kL2Eps = 1e-6f;

// ---------------------------------------------------------------------------
// element I/O
// ---------------------------------------------------------------------------
GDN2_DEV float to_f(float x) { return x; }
GDN2_DEV float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> GDN2_DEV T from_f(float x);
template <> GDN2_DEV float from_f<float>(float x) { return x; }
template <> GDN2_DEV __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <typename T>
GDN2_DEV float ldf(const T* p) { return to_f(p[0]); }

GDN2_DEV uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
GDN2_DEV float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// 8 consecutive elements (16-byte aligned for bf16, 32-byte for fp32) <-> registers
GDN2_DEV void ld8(const float* p, float* x) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
GDN2_DEV void ld8(const __nv_bfloat16* p, float* x) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h2 = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
    x[2 * i] = __low2float(h2);
    x[2 * i + 1] = __high2float(h2);
  }
}
// pulls [p, p + bytes) into L2 without waiting (p 16-byte aligned, bytes % 16 == 0)
GDN2_DEV void l2_prefetch(const void* p, int bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// SMs of the current device (the co-resident CTAs of a one-CTA-per-SM kernel)
inline int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  return n;
}

// 2 consecutive elements (8-byte aligned for fp32, 4-byte for bf16)
GDN2_DEV float2 ld2(const float* p) { return *reinterpret_cast<const float2*>(p); }
GDN2_DEV float2 ld2(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
GDN2_DEV uint4 pack8(const float* x) {
  uint4 pk;
  pk.x = pack_bf16(x[0], x[1]);
  pk.y = pack_bf16(x[2], x[3]);
  pk.z = pack_bf16(x[4], x[5]);
  pk.w = pack_bf16(x[6], x[7]);
  return pk;
}
GDN2_DEV void st8(__nv_bfloat16* p, const float* x) { *reinterpret_cast<uint4*>(p) = pack8(x); }
GDN2_DEV void st8(float* p, const float* x) {
  *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(x[4], x[5], x[6], x[7]);
}

GDN2_DEV float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// softplus with the pass-through above 20 used by the reference's gate:
// softplus(x) = max(x, 0) + log1p(y), y = e^-|x| in (0, 1].  log1p(y) from the
// series ln((1+s)/(1-s)) = 2 (s + s^3/3 + s^5/5 + ...) with s = y / (2 + y) <= 1/3
// (Abramowitz & Stegun 4.1.27); eight terms leave a truncation error below
// (1/3)^16 / 17 < 2e-9 relative.  Short and branch-free, unlike a general log1p.
GDN2_DEV float softplus_f(float x) {
  if (x > 20.f) return x;
  const float y = __expf(-fabsf(x));
  const float s = __fdividef(y, 2.f + y), s2 = s * s;
  float p = 1.f / 15.f;
  p = fmaf(p, s2, 1.f / 13.f);
  p = fmaf(p, s2, 1.f / 11.f);
  p = fmaf(p, s2, 1.f / 9.f);
  p = fmaf(p, s2, 1.f / 7.f);
  p = fmaf(p, s2, 1.f / 5.f);
  p = fmaf(p, s2, 1.f / 3.f);
  p = fmaf(p, s2, 1.f);
  return fmaxf(x, 0.f) + 2.f * s * p;
}
// fast reciprocal (__fdividef, a few ulp): every use feeds fp32 math or a bf16 result
GDN2_DEV float sigmoid_f(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// ---------------------------------------------------------------------------
// bf16 mma.sync m16n8k16 fragments (row.col, fp32 accumulate)
// ---------------------------------------------------------------------------
GDN2_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

GDN2_DEV void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}
GDN2_DEV void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}

GDN2_DEV void mma_bf16(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Shared-memory bf16 matrix view: element (r, c) at base[r * ld + c].
struct Smem {
  __nv_bfloat16* p;
  int ld;
  GDN2_DEV __nv_bfloat16* at(int r, int c) const { return p + r * ld + c; }
};

// A fragment (16x16 slice of the logical A[m][k]) at (m0, k0).
// kTrans=false: A stored row-major [m][k]; true: stored [k][m] (use A^T of a stored matrix).
template <bool kTrans, typename SM>
GDN2_DEV void load_a(uint32_t* a, SM s, int m0, int k0, int lane) {
  if (!kTrans) {
    const int r = m0 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int c = k0 + (lane >> 4) * 8;
    ldsm_x4(a[0], a[1], a[2], a[3], s.at(r, c));
  } else {
    const int kr = k0 + (lane & 7) + (lane >> 4) * 8;
    const int mc = m0 + ((lane >> 3) & 1) * 8;
    ldsm_x4_t(a[0], a[1], a[2], a[3], s.at(kr, mc));
  }
}

// Two B fragments (k 16 x n 16 of the logical B[k][n]) at (k0, n0): b[0..1] for
// n0..n0+7 and b[2..3] for n0+8..n0+15.
// kNK=false: B stored row-major [k][n]; true: stored [n][k] (B^T row-major).
template <bool kNK, typename SM>
GDN2_DEV void load_b2(uint32_t* b, SM s, int k0, int n0, int lane) {
  if (kNK) {
    const int nr = n0 + (lane & 7) + (lane >> 4) * 8;
    const int kc = k0 + ((lane >> 3) & 1) * 8;
    ldsm_x4(b[0], b[1], b[2], b[3], s.at(nr, kc));
  } else {
    const int kr = k0 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int nc = n0 + (lane >> 4) * 8;
    ldsm_x4_t(b[0], b[1], b[2], b[3], s.at(kr, nc));
  }
}

// Warp tile: acc[MT][NT][4] += A[m0 : m0+16*MT, 0:kdim] * B[0:kdim, n0 : n0+8*NT]
// (NT even).  Accumulator layout per (i, j): c0,c1 at row m0+16i+g, cols
// n0+8j+2t, +1; c2,c3 at row +8.
// (SA, SB: any shared-memory view with at(r, c) -> the 16-byte row segment of
// element (r, c), c % 8 == 0: padded rows (Smem) or swizzled tiles)
template <int MT, int NT, bool kATrans, bool kBNK, typename SA = Smem, typename SB = Smem>
GDN2_DEV void warp_mma(float (&acc)[MT][NT][4], SA A, int m0, SB B, int n0, int k_begin,
                       int k_end, int lane) {
  static_assert(NT % 2 == 0, "NT must be even");
#pragma unroll 2
  for (int k0 = k_begin; k0 < k_end; k0 += 16) {
    uint32_t af[MT][4];
#pragma unroll
    for (int i = 0; i < MT; ++i) load_a<kATrans>(af[i], A, m0 + 16 * i, k0, lane);
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      uint32_t bf[4];
      load_b2<kBNK>(bf, B, k0, n0 + 8 * j, lane);
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        mma_bf16(acc[i][j], af[i], bf);
        mma_bf16(acc[i][j + 1], af[i], bf + 2);
      }
    }
  }
}

// Same product with the reduction split over KS independent accumulator sets
// (k-steps dealt round-robin) that are summed at the end: a dependent chain
// of k_len/16/KS tensor-core ops instead of k_len/16, for latency-bound loops.
template <int KS, int MT, int NT, bool kATrans, bool kBNK>
GDN2_DEV void warp_mma_ks(float (&acc)[MT][NT][4], Smem A, int m0, Smem B, int n0, int k_begin, int k_end,
                          int lane) {
  static_assert(NT % 2 == 0, "NT must be even");
  float part[KS][MT][NT][4];
#pragma unroll
  for (int s = 0; s < KS; ++s)
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) part[s][i][j][e] = 0.f;
  for (int k0 = k_begin; k0 < k_end; k0 += 16 * KS) {
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      const int kk = k0 + 16 * s;
      if (kk < k_end) {
        uint32_t af[MT][4];
#pragma unroll
        for (int i = 0; i < MT; ++i) load_a<kATrans>(af[i], A, m0 + 16 * i, kk, lane);
#pragma unroll
        for (int j = 0; j < NT; j += 2) {
          uint32_t bf[4];
          load_b2<kBNK>(bf, B, kk, n0 + 8 * j, lane);
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            mma_bf16(part[s][i][j], af[i], bf);
            mma_bf16(part[s][i][j + 1], af[i], bf + 2);
          }
        }
      }
    }
  }
#pragma unroll
  for (int s = 0; s < KS; ++s)
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][j][e] += part[s][i][j][e];
}

template <int MT, int NT>
GDN2_DEV void zero_acc(float (&acc)[MT][NT][4]) {
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;
}

// Visit every accumulator element with its (row, col).
template <int MT, int NT, typename F>
GDN2_DEV void acc_foreach(float (&acc)[MT][NT][4], int m0, int n0, int lane, F f) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = m0 + 16 * i + g + (e >> 1) * 8;
        const int c = n0 + 8 * j + 2 * t + (e & 1);
        f(acc[i][j][e], r, c);
      }
}

// ---------------------------------------------------------------------------
// varlen / dense sequence geometry
// ---------------------------------------------------------------------------
struct SeqGeom {
  const int64_t* cu;   // [N+1] or nullptr (dense)
  const int32_t* cidx; // [NT,2] (seq, chunk-in-seq) or nullptr
  const int32_t* coff; // [N+1] first global chunk per sequence, or nullptr
  int64_t T;           // dense per-sequence length
  int64_t NTseq;       // dense chunks per sequence
  GDN2_DEV void seq(int64_t n, int64_t& bos, int64_t& len) const {
    if (cu) {
      bos = cu[n];
      len = cu[n + 1] - bos;
    } else {
      bos = n * T;
      len = T;
    }
  }
  GDN2_DEV int64_t chunk0(int64_t n) const { return coff ? (int64_t)coff[n] : n * NTseq; }
  // global chunk -> (sequence, chunk within the sequence)
  GDN2_DEV void chunk(int64_t c, int64_t& n, int64_t& i) const {
    if (cidx) {
      n = cidx[2 * c];
      i = cidx[2 * c + 1];
    } else if (c < (1ll << 31) && NTseq < (1ll << 31)) {
      // 32-bit division: a short instruction sequence where the 64-bit one is a
      // long dependent chain on every CTA's critical path
      const uint32_t q = static_cast<uint32_t>(c) / static_cast<uint32_t>(NTseq);
      n = q;
      i = c - static_cast<int64_t>(q) * NTseq;
    } else {
      n = c / NTseq;
      i = c % NTseq;
    }
  }
};

}  // namespace gdn2

#define GDN2_CUDA_TRY(expr)                              \
  do {                                                   \
    cudaError_t e_ = (expr);                             \
    if (e_ != cudaSuccess) return -static_cast<int>(e_); \
  } while (0)

#define GDN2_LAUNCH_CHECK()                                      \
  do {                                                           \
    cudaError_t e_ = cudaGetLastError();                         \
    if (e_ != cudaSuccess) return -static_cast<int>(e_);         \
  } while (0)
