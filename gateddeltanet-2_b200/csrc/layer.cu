// The GatedDeltaNet2 layer's memory-bound passes around the operator
// (lit_gpt/gdn2.py:282-464), each one read and one write of its tensors:
//
//   layer_prep_fwd_kernel  merged projection rows q|k|v|b|w|f0|g0 ->
//                          SiLU(short causal depthwise conv) for q, k, v
//                          (fla ShortConvolution, gdn2.py:342-367), sigmoid
//                          gates b, w (gdn2.py:398-399, :412-420), contiguous
//                          f0, g0 for the second-stage GEMMs;
//   layer_prep_bwd_kernel  the reverse pass, with per-CTA conv weight / bias
//                          partial sums reduced in a fixed order;
//   norm_gate_fwd/bwd      FusedRMSNormSwishGate (gdn2.py:462; fla
//                          fused_norm_gate.py:35-104).
//
// Thread layout of the prep kernels: a lane owns NV consecutive channels (a
// 16-byte vector of a row in the forward, 8-byte in the backward, so a warp
// touches 512 or 256 contiguous bytes of each row) and a warp walks a segment
// of kPrepRows rows; the 8 warps of a CTA take 8 consecutive segments of the
// same 32 x NV channels.  The conv taps of a row are
// the previous W-1 rows of the same sequence, held in registers while the
// warp walks forward (forward) or reloaded through L1 (backward, which walks
// backward so that the W cotangents a row needs are already computed).
#include <algorithm>

#include "chunk_layout.cuh"
#include "common.cuh"
#include "profile.cuh"

namespace gdn2 {
namespace {

using bf16 = __nv_bfloat16;

constexpr int kPrepWarps = 8;
constexpr int kPrepRows = 32;
constexpr int kPrepRowsPerCta = kPrepWarps * kPrepRows;
constexpr int kNormBwdMaxCtas = 1184;  // fixed so the dweight reduction order never depends on the device

struct PrepGeom {
  int64_t C;                 // conv channels 2Dk+Dv (= proj column of b_raw)
  int64_t Gc, Gs, Gf, G;     // NV-channel groups: conv, sigmoid, copy, total
  int64_t off_f;             // proj column of f0 (g0 follows)
  int64_t grid_y;            // row tiles of kPrepRowsPerCta
};

// NV: channels per lane (8 in the forward, 4 in the backward, whose lanes
// hold W x NV taps, W x NV conv cotangents and (W+1) x NV partial sums)
PrepGeom prep_geom(const gdn2_prep_args& a, int NV) {
  PrepGeom g;
  g.C = 2 * a.Dk + a.Dv;
  g.Gc = g.C / NV;
  g.Gs = (a.Dk + a.Dv) / NV;
  g.Gf = a.f0 ? 2 * a.Dfg / NV : 0;
  g.G = g.Gc + g.Gs + g.Gf;
  g.off_f = g.C + a.Dk + a.Dv;
  g.grid_y = (a.rows + kPrepRowsPerCta - 1) / kPrepRowsPerCta;
  return g;
}

struct Seq {
  int64_t n, s, e;  // index, first row, one past the last row
};

// sequence containing row r (with cu_seqlens: the last n with cu[n] <= r, which
// skips empty sequences)
GDN2_DEV Seq seq_of(const gdn2_prep_args& a, int64_t r) {
  if (!a.cu_seqlens) {
    const int64_t n = r / a.T;
    return {n, n * a.T, n * a.T + a.T};
  }
  int64_t lo = 0, hi = a.N - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (a.cu_seqlens[mid] <= r) lo = mid;
    else hi = mid - 1;
  }
  return {lo, a.cu_seqlens[lo], a.cu_seqlens[lo + 1]};
}

GDN2_DEV float silu(float z) { return z / (1.f + __expf(-z)); }
GDN2_DEV float silu_grad(float z) {
  const float s = sigmoid_f(z);
  return s * (1.f + z * (1.f - s));
}

// NV consecutive bf16 <-> fp32 registers (16-byte or 8-byte vectors)
template <int NV>
GDN2_DEV void ldv(const bf16* p, float* x) {
  if constexpr (NV == 8) {
    ld8(p, x);
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
  }
}
template <int NV>
GDN2_DEV void stv(bf16* p, const float* x) {
  if constexpr (NV == 8) {
    st8(p, x);
  } else {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]));
  }
}

// conv input of row `row` for channels c0..c0+NV-1 of sequence sq: the
// projection inside the sequence, the cached history (entry W - (s - row)) before it
template <int W, int NV>
GDN2_DEV void conv_tap(const gdn2_prep_args& a, const PrepGeom& g, const Seq& sq, int64_t row, int64_t c0,
                       float* x) {
  if (row >= sq.s) {
    ldv<NV>(reinterpret_cast<const bf16*>(a.proj) + row * a.proj_stride + c0, x);
  } else if (a.conv_state_in && sq.s - row < W) {  // (a malformed cu_seqlens reads zeros, never out of the cache)
    const bf16* p = reinterpret_cast<const bf16*>(a.conv_state_in) + (sq.n * g.C + c0) * W + (W - (sq.s - row));
#pragma unroll
    for (int i = 0; i < NV; ++i) x[i] = __bfloat162float(p[i * W]);
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i) x[i] = 0.f;
  }
}

struct OutSlot {
  bf16* p;
  int64_t ld, col;
};

// output tensor, its row length and column of conv channel c0 (q | k | v)
GDN2_DEV OutSlot conv_slot(const gdn2_prep_args& a, int64_t c0) {
  if (c0 < a.Dk) return {reinterpret_cast<bf16*>(a.q), a.Dk, c0};
  if (c0 < 2 * a.Dk) return {reinterpret_cast<bf16*>(a.k), a.Dk, c0 - a.Dk};
  return {reinterpret_cast<bf16*>(a.v), a.Dv, c0 - 2 * a.Dk};
}

template <int W, int NV>
__global__ void __launch_bounds__(kPrepWarps * 32) layer_prep_fwd_kernel(gdn2_prep_args a, PrepGeom g) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t grp = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  const int64_t r0 = (static_cast<int64_t>(blockIdx.y) * kPrepWarps + warp) * kPrepRows;
  if (grp >= g.G || r0 >= a.rows) return;
  const int64_t r1 = min(r0 + kPrepRows, a.rows);
  const bf16* proj = reinterpret_cast<const bf16*>(a.proj);
  const int64_t ld = a.proj_stride;

  if (grp < g.Gc) {  // ---- q, k, v: SiLU(conv) --------------------------------
    const int64_t c0 = grp * NV;
    const OutSlot o = conv_slot(a, c0);
    if constexpr (W == 0) {
      for (int64_t r = r0; r < r1; ++r) {
        float x[NV];
        ldv<NV>(proj + r * ld + c0, x);
#pragma unroll
        for (int i = 0; i < NV; ++i) x[i] = silu(x[i]);
        stv<NV>(o.p + r * o.ld + o.col, x);
      }
    } else {
      float wt[W][NV], bias[NV];
#pragma unroll
      for (int i = 0; i < NV; ++i) {
#pragma unroll
        for (int j = 0; j < W; ++j) wt[j][i] = a.conv_weight[(c0 + i) * W + j];
        bias[i] = a.conv_bias ? a.conv_bias[c0 + i] : 0.f;
      }
      float win[W - 1][NV];  // win[j]: input of row r - (W-1) + j
      Seq sq = seq_of(a, r0);
#pragma unroll
      for (int j = 0; j < W - 1; ++j) conv_tap<W, NV>(a, g, sq, r0 - (W - 1) + j, c0, win[j]);
      bf16* st_out = reinterpret_cast<bf16*>(a.conv_state_out);
      for (int64_t r = r0; r < r1; ++r) {
        if (r == sq.e) {  // a new sequence starts: its history is its cache
          sq = seq_of(a, r);
#pragma unroll
          for (int j = 0; j < W - 1; ++j) conv_tap<W, NV>(a, g, sq, r - (W - 1) + j, c0, win[j]);
        }
        float x[NV], y[NV];
        ldv<NV>(proj + r * ld + c0, x);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          float z = bias[i] + wt[W - 1][i] * x[i];
#pragma unroll
          for (int j = 0; j < W - 1; ++j) z += wt[j][i] * win[j][i];
          y[i] = silu(z);
        }
        stv<NV>(o.p + r * o.ld + o.col, y);
        if (st_out && r == sq.e - 1) {  // the sequence's last W inputs
          bf16* p = st_out + (sq.n * g.C + c0) * W;
#pragma unroll
          for (int i = 0; i < NV; ++i) {
#pragma unroll
            for (int j = 0; j < W - 1; ++j) p[i * W + j] = __float2bfloat16_rn(win[j][i]);
            p[i * W + W - 1] = __float2bfloat16_rn(x[i]);
          }
        }
#pragma unroll
        for (int j = 0; j < W - 2; ++j) {
#pragma unroll
          for (int i = 0; i < NV; ++i) win[j][i] = win[j + 1][i];
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) win[W - 2][i] = x[i];
      }
    }
  } else if (grp < g.Gc + g.Gs) {  // ---- b, w: sigmoid gates ----------------
    const int64_t s0 = (grp - g.Gc) * NV;
    const bool is_b = s0 < a.Dk;
    bf16* out = reinterpret_cast<bf16*>(is_b ? a.b : a.w);
    const int64_t old = is_b ? a.Dk : a.Dv, oc = is_b ? s0 : s0 - a.Dk;
    const float sc = is_b ? a.b_scale : 1.f;
    for (int64_t r = r0; r < r1; ++r) {
      float x[NV];
      ldv<NV>(proj + r * ld + g.C + s0, x);
#pragma unroll
      for (int i = 0; i < NV; ++i) x[i] = sc * sigmoid_f(x[i]);
      stv<NV>(out + r * old + oc, x);
    }
  } else {  // ---- f0, g0: contiguous copies ------------------------------------
    const int64_t f = (grp - g.Gc - g.Gs) * NV;
    const bool is_f = f < a.Dfg;
    bf16* out = reinterpret_cast<bf16*>(is_f ? a.f0 : a.g0);
    const int64_t oc = is_f ? f : f - a.Dfg;
    for (int64_t r = r0; r < r1; ++r) {
      float x[NV];
      ldv<NV>(proj + r * ld + g.off_f + f, x);
      stv<NV>(out + r * a.Dfg + oc, x);
    }
  }
}

// Partial sums per CTA row tile: part[tile][C*W + C] (weights c*W + j, then bias).
template <int W, int NV>
__global__ void __launch_bounds__(kPrepWarps * 32)
    layer_prep_bwd_kernel(gdn2_prep_args a, gdn2_prep_grads gr, PrepGeom g, float* part) {
  constexpr int kAcc = (W > 0 ? W + 1 : 1) * NV;  // conv weight + bias sums of a lane's channels
  __shared__ float red[W > 0 ? kAcc * kPrepWarps * 32 : 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t grp = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  const int64_t r0 = (static_cast<int64_t>(blockIdx.y) * kPrepWarps + warp) * kPrepRows;
  const bool active = grp < g.G && r0 < a.rows;
  const int64_t r1 = min(r0 + kPrepRows, a.rows);
  const bf16* proj = reinterpret_cast<const bf16*>(a.proj);
  bf16* dproj = reinterpret_cast<bf16*>(gr.dproj);
  const int64_t ld = a.proj_stride;
  float acc[kAcc];
#pragma unroll
  for (int i = 0; i < kAcc; ++i) acc[i] = 0.f;

  if (active && grp < g.Gc) {  // ---- q, k, v --------------------------------------
    const int64_t c0 = grp * NV;
    const int64_t sec = c0 < a.Dk ? 0 : (c0 < 2 * a.Dk ? 1 : 2);
    const bf16* dy_p = reinterpret_cast<const bf16*>(sec == 0 ? gr.dq : (sec == 1 ? gr.dk : gr.dv));
    const int64_t dld = sec == 2 ? a.Dv : a.Dk, dcol = c0 - sec * a.Dk;
    if constexpr (W == 0) {
      for (int64_t r = r0; r < r1; ++r) {
        float x[NV], dy[NV];
        ldv<NV>(proj + r * ld + c0, x);
        ldv<NV>(dy_p + r * dld + dcol, dy);
#pragma unroll
        for (int i = 0; i < NV; ++i) dy[i] *= silu_grad(x[i]);
        stv<NV>(dproj + r * ld + c0, dy);
      }
    } else {
      float wt[W][NV], bias[NV];
#pragma unroll
      for (int i = 0; i < NV; ++i) {
#pragma unroll
        for (int j = 0; j < W; ++j) wt[j][i] = a.conv_weight[(c0 + i) * W + j];
        bias[i] = a.conv_bias ? a.conv_bias[c0 + i] : 0.f;
      }
      float ring[W][NV];  // ring[m]: d(pre-activation) of row t + m (0 past the sequence)
#pragma unroll
      for (int m = 0; m < W; ++m)
#pragma unroll
        for (int i = 0; i < NV; ++i) ring[m][i] = 0.f;
      const int64_t t_hi = min(r1 + W - 1, a.rows) - 1;
      Seq sq = seq_of(a, t_hi);
      for (int64_t t = t_hi; t >= r0; --t) {
        if (t < sq.s) {  // crossed into the previous sequence
          sq = seq_of(a, t);
#pragma unroll
          for (int m = 0; m < W; ++m)
#pragma unroll
            for (int i = 0; i < NV; ++i) ring[m][i] = 0.f;
        }
        float xt[W][NV], dy[NV];
#pragma unroll
        for (int j = 0; j < W; ++j) conv_tap<W, NV>(a, g, sq, t - (W - 1) + j, c0, xt[j]);
        ldv<NV>(dy_p + t * dld + dcol, dy);
#pragma unroll
        for (int m = W - 1; m > 0; --m)
#pragma unroll
          for (int i = 0; i < NV; ++i) ring[m][i] = ring[m - 1][i];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          float z = bias[i];
#pragma unroll
          for (int j = 0; j < W; ++j) z += wt[j][i] * xt[j][i];
          ring[0][i] = dy[i] * silu_grad(z);
        }
        if (t < r1) {
          float dx[NV];
#pragma unroll
          for (int i = 0; i < NV; ++i) {
            float sacc = 0.f;
#pragma unroll
            for (int m = 0; m < W; ++m) sacc += wt[W - 1 - m][i] * ring[m][i];
            dx[i] = sacc;
#pragma unroll
            for (int j = 0; j < W; ++j) acc[j * NV + i] += ring[0][i] * xt[j][i];
            acc[W * NV + i] += ring[0][i];
          }
          stv<NV>(dproj + t * ld + c0, dx);
        }
      }
    }
  } else if (active && grp < g.Gc + g.Gs) {  // ---- b, w ------------------------------
    const int64_t s0 = (grp - g.Gc) * NV;
    const bool is_b = s0 < a.Dk;
    const bf16* dg = reinterpret_cast<const bf16*>(is_b ? gr.db : gr.dw);
    const int64_t old = is_b ? a.Dk : a.Dv, oc = is_b ? s0 : s0 - a.Dk;
    const float sc = is_b ? a.b_scale : 1.f;
    for (int64_t r = r0; r < r1; ++r) {
      float x[NV], d[NV];
      ldv<NV>(proj + r * ld + g.C + s0, x);
      ldv<NV>(dg + r * old + oc, d);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const float sg = sigmoid_f(x[i]);
        d[i] *= sc * sg * (1.f - sg);
      }
      stv<NV>(dproj + r * ld + g.C + s0, d);
    }
  } else if (active) {  // ---- f0, g0 ------------------------------------------------
    const int64_t f = (grp - g.Gc - g.Gs) * NV;
    const bool is_f = f < a.Dfg;
    const bf16* src = reinterpret_cast<const bf16*>(is_f ? gr.df0 : gr.dg0);
    const int64_t oc = is_f ? f : f - a.Dfg;
    for (int64_t r = r0; r < r1; ++r) {
      float x[NV];
      if (src) {
        ldv<NV>(src + r * a.Dfg + oc, x);
      } else {
#pragma unroll
        for (int i = 0; i < NV; ++i) x[i] = 0.f;
      }
      stv<NV>(dproj + r * ld + g.off_f + f, x);
    }
  }

  if constexpr (W > 0) {
    // CTA-uniform: only column tiles holding conv channels reduce
    if (static_cast<int64_t>(blockIdx.x) * 32 >= g.Gc) return;
#pragma unroll
    for (int k = 0; k < kAcc; ++k) red[(k * kPrepWarps + warp) * 32 + lane] = acc[k];
    __syncthreads();
    for (int o = threadIdx.x; o < kAcc * 32; o += kPrepWarps * 32) {
      const int k = o / 32, ln = o % 32;
      float sacc = 0.f;
#pragma unroll
      for (int w = 0; w < kPrepWarps; ++w) sacc += red[(k * kPrepWarps + w) * 32 + ln];
      const int64_t gg = static_cast<int64_t>(blockIdx.x) * 32 + ln;
      if (gg >= g.Gc) continue;
      const int j = k / NV, i = k % NV;
      const int64_t c = gg * NV + i;
      float* pt = part + static_cast<int64_t>(blockIdx.y) * g.C * (W + 1);
      if (j < W) pt[c * W + j] = sacc;
      else pt[g.C * W + c] = sacc;
    }
  }
}

// out_a[i] (i < na) / out_b[i - na] = sum over p of part[p * (na + nb) + i]
__global__ void reduce_partials_kernel(const float* part, int64_t nparts, int64_t na, int64_t nb, float* out_a,
                                       float* out_b) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t n = na + nb;
  if (i >= n) return;
  float s = 0.f;
  for (int64_t p = 0; p < nparts; ++p) s += part[p * n + i];
  if (i < na) out_a[i] = s;
  else if (out_b) out_b[i - na] = s;
}

// ---------------------------------------------------------------------------
// gated RMSNorm: D/8 lanes per row, 32/(D/8) rows per warp
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) norm_gate_fwd_kernel(const bf16* x, const bf16* gate, const float* weight,
                                                           float eps, int64_t rows, bf16* y, float* rstd) {
  constexpr int LPR = D / 8, RPW = 32 / LPR;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * 8 + warp) * RPW + lane / LPR;
  const int c0 = (lane % LPR) * 8;
  const bool ok = row < rows;
  float xv[8], gv[8], wv[8];
  if (ok) {
    ld8(x + row * D + c0, xv);
    ld8(gate + row * D + c0, gv);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = gv[i] = 0.f;
  }
  ld8(weight + c0, wv);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += xv[i] * xv[i];
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rs = rsqrtf(ss / D + eps);
  if (!ok) return;
#pragma unroll
  for (int i = 0; i < 8; ++i) xv[i] = xv[i] * rs * wv[i] * gv[i] * sigmoid_f(gv[i]);
  st8(y + row * D + c0, xv);
  if (lane % LPR == 0) rstd[row] = rs;
}

template <int D>
__global__ void __launch_bounds__(256)
    norm_gate_bwd_kernel(const bf16* dy, const bf16* x, const bf16* gate, const float* weight, const float* rstd,
                         int64_t rows, bf16* dx, bf16* dgate, float* part) {
  constexpr int LPR = D / 8, RPW = 32 / LPR, kRowsPerCta = 8 * RPW;
  __shared__ float red[8][256];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = (lane % LPR) * 8;
  float wv[8], dwa[8];
  ld8(weight + c0, wv);
#pragma unroll
  for (int i = 0; i < 8; ++i) dwa[i] = 0.f;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kRowsPerCta; base < rows;
       base += static_cast<int64_t>(gridDim.x) * kRowsPerCta) {
    const int64_t row = base + warp * RPW + lane / LPR;
    const bool ok = row < rows;
    float xv[8], gv[8], dv[8], dxh[8];
    float rs = 0.f;
    if (ok) {
      ld8(x + row * D + c0, xv);
      ld8(gate + row * D + c0, gv);
      ld8(dy + row * D + c0, dv);
      rs = rstd[row];
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) xv[i] = gv[i] = dv[i] = 0.f;
    }
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float s = sigmoid_f(gv[i]);
      const float xh = xv[i] * rs;
      const float dyn = dv[i] * gv[i] * s;                         // d(normalised * weight)
      gv[i] = dv[i] * xh * wv[i] * s * (1.f + gv[i] * (1.f - s));  // dgate
      dwa[i] += dyn * xh;
      dxh[i] = dyn * wv[i];
      dot += dxh[i] * xh;
      xv[i] = xh;
    }
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    if (ok) {
      const float mdot = dot / D;
#pragma unroll
      for (int i = 0; i < 8; ++i) dxh[i] = rs * (dxh[i] - xv[i] * mdot);
      st8(dx + row * D + c0, dxh);
      st8(dgate + row * D + c0, gv);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red[i][threadIdx.x] = dwa[i];
  __syncthreads();
  if (threadIdx.x < D) {
    const int c = threadIdx.x, gi = c / 8, i = c % 8;
    float s = 0.f;
    for (int w = 0; w < 8; ++w)
      for (int rr = 0; rr < RPW; ++rr) s += red[i][w * 32 + rr * LPR + gi];
    part[static_cast<int64_t>(blockIdx.x) * D + c] = s;
  }
}

int64_t norm_bwd_ctas(int64_t rows, int64_t D) {
  const int64_t rpc = 8 * (32 / (D / 8));
  return std::min<int64_t>((rows + rpc - 1) / rpc, kNormBwdMaxCtas);
}

bool aligned16(const void* p) { return !(reinterpret_cast<uintptr_t>(p) & 15); }

int check_prep(const gdn2_prep_args* a, bool need_ptrs = true) {
  if (!a) return GDN2_ERR_NULL_POINTER;
  if (a->rows < 0 || a->N < 0 || a->Dk <= 0 || a->Dv <= 0 || a->Dfg < 0) return GDN2_ERR_SHAPE;
  if (a->Dk % 8 || a->Dv % 8 || a->Dfg % 8) return GDN2_ERR_SHAPE;
  if (a->conv_size != 0 && (a->conv_size < 2 || a->conv_size > 4)) return GDN2_ERR_SHAPE;
  if (a->proj_stride % 8 || a->proj_stride < 3 * a->Dk + 2 * a->Dv + 2 * a->Dfg) return GDN2_ERR_SHAPE;
  if (a->flags != 0) return GDN2_ERR_FLAGS;
  if (a->cu_seqlens) {
    if (a->N < 1) return GDN2_ERR_SHAPE;
  } else if (a->rows > 0) {
    if (a->T <= 0 || a->rows % a->T || a->N != a->rows / a->T) return GDN2_ERR_SHAPE;
  }
  if (!need_ptrs) return GDN2_OK;
  if (a->rows > 0 && (!a->proj || !a->q || !a->k || !a->v || !a->b || !a->w)) return GDN2_ERR_NULL_POINTER;
  if ((a->f0 == nullptr) != (a->g0 == nullptr)) return GDN2_ERR_NULL_POINTER;
  if (a->f0 && a->Dfg == 0) return GDN2_ERR_SHAPE;
  if (a->conv_size > 0 && !a->conv_weight) return GDN2_ERR_NULL_POINTER;
  if (a->conv_size == 0 && (a->conv_state_in || a->conv_state_out)) return GDN2_ERR_FLAGS;
  if (a->conv_state_out && a->conv_state_out == a->conv_state_in && a->rows != a->N) return GDN2_ERR_FLAGS;
  const void* ptrs[] = {a->proj, a->q, a->k, a->v, a->b, a->w, a->f0, a->g0};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return GDN2_ERR_ALIGNMENT;
  return GDN2_OK;
}

constexpr int kFwdNV = 8, kBwdNV = 4;

template <int W>
cudaError_t prep_fwd_launch(const gdn2_prep_args& a, cudaStream_t s) {
  const PrepGeom g = prep_geom(a, kFwdNV);
  const dim3 grid(static_cast<unsigned>((g.G + 31) / 32), static_cast<unsigned>(g.grid_y));
  ProfScope ps(kKLayerPrepFwd, s);
  layer_prep_fwd_kernel<W, kFwdNV><<<grid, kPrepWarps * 32, 0, s>>>(a, g);
  return cudaGetLastError();
}

template <int W>
cudaError_t prep_bwd_launch(const gdn2_prep_args& a, const gdn2_prep_grads& gr, float* part, cudaStream_t s) {
  const PrepGeom g = prep_geom(a, kBwdNV);
  const dim3 grid(static_cast<unsigned>((g.G + 31) / 32), static_cast<unsigned>(g.grid_y));
  {
    ProfScope ps(kKLayerPrepBwd, s);
    layer_prep_bwd_kernel<W, kBwdNV><<<grid, kPrepWarps * 32, 0, s>>>(a, gr, g, part);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || W == 0) return e;
  const int64_t na = g.C * W, nb = g.C;
  reduce_partials_kernel<<<static_cast<unsigned>((na + nb + 255) / 256), 256, 0, s>>>(part, g.grid_y, na, nb,
                                                                                     gr.dconv_weight, gr.dconv_bias);
  return cudaGetLastError();
}

}  // namespace
}  // namespace gdn2

using namespace gdn2;

extern "C" {

int gdn2_layer_prep_fwd(const gdn2_prep_args* a, gdn2_stream_t stream) {
  const int st = check_prep(a);
  if (st) return st;
  if (a->rows == 0) return GDN2_OK;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (a->conv_size) {
    case 0: e = prep_fwd_launch<0>(*a, s); break;
    case 2: e = prep_fwd_launch<2>(*a, s); break;
    case 3: e = prep_fwd_launch<3>(*a, s); break;
    default: e = prep_fwd_launch<4>(*a, s); break;
  }
  return e == cudaSuccess ? GDN2_OK : -static_cast<int>(e);
}

size_t gdn2_layer_prep_bwd_workspace_size(const gdn2_prep_args* a) {
  if (check_prep(a, false) != GDN2_OK || a->conv_size == 0) return 0;
  const PrepGeom g = prep_geom(*a, kBwdNV);
  return static_cast<size_t>(g.grid_y * g.C * (a->conv_size + 1)) * sizeof(float);
}

int gdn2_layer_prep_bwd(const gdn2_prep_args* a, const gdn2_prep_grads* gr, void* workspace, size_t workspace_bytes,
                        gdn2_stream_t stream) {
  const int st = check_prep(a);
  if (st) return st;
  if (!gr) return GDN2_ERR_NULL_POINTER;
  if (a->rows > 0 && (!gr->dq || !gr->dk || !gr->dv || !gr->db || !gr->dw || !gr->dproj))
    return GDN2_ERR_NULL_POINTER;
  if (a->conv_size > 0 && !gr->dconv_weight) return GDN2_ERR_NULL_POINTER;
  if (a->conv_bias && a->conv_size > 0 && !gr->dconv_bias) return GDN2_ERR_NULL_POINTER;
  const void* ptrs[] = {gr->dq, gr->dk, gr->dv, gr->db, gr->dw, gr->df0, gr->dg0, gr->dproj};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return GDN2_ERR_ALIGNMENT;
  const size_t need = gdn2_layer_prep_bwd_workspace_size(a);
  if (need > workspace_bytes || (need > 0 && !workspace)) return GDN2_ERR_WORKSPACE;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (a->rows == 0) {
    // no rows: the parameter gradients are zero
    if (a->conv_size > 0) {
      const int64_t C = 2 * a->Dk + a->Dv;
      cudaError_t e = cudaMemsetAsync(gr->dconv_weight, 0, C * a->conv_size * sizeof(float), s);
      if (e == cudaSuccess && gr->dconv_bias) e = cudaMemsetAsync(gr->dconv_bias, 0, C * sizeof(float), s);
      if (e != cudaSuccess) return -static_cast<int>(e);
    }
    return GDN2_OK;
  }
  float* part = reinterpret_cast<float*>(workspace);
  cudaError_t e;
  switch (a->conv_size) {
    case 0: e = prep_bwd_launch<0>(*a, *gr, part, s); break;
    case 2: e = prep_bwd_launch<2>(*a, *gr, part, s); break;
    case 3: e = prep_bwd_launch<3>(*a, *gr, part, s); break;
    default: e = prep_bwd_launch<4>(*a, *gr, part, s); break;
  }
  return e == cudaSuccess ? GDN2_OK : -static_cast<int>(e);
}

int gdn2_norm_gate_fwd(const void* x, const void* gate, const float* weight, float eps, int64_t rows, int64_t D,
                       void* y, float* rstd, gdn2_stream_t stream) {
  if (rows < 0) return GDN2_ERR_SHAPE;
  if (D != 64 && D != 128 && D != 256) return GDN2_ERR_UNSUPPORTED_DIM;
  if (rows == 0) return GDN2_OK;
  if (!x || !gate || !weight || !y || !rstd) return GDN2_ERR_NULL_POINTER;
  if (!aligned16(x) || !aligned16(gate) || !aligned16(weight) || !aligned16(y)) return GDN2_ERR_ALIGNMENT;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t rpc = 8 * (32 / (D / 8));
  const unsigned grid = static_cast<unsigned>((rows + rpc - 1) / rpc);
  const bf16* xb = reinterpret_cast<const bf16*>(x);
  const bf16* gb = reinterpret_cast<const bf16*>(gate);
  bf16* yb = reinterpret_cast<bf16*>(y);
  {
    ProfScope ps(kKNormGateFwd, s);
    if (D == 64) norm_gate_fwd_kernel<64><<<grid, 256, 0, s>>>(xb, gb, weight, eps, rows, yb, rstd);
    else if (D == 128) norm_gate_fwd_kernel<128><<<grid, 256, 0, s>>>(xb, gb, weight, eps, rows, yb, rstd);
    else norm_gate_fwd_kernel<256><<<grid, 256, 0, s>>>(xb, gb, weight, eps, rows, yb, rstd);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GDN2_OK : -static_cast<int>(e);
}

size_t gdn2_norm_gate_bwd_workspace_size(int64_t rows, int64_t D) {
  if (rows <= 0 || (D != 64 && D != 128 && D != 256)) return 0;
  return static_cast<size_t>(norm_bwd_ctas(rows, D) * D) * sizeof(float);
}

int gdn2_norm_gate_bwd(const void* dy, const void* x, const void* gate, const float* weight, const float* rstd,
                       int64_t rows, int64_t D, void* dx, void* dgate, float* dweight, void* workspace,
                       size_t workspace_bytes, gdn2_stream_t stream) {
  if (rows < 0) return GDN2_ERR_SHAPE;
  if (D != 64 && D != 128 && D != 256) return GDN2_ERR_UNSUPPORTED_DIM;
  if (!dweight) return GDN2_ERR_NULL_POINTER;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (rows == 0) {
    const cudaError_t e = cudaMemsetAsync(dweight, 0, D * sizeof(float), s);
    return e == cudaSuccess ? GDN2_OK : -static_cast<int>(e);
  }
  if (!dy || !x || !gate || !weight || !rstd || !dx || !dgate) return GDN2_ERR_NULL_POINTER;
  const void* ptrs[] = {dy, x, gate, weight, dx, dgate};
  for (const void* p : ptrs)
    if (!aligned16(p)) return GDN2_ERR_ALIGNMENT;
  const size_t need = gdn2_norm_gate_bwd_workspace_size(rows, D);
  if (need > workspace_bytes || !workspace) return GDN2_ERR_WORKSPACE;
  const int64_t nct = norm_bwd_ctas(rows, D);
  float* part = reinterpret_cast<float*>(workspace);
  const bf16 *dyb = reinterpret_cast<const bf16*>(dy), *xb = reinterpret_cast<const bf16*>(x),
             *gb = reinterpret_cast<const bf16*>(gate);
  bf16 *dxb = reinterpret_cast<bf16*>(dx), *dgb = reinterpret_cast<bf16*>(dgate);
  {
    ProfScope ps(kKNormGateBwd, s);
    const unsigned grid = static_cast<unsigned>(nct);
    if (D == 64) norm_gate_bwd_kernel<64><<<grid, 256, 0, s>>>(dyb, xb, gb, weight, rstd, rows, dxb, dgb, part);
    else if (D == 128) norm_gate_bwd_kernel<128><<<grid, 256, 0, s>>>(dyb, xb, gb, weight, rstd, rows, dxb, dgb, part);
    else norm_gate_bwd_kernel<256><<<grid, 256, 0, s>>>(dyb, xb, gb, weight, rstd, rows, dxb, dgb, part);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return -static_cast<int>(e);
  reduce_partials_kernel<<<static_cast<unsigned>((D + 255) / 256), 256, 0, s>>>(part, nct, D, 0, dweight, nullptr);
  e = cudaGetLastError();
  return e == cudaSuccess ? GDN2_OK : -static_cast<int>(e);
}

}  // extern "C"
