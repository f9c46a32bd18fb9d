// The GatedDeltaNet2 layer's memory-bound passes around the operator
// (lit_gpt/gdn2.py:282-464), each one read and one write of its tensors:
//
//   layer_prep_fwd_kernel  merged projection rows q|k|v|b|w|f0|g0 ->
//                          SiLU(short causal depthwise conv) for q, k, v
//                          (fla ShortConvolution, gdn2.py:342-367), sigmoid
//                          gates b, w (gdn2.py:383-384, :410-412), contiguous
//                          f0, g0 for the second-stage GEMMs;
//   layer_prep_bwd_kernel  the reverse pass, with per-CTA conv weight / bias
//                          partial sums reduced in a fixed order;
//   norm_gate_fwd/bwd      FusedRMSNormSwishGate (gdn2.py:462; fla
//                          fused_norm_gate.py:35-104).
//
// Thread layout of the prep kernels: a lane owns NV = 4 consecutive channels
// (an 8-byte vector of a row, so a warp touches 256 contiguous bytes of each
// row) and a warp walks a segment of kPrepRows rows, kPrepU rows per group of
// loads; the 8 warps of a CTA take 8 consecutive segments of the same 128
// channels.  The conv taps of a row are the previous W-1 rows of the same
// sequence, held in registers while the warp walks forward.
#include <algorithm>

#include "chunk_layout.cuh"
#include "common.cuh"
#include "profile.cuh"
#include "tc.cuh"

namespace gdn2 {
namespace {

using bf16 = __nv_bfloat16;

constexpr int kPrepWarps = 8;
constexpr int kPrepRows = 32;
constexpr int kPrepRowsPerCta = kPrepWarps * kPrepRows;
constexpr int kBwdRows = 16;  // backward rows per warp (plus W-1 staged rows after them)
constexpr int kNV = 4;        // channels per lane
constexpr int kNormBwdMaxCtas = 1184;  // fixed so the dweight reduction order never depends on the device

struct PrepGeom {
  int64_t C;                 // conv channels 2Dk+Dv (= proj column of b_raw)
  int64_t Gc, Gs, Gf, G;     // 4-channel groups: conv, sigmoid, copy, total
  int64_t off_f;             // proj column of f0 (g0 follows)
  int64_t grid_y;            // row tiles (rows per CTA: 8 warps x rows per warp)
};

PrepGeom prep_geom(const gdn2_prep_args& a, int NV, int rows_per_cta) {
  PrepGeom g;
  g.C = 2 * a.Dk + a.Dv;
  g.Gc = g.C / NV;
  g.Gs = (a.Dk + a.Dv) / NV;
  g.Gf = a.f0 ? 2 * a.Dfg / NV : 0;
  g.G = g.Gc + g.Gs + g.Gf;
  g.off_f = g.C + a.Dk + a.Dv;
  g.grid_y = (a.rows + rows_per_cta - 1) / rows_per_cta;
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

GDN2_DEV float silu(float z) { return __fdividef(z, 1.f + __expf(-z)); }
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

// Fault word of the layer kernels: bit 1 = a bounded wait on a staging
// barrier gave up (that launch's outputs are invalid).
__device__ unsigned int g_layer_fault;

// ---------------------------------------------------------------------------
// bulk staging of a warp's strip: rows [r, r + n) x channels [col0, col0 + 128)
// ---------------------------------------------------------------------------
constexpr int kStripCh = 32 * kNV;         // channels of a column tile (a warp's strip)
constexpr int kStripBytes = kStripCh * 2;  // bf16

// Lane 0 only.  Copies rows [r, r + n) of columns [lo, hi) (channels of the
// strip starting at col0) from `src` (row stride ld, column c at src + c - base)
// into buf (kStripCh bf16 per row); returns the bytes it queued.
GDN2_DEV uint32_t stage_rows(bf16* buf, const bf16* src, int64_t ld, int64_t base, int64_t col0, int64_t lo,
                             int64_t hi, int64_t r, int n, uint64_t* bar) {
  if (hi <= lo || !src) return 0;
  const uint32_t bytes = static_cast<uint32_t>((hi - lo) * 2);
  const bf16* p = src + r * ld + (lo - base);
  bf16* d = buf + (lo - col0);
  for (int i = 0; i < n; ++i) tc::bulk_load(d + i * kStripCh, p + i * ld, bytes, bar);
  return bytes * n;
}

// waits for the strip; on a timeout records it, gives the copies one more
// bounded wait and reports failure (the caller abandons its rows)
GDN2_DEV bool strip_wait(uint64_t* bar) {
  if (tc::mbar_wait(bar, 0)) return true;
  atomicOr(&g_layer_fault, 2u);
  tc::mbar_wait(bar, 0);
  return false;
}

// Forward.  Each warp stages its kPrepRows x 128-channel strip of the
// projection with bulk copies (all rows in flight at once), then every lane
// computes its 4 channels row by row from shared memory.
template <int W>
__global__ void __launch_bounds__(kPrepWarps * 32, 3) layer_prep_fwd_kernel(gdn2_prep_args a, PrepGeom g) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t r0 = (static_cast<int64_t>(blockIdx.y) * kPrepWarps + warp) * kPrepRows;
  if (r0 >= a.rows) return;  // warps are independent: no CTA barrier below
  const int64_t r1 = min(r0 + kPrepRows, a.rows);
  const int nrow = static_cast<int>(r1 - r0);
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * kStripCh;
  const int64_t width = g.G * kNV;  // staged columns: q|k|v|b|w (|f0|g0)
  bf16* buf = reinterpret_cast<bf16*>(smem_raw) + warp * kPrepRows * kStripCh;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw + kPrepWarps * kPrepRows * kStripBytes) + warp;
  const bf16* proj = reinterpret_cast<const bf16*>(a.proj);
  if (lane == 0) {
    tc::mbar_init(bar, 1);
    tc::mbar_fence_init();
    const uint32_t bytes = static_cast<uint32_t>((min(col0 + kStripCh, width) - col0) * 2) * nrow;
    tc::mbar_arrive_expect_tx(bar, bytes);
    stage_rows(buf, proj, a.proj_stride, 0, col0, col0, min(col0 + kStripCh, width), r0, nrow, bar);
  }
  __syncwarp();
  const int64_t grp = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  const bf16* xrow = buf + lane * kNV;  // this lane's 4 channels of staged row 0

  if (grp < g.Gc) {  // ---- q, k, v: SiLU(conv) --------------------------------
    const int64_t c0 = grp * kNV;
    const OutSlot o = conv_slot(a, c0);
    float wt[W > 0 ? W : 1][kNV], bias[kNV];
    float win[W > 1 ? W - 1 : 1][kNV];  // win[j]: input of row r - (W-1) + j
    Seq sq{0, 0, 0};
    bf16* st_out = reinterpret_cast<bf16*>(a.conv_state_out);
    if constexpr (W > 0) {  // set up while the strip is in flight
#pragma unroll
      for (int i = 0; i < kNV; ++i) {
#pragma unroll
        for (int j = 0; j < W; ++j) wt[j][i] = a.conv_weight[(c0 + i) * W + j];
        bias[i] = a.conv_bias ? a.conv_bias[c0 + i] : 0.f;
      }
      sq = seq_of(a, r0);
#pragma unroll
      for (int j = 0; j < W - 1; ++j) conv_tap<W, kNV>(a, g, sq, r0 - (W - 1) + j, c0, win[j]);
    }
    if (!strip_wait(bar)) return;
    bf16* op = o.p + r0 * o.ld + o.col;
#pragma unroll 4
    for (int i = 0; i < nrow; ++i, op += o.ld) {
      const int64_t r = r0 + i;
      float x[kNV], y[kNV];
      ldv<kNV>(xrow + i * kStripCh, x);
      if constexpr (W == 0) {
#pragma unroll
        for (int c = 0; c < kNV; ++c) y[c] = silu(x[c]);
      } else {
        if (r == sq.e) {  // a new sequence starts: its history is its cache
          sq = seq_of(a, r);
#pragma unroll
          for (int j = 0; j < W - 1; ++j) conv_tap<W, kNV>(a, g, sq, r - (W - 1) + j, c0, win[j]);
        }
#pragma unroll
        for (int c = 0; c < kNV; ++c) {
          float z = bias[c] + wt[W - 1][c] * x[c];
#pragma unroll
          for (int j = 0; j < W - 1; ++j) z += wt[j][c] * win[j][c];
          y[c] = silu(z);
        }
        if (st_out && r == sq.e - 1) {  // the sequence's last W inputs
          bf16* p = st_out + (sq.n * g.C + c0) * W;
#pragma unroll
          for (int c = 0; c < kNV; ++c) {
#pragma unroll
            for (int j = 0; j < W - 1; ++j) p[c * W + j] = __float2bfloat16_rn(win[j][c]);
            p[c * W + W - 1] = __float2bfloat16_rn(x[c]);
          }
        }
#pragma unroll
        for (int j = 0; j + 1 < W - 1; ++j)
#pragma unroll
          for (int c = 0; c < kNV; ++c) win[j][c] = win[j + 1][c];
#pragma unroll
        for (int c = 0; c < kNV; ++c) win[W - 2][c] = x[c];
      }
      stv<kNV>(op, y);
    }
  } else if (grp < g.Gc + g.Gs) {  // ---- b, w: sigmoid gates ----------------
    const int64_t s0 = (grp - g.Gc) * kNV;
    const bool is_b = s0 < a.Dk;
    bf16* out = reinterpret_cast<bf16*>(is_b ? a.b : a.w);
    const int64_t old = is_b ? a.Dk : a.Dv, oc = is_b ? s0 : s0 - a.Dk;
    const float sc = is_b ? a.b_scale : 1.f;
    if (!strip_wait(bar)) return;
    bf16* op = out + r0 * old + oc;
#pragma unroll 4
    for (int i = 0; i < nrow; ++i, op += old) {
      float x[kNV];
      ldv<kNV>(xrow + i * kStripCh, x);
#pragma unroll
      for (int c = 0; c < kNV; ++c) x[c] = sc * sigmoid_f(x[c]);
      stv<kNV>(op, x);
    }
  } else if (grp < g.G) {  // ---- f0, g0: contiguous copies ---------------------
    const int64_t f = (grp - g.Gc - g.Gs) * kNV;
    const bool is_f = f < a.Dfg;
    bf16* out = reinterpret_cast<bf16*>(is_f ? a.f0 : a.g0);
    const int64_t oc = is_f ? f : f - a.Dfg;
    if (!strip_wait(bar)) return;
    bf16* op = out + r0 * a.Dfg + oc;
#pragma unroll 4
    for (int i = 0; i < nrow; ++i, op += a.Dfg)
      *reinterpret_cast<uint2*>(op) = *reinterpret_cast<const uint2*>(xrow + i * kStripCh);
  } else {
    strip_wait(bar);  // no channels: still let the copies land before the warp exits
  }
}

// Backward.  Each warp stages the projection and the cotangents of rows
// [r0, t_end) (its kBwdRows rows and, for the convolution, the W-1 rows after
// them) with bulk copies; the cotangent strip is assembled from the section
// tensors it crosses (dq | dk | dv | db | dw | df0 | dg0).  A lane then walks
// its rows forward: d(pre-activation) dz_t needs the conv inputs of rows
// t-(W-1)..t (register window, as in the forward) and feeds the input
// cotangents of rows t-(W-1)..t, whose sums stay pending in registers; row
// t-(W-1) is complete (and stored) at step t.  Partial sums of the conv
// parameter gradients per CTA row tile: part[tile][C*W + C] (weights c*W + j,
// then bias).
template <int W>
__global__ void __launch_bounds__(kPrepWarps * 32, 2)
    layer_prep_bwd_kernel(gdn2_prep_args a, gdn2_prep_grads gr, PrepGeom g, float* part) {
  constexpr int kAcc = (W > 0 ? W + 1 : 1) * kNV;  // conv weight + bias sums of a lane's channels
  constexpr int kRowsSt = kBwdRows + (W > 0 ? W - 1 : 0);
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t r0 = (static_cast<int64_t>(blockIdx.y) * kPrepWarps + warp) * kBwdRows;
  const bool rows_ok = r0 < a.rows;
  const int64_t r1 = min(r0 + kBwdRows, a.rows);
  const int64_t t_end = W > 0 ? min(r1 + W - 1, a.rows) : r1;
  const int nst = rows_ok ? static_cast<int>(t_end - r0) : 0;
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * kStripCh;
  const int64_t width = g.G * kNV;
  const int64_t col1 = min(col0 + kStripCh, width);
  bf16* bx = reinterpret_cast<bf16*>(smem_raw) + warp * 2 * kRowsSt * kStripCh;
  bf16* bd = bx + kRowsSt * kStripCh;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw + kPrepWarps * 2 * kRowsSt * kStripBytes) + warp;
  const bf16* proj = reinterpret_cast<const bf16*>(a.proj);
  bf16* dproj = reinterpret_cast<bf16*>(gr.dproj);
  const int64_t ld = a.proj_stride;
  if (rows_ok && lane == 0) {
    tc::mbar_init(bar, 1);
    tc::mbar_fence_init();
    // sections of the strip's columns: [start, end) in proj order, source, row stride
    const int64_t Dk = a.Dk, Dv = a.Dv, C = g.C, F = g.off_f;
    const int64_t st[7] = {0, Dk, 2 * Dk, C, C + Dk, F, F + a.Dfg};
    const int64_t en[7] = {Dk, 2 * Dk, C, C + Dk, C + Dk + Dv, F + a.Dfg, F + 2 * a.Dfg};
    const bf16* srcs[7] = {reinterpret_cast<const bf16*>(gr.dq), reinterpret_cast<const bf16*>(gr.dk),
                           reinterpret_cast<const bf16*>(gr.dv), reinterpret_cast<const bf16*>(gr.db),
                           reinterpret_cast<const bf16*>(gr.dw), reinterpret_cast<const bf16*>(gr.df0),
                           reinterpret_cast<const bf16*>(gr.dg0)};
    const int64_t lds[7] = {Dk, Dk, Dv, Dk, Dv, a.Dfg, a.Dfg};
    uint32_t bytes = static_cast<uint32_t>((col1 - col0) * 2) * nst;
    for (int k = 0; k < 7; ++k) {
      const int64_t lo = max(col0, st[k]), hi = min(col1, en[k]);
      if (hi > lo && srcs[k]) bytes += static_cast<uint32_t>((hi - lo) * 2) * nst;
    }
    tc::mbar_arrive_expect_tx(bar, bytes);
    stage_rows(bx, proj, ld, 0, col0, col0, col1, r0, nst, bar);
    for (int k = 0; k < 7; ++k)
      stage_rows(bd, srcs[k], lds[k], st[k], col0, max(col0, st[k]), min(col1, en[k]), r0, nst, bar);
  }
  __syncwarp();
  const int64_t grp = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  const bool active = rows_ok && grp < g.G;
  const bf16* xrow = bx + lane * kNV;
  const bf16* drow = bd + lane * kNV;
  float acc[kAcc];
#pragma unroll
  for (int i = 0; i < kAcc; ++i) acc[i] = 0.f;
  bool staged = true;
  if (rows_ok) staged = strip_wait(bar);

  if (active && staged && grp < g.Gc) {  // ---- q, k, v ------------------------------
    const int64_t c0 = grp * kNV;
    if constexpr (W == 0) {
      for (int i = 0; i < nst; ++i) {
        float x[kNV], dy[kNV];
        ldv<kNV>(xrow + i * kStripCh, x);
        ldv<kNV>(drow + i * kStripCh, dy);
#pragma unroll
        for (int c = 0; c < kNV; ++c) dy[c] *= silu_grad(x[c]);
        stv<kNV>(dproj + (r0 + i) * ld + c0, dy);
      }
    } else {
      float wt[W][kNV], bias[kNV];
#pragma unroll
      for (int c = 0; c < kNV; ++c) {
#pragma unroll
        for (int j = 0; j < W; ++j) wt[j][c] = a.conv_weight[(c0 + c) * W + j];
        bias[c] = a.conv_bias ? a.conv_bias[c0 + c] : 0.f;
      }
      float win[W - 1][kNV];   // conv inputs of rows t-(W-1) .. t-1
      float pend[W - 1][kNV];  // pending input cotangents of rows t-(W-1) .. t-1
      Seq sq = seq_of(a, r0);
#pragma unroll
      for (int j = 0; j < W - 1; ++j) {
        conv_tap<W, kNV>(a, g, sq, r0 - (W - 1) + j, c0, win[j]);
#pragma unroll
        for (int c = 0; c < kNV; ++c) pend[j][c] = 0.f;
      }
      // row `row` is ours to store when it lies in [r0, r1) and in the lane's current sequence
      auto emit = [&](int64_t row, const float* v) {
        if (row >= r0 && row < r1 && row >= sq.s) stv<kNV>(dproj + row * ld + c0, v);
      };
      bool done = false;
      for (int i = 0; i < nst; ++i) {
        const int64_t t = r0 + i;
        if (t == sq.e) {  // the pending rows of the finished sequence are complete
#pragma unroll
          for (int j = 0; j < W - 1; ++j) emit(t - (W - 1) + j, pend[j]);
          if (t >= r1) {
            done = true;
            break;
          }
          sq = seq_of(a, t);
#pragma unroll
          for (int j = 0; j < W - 1; ++j) {
            conv_tap<W, kNV>(a, g, sq, t - (W - 1) + j, c0, win[j]);
#pragma unroll
            for (int c = 0; c < kNV; ++c) pend[j][c] = 0.f;
          }
        }
        float x[kNV], dy[kNV], dz[kNV], fin[kNV];
        ldv<kNV>(xrow + i * kStripCh, x);
        ldv<kNV>(drow + i * kStripCh, dy);
#pragma unroll
        for (int c = 0; c < kNV; ++c) {
          float z = bias[c] + wt[W - 1][c] * x[c];
#pragma unroll
          for (int j = 0; j < W - 1; ++j) z += wt[j][c] * win[j][c];
          dz[c] = dy[c] * silu_grad(z);
          fin[c] = pend[0][c] + wt[0][c] * dz[c];  // row t-(W-1) is complete
        }
        emit(t - (W - 1), fin);
        if (t < r1) {
#pragma unroll
          for (int c = 0; c < kNV; ++c) {
#pragma unroll
            for (int j = 0; j < W - 1; ++j) acc[j * kNV + c] += dz[c] * win[j][c];
            acc[(W - 1) * kNV + c] += dz[c] * x[c];
            acc[W * kNV + c] += dz[c];
          }
        }
        // shift: pend[j] <- pend[j+1] + wt[j+1] dz ; the newest pending row is t
#pragma unroll
        for (int j = 0; j < W - 1; ++j)
#pragma unroll
          for (int c = 0; c < kNV; ++c)
            pend[j][c] = (j + 1 < W - 1 ? pend[j + 1][c] : 0.f) + wt[j + 1][c] * dz[c];
#pragma unroll
        for (int j = 0; j + 1 < W - 1; ++j)
#pragma unroll
          for (int c = 0; c < kNV; ++c) win[j][c] = win[j + 1][c];
#pragma unroll
        for (int c = 0; c < kNV; ++c) win[W - 2][c] = x[c];
      }
      // the end of the data completes the rows still pending
      if (!done && t_end == a.rows) {
#pragma unroll
        for (int j = 0; j < W - 1; ++j) emit(t_end - (W - 1) + j, pend[j]);
      }
    }
  } else if (active && staged && grp < g.Gc + g.Gs) {  // ---- b, w --------------------
    const int64_t s0 = (grp - g.Gc) * kNV;
    const float sc = s0 < a.Dk ? a.b_scale : 1.f;
    bf16* op = dproj + r0 * ld + g.C + s0;
    const int n = static_cast<int>(r1 - r0);
#pragma unroll 4
    for (int i = 0; i < n; ++i, op += ld) {
      float x[kNV], d[kNV];
      ldv<kNV>(xrow + i * kStripCh, x);
      ldv<kNV>(drow + i * kStripCh, d);
#pragma unroll
      for (int c = 0; c < kNV; ++c) {
        const float sg = sigmoid_f(x[c]);
        d[c] *= sc * sg * (1.f - sg);
      }
      stv<kNV>(op, d);
    }
  } else if (active && staged) {  // ---- f0, g0 ----------------------------------------
    const int64_t f = (grp - g.Gc - g.Gs) * kNV;
    const bool has = f < a.Dfg ? gr.df0 != nullptr : gr.dg0 != nullptr;
    for (int64_t r = r0; r < r1; ++r) {
      const int i = static_cast<int>(r - r0);
      *reinterpret_cast<uint2*>(dproj + r * ld + g.off_f + f) =
          has ? *reinterpret_cast<const uint2*>(drow + i * kStripCh) : make_uint2(0, 0);
    }
  }

  if constexpr (W > 0) {
    // CTA-uniform: only column tiles holding conv channels reduce.  The
    // staging buffers are free once every warp is past its rows.
    if (static_cast<int64_t>(blockIdx.x) * 32 >= g.Gc) return;
    __syncthreads();
    float* red = reinterpret_cast<float*>(smem_raw);
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
      const int j = k / kNV, i = k % kNV;
      const int64_t c = gg * kNV + i;
      float* pt = part + static_cast<int64_t>(blockIdx.y) * g.C * (W + 1);
      if (j < W) pt[c * W + j] = sacc;
      else pt[g.C * W + c] = sacc;
    }
  }
}

template <int W>
constexpr size_t bwd_smem_bytes() {
  return static_cast<size_t>(kPrepWarps) * 2 * (kBwdRows + (W > 0 ? W - 1 : 0)) * kStripBytes +
         kPrepWarps * sizeof(uint64_t);
}
constexpr size_t kFwdSmemBytes = static_cast<size_t>(kPrepWarps) * kPrepRows * kStripBytes + kPrepWarps * sizeof(uint64_t);

// out_a[i] (i < na) / out_b[i - na] = sum over p < nparts of part[p * (na + nb) + i].
// A CTA owns 32 columns; thread (x, y) sums partials y, y + 32, ... of column
// x with four running sums (independent loads in flight), then the 32 sums of
// a column are added in y order: a fixed order, so the result is reproducible.
constexpr int kRedThreads = 1024;
__global__ void __launch_bounds__(kRedThreads) reduce_partials_kernel(const float* part, int64_t nparts, int64_t na,
                                                                      int64_t nb, float* out_a, float* out_b) {
  __shared__ float red[32][33];
  const int x = threadIdx.x & 31, y = threadIdx.x >> 5;
  const int64_t n = na + nb, i = static_cast<int64_t>(blockIdx.x) * 32 + x;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (i < n) {
    int64_t p = y;
    for (; p + 96 < nparts; p += 128) {
      s0 += part[p * n + i];
      s1 += part[(p + 32) * n + i];
      s2 += part[(p + 64) * n + i];
      s3 += part[(p + 96) * n + i];
    }
    for (; p < nparts; p += 32) s0 += part[p * n + i];
  }
  red[y][x] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (y == 0 && i < n) {
    float t = 0.f;
#pragma unroll 8
    for (int k = 0; k < 32; ++k) t += red[k][x];
    if (i < na) out_a[i] = t;
    else if (out_b) out_b[i - na] = t;
  }
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

template <int W>
cudaError_t prep_fwd_launch(const gdn2_prep_args& a, cudaStream_t s) {
  const PrepGeom g = prep_geom(a, kNV, kPrepRowsPerCta);
  const dim3 grid(static_cast<unsigned>((g.G + 31) / 32), static_cast<unsigned>(g.grid_y));
  cudaError_t e = cudaFuncSetAttribute(layer_prep_fwd_kernel<W>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kFwdSmemBytes));
  if (e != cudaSuccess) return e;
  ProfScope ps(kKLayerPrepFwd, s);
  layer_prep_fwd_kernel<W><<<grid, kPrepWarps * 32, kFwdSmemBytes, s>>>(a, g);
  return cudaGetLastError();
}

template <int W>
cudaError_t prep_bwd_launch(const gdn2_prep_args& a, const gdn2_prep_grads& gr, float* part, cudaStream_t s) {
  const PrepGeom g = prep_geom(a, kNV, kPrepWarps * kBwdRows);
  const dim3 grid(static_cast<unsigned>((g.G + 31) / 32), static_cast<unsigned>(g.grid_y));
  constexpr size_t smem = bwd_smem_bytes<W>();
  cudaError_t e = cudaFuncSetAttribute(layer_prep_bwd_kernel<W>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  {
    ProfScope ps(kKLayerPrepBwd, s);
    layer_prep_bwd_kernel<W><<<grid, kPrepWarps * 32, smem, s>>>(a, gr, g, part);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess || W == 0) return e;
  const int64_t na = g.C * W, nb = g.C;
  reduce_partials_kernel<<<static_cast<unsigned>((na + nb + 31) / 32), kRedThreads, 0, s>>>(
      part, g.grid_y, na, nb, gr.dconv_weight, gr.dconv_bias);
  return cudaGetLastError();
}

}  // namespace

int layer_fault_read(int clear, unsigned int* out) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_layer_fault, sizeof(v));
  if (e == cudaSuccess && clear && v) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_layer_fault, &z, sizeof(z));
  }
  *out = v;
  return e == cudaSuccess ? 0 : -static_cast<int>(e);
}

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
  const PrepGeom g = prep_geom(*a, kNV, kPrepWarps * kBwdRows);
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
  reduce_partials_kernel<<<static_cast<unsigned>((D + 31) / 32), kRedThreads, 0, s>>>(part, nct, D, 0, dweight,
                                                                                        nullptr);
  e = cudaGetLastError();
  return e == cudaSuccess ? GDN2_OK : -static_cast<int>(e);
}

}  // extern "C"
