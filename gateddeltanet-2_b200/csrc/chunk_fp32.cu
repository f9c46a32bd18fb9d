// The chunk op for fp32 inputs: token-serial fp32 arithmetic end to end, so
// fp32 callers get the recurrence to fp32 rounding (the bf16 tensor-core path
// rounds its operands to bf16).  The reference computes fp32 inputs in fp32
// as well (chunk_gdn2.py:1205-1359 with fp32 dots; to ~5e-7 of the naive fp32
// recurrence under the Triton interpreter).
//
//   fp32_prep_kernel      l2norm of q, k (fla l2norm_fwd, eps 1e-6 inside the
//                         sqrt) and the gate activation, once per token row;
//   recurrent_kernel      (recurrent.cu) the forward, which also keeps the
//                         fp32 state entering every 64-token chunk;
//   chunk_bwd_fp32_kernel the reverse pass, one CTA per (sequence, head): per
//                         chunk (last first) it recomputes the states entering
//                         each token from the chunk's checkpoint, then runs the
//                         reverse-mode recurrence token by token;
//   fp32_epilogue_kernel  the l2norm and gate VJPs (dA_log, ddt_bias).
//
// Per token, with S' = Diag(exp g) S_prev, u = w*v - S'^T(b*k),
// S = S' + k u^T, o = S^T (scale q), and dS the cotangent of S:
//   dSt = dS + scale q do^T ;  dq = scale S do ;  du = dSt^T k ;  dk = dSt u
//   dS' = dSt - (b*k) du^T ;  d(b*k) = -S' du  (db = d(b*k) k, dk += d(b*k) b)
//   dg = rowsum(dS' * S') ;  dv = du * w ;  dw = du * v ;  dS_prev = Diag(exp g) dS'
#include "chunk_layout.cuh"
#include "common.cuh"
#include "profile.cuh"

namespace gdn2 {
namespace {

GDN2_DEV float softplus_exact(float x) { return x > 20.f ? x : log1pf(expf(x)); }
GDN2_DEV float sigmoid_exact(float x) { return 1.f / (1.f + expf(-x)); }

// ---------------------------------------------------------------------------
// prep: one warp per (token, head) row
// ---------------------------------------------------------------------------
constexpr int kPrepRows = 8;

template <int K>
__global__ void __launch_bounds__(32 * kPrepRows)
fp32_prep_kernel(const gdn2_chunk_args a, const ChunkWs ws, int64_t rows) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kPrepRows + warp;  // token * H + head
  if (row >= rows) return;
  const int64_t h = row % a.H;
  constexpr int E = K / 32;
  if (a.flags & GDN2_L2NORM_QK) {
    const float* q = static_cast<const float*>(a.q) + row * K;
    const float* k = static_cast<const float*>(a.k) + row * K;
    float qv[E], kv[E], sq = 0.f, sk = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      qv[e] = q[lane + 32 * e];
      kv[e] = k[lane + 32 * e];
      sq += qv[e] * qv[e];
      sk += kv[e] * kv[e];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      sq += __shfl_xor_sync(0xffffffffu, sq, off);
      sk += __shfl_xor_sync(0xffffffffu, sk, off);
    }
    const float rq = 1.f / sqrtf(sq + kL2Eps), rk = 1.f / sqrtf(sk + kL2Eps);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      ws.qf[row * K + lane + 32 * e] = qv[e] * rq;
      ws.kf[row * K + lane + 32 * e] = kv[e] * rk;
    }
    if (lane == 0) {
      ws.q_rstd[row] = rq;
      ws.k_rstd[row] = rk;
    }
  }
  if (a.flags & GDN2_GATE_IN_KERNEL) {
    const float* g = static_cast<const float*>(a.g) + row * K;
    const float A = expf(a.A_log[h]);
    const bool lb = a.flags & GDN2_LOWER_BOUND;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int c = lane + 32 * e;
      const float x = g[c] + (a.dt_bias ? a.dt_bias[h * K + c] : 0.f);
      ws.gf[row * K + c] = lb ? a.lower_bound * sigmoid_exact(A * x) : -A * softplus_exact(x);
    }
  }
}

// ---------------------------------------------------------------------------
// reverse pass: one CTA per (sequence, head), 512 threads.  Thread (r, q)
// holds row r of the state (and of its cotangent) for the CPT columns of
// column group q; the G = 512 / K threads of a row are adjacent lanes.
// ---------------------------------------------------------------------------
constexpr int kB32Threads = 512;

template <int K, int V>
__global__ void __launch_bounds__(kB32Threads, 1)
chunk_bwd_fp32_kernel(const gdn2_chunk_args a, const gdn2_chunk_grads gr, const ChunkWs ws, const BwdWs bw) {
  constexpr int G = kB32Threads / K, CPT = V / G, RW = 32 / G, NW = kB32Threads / 32;
  __shared__ float s_q[K], s_k[K], s_b[K], s_bk[K], s_al[K];
  __shared__ float s_v[V], s_w[V], s_do[V], s_du[V];
  __shared__ __align__(16) float s_u[64][V];  // u of every token of the chunk
  __shared__ float s_red[NW][V];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r = warp * RW + lane / G, q = lane % G, j0 = q * CPT;
  const int64_t H = a.H, nh = blockIdx.x, n = nh / H, h = nh % H;
  SeqGeom geo{a.cu_seqlens, a.chunk_index, a.chunk_offset, a.T, (a.T + kChunk - 1) / kChunk};
  int64_t bos, len;
  geo.seq(n, bos, len);
  const int nchunks = (int)((len + kChunk - 1) / kChunk);
  const int64_t c0 = geo.chunk0(n);
  const bool tr = a.flags & GDN2_TRANSPOSE_STATE;
  const bool state_only = a.flags & GDN2_BWD_STATE_ONLY;
  const bool l2 = a.flags & GDN2_L2NORM_QK, gate = a.flags & GDN2_GATE_IN_KERNEL;
  const float scale = a.scale;
  const float* qf = ws.qf;
  const float* kf = ws.kf;
  const float* gf = ws.gf;
  const float* bb = static_cast<const float*>(a.b);
  const float* vv = static_cast<const float*>(a.v);
  const float* ww = static_cast<const float*>(a.w);
  const float* dout = static_cast<const float*>(gr.dout);
  float* dq_out = l2 ? bw.dqf : static_cast<float*>(gr.dq);
  float* dk_out = l2 ? bw.dkf : static_cast<float*>(gr.dk);
  float* dg_out = gate ? bw.dgf : static_cast<float*>(gr.dg);
  float* db_out = static_cast<float*>(gr.db);
  float* dv_out = static_cast<float*>(gr.dv);
  float* dw_out = static_cast<float*>(gr.dw);
  float* stp = bw.tok_states + nh * (int64_t)kChunk * K * V;

  // K-vectors by threads [0, K), V-vectors by threads [K, K + V)
  auto load_vectors = [&](int64_t tok, bool with_q) {
    if (tid < K) {
      const int64_t i = (tok * H + h) * K + tid;
      const float kv = kf[i], bv = bb[i];
      s_k[tid] = kv;
      s_b[tid] = bv;
      s_bk[tid] = bv * kv;
      s_al[tid] = expf(gf[i]);
      if (with_q) s_q[tid] = qf[i];
    } else if (tid < K + V) {
      const int c = tid - K;
      const int64_t i = (tok * H + h) * V + c;
      s_v[c] = vv[i];
      s_w[c] = ww[i];
      if (with_q) s_do[c] = dout[i];
    }
  };
  // column sums over the K rows of x[CPT] (this thread's columns) -> s_du-like target
  auto column_sum = [&](float (&x)[CPT], float* target) {
#pragma unroll
    for (int e = 0; e < CPT; ++e)
#pragma unroll
      for (int off = G; off < 32; off <<= 1) x[e] += __shfl_xor_sync(0xffffffffu, x[e], off);
    if (lane < G) {
#pragma unroll
      for (int e = 0; e < CPT; ++e) s_red[warp][j0 + e] = x[e];
    }
    __syncthreads();
    if (tid < V) {
      float acc = 0.f;
#pragma unroll
      for (int w2 = 0; w2 < NW; ++w2) acc += s_red[w2][tid];
      target[tid] = acc;
    }
    __syncthreads();
  };
  auto row_sum = [&](float x) {
#pragma unroll
    for (int off = 1; off < G; off <<= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    return x;
  };

  float dS[CPT];
#pragma unroll
  for (int e = 0; e < CPT; ++e) {
    const float* d = gr.dht ? gr.dht + nh * (int64_t)K * V : nullptr;
    dS[e] = d ? (tr ? d[(int64_t)(j0 + e) * K + r] : d[(int64_t)r * V + j0 + e]) : 0.f;
  }
  for (int c = nchunks - 1; c >= 0; --c) {
    const int64_t t0 = bos + (int64_t)c * kChunk;
    const int64_t rem = len - (int64_t)c * kChunk;
    const int L = (int)(rem < kChunk ? rem : kChunk);
    // forward over the chunk from its checkpoint: keep each token's entering
    // state (global scratch) and its u (shared memory)
    float S[CPT];
    {
      const float* ck = ws.ckpt + ((c0 + c) * H + h) * (int64_t)K * V + (int64_t)r * V + j0;
#pragma unroll
      for (int e = 0; e < CPT; e += 4) {
        const float4 x = *reinterpret_cast<const float4*>(ck + e);
        S[e] = x.x, S[e + 1] = x.y, S[e + 2] = x.z, S[e + 3] = x.w;
      }
    }
    for (int i = 0; i < L; ++i) {
      __syncthreads();  // the previous token's vectors are no longer read
      load_vectors(t0 + i, false);
      float* sp = stp + ((int64_t)i * K + r) * V + j0;
#pragma unroll
      for (int e = 0; e < CPT; e += 4) *reinterpret_cast<float4*>(sp + e) = make_float4(S[e], S[e + 1], S[e + 2], S[e + 3]);
      __syncthreads();
      const float al = s_al[r], bk = s_bk[r], kr = s_k[r];
      float p[CPT];
#pragma unroll
      for (int e = 0; e < CPT; ++e) {
        S[e] *= al;
        p[e] = S[e] * bk;
      }
      column_sum(p, s_du);
      if (tid < V) s_u[i][tid] = s_w[tid] * s_v[tid] - s_du[tid];
      __syncthreads();
#pragma unroll
      for (int e = 0; e < CPT; ++e) S[e] += kr * s_u[i][j0 + e];
    }
    // reverse over the chunk's tokens
    for (int i = L - 1; i >= 0; --i) {
      const int64_t tok = t0 + i;
      __syncthreads();
      load_vectors(tok, true);
      __syncthreads();
      const float al = s_al[r], bk = s_bk[r], kr = s_k[r], br = s_b[r], qr = s_q[r] * scale;
      const float* sp = stp + ((int64_t)i * K + r) * V + j0;
      // two sweeps over the entering state (re-read from L1/L2) keep the live
      // registers at dS plus one column vector
      float x[CPT];
      float dq_p = 0.f, dk_p = 0.f;
#pragma unroll
      for (int e = 0; e < CPT; e += 4) {
        const float4 y4 = *reinterpret_cast<const float4*>(sp + e);
        const float y[4] = {y4.x, y4.y, y4.z, y4.w};
#pragma unroll
        for (int f = 0; f < 4; ++f) {
          const float u = s_u[i][j0 + e + f], d = s_do[j0 + e + f];
          const float Sd = al * y[f];
          const float dSt = dS[e + f] + qr * d;
          dq_p += (Sd + kr * u) * d;  // S = S' + k u^T
          dk_p += dSt * u;
          x[e + f] = dSt * kr;
        }
      }
      column_sum(x, s_du);  // du = dSt^T k
      float dbk_p = 0.f, dg_p = 0.f;
#pragma unroll
      for (int e = 0; e < CPT; e += 4) {
        const float4 y4 = *reinterpret_cast<const float4*>(sp + e);
        const float y[4] = {y4.x, y4.y, y4.z, y4.w};
#pragma unroll
        for (int f = 0; f < 4; ++f) {
          const float Sd = al * y[f];
          const float du = s_du[j0 + e + f];
          const float dSp = dS[e + f] + qr * s_do[j0 + e + f] - bk * du;
          dbk_p -= Sd * du;
          dg_p += dSp * Sd;
          dS[e + f] = al * dSp;
        }
      }
      dq_p = row_sum(dq_p);
      dk_p = row_sum(dk_p);
      dbk_p = row_sum(dbk_p);
      dg_p = row_sum(dg_p);
      if (!state_only) {
        if (q == 0) {
          const int64_t o = (tok * H + h) * K + r;
          dq_out[o] = scale * dq_p;
          dk_out[o] = dk_p + dbk_p * br;
          db_out[o] = dbk_p * kr;
          dg_out[o] = dg_p;
        }
        if (tid < V) {
          const int64_t o = (tok * H + h) * V + tid;
          dv_out[o] = s_du[tid] * s_w[tid];
          dw_out[o] = s_du[tid] * s_v[tid];
        }
      }
    }
  }
  if (gr.dh0) {
    float* d = gr.dh0 + nh * (int64_t)K * V;
#pragma unroll
    for (int e = 0; e < CPT; ++e) {
      if (tr) d[(int64_t)(j0 + e) * K + r] = dS[e];
      else d[(int64_t)r * V + j0 + e] = dS[e];
    }
  }
}

// ---------------------------------------------------------------------------
// epilogue: one warp per (token, head) row; the l2norm VJP
// dx = (dy - (dy . y) y) rstd (fla l2norm_bwd) and the gate VJP
// ---------------------------------------------------------------------------
template <int K>
__global__ void __launch_bounds__(32 * kPrepRows)
fp32_epilogue_kernel(const gdn2_chunk_args a, const gdn2_chunk_grads gr, const ChunkWs ws, const BwdWs bw,
                     int64_t rows) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kPrepRows + warp;
  if (row >= rows) return;
  const int64_t h = row % a.H;
  constexpr int E = K / 32;
  if (a.flags & GDN2_L2NORM_QK) {
    float dq[E], dk[E], yq[E], yk[E], sq = 0.f, sk = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int64_t i = row * K + lane + 32 * e;
      dq[e] = bw.dqf[i];
      dk[e] = bw.dkf[i];
      yq[e] = ws.qf[i];
      yk[e] = ws.kf[i];
      sq += dq[e] * yq[e];
      sk += dk[e] * yk[e];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      sq += __shfl_xor_sync(0xffffffffu, sq, off);
      sk += __shfl_xor_sync(0xffffffffu, sk, off);
    }
    const float rq = ws.q_rstd[row], rk = ws.k_rstd[row];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int64_t i = row * K + lane + 32 * e;
      static_cast<float*>(gr.dq)[i] = (dq[e] - sq * yq[e]) * rq;
      static_cast<float*>(gr.dk)[i] = (dk[e] - sk * yk[e]) * rk;
    }
  }
  if (a.flags & GDN2_GATE_IN_KERNEL) {
    const float* g = static_cast<const float*>(a.g) + row * K;
    const float A = expf(a.A_log[h]);
    const bool lb = a.flags & GDN2_LOWER_BOUND;
    float dA = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int c = lane + 32 * e;
      const float x = g[c] + (a.dt_bias ? a.dt_bias[h * K + c] : 0.f);
      const float dy = bw.dgf[row * K + c];
      float fo, fa;
      if (lb) {
        const float s2 = sigmoid_exact(A * x);
        fo = a.lower_bound * s2 * (1.f - s2) * A;
        fa = fo * x;
      } else {
        fo = -A * sigmoid_exact(x);
        fa = -A * softplus_exact(x);
      }
      const float dg = dy * fo;
      static_cast<float*>(gr.dg)[row * K + c] = dg;
      dA += dy * fa;
      if (a.dt_bias) atomicAdd(&gr.ddt_bias[h * K + c], dg);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dA += __shfl_xor_sync(0xffffffffu, dA, off);
    if (lane == 0) atomicAdd(&gr.dA_log[h], dA);
  }
}

template <int K, int V>
int launch_bwd_fp32_kv(const gdn2_chunk_args& a, const gdn2_chunk_grads& g, const ChunkWs& ws, const BwdWs& bw,
                       cudaStream_t s) {
  if (a.N * a.H > 0) {
    ProfScope ps(kKBwdFp32, s);
    chunk_bwd_fp32_kernel<K, V><<<(unsigned)(a.N * a.H), kB32Threads, 0, s>>>(a, g, ws, bw);
    GDN2_LAUNCH_CHECK();
  }
  const int64_t rows = a.B * a.T * a.H;
  if ((a.flags & (GDN2_L2NORM_QK | GDN2_GATE_IN_KERNEL)) && !(a.flags & GDN2_BWD_STATE_ONLY) && rows > 0) {
    ProfScope ps(kKFp32Aux, s);
    fp32_epilogue_kernel<K><<<(unsigned)((rows + kPrepRows - 1) / kPrepRows), 32 * kPrepRows, 0, s>>>(a, g, ws, bw,
                                                                                                     rows);
    GDN2_LAUNCH_CHECK();
  }
  return 0;
}

}  // namespace

int chunk_fwd_fp32_launch(const gdn2_chunk_args& a, const ChunkWs& ws, cudaStream_t s) {
  const int64_t rows = a.B * a.T * a.H;
  if ((a.flags & (GDN2_L2NORM_QK | GDN2_GATE_IN_KERNEL)) && rows > 0) {
    ProfScope ps(kKFp32Aux, s);
    const unsigned grid = (unsigned)((rows + kPrepRows - 1) / kPrepRows);
    if (a.K == 128) fp32_prep_kernel<128><<<grid, 32 * kPrepRows, 0, s>>>(a, ws, rows);
    else fp32_prep_kernel<64><<<grid, 32 * kPrepRows, 0, s>>>(a, ws, rows);
    GDN2_LAUNCH_CHECK();
  }
  gdn2_recurrent_args r{};
  r.B = a.B, r.T = a.T, r.H = a.H, r.HV = a.H, r.K = a.K, r.V = a.V, r.N = a.N;
  r.cu_seqlens = a.cu_seqlens;
  r.state_slot_stride_in = r.state_slot_stride_out = a.H * a.K * a.V;
  r.scale = a.scale;
  r.flags = a.flags & (GDN2_HAS_H0 | GDN2_STORE_FINAL | GDN2_TRANSPOSE_STATE);
  r.dtype_qkv = GDN2_F32, r.dtype_gbw = GDN2_F32;
  r.q = ws.qf, r.k = ws.kf, r.v = a.v, r.g = ws.gf, r.b = a.b, r.w = a.w;
  r.h0 = a.h0, r.ht = a.ht, r.o = a.o;
  RecCheckpoints ck;
  ck.states = ws.ckpt;  // nullptr unless the backward (or the chunk states) is wanted
  ck.chunk_offset = a.chunk_offset;
  ck.chunks_per_seq = (a.T + kChunk - 1) / kChunk;
  return recurrent_fwd(r, s, ck);
}

int chunk_bwd_fp32_launch(const gdn2_chunk_args& a, const gdn2_chunk_grads& g, const ChunkWs& ws, const BwdWs& bw,
                          cudaStream_t s) {
  if (a.K == 128 && a.V == 128) return launch_bwd_fp32_kv<128, 128>(a, g, ws, bw, s);
  if (a.K == 128 && a.V == 64) return launch_bwd_fp32_kv<128, 64>(a, g, ws, bw, s);
  if (a.K == 64 && a.V == 128) return launch_bwd_fp32_kv<64, 128>(a, g, ws, bw, s);
  return launch_bwd_fp32_kv<64, 64>(a, g, ws, bw, s);
}

}  // namespace gdn2
