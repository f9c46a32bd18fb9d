// Token-serial GDN2 recurrence (decode / short prefill).
//
// Same per-token math as the reference kernel fused_recurrent_gdn2_fwd_kernel
// (lit_gpt/gdn2_ops/fused_recurrent_gdn2.py:193-243):
//     S <- Diag(exp(g)) S ; u = w*v - S^T(b*k) ; S <- S + k u^T ; o = S^T(scale q)
// B200 design: one CTA per (sequence, value head, 32-column V tile); the
// [K x 32] fp32 state tile lives in registers (each thread owns 8 rows x one
// float4 of columns), is read once with coalesced 128-bit loads and written
// once with 128-bit stores.  Both K-reductions (S^T(b*k) and S^T q) come out
// of the same pass over the tile: warp shuffles, then a cross-warp smem step.
// o uses S_new^T q = S_dec^T q + u (k.q), so the state is touched once per token.
#include <type_traits>

#include "chunk_layout.cuh"
#include "common.cuh"
#include "profile.cuh"

namespace gdn2 {

namespace {

constexpr int kRecThreads = 128;
constexpr int kRecBV = 32;                  // state columns per CTA
constexpr int kRecColGroups = kRecBV / 4;   // float4 groups per row (8)
constexpr int kRecRowStep = kRecThreads / kRecColGroups;  // 16 rows per pass

// 8 resident CTAs per SM (64 registers a thread): the 16 KiB state tiles of
// eight CTAs in flight per SM keep the HBM pipe full (measured 83% of the copy
// bandwidth at 256 x 16 heads, against 66% at the unconstrained 127 registers).
template <typename TQ, typename TG, int K, bool kTransposed, bool kCkpt>
__global__ void __launch_bounds__(kRecThreads, 8)
recurrent_kernel(gdn2_recurrent_args a, RecCheckpoints ck) {
  constexpr int kRows = K / kRecRowStep;  // rows per thread (8 for K=128)
  __shared__ float s_q[K], s_k[K], s_bk[K], s_alpha[K];
  __shared__ float s_v[kRecBV], s_w[kRecBV];
  __shared__ float s_red[kRecThreads / 32][2][kRecBV];
  __shared__ float s_scal[kRecThreads / 32][3];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t V = a.V, H = a.H, HV = a.HV;
  const int nvt = (int)(V / kRecBV);
  const int64_t pid = blockIdx.x;
  const int iv = (int)(pid % nvt);
  const int64_t nh = pid / nvt;
  const int64_t n = nh / HV;
  const int64_t hv = nh % HV;
  const int64_t h = hv / (HV / H);  // key head (grouped value heads)

  int64_t bos, T;
  if (a.cu_seqlens) {
    bos = a.cu_seqlens[n];
    T = a.cu_seqlens[n + 1] - bos;
  } else {
    bos = n * a.T;
    T = a.T;
  }
  if (T <= 0) return;

  const int cg = tid % kRecColGroups;   // float4 column group
  const int r0 = tid / kRecColGroups;   // first row
  const int c0 = iv * kRecBV + cg * 4;  // global V column of this thread's float4

  // ---- initial state ---------------------------------------------------------
  float st[kRows][4];
  const float* h0 = nullptr;
  if (a.flags & GDN2_HAS_H0) {
    int64_t slot = n;
    if (a.ssm_state_indices) {
      int64_t i0 = a.num_accepted_tokens ? (int64_t)a.num_accepted_tokens[n] - 1 : 0;
      slot = a.ssm_state_indices[n * a.stride_indices_seq + i0];
    }
    h0 = a.h0 + slot * a.state_slot_stride_in + hv * (int64_t)K * V;
  }
#pragma unroll
  for (int i = 0; i < kRows; ++i) {
    const int r = r0 + i * kRecRowStep;
    if (h0) {
      if (!kTransposed) {
        const float4 x = *reinterpret_cast<const float4*>(h0 + (int64_t)r * V + c0);
        st[i][0] = x.x; st[i][1] = x.y; st[i][2] = x.z; st[i][3] = x.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) st[i][e] = h0[(int64_t)(c0 + e) * K + r];
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) st[i][e] = 0.f;
    }
  }

  const bool l2 = a.flags & GDN2_L2NORM_QK;
  const bool gate = a.flags & GDN2_GATE_IN_KERNEL;
  const bool lb = a.flags & GDN2_LOWER_BOUND;
  const float A = gate ? __expf(a.A_log[h]) : 0.f;
  const TQ* q = static_cast<const TQ*>(a.q);
  const TQ* k = static_cast<const TQ*>(a.k);
  const TQ* v = static_cast<const TQ*>(a.v);
  const TG* g = static_cast<const TG*>(a.g);
  const TG* b = static_cast<const TG*>(a.b);
  const TG* w = static_cast<const TG*>(a.w);
  TQ* o = static_cast<TQ*>(a.o);

  for (int64_t t = 0; t < T; ++t) {
    const int64_t tok = bos + t;
    // the chunked fp32 path keeps the state entering every 64-token chunk
    if (kCkpt && (t & 63) == 0) {
      const int64_t c = (ck.chunk_offset ? (int64_t)ck.chunk_offset[n] : n * ck.chunks_per_seq) + (t >> 6);
      float* dst = ck.states + (c * HV + hv) * (int64_t)K * V;
#pragma unroll
      for (int i = 0; i < kRows; ++i)
        *reinterpret_cast<float4*>(dst + (int64_t)(r0 + i * kRecRowStep) * V + c0) =
            make_float4(st[i][0], st[i][1], st[i][2], st[i][3]);
    }
    // ---- per-token vectors into smem, with l2norm / gate activation ----------
    float pq = 0.f, pk = 0.f, pqk = 0.f;
    for (int c = tid; c < K; c += kRecThreads) {
      const float qv = to_f(q[(tok * H + h) * K + c]);
      const float kv = to_f(k[(tok * H + h) * K + c]);
      s_q[c] = qv;
      s_k[c] = kv;
      pq += qv * qv;
      pk += kv * kv;
      pqk += qv * kv;
      float gv = to_f(g[(tok * HV + hv) * K + c]);
      if (gate) {
        if (a.dt_bias) gv += a.dt_bias[h * K + c];
        gv = lb ? a.lower_bound * sigmoid_f(A * gv) : -A * softplus_f(gv);
      }
      s_alpha[c] = __expf(gv);
      s_bk[c] = to_f(b[(tok * HV + hv) * K + c]);  // times k below
    }
    if (tid < kRecBV) {
      const int64_t vi = (tok * HV + hv) * V + iv * kRecBV + tid;
      s_v[tid] = to_f(v[vi]);
      s_w[tid] = to_f(w[vi]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      pq += __shfl_xor_sync(0xffffffffu, pq, off);
      pk += __shfl_xor_sync(0xffffffffu, pk, off);
      pqk += __shfl_xor_sync(0xffffffffu, pqk, off);
    }
    if (lane == 0) {
      s_scal[warp][0] = pq;
      s_scal[warp][1] = pk;
      s_scal[warp][2] = pqk;
    }
    __syncthreads();
    float sq = 0.f, sk = 0.f, sqk = 0.f;
#pragma unroll
    for (int i = 0; i < kRecThreads / 32; ++i) {
      sq += s_scal[i][0];
      sk += s_scal[i][1];
      sqk += s_scal[i][2];
    }
    const float rq = l2 ? rsqrtf(sq + kL2Eps) : 1.f;
    const float rk = l2 ? rsqrtf(sk + kL2Eps) : 1.f;
    const float qscale = rq * a.scale;  // q_eff = q * rq * scale
    const float kdotq = sqk * rk * qscale;

    // ---- decay + both K-reductions in one pass ------------------------------
    float er[4] = {0.f, 0.f, 0.f, 0.f}, qs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int r = r0 + i * kRecRowStep;
      const float al = s_alpha[r];
      const float kr = s_k[r] * rk;
      const float bkr = s_bk[r] * kr;
      const float qr = s_q[r] * qscale;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        st[i][e] *= al;
        er[e] += st[i][e] * bkr;
        qs[e] += st[i][e] * qr;
      }
    }
    // lanes l, l^8, l^16, l^24 share the column group
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      er[e] += __shfl_xor_sync(0xffffffffu, er[e], 8);
      er[e] += __shfl_xor_sync(0xffffffffu, er[e], 16);
      qs[e] += __shfl_xor_sync(0xffffffffu, qs[e], 8);
      qs[e] += __shfl_xor_sync(0xffffffffu, qs[e], 16);
    }
    if (lane < kRecColGroups) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s_red[warp][0][cg * 4 + e] = er[e];
        s_red[warp][1][cg * 4 + e] = qs[e];
      }
    }
    __syncthreads();
    float u[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float E = 0.f;
#pragma unroll
      for (int wi = 0; wi < kRecThreads / 32; ++wi) E += s_red[wi][0][cg * 4 + e];
      u[e] = s_w[cg * 4 + e] * s_v[cg * 4 + e] - E;
    }
    // o = S_dec^T q + u (k.q): one thread per column
    if (tid < kRecBV) {
      float Q = 0.f;
#pragma unroll
      for (int wi = 0; wi < kRecThreads / 32; ++wi) Q += s_red[wi][1][tid];
      float E = 0.f;
#pragma unroll
      for (int wi = 0; wi < kRecThreads / 32; ++wi) E += s_red[wi][0][tid];
      const float uc = s_w[tid] * s_v[tid] - E;
      o[(tok * HV + hv) * V + iv * kRecBV + tid] = from_f<TQ>(Q + uc * kdotq);
    }
    // rank-one write
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const float kr = s_k[r0 + i * kRecRowStep] * rk;
#pragma unroll
      for (int e = 0; e < 4; ++e) st[i][e] += kr * u[e];
    }
    // serving pool: every token's state goes to its slot
    if (a.ssm_state_indices && (a.flags & GDN2_STORE_FINAL)) {
      int64_t slot;
      if (a.inplace) slot = a.ssm_state_indices[n * a.stride_indices_seq + t];
      else slot = tok;
      float* dst = a.ht + slot * a.state_slot_stride_out + hv * (int64_t)K * V;
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        const int r = r0 + i * kRecRowStep;
        if (!kTransposed) {
          *reinterpret_cast<float4*>(dst + (int64_t)r * V + c0) =
              make_float4(st[i][0], st[i][1], st[i][2], st[i][3]);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) dst[(int64_t)(c0 + e) * K + r] = st[i][e];
        }
      }
    }
    __syncthreads();  // smem vectors are rewritten by the next token
  }

  if (!a.ssm_state_indices && (a.flags & GDN2_STORE_FINAL)) {
    float* dst = a.ht + n * a.state_slot_stride_out + hv * (int64_t)K * V;
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int r = r0 + i * kRecRowStep;
      if (!kTransposed) {
        *reinterpret_cast<float4*>(dst + (int64_t)r * V + c0) =
            make_float4(st[i][0], st[i][1], st[i][2], st[i][3]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) dst[(int64_t)(c0 + e) * K + r] = st[i][e];
      }
    }
  }
}

template <typename TQ, typename TG, int K>
cudaError_t launch_rec(const gdn2_recurrent_args& a, const RecCheckpoints& ck, cudaStream_t s) {
  const int64_t grid = a.N * a.HV * (a.V / kRecBV);
  if (grid == 0) return cudaSuccess;
  ProfScope ps(kKRecurrent, s);
  const bool tr = a.flags & GDN2_TRANSPOSE_STATE;
  if (ck.states) {  // the chunked fp32 path (fp32 inputs only)
    if constexpr (std::is_same<TQ, float>::value && std::is_same<TG, float>::value) {
      if (tr) recurrent_kernel<TQ, TG, K, true, true><<<(unsigned)grid, kRecThreads, 0, s>>>(a, ck);
      else recurrent_kernel<TQ, TG, K, false, true><<<(unsigned)grid, kRecThreads, 0, s>>>(a, ck);
      return cudaGetLastError();
    }
    return cudaErrorInvalidValue;
  }
  if (tr) recurrent_kernel<TQ, TG, K, true, false><<<(unsigned)grid, kRecThreads, 0, s>>>(a, ck);
  else recurrent_kernel<TQ, TG, K, false, false><<<(unsigned)grid, kRecThreads, 0, s>>>(a, ck);
  return cudaGetLastError();
}

template <typename TQ, typename TG>
cudaError_t dispatch_k(const gdn2_recurrent_args& a, const RecCheckpoints& ck, cudaStream_t s) {
  if (a.K == 128) return launch_rec<TQ, TG, 128>(a, ck, s);
  return launch_rec<TQ, TG, 64>(a, ck, s);
}

}  // namespace

int recurrent_fwd(const gdn2_recurrent_args& a, cudaStream_t s, const RecCheckpoints& ck) {
  cudaError_t e;
  const bool qbf = a.dtype_qkv == GDN2_BF16, gbf = a.dtype_gbw == GDN2_BF16;
  if (qbf && gbf) e = dispatch_k<__nv_bfloat16, __nv_bfloat16>(a, ck, s);
  else if (qbf) e = dispatch_k<__nv_bfloat16, float>(a, ck, s);
  else if (gbf) e = dispatch_k<float, __nv_bfloat16>(a, ck, s);
  else e = dispatch_k<float, float>(a, ck, s);
  return e == cudaSuccess ? 0 : -static_cast<int>(e);
}

}  // namespace gdn2
