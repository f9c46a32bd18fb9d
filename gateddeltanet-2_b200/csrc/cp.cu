// Context-parallel (T sharded over ranks) pieces of the chunkwise forward.
//
// A shard of a sequence maps the state it receives affinely:
//     S_out = M S_in + h_e,   M = prod_c (Diag(2^G_last,c) - kg_c^T Y_c)  (K x K)
// because within a chunk  S' = Diag(2^G_last) S + kg^T (U - Y S).
// gdn2_cp_transition runs the intra kernel on the shard and the scan on the
// augmented state [S_M | S] (chunk_fwd.cu, kTrans): no K x K x K products.
// gdn2_cp_compose folds the gathered maps of the ranks before this one into
// the entering state, S <- M_j S + h_j for j = 0 .. rank-1, in fp32; the
// caller then reruns gdn2_chunk_fwd on its shard from that state.
// This mirrors the KDA context-parallel pre-process / merge of the reference
// (lit_gpt/gdn2_ops/chunk_kda.py:102-330, :346-482, :774-852), which GDN2
// shares the scan kernels with but never enables (chunk_gdn2.py:86-92).
#include "chunk_layout.cuh"
#include "common.cuh"
#include "profile.cuh"

namespace {

constexpr int kComposeThreads = 256;
constexpr int kComposeBV = 32;

// one CTA per (sequence x head, 32-column tile of the state)
template <int K>
__global__ void __launch_bounds__(kComposeThreads)
cp_compose_kernel(const float* __restrict__ maps, int rank, int64_t NH, int64_t V, float* __restrict__ state) {
  extern __shared__ float cp_smem[];
  float (*Ms)[K + 1] = reinterpret_cast<float (*)[K + 1]>(cp_smem);
  float (*Ss)[kComposeBV + 1] = reinterpret_cast<float (*)[kComposeBV + 1]>(cp_smem + K * (K + 1));
  const int tid = threadIdx.x;
  const int64_t nh = blockIdx.y;
  const int v0 = blockIdx.x * kComposeBV;
  const int64_t W = K + V;
  float* st = state + nh * (int64_t)K * V;
  for (int i = tid; i < K * kComposeBV; i += kComposeThreads) {
    const int r = i / kComposeBV, c = i % kComposeBV;
    Ss[r][c] = st[(int64_t)r * V + v0 + c];
  }
  constexpr int kPer = K * kComposeBV / kComposeThreads;
  for (int j = 0; j < rank; ++j) {
    const float* mp = maps + ((int64_t)j * NH + nh) * K * W;
    __syncthreads();
    for (int i = tid; i < K * K; i += kComposeThreads) Ms[i / K][i % K] = mp[(int64_t)(i / K) * W + (i % K)];
    __syncthreads();
    float out[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int i = tid + u * kComposeThreads, r = i / kComposeBV, c = i % kComposeBV;
      float acc = mp[(int64_t)r * W + K + v0 + c];
      for (int x = 0; x < K; ++x) acc = fmaf(Ms[r][x], Ss[x][c], acc);
      out[u] = acc;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int i = tid + u * kComposeThreads;
      Ss[i / kComposeBV][i % kComposeBV] = out[u];
    }
  }
  __syncthreads();
  for (int i = tid; i < K * kComposeBV; i += kComposeThreads) {
    const int r = i / kComposeBV, c = i % kComposeBV;
    st[(int64_t)r * V + v0 + c] = Ss[r][c];
  }
}

// Backward fold over the ranks after `rank`, one CTA per (sequence x head,
// 32-column tile): X <- M_j^T X + g_j for j = world-1 .. rank+1 (X = 0 first),
// then dstate += X.
template <int K>
__global__ void __launch_bounds__(kComposeThreads)
cp_compose_bwd_kernel(const float* __restrict__ maps, const float* __restrict__ gs, int rank, int world, int64_t NH,
                      int64_t V, float* __restrict__ dstate) {
  extern __shared__ float cp_smem[];
  float (*Mt)[K + 1] = reinterpret_cast<float (*)[K + 1]>(cp_smem);  // Mt[x][r] = M[r][x]
  float (*Xs)[kComposeBV + 1] = reinterpret_cast<float (*)[kComposeBV + 1]>(cp_smem + K * (K + 1));
  const int tid = threadIdx.x;
  const int64_t nh = blockIdx.y;
  const int v0 = blockIdx.x * kComposeBV;
  const int64_t W = K + V;
  for (int i = tid; i < K * kComposeBV; i += kComposeThreads) Xs[i / kComposeBV][i % kComposeBV] = 0.f;
  constexpr int kPer = K * kComposeBV / kComposeThreads;
  for (int j = world - 1; j > rank; --j) {
    const float* mp = maps + ((int64_t)j * NH + nh) * K * W;
    const float* gp = gs + ((int64_t)j * NH + nh) * K * V;
    __syncthreads();
    for (int i = tid; i < K * K; i += kComposeThreads) Mt[i % K][i / K] = mp[(int64_t)(i / K) * W + (i % K)];
    __syncthreads();
    float out[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int i = tid + u * kComposeThreads, r = i / kComposeBV, c = i % kComposeBV;
      float acc = gp[(int64_t)r * V + v0 + c];
      for (int x = 0; x < K; ++x) acc = fmaf(Mt[r][x], Xs[x][c], acc);
      out[u] = acc;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int i = tid + u * kComposeThreads;
      Xs[i / kComposeBV][i % kComposeBV] = out[u];
    }
  }
  __syncthreads();
  float* st = dstate + nh * (int64_t)K * V;
  for (int i = tid; i < K * kComposeBV; i += kComposeThreads) {
    const int r = i / kComposeBV, c = i % kComposeBV;
    st[(int64_t)r * V + v0 + c] += Xs[r][c];
  }
}

bool dim_ok(int64_t d) { return d == 64 || d == 128; }

}  // namespace

using namespace gdn2;

extern "C" int gdn2_cp_transition(const gdn2_chunk_args* a, float* maps, void* workspace, size_t workspace_bytes,
                                  gdn2_stream_t stream) {
  if (!a || !maps) return GDN2_ERR_NULL_POINTER;
  if (a->cu_seqlens) return GDN2_ERR_SHAPE;  // shards are dense [B, T_shard]
  if (a->flags & (GDN2_SAVE_FOR_BWD | GDN2_STORE_FINAL | GDN2_TRANSPOSE_STATE)) return GDN2_ERR_FLAGS;
  if (!dim_ok(a->K) || !dim_ok(a->V)) return GDN2_ERR_UNSUPPORTED_DIM;
  if (a->dtype_qkv != GDN2_BF16 || (a->dtype_bw != GDN2_BF16 && a->dtype_bw != GDN2_F32)) return GDN2_ERR_DTYPE;
  if (a->B < 0 || a->T < 0 || a->H <= 0 || a->N != a->B || a->NT != a->B * ((a->T + 63) / 64))
    return GDN2_ERR_SHAPE;
  if (a->B * a->T > 0 && (!a->q || !a->k || !a->v || !a->g || !a->b || !a->w)) return GDN2_ERR_NULL_POINTER;
  if ((a->flags & GDN2_GATE_IN_KERNEL) && !a->A_log) return GDN2_ERR_NULL_POINTER;
  if ((a->flags & GDN2_HAS_H0) && !a->h0) return GDN2_ERR_NULL_POINTER;
  const void* ptrs[] = {a->q, a->k, a->v, a->b, a->w, a->g};
  for (const void* p : ptrs)
    if (p && (reinterpret_cast<uintptr_t>(p) & 15)) return GDN2_ERR_ALIGNMENT;
  const size_t need = chunk_ws_layout(*a, nullptr, nullptr);
  if (need > workspace_bytes || (need > 0 && !workspace)) return GDN2_ERR_WORKSPACE;
  if (a->N == 0 || a->B * a->T == 0) return GDN2_OK;
  ChunkWs ws;
  chunk_ws_layout(*a, workspace, &ws);
  return chunk_transition_launch(*a, ws, maps, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int gdn2_cp_compose(const float* gathered_maps, int32_t rank, int64_t N, int64_t H, int64_t K, int64_t V,
                               float* state, gdn2_stream_t stream) {
  if (!gathered_maps || !state) return GDN2_ERR_NULL_POINTER;
  if (rank < 0 || N < 0 || H <= 0) return GDN2_ERR_SHAPE;
  if (!dim_ok(K) || !dim_ok(V)) return GDN2_ERR_UNSUPPORTED_DIM;
  if (rank == 0 || N == 0) return GDN2_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid((unsigned)(V / kComposeBV), (unsigned)(N * H));
  ProfScope ps(kKCp, s);
  if (K == 128) {
    const int sm = (128 * 129 + 128 * (kComposeBV + 1)) * 4;
    cudaError_t e = cudaFuncSetAttribute(cp_compose_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
    if (e != cudaSuccess) return -static_cast<int>(e);
    cp_compose_kernel<128><<<grid, kComposeThreads, sm, s>>>(gathered_maps, rank, N * H, V, state);
  } else {
    const int sm = (64 * 65 + 64 * (kComposeBV + 1)) * 4;
    cp_compose_kernel<64><<<grid, kComposeThreads, sm, s>>>(gathered_maps, rank, N * H, V, state);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : -static_cast<int>(e);
}

extern "C" int gdn2_cp_compose_bwd(const float* gathered_maps, const float* gathered_g, int32_t rank, int32_t world,
                                   int64_t N, int64_t H, int64_t K, int64_t V, float* dstate, gdn2_stream_t stream) {
  if (!gathered_maps || !gathered_g || !dstate) return GDN2_ERR_NULL_POINTER;
  if (rank < 0 || world <= rank || N < 0 || H <= 0) return GDN2_ERR_SHAPE;
  if (!dim_ok(K) || !dim_ok(V)) return GDN2_ERR_UNSUPPORTED_DIM;
  if (rank == world - 1 || N == 0) return GDN2_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid((unsigned)(V / kComposeBV), (unsigned)(N * H));
  ProfScope ps(kKCp, s);
  if (K == 128) {
    const int sm = (128 * 129 + 128 * (kComposeBV + 1)) * 4;
    cudaError_t e =
        cudaFuncSetAttribute(cp_compose_bwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm);
    if (e != cudaSuccess) return -static_cast<int>(e);
    cp_compose_bwd_kernel<128><<<grid, kComposeThreads, sm, s>>>(gathered_maps, gathered_g, rank, world, N * H,
                                                                 V, dstate);
  } else {
    const int sm = (64 * 65 + 64 * (kComposeBV + 1)) * 4;
    cp_compose_bwd_kernel<64><<<grid, kComposeThreads, sm, s>>>(gathered_maps, gathered_g, rank, world, N * H, V,
                                                                dstate);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : -static_cast<int>(e);
}
