// Chunkwise GDN2 backward (C = 64): the reference pipeline
//   chunk_gdn2_bwd (lit_gpt/gdn2_ops/chunk_gdn2.py:2330-2493)
//   = dAv (chunk_kda.py:3769-3831) -> dhu reverse scan (:1356-1669)
//     -> gate-aware WY VJP (chunk_gdn2.py:1554-1735) -> intra VJP (:1759-2019)
//     -> reverse cumsum of dg (:2477-2483) -> gate VJP (chunk_kda.py:2420-2555)
//     -> l2norm VJP (chunk_gdn2.py:2638-2640)
// as two B200 kernels.  The forward saved G, Aqk, A = (I+T)^-1, Y, kg, qg,
// v_new and the per-chunk entering states h, so nothing is recomputed.
//
// chunk_scan_bwd_kernel (one CTA per (sequence, head, 64-column V tile)),
// serial over chunks in reverse with the state cotangent dS [K x 64] in
// tensor-core accumulators:
//   dh[c]  = dS                                   (cotangent of the chunk's exit state)
//   dv_new = Aqk^T do + kg dS
//   dS    <- 2^G_last dS + qg^T do - Y^T dv_new     (qg carries the output scale)
//
// chunk_bwd_intra_kernel (one CTA per (chunk, head)), everything else in one
// pass with all [64 x K] accumulators (dq, dk, db, dG) in registers:
//   dq  = scale (do h^T) 2^G + intra ;  dk = (v_new dh^T) 2^(G_last-G) + ...
//   dY  = -dv_new h^T ;  d(w v) = A^T dv_new -> dv, dw
//   dA  = dv_new (w v)^T + dY (b k 2^G)^T ;  dT = -A^T dA A^T (strictly lower)
//   d(b k 2^G) = A^T dY -> db, dk, dG
//   intra: dAqk = scale do v_new^T, dT through the anchored score factors
//   (exact per-pair path for the (block, channel)s the forward flagged)
//   dG -> in-chunk reverse cumsum -> gate VJP; l2norm VJP on dq, dk.
#include <type_traits>

#include "common.cuh"
#include "chunk_layout.cuh"
#include "profile.cuh"
#include "tc.cuh"

namespace gdn2 {

GDN2_DEV void cp_async16b(void* dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)), "l"(src), "r"(n));
}
GDN2_DEV void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
GDN2_DEV void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// ---------------------------------------------------------------------------
// B2: reverse scan of the state cotangent
// ---------------------------------------------------------------------------
constexpr int kBScanThreads = 256;
constexpr int kBScanBV = 64;

template <int K>
struct BScanStage {
  static constexpr int LK = K + 8, LV = kBScanBV + 8, LA = kChunk + 8;
  alignas(16) __nv_bfloat16 Y[kChunk][LK];
  alignas(16) __nv_bfloat16 QG[kChunk][LK];
  alignas(16) __nv_bfloat16 KG[kChunk][LK];
  alignas(16) __nv_bfloat16 Aqk[kChunk][LA];
  alignas(16) __nv_bfloat16 DO[kChunk][LV];
  alignas(16) float glast[K];
};

template <int K>
struct BScanSmem {
  BScanStage<K> st[2];
  alignas(16) __nv_bfloat16 DSb[K][kBScanBV + 8];
  alignas(16) __nv_bfloat16 DV[kChunk][kBScanBV + 8];
};

template <int K, int V>
GDN2_DEV void bscan_prefetch(BScanStage<K>& st, const ChunkWs& ws, const __nv_bfloat16* dout,
                             const gdn2_chunk_args& a, int64_t t0, int L, int64_t h, int v0, int tid) {
  const int64_t H = a.H;
  for (int i = tid; i < kChunk * (K / 8); i += kBScanThreads) {
    const int r = i / (K / 8), p = (i % (K / 8)) * 8;
    const bool ok = r < L;
    const int64_t gi = ((t0 + (ok ? r : 0)) * H + h) * K + p;
    cp_async16b(&st.Y[r][p], ws.Y + gi, ok);
    cp_async16b(&st.QG[r][p], ws.qg + gi, ok);
    cp_async16b(&st.KG[r][p], ws.kg + gi, ok);
  }
  for (int i = tid; i < kChunk * (kChunk / 8); i += kBScanThreads) {
    const int r = i / (kChunk / 8), p = (i % (kChunk / 8)) * 8;
    const bool ok = r < L;
    cp_async16b(&st.Aqk[r][p], ws.Aqk + ((t0 + (ok ? r : 0)) * H + h) * kChunk + p, ok);
  }
  for (int i = tid; i < kChunk * (kBScanBV / 8); i += kBScanThreads) {
    const int r = i / (kBScanBV / 8), p = (i % (kBScanBV / 8)) * 8;
    const bool ok = r < L;
    cp_async16b(&st.DO[r][p], dout + ((t0 + (ok ? r : 0)) * H + h) * V + v0 + p, ok);
  }
  for (int i = tid; i < K / 4; i += kBScanThreads)
    cp_async16b(&st.glast[i * 4], ws.G + ((t0 + L - 1) * H + h) * K + i * 4, true);
}

template <int K, int V>
__global__ void __launch_bounds__(kBScanThreads, 1)
chunk_scan_bwd_kernel(gdn2_chunk_args a, gdn2_chunk_grads gr, ChunkWs ws, BwdWs bw) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  BScanSmem<K>& sm = *reinterpret_cast<BScanSmem<K>*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t H = a.H;
  const int v0 = blockIdx.x * kBScanBV;
  const int64_t n = blockIdx.y / H, h = blockIdx.y % H;
  SeqGeom geo{a.cu_seqlens, a.chunk_index, a.chunk_offset, a.T, (a.T + kChunk - 1) / kChunk};
  int64_t bos, len;
  geo.seq(n, bos, len);
  const int64_t nchunks = (len + kChunk - 1) / kChunk;
  const int64_t c0 = geo.chunk0(n);
  const bool tr = a.flags & GDN2_TRANSPOSE_STATE;
  const __nv_bfloat16* dout = static_cast<const __nv_bfloat16*>(gr.dout);

  constexpr int kRowsPerWarp = K / 8;
  constexpr int MT = kRowsPerWarp >= 16 ? kRowsPerWarp / 16 : 1;
  constexpr int NT = kBScanBV / 8;
  const bool srows = kRowsPerWarp >= 16;
  const bool sown = srows || warp < 4;
  const int sr0 = srows ? warp * kRowsPerWarp : warp * 16;
  float dS[MT][NT][4];
  acc_foreach(dS, sr0, 0, lane, [&](float& v, int r, int c) {
    float x = 0.f;
    if (sown && gr.dht) {
      const float* d = gr.dht + (n * H + h) * (int64_t)K * V;
      x = tr ? d[(int64_t)(v0 + c) * K + r] : d[(int64_t)r * V + v0 + c];
    }
    v = x;
  });

  auto chunk_len = [&](int64_t ci) {
    const int64_t rem = len - ci * kChunk;
    return (int)(rem < kChunk ? rem : kChunk);
  };
  if (nchunks > 0)
    bscan_prefetch<K, V>(sm.st[(nchunks - 1) & 1], ws, dout, a, bos + (nchunks - 1) * kChunk,
                         chunk_len(nchunks - 1), h, v0, tid);
  cp_commit();

  for (int64_t ci = nchunks - 1; ci >= 0; --ci) {
    const int64_t t0 = bos + ci * kChunk;
    const int L = chunk_len(ci);
    BScanStage<K>& st = sm.st[ci & 1];
    if (sown) acc_foreach(dS, sr0, 0, lane, [&](float& v, int r, int c) { sm.DSb[r][c] = __float2bfloat16_rn(v); });
    if (ci > 0) bscan_prefetch<K, V>(sm.st[(ci - 1) & 1], ws, dout, a, t0 - kChunk, chunk_len(ci - 1), h, v0, tid);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    {  // dh of this chunk, transposed (dh^T [v][k]), 16-byte stores
      __nv_bfloat16* dst = bw.dh + ((c0 + ci) * H + h) * (int64_t)K * V + (int64_t)v0 * K;
      for (int i = tid; i < kBScanBV * (K / 8); i += kBScanThreads) {
        const int c = i / (K / 8), p = (i % (K / 8)) * 8;
        uint4 pk;
        pk.x = pack_bf16(__bfloat162float(sm.DSb[p + 0][c]), __bfloat162float(sm.DSb[p + 1][c]));
        pk.y = pack_bf16(__bfloat162float(sm.DSb[p + 2][c]), __bfloat162float(sm.DSb[p + 3][c]));
        pk.z = pack_bf16(__bfloat162float(sm.DSb[p + 4][c]), __bfloat162float(sm.DSb[p + 5][c]));
        pk.w = pack_bf16(__bfloat162float(sm.DSb[p + 6][c]), __bfloat162float(sm.DSb[p + 7][c]));
        *reinterpret_cast<uint4*>(dst + (int64_t)c * K + p) = pk;
      }
    }

    // dv_new = Aqk^T do + kg dS      (warp tile 16 x 32)
    const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 32;
    {
      float acc[1][4][4];
      zero_acc(acc);
      warp_mma_ks<2, 1, 4, true, false>(acc, Smem{&st.Aqk[0][0], BScanStage<K>::LA}, m0,
                                        Smem{&st.DO[0][0], BScanStage<K>::LV}, n0, 0, kChunk, lane);
      warp_mma_ks<2, 1, 4, false, false>(acc, Smem{&st.KG[0][0], BScanStage<K>::LK}, m0,
                                         Smem{&sm.DSb[0][0], kBScanBV + 8}, n0, 0, K, lane);
      acc_foreach(acc, m0, n0, lane, [&](float v, int r, int c) { sm.DV[r][c] = __float2bfloat16_rn(r < L ? v : 0.f); });
    }
    __syncthreads();
    for (int i = tid; i < L * (kBScanBV / 8); i += kBScanThreads) {
      const int r = i / (kBScanBV / 8), p = (i % (kBScanBV / 8)) * 8;
      *reinterpret_cast<uint4*>(bw.dvn + ((t0 + r) * H + h) * V + v0 + p) = *reinterpret_cast<const uint4*>(&sm.DV[r][p]);
    }
    // dS <- 2^G_last dS + qg^T do - Y^T dv_new
    if (sown) {
      float t1[MT][NT][4], t2[MT][NT][4];
      zero_acc(t1);
      zero_acc(t2);
      warp_mma<MT, NT, true, false>(t1, Smem{&st.QG[0][0], BScanStage<K>::LK}, sr0,
                                    Smem{&st.DO[0][0], BScanStage<K>::LV}, 0, 0, kChunk, lane);
      warp_mma<MT, NT, true, false>(t2, Smem{&st.Y[0][0], BScanStage<K>::LK}, sr0,
                                    Smem{&sm.DV[0][0], kBScanBV + 8}, 0, 0, kChunk, lane);
      float dec[MT][2];
#pragma unroll
      for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int x = 0; x < 2; ++x) dec[i][x] = exp2_approx(st.glast[sr0 + 16 * i + (lane >> 2) + 8 * x]);
#pragma unroll
      for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            dS[i][j][e] = dS[i][j][e] * dec[i][e >> 1] + t1[i][j][e] - t2[i][j][e];
    }
    __syncthreads();
  }
  cp_wait<0>();
  if (sown && gr.dh0) {
    float* d = gr.dh0 + (n * H + h) * (int64_t)K * V;
    acc_foreach(dS, sr0, 0, lane, [&](float& v, int r, int c) {
      if (tr) d[(int64_t)(v0 + c) * K + r] = v;
      else d[(int64_t)r * V + v0 + c] = v;
    });
  }
}

// ---------------------------------------------------------------------------
// B3: chunk-parallel WY + intra backward
// ---------------------------------------------------------------------------
// 16 warps: warp w owns rows [16 (w & 3), +16) and columns [(w >> 2) K/4, +K/4)
// of every [64 x K] accumulator (dq, dk, db, dG), 16 fp32 registers each.
constexpr int kBIntraThreads = 512;
constexpr float kAnchorRangeB = 96.f;  // must match the forward's anchored range

template <int K, int V, typename TB>
struct BIntraSmem {
  // padded rows: accumulator-pattern accesses (8 rows x 4 column pairs per
  // warp instruction) then fall in distinct banks
  static constexpr int LK = K + 8, LV = V + 8, LA = kChunk + 8, LG = K + 4;
  static constexpr int LB = K + 16 / (int)sizeof(TB);  // staged db rows (16-byte aligned)
  alignas(16) float G[kChunk][LG];         // later reused for dG
  alignas(16) __nv_bfloat16 A[kChunk][LA];
  alignas(16) __nv_bfloat16 DAqk[kChunk][LA];
  alignas(16) __nv_bfloat16 DT[kChunk][LA];
  alignas(16) float last[K];               // dgk_last + sum_r k dk_inter
  alignas(16) float rsum[kChunk][4][2];    // l2norm row sums (q, k) per column group
  alignas(16) uint8_t flag[4][K];
  alignas(16) float ptot[kBIntraThreads / K][K];  // per-part sums of the dg reverse cumsum
  int nflag;
  // phase 1 needs h, dh, do, v_new, dv_new; phase 2 the WY operands; phase 3
  // the anchored score operands.  q, k, b are staged once phase 1's products
  // are done, in the part of the union phases 2 and 3 leave free.
  struct P1 {
    alignas(16) __nv_bfloat16 DVN[kChunk][LV];
    alignas(16) __nv_bfloat16 DY[kChunk][LK];
    alignas(16) __nv_bfloat16 HsT[V][LK];  // h^T: the chunk's entering state, [v][k]
    alignas(16) __nv_bfloat16 DHT[V][LK];  // dh^T: the chunk's exit-state cotangent, [v][k]
    alignas(16) __nv_bfloat16 DO[kChunk][LV];
    alignas(16) __nv_bfloat16 VN[kChunk][LV];
  };
  struct P2 {
    alignas(16) __nv_bfloat16 DVN[kChunk][LV];
    alignas(16) __nv_bfloat16 DY[kChunk][LK];
    alignas(16) __nv_bfloat16 KB2G[kChunk][LK];
    alignas(16) __nv_bfloat16 WV[kChunk][LV];
    alignas(16) __nv_bfloat16 DA[kChunk][LA];
    alignas(16) __nv_bfloat16 X[kChunk][LA];
  };
  struct P3 {
    alignas(16) __nv_bfloat16 QG[kChunk][LK];
    alignas(16) __nv_bfloat16 KBG[kChunk][LK];
    alignas(16) __nv_bfloat16 KN[160][LK];
  };
  static constexpr size_t kStageOff =
      ((sizeof(P2) > sizeof(P3) ? sizeof(P2) : sizeof(P3)) + 127) / 128 * 128;
  struct Staged {
    alignas(16) __nv_bfloat16 Q[kChunk][LK];
    alignas(16) __nv_bfloat16 Kk[kChunk][LK];
    alignas(16) TB Bg[kChunk][K + 16 / sizeof(TB)];
  };
  static constexpr size_t kUnion =
      sizeof(P1) > kStageOff + sizeof(Staged) ? sizeof(P1) : kStageOff + sizeof(Staged);
  alignas(128) unsigned char u[kUnion];
  GDN2_DEV P1& p1() { return *reinterpret_cast<P1*>(u); }
  GDN2_DEV P2& p2() { return *reinterpret_cast<P2*>(u); }
  GDN2_DEV P3& p3() { return *reinterpret_cast<P3*>(u); }
  GDN2_DEV Staged& st() { return *reinterpret_cast<Staged*>(u + kStageOff); }
};

// d_k = d_v = 128: the products with the chunk's states and the WY products
// (dq, dk, dY, dAqk, d(wv), dA, d(b k 2^G)) run on tcgen05 with M = 64
// accumulators in TMEM, read back with the 16x256b shape straight into the
// mma.sync fragment layout the 16 warps use for everything else.  A
// tcgen05 product reads each operand tile from shared memory once, where 16
// mma.sync warps read every operand four times over (ldmatrix per warp tile).
// Their operands are 128-byte-swizzled [rows x 64] bf16 tiles (tc.cuh); the
// 64 x 64 x 64 products X = dA A^T and A^T X run on mma.sync from those same
// swizzled tiles, the anchored row / column parts on padded tiles.
template <typename TB>
struct BIntraSmemTc {
  static constexpr int K = 128, V = 128;
  static constexpr int LK = K + 8, LV = V + 8, LA = kChunk + 8, LG = K + 4;
  static constexpr int LB = K + 16 / (int)sizeof(TB);
  static constexpr uint32_t kT = 64 * 128;  // one [64 rows x 64] bf16 swizzled tile, bytes
  alignas(1024) unsigned char A[kT];        // (I+T)^-1 as [t][s]
  alignas(16) float G[kChunk][LG];
  alignas(16) __nv_bfloat16 DAqk[kChunk][LA];
  alignas(16) __nv_bfloat16 DT[kChunk][LA];
  alignas(16) float last[K];
  alignas(16) float rsum[kChunk][4][2];
  alignas(16) uint8_t flag[4][K];
  alignas(16) float ptot[kBIntraThreads / K][K];
  alignas(8) uint64_t bar[3];  // completion of the three groups of tcgen05 products
  uint32_t tbase;              // TMEM base address (512 columns)
  int nflag;
  // tiles of 64-column blocks: [block][row][64]
  struct P1 {
    alignas(1024) unsigned char DVN[2 * kT];  // dv_new [t][v]
    unsigned char DY[2 * kT];                 // -dY [t][k]
    unsigned char HsT[4 * kT];                // h^T [v][k] (128 rows per k block)
    unsigned char DHT[4 * kT];                // dh^T [v][k]
    unsigned char DO[2 * kT];                 // do [t][v]
    unsigned char VN[2 * kT];                 // v_new [t][v]
  };
  struct P2 {
    alignas(1024) unsigned char DVN[2 * kT];  // as in P1
    unsigned char DY[2 * kT];
    unsigned char KB2G[2 * kT];  // b k 2^G [s][k] (first: dv staged for 16-byte stores)
    unsigned char WV[2 * kT];    // w v [s][v]
    unsigned char DA[kT];        // dA [t][u]
    unsigned char X[kT];         // dA A^T [t][t']
  };
  struct P3 {
    alignas(16) __nv_bfloat16 QG[kChunk][LK];
    alignas(16) __nv_bfloat16 KBG[kChunk][LK];
    alignas(16) __nv_bfloat16 KN[160][LK];
  };
  static constexpr size_t kStageOff =
      ((sizeof(P2) > sizeof(P3) ? sizeof(P2) : sizeof(P3)) + 127) / 128 * 128;
  struct Staged {
    alignas(16) __nv_bfloat16 Q[kChunk][LK];
    alignas(16) __nv_bfloat16 Kk[kChunk][LK];
    alignas(16) TB Bg[kChunk][K + 16 / sizeof(TB)];
  };
  static constexpr size_t kUnion =
      sizeof(P1) > kStageOff + sizeof(Staged) ? sizeof(P1) : kStageOff + sizeof(Staged);
  alignas(1024) unsigned char u[kUnion];
  GDN2_DEV P1& p1() { return *reinterpret_cast<P1*>(u); }
  GDN2_DEV P2& p2() { return *reinterpret_cast<P2*>(u); }
  GDN2_DEV P3& p3() { return *reinterpret_cast<P3*>(u); }
  GDN2_DEV Staged& st() { return *reinterpret_cast<Staged*>(u + kStageOff); }
};
static_assert(sizeof(BIntraSmemTc<float>) + 1024 <= 227 * 1024, "B3 (tcgen05) shared memory");
static_assert(offsetof(BIntraSmemTc<float>::P2, DVN) == offsetof(BIntraSmemTc<float>::P1, DVN) &&
                  offsetof(BIntraSmemTc<float>::P2, DY) == offsetof(BIntraSmemTc<float>::P1, DY),
              "dv_new and dY stay in place from phase 1 to phase 2");

using BIntraSmem128x128 = BIntraSmem<128, 128, float>;
static_assert(offsetof(BIntraSmem128x128, u) % 128 == 0, "cp.async/ldmatrix targets need 16B alignment");
static_assert(sizeof(BIntraSmem128x128) <= 227 * 1024, "B3 shared memory");
using BIntraSmem64x64 = BIntraSmem<64, 64, float>;
static_assert(offsetof(BIntraSmem64x64, u) % 128 == 0, "cp.async/ldmatrix targets need 16B alignment");
using BScanSmem128 = BScanSmem<128>;
static_assert(offsetof(BScanSmem128, DSb) % 16 == 0 && sizeof(BScanStage<128>) % 16 == 0, "stage alignment");

template <typename TB>
GDN2_DEV void store2(TB* p, float x0, float x1);
template <>
GDN2_DEV void store2<float>(float* p, float x0, float x1) { *reinterpret_cast<float2*>(p) = make_float2(x0, x1); }
template <>
GDN2_DEV void store2<__nv_bfloat16>(__nv_bfloat16* p, float x0, float x1) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(x0, x1);
}

template <typename TB>
GDN2_DEV float ldb(const void* p, int64_t i) {
  return to_f(static_cast<const TB*>(p)[i]);
}

__device__ unsigned int g_b3_fault;  // bit 0: a bounded wait of the backward intra kernel gave up

// Bounded wait on a tcgen05 commit, with the same outcome on every lane (the
// warp-collective TMEM loads after it must not diverge); a timeout is recorded
// and the kernel carries on, so every thread still meets every barrier.
GDN2_DEV void b3_wait(uint64_t* bar) {
  const bool ok = __all_sync(0xffffffffu, tc::mbar_wait(bar, 0));
  if (!ok && (threadIdx.x & 31) == 0) atomicOr(&g_b3_fault, 1u);
  tc::tc_fence_after();
}
// a [64 x 64] bf16 tile in the 128-byte-swizzled layout, as an mma.sync operand
struct SmemSw {
  unsigned char* p;
  GDN2_DEV __nv_bfloat16* at(int r, int c) const {
    return reinterpret_cast<__nv_bfloat16*>(p + tc::sw128_off(r, c));
  }
};
GDN2_DEV uint64_t b3_kmaj(uint32_t a) { return tc::sdesc_sw128(a, 16, 1024); }
GDN2_DEV uint64_t b3_mnmaj(uint32_t a, uint32_t lbo) { return tc::sdesc_sw128(a, lbo, 1024); }
// bf16 pair (c even) of element (r, c) of a tile of 64-column swizzled blocks
// `block` bytes apart
GDN2_DEV uint32_t b3_off(int r, int c, uint32_t block) { return (c >> 6) * block + tc::sw128_off(r, c & 63); }

// L2 prefetch maps of the backward intra kernel's first operands: the chunk's
// states h, dh, its do, v_new, dv_new rows, A and G
struct BwdIntraPrefetch {
  CUtensorMap h, dh, dout, vn, dvn, A, G;
  CUtensorMap q, k, b, w, v, g;  // and this CTA's own later operands
};

template <int K, int V, typename TB>
__global__ void __launch_bounds__(kBIntraThreads, 1)
chunk_bwd_intra_kernel(gdn2_chunk_args a, gdn2_chunk_grads gr, ChunkWs ws, BwdWs bw, int pf_stride,
                       const __grid_constant__ BwdIntraPrefetch pm) {
  extern __shared__ __align__(1024) unsigned char smem_b3[];
  unsigned char* smem_raw = smem_b3;
  constexpr bool kTc = K == 128 && V == 128;
  using S = std::conditional_t<kTc, BIntraSmemTc<TB>, BIntraSmem<K, V, TB>>;
  // tcgen05 operand tiles start on 1024-byte boundaries; the offset is applied to
  // smem_raw itself so that every access stays a shared-memory access
  S& sm = *reinterpret_cast<S*>(smem_raw + (kTc ? (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u : 0u));
  auto& p1 = sm.p1();
  auto& p2 = sm.p2();
  auto& p3 = sm.p3();
  auto& sg = sm.st();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t H = a.H, h = blockIdx.y, cglob = blockIdx.x;
  SeqGeom geo{a.cu_seqlens, a.chunk_index, a.chunk_offset, a.T, (a.T + kChunk - 1) / kChunk};
  int64_t n, ci, bos, len;
  geo.chunk(cglob, n, ci);
  geo.seq(n, bos, len);
  const int64_t t0 = bos + ci * kChunk;
  const int64_t rem = len - ci * kChunk;
  const int L = (int)(rem < kChunk ? rem : kChunk);
  const int64_t cidx = geo.chunk0(n) + ci;
  const float scale = a.scale;
  const __nv_bfloat16* vin = static_cast<const __nv_bfloat16*>(a.v);
  const __nv_bfloat16* dout = static_cast<const __nv_bfloat16*>(gr.dout);
  auto tokK = [&](int r, int c) { return ((t0 + r) * H + h) * K + c; };
  auto tokV = [&](int r, int c) { return ((t0 + r) * H + h) * V + c; };
  // staged q, k, b (zero past the sequence end)
  auto qv = [&](int r, int c) { return __bfloat162float(sg.Q[r][c]); };
  auto kv = [&](int r, int c) { return __bfloat162float(sg.Kk[r][c]); };
  auto bv = [&](int r, int c) { return to_f(sg.Bg[r][c]); };

  // ---- loads -----------------------------------------------------------------
  {
    const __nv_bfloat16* hsrc = ws.h + (cidx * H + h) * (int64_t)K * V;
    const __nv_bfloat16* dhsrc = bw.dh + (cidx * H + h) * (int64_t)K * V;
    if constexpr (kTc) {
      // swizzled tiles: 16-byte piece (r, p) of 64-column block b at b * block + sw128_off(r, p)
      for (int i = tid; i < V * (K / 8); i += kBIntraThreads) {
        const int r = i / (K / 8), p = (i % (K / 8)) * 8;
        const uint32_t o = b3_off(r, p, 2 * S::kT);  // 128 rows per block
        cp_async16b(p1.HsT + o, hsrc + (int64_t)r * K + p, true);
        cp_async16b(p1.DHT + o, dhsrc + (int64_t)r * K + p, true);
      }
      for (int i = tid; i < kChunk * (V / 8); i += kBIntraThreads) {
        const int r = i / (V / 8), p = (i % (V / 8)) * 8;
        const bool ok = r < L;
        const int64_t gi = tokV(ok ? r : 0, p);
        const uint32_t o = b3_off(r, p, S::kT);
        cp_async16b(p1.DO + o, dout + gi, ok);
        cp_async16b(p1.VN + o, ws.v_new + gi, ok);
        cp_async16b(p1.DVN + o, bw.dvn + gi, ok);
      }
    } else {
      for (int i = tid; i < V * (K / 8); i += kBIntraThreads) {
        const int r = i / (K / 8), p = (i % (K / 8)) * 8;
        cp_async16b(&p1.HsT[r][p], hsrc + (int64_t)r * K + p, true);
        cp_async16b(&p1.DHT[r][p], dhsrc + (int64_t)r * K + p, true);
      }
      for (int i = tid; i < kChunk * (V / 8); i += kBIntraThreads) {
        const int r = i / (V / 8), p = (i % (V / 8)) * 8;
        const bool ok = r < L;
        const int64_t gi = tokV(ok ? r : 0, p);
        cp_async16b(&p1.DO[r][p], dout + gi, ok);
        cp_async16b(&p1.VN[r][p], ws.v_new + gi, ok);
        cp_async16b(&p1.DVN[r][p], bw.dvn + gi, ok);
      }
    }
    cp_commit();  // group 1: the phase-1 operands
    // group 2: A and G, first needed after the phase-1 products
    for (int i = tid; i < kChunk * (kChunk / 8); i += kBIntraThreads) {
      const int r = i / (kChunk / 8), p = (i % (kChunk / 8)) * 8;
      const bool ok = r < L;
      const __nv_bfloat16* src = ws.Akk + ((t0 + (ok ? r : 0)) * H + h) * kChunk + p;
      if constexpr (kTc) cp_async16b(sm.A + tc::sw128_off(r, p), src, ok);
      else cp_async16b(&sm.A[r][p], src, ok);
    }
    for (int i = tid; i < kChunk * (K / 4); i += kBIntraThreads) {
      const int r = i / (K / 4), p = (i % (K / 4)) * 4;
      const bool ok = r < L;
      cp_async16b(&sm.G[r][p], ws.G + tokK(ok ? r : L - 1, p), true);  // padded rows repeat G_last
    }
    cp_commit();
    for (int c = tid; c < K; c += kBIntraThreads) sm.last[c] = 0.f;
    if (tid == 0) sm.nflag = 0;
    if constexpr (kTc) {
      if (warp == 0) tc::tmem_alloc(&sm.tbase, 512);
      if (tid == 0) {
        for (int i = 0; i < 3; ++i) tc::mbar_init(&sm.bar[i], 1);
        tc::mbar_fence_init();
      }
    }
    cp_wait<1>();
    if constexpr (kTc) {
      tc::fence_proxy_async();  // the copied tiles -> the tensor core's proxy
      tc::tc_fence_before();
    }
    __syncthreads();
    if constexpr (kTc) {
      tc::tc_fence_after();
      // product group 1 (TMEM columns: dq [0,128), dk [128,256), -dY [256,384), dAqk [384,448)):
      //   dq = do h, dk = v_new dh, dY = dv_new h over v (h^T tiles as N-major B), dAqk = do v_new^T
      if (tid == 0) {
        constexpr uint32_t iN = tc::idesc_bf16(64, 128, 0, 1), i64 = tc::idesc_bf16(64, 64, 0, 0);
        const uint32_t tb = sm.tbase, sH = smem_u32(p1.HsT), sDH = smem_u32(p1.DHT), sDO = smem_u32(p1.DO),
                       sVN = smem_u32(p1.VN), sDVN = smem_u32(p1.DVN);
#pragma unroll 1
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t ko = (kk >> 2) * S::kT + (kk & 3) * 32, hk = kk * 2048;
          tc::mma_bf16(tb + 0, b3_kmaj(sDO + ko), b3_mnmaj(sH + hk, 2 * S::kT), iN, kk > 0);
          tc::mma_bf16(tb + 128, b3_kmaj(sVN + ko), b3_mnmaj(sDH + hk, 2 * S::kT), iN, kk > 0);
          tc::mma_bf16(tb + 256, b3_kmaj(sDVN + ko), b3_mnmaj(sH + hk, 2 * S::kT), iN, kk > 0);
          tc::mma_bf16(tb + 384, b3_kmaj(sDO + ko), b3_kmaj(sVN + ko), i64, kk > 0);
        }
        tc::mma_commit(&sm.bar[0]);
      }
    }
    // q, k, b (staged after phase 1) and w, v (read from global in the d(w v)
    // step) go to L2 now: one tensor prefetch each, from one thread
    if (pf_stride > 0 && tid == 0) {
      const int tt = (int)t0, hh = (int)h;
      tc::tma_prefetch_3d(&pm.q, 0, hh, tt);
      tc::tma_prefetch_3d(&pm.k, 0, hh, tt);
      tc::tma_prefetch_3d(&pm.b, 0, hh, tt);
      tc::tma_prefetch_3d(&pm.w, 0, hh, tt);
      tc::tma_prefetch_3d(&pm.v, 0, hh, tt);
    }
  }

  const int rb = warp & 3, ch = warp >> 2;
  const int m0 = rb * 16;
  constexpr int NTk = K / 32, NTv = V / 32;
  const int n0 = ch * (K / 4), n0v = ch * (V / 4);
  // 64x64 products: warp tile 16 x 16
  const int mm = (warp & 3) * 16, nn = (warp >> 2) * 16;
  float dq[1][NTk][4], dk[1][NTk][4], db[1][NTk][4], dG[1][NTk][4];
  zero_acc(dq);
  zero_acc(dk);
  zero_acc(db);
  zero_acc(dG);
  const float* Glast = &sm.G[kChunk - 1][0];

  // ---- phase 1: products with h, dh ------------------------------------------
  // bf16 element (r, c) of the tiles both variants write: dY, w v, b k 2^G and
  // the staged dv (padded rows for mma.sync, swizzled blocks for tcgen05)
  auto pDY = [&](int r, int c) -> __nv_bfloat16* {
    if constexpr (kTc) return reinterpret_cast<__nv_bfloat16*>(p1.DY + b3_off(r, c, S::kT));
    else return &p1.DY[r][c];
  };
  auto pWV = [&](int r, int c) -> __nv_bfloat16* {
    if constexpr (kTc) return reinterpret_cast<__nv_bfloat16*>(p2.WV + b3_off(r, c, S::kT));
    else return &p2.WV[r][c];
  };
  auto pKB2G = [&](int r, int c) -> __nv_bfloat16* {
    if constexpr (kTc) return reinterpret_cast<__nv_bfloat16*>(p2.KB2G + b3_off(r, c, S::kT));
    else return &p2.KB2G[r][c];
  };
  // dv is staged in the b k 2^G tile (free until phase 2) for 16-byte stores
  constexpr bool kStageDv = K == V;
  auto pSDV = [&](int r, int c) -> __nv_bfloat16* {
    if constexpr (kTc) return reinterpret_cast<__nv_bfloat16*>(p2.KB2G + b3_off(r, c, S::kT));
    else return &p2.KB2G[0][0] + r * S::LV + c;
  };
  // this warp's TMEM lane quarter: rows [m0, m0 + 16) of every M = 64 accumulator
  uint32_t tl = 0;
  if constexpr (kTc) tl = tc::tmem_addr(sm.tbase, 32 * (warp & 3), 0);

  if constexpr (!kTc) {
    warp_mma<1, NTk, false, false>(dq, Smem{&p1.DO[0][0], S::LV}, m0, Smem{&p1.HsT[0][0], S::LK}, n0, 0, V, lane);
    warp_mma<1, NTk, false, false>(dk, Smem{&p1.VN[0][0], S::LV}, m0, Smem{&p1.DHT[0][0], S::LK}, n0, 0, V, lane);
    float t[1][NTk][4];
    zero_acc(t);
    warp_mma<1, NTk, false, false>(t, Smem{&p1.DVN[0][0], S::LV}, m0, Smem{&p1.HsT[0][0], S::LK}, n0, 0, V, lane);
    acc_foreach(t, m0, n0, lane, [&](float v, int r, int c) { *pDY(r, c) = __float2bfloat16_rn(-v); });
  }
  cp_wait<0>();  // A and G
  if constexpr (kTc) tc::fence_proxy_async();  // A is a tcgen05 operand from product group 2 on
  __syncthreads();
  // the forward's exactness flags (same criterion, same G)
  for (int i = tid; i < 4 * K; i += kBIntraThreads) {
    const int blk = i / K, c = i % K, a0 = blk * 16;
    const int alast = min(a0 + 15, max(L - 1, 0));
    const uint8_t f = (sm.G[a0][c] - sm.G[alast][c]) > kAnchorRangeB ? 1 : 0;
    sm.flag[blk][c] = f;
    if (f) atomicAdd(&sm.nflag, 1);
  }
  // dgk_last = 2^G_last * sum_v h dh: a thread owns two state rows and a
  // slice of v (paired loads along the rows, conflict-free), partials summed
  // into last[] with shared atomics
  {
    constexpr int kPairs = K / 2, kParts = kBIntraThreads / kPairs, kVPer = V / kParts;
    const int r = 2 * (tid % kPairs), part = tid / kPairs;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 4
    for (int v = part * kVPer; v < (part + 1) * kVPer; ++v) {
      float2 hh, dd;
      if constexpr (kTc) {
        const uint32_t o = b3_off(v, r, 2 * S::kT);
        hh = ld2(reinterpret_cast<const __nv_bfloat16*>(p1.HsT + o));
        dd = ld2(reinterpret_cast<const __nv_bfloat16*>(p1.DHT + o));
      } else {
        hh = ld2(&p1.HsT[v][r]);
        dd = ld2(&p1.DHT[v][r]);
      }
      s0 += hh.x * dd.x;
      s1 += hh.y * dd.y;
    }
    atomicAdd(&sm.last[r], s0 * exp2_approx(Glast[r]));
    atomicAdd(&sm.last[r + 1], s1 * exp2_approx(Glast[r + 1]));
  }
  // dAqk = scale do v_new^T (lower incl. diagonal)
  {
    float t[1][2][4];
    if constexpr (kTc) {
      // product group 1's accumulators: dq, dk to registers, -dY to its operand tile
      b3_wait(&sm.bar[0]);
      {
        float y[1][NTk][4];
        tc::tmem_ld_frag<NTk>(tl + 256 + n0, y[0]);
        tc::tmem_wait_ld();
        acc_foreach(y, m0, n0, lane, [&](float v, int r, int c) { *pDY(r, c) = __float2bfloat16_rn(-v); });
      }
      tc::tmem_ld_frag<NTk>(tl + 0 + n0, dq[0]);
      tc::tmem_ld_frag<NTk>(tl + 128 + n0, dk[0]);
      tc::tmem_ld_frag<2>(tl + 384 + nn, t[0]);
      tc::tmem_wait_ld();
    } else {
      zero_acc(t);
      warp_mma<1, 2, false, true>(t, Smem{&p1.DO[0][0], S::LV}, mm, Smem{&p1.VN[0][0], S::LV}, nn, 0, V, lane);
    }
    acc_foreach(t, mm, nn, lane, [&](float v, int r, int s) {
      sm.DAqk[r][s] = __float2bfloat16_rn((s <= r && r < L) ? v * scale : 0.f);
    });
  }
  if constexpr (kTc) {
    tc::fence_proxy_async();  // -dY -> the tensor core
    tc::tc_fence_before();    // product group 1's columns are drained
  }
  __syncthreads();  // h, dh, do, v_new are dead: stage q, k, b in their place
  if constexpr (kTc) {
    tc::tc_fence_after();
    // product group 2: d(w v) = A^T dv_new -> columns [256,384), d(b k 2^G) = A^T dY -> [0,128)
    // (A as an M-major operand, dv_new and dY as N-major ones)
    if (tid == 0) {
      constexpr uint32_t iT = tc::idesc_bf16(64, 128, 1, 1);
      const uint32_t tb = sm.tbase, sA = smem_u32(sm.A), sDVN = smem_u32(p2.DVN), sDY = smem_u32(p2.DY);
#pragma unroll 1
      for (int kk = 0; kk < 4; ++kk) {
        tc::mma_bf16(tb + 256, b3_mnmaj(sA + kk * 2048, S::kT), b3_mnmaj(sDVN + kk * 2048, S::kT), iT, kk > 0);
        tc::mma_bf16(tb + 0, b3_mnmaj(sA + kk * 2048, S::kT), b3_mnmaj(sDY + kk * 2048, S::kT), iT, kk > 0);
      }
      tc::mma_commit(&sm.bar[1]);
    }
  }
  for (int i = tid; i < kChunk * (K / 8); i += kBIntraThreads) {
    const int r = i / (K / 8), p = (i % (K / 8)) * 8;
    const bool ok = r < L;
    const int64_t gi = tokK(ok ? r : 0, p);
    cp_async16b(&sg.Q[r][p], ws.qn + gi, ok);
    cp_async16b(&sg.Kk[r][p], ws.kn + gi, ok);
  }
  constexpr int kBPer16 = 16 / sizeof(TB);
  for (int i = tid; i < kChunk * (K / kBPer16); i += kBIntraThreads) {
    const int r = i / (K / kBPer16), p = (i % (K / kBPer16)) * kBPer16;
    const bool ok = r < L;
    cp_async16b(&sg.Bg[r][p], static_cast<const TB*>(a.b) + tokK(ok ? r : 0, p), ok);
  }
  cp_commit();
  // d(w v) = A^T dv_new  ->  dv = w d(wv), dw = v d(wv); the same registers of
  // w and v also form WV = w v for phase 2 (w, v are read from HBM once).
  {
    __nv_bfloat16* dv = static_cast<__nv_bfloat16*>(gr.dv);
    TB* dw = static_cast<TB*>(gr.dw);
    float wl[NTv][4], vl[NTv][4];
#pragma unroll
    for (int j = 0; j < NTv; ++j)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int r = m0 + (lane >> 2) + x * 8, c = n0v + 8 * j + 2 * (lane & 3);
        float2 w2 = make_float2(0.f, 0.f), v2 = make_float2(0.f, 0.f);
        if (r < L) {
          w2 = ld2(static_cast<const TB*>(a.w) + tokV(r, c));
          v2 = ld2(vin + tokV(r, c));
        }
        wl[j][2 * x] = w2.x;
        wl[j][2 * x + 1] = w2.y;
        vl[j][2 * x] = v2.x;
        vl[j][2 * x + 1] = v2.y;
      }
    float t[1][NTv][4];
    if constexpr (kTc) {
      b3_wait(&sm.bar[1]);
      tc::tmem_ld_frag<NTv>(tl + 256 + n0v, t[0]);
      tc::tmem_wait_ld();
    } else {
      zero_acc(t);
      warp_mma<1, NTv, true, false>(t, Smem{&sm.A[0][0], S::LA}, m0, Smem{&p1.DVN[0][0], S::LV}, n0v, 0, kChunk,
                                    lane);
    }
#pragma unroll
    for (int j = 0; j < NTv; ++j)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int r = m0 + (lane >> 2) + x * 8, c = n0v + 8 * j + 2 * (lane & 3);
        *reinterpret_cast<__nv_bfloat162*>(pWV(r, c)) =
            __floats2bfloat162_rn(wl[j][2 * x] * vl[j][2 * x], wl[j][2 * x + 1] * vl[j][2 * x + 1]);
        const __nv_bfloat162 dv2 =
            __floats2bfloat162_rn(t[0][j][2 * x] * wl[j][2 * x], t[0][j][2 * x + 1] * wl[j][2 * x + 1]);
        if constexpr (kStageDv) *reinterpret_cast<__nv_bfloat162*>(pSDV(r, c)) = dv2;
        if (r < L) {
          const int64_t gi = tokV(r, c);
          if constexpr (!kStageDv) *reinterpret_cast<__nv_bfloat162*>(dv + gi) = dv2;
          store2<TB>(dw + gi, t[0][j][2 * x] * vl[j][2 * x], t[0][j][2 * x + 1] * vl[j][2 * x + 1]);
        }
      }
  }
  cp_wait<0>();
  __syncthreads();
  if constexpr (kStageDv) {  // dv out of its staging tile with 16-byte stores
    __nv_bfloat16* dv = static_cast<__nv_bfloat16*>(gr.dv);
    for (int i = tid; i < L * (V / 8); i += kBIntraThreads) {
      const int r = i / (V / 8), p = (i % (V / 8)) * 8;
      *reinterpret_cast<uint4*>(dv + tokV(r, p)) = *reinterpret_cast<const uint4*>(pSDV(r, p));
    }
  }
  // inter-chunk parts: dq = scale (do h^T) 2^G ; dk = (v_new dh^T) 2^(G_last - G)
  {
    float colsum[NTk][2];
#pragma unroll
    for (int j = 0; j < NTk; ++j) colsum[j][0] = colsum[j][1] = 0.f;
#pragma unroll
    for (int j = 0; j < NTk; ++j)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int r = m0 + (lane >> 2) + x * 8, c = n0 + 8 * j + 2 * (lane & 3);
        const float2 G2 = ld2(&sm.G[r][c]), Gl2 = ld2(&Glast[c]);
        const float2 q2 = ld2(&sg.Q[r][c]), k2 = ld2(&sg.Kk[r][c]);
        const float Gr[2] = {G2.x, G2.y}, Gl[2] = {Gl2.x, Gl2.y}, qq[2] = {q2.x, q2.y}, kk[2] = {k2.x, k2.y};
#pragma unroll
        for (int y = 0; y < 2; ++y) {
          const int e = 2 * x + y;
          const float dqi = r < L ? dq[0][j][e] * scale * exp2_approx(Gr[y]) : 0.f;
          const float dki = r < L ? dk[0][j][e] * exp2_approx(Gl[y] - Gr[y]) : 0.f;
          dq[0][j][e] = dqi;
          dk[0][j][e] = dki;
          dG[0][j][e] = qq[y] * dqi - kk[y] * dki;
          colsum[j][y] += kk[y] * dki;
        }
      }
#pragma unroll
    for (int j = 0; j < NTk; ++j)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        float s = colsum[j][x];
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        s += __shfl_xor_sync(0xffffffffu, s, 8);
        s += __shfl_xor_sync(0xffffffffu, s, 16);
        if (lane < 4) atomicAdd(&sm.last[n0 + 8 * j + 2 * lane + x], s);
      }
  }

  if constexpr (kStageDv) __syncthreads();  // the staged dv is read before KB2G overwrites it

  // ---- phase 2: WY factors -----------------------------------------------------
  for (int g = tid; g < kChunk * K / 8; g += kBIntraThreads) {
    const int r = g / (K / 8), c0 = (g % (K / 8)) * 8;
    float b8[8], k8[8], G8[8];
    ld8(&sg.Bg[r][c0], b8);
    ld8(&sg.Kk[r][c0], k8);
    ld8(&sm.G[r][c0], G8);
#pragma unroll
    for (int e = 0; e < 8; ++e) b8[e] = b8[e] * k8[e] * exp2_approx(G8[e]);
    st8(pKB2G(r, c0), b8);
  }
  if constexpr (kTc) tc::fence_proxy_async();  // w v and b k 2^G -> the tensor core
  __syncthreads();
  float tA[1][2][4];  // dA = dv_new (w v)^T + dY (b k 2^G)^T
  if constexpr (kTc) {
    tc::tc_fence_after();
    // product group 3: dA -> columns [384,448)
    if (tid == 0) {
      constexpr uint32_t i64 = tc::idesc_bf16(64, 64, 0, 0);
      const uint32_t tb = sm.tbase, sDVN = smem_u32(p2.DVN), sWV = smem_u32(p2.WV), sDY = smem_u32(p2.DY),
                     sKB = smem_u32(p2.KB2G);
#pragma unroll 1
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t ko = (kk >> 2) * S::kT + (kk & 3) * 32;
        tc::mma_bf16(tb + 384, b3_kmaj(sDVN + ko), b3_kmaj(sWV + ko), i64, kk > 0);
      }
#pragma unroll 1
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t ko = (kk >> 2) * S::kT + (kk & 3) * 32;
        tc::mma_bf16(tb + 384, b3_kmaj(sDY + ko), b3_kmaj(sKB + ko), i64, 1);
      }
      tc::mma_commit(&sm.bar[2]);
    }
  } else {
    zero_acc(tA);
    warp_mma<1, 2, false, true>(tA, Smem{&p2.DVN[0][0], S::LV}, mm, Smem{&p2.WV[0][0], S::LV}, nn, 0, V, lane);
    warp_mma<1, 2, false, true>(tA, Smem{&p2.DY[0][0], S::LK}, mm, Smem{&p2.KB2G[0][0], S::LK}, nn, 0, K, lane);
    acc_foreach(tA, mm, nn, lane, [&](float v, int r, int s) {
      p2.DA[r][s] = __float2bfloat16_rn((s < r && r < L) ? v : 0.f);
    });
  }
  // d(b k 2^G) = A^T dY (tcgen05: product group 2, complete since the d(w v) step)
  {
    float t[1][NTk][4];
    if constexpr (kTc) {
      tc::tmem_ld_frag<NTk>(tl + 0 + n0, t[0]);
      tc::tmem_wait_ld();
    } else {
      zero_acc(t);
      warp_mma<1, NTk, true, false>(t, Smem{&sm.A[0][0], S::LA}, m0, Smem{&p2.DY[0][0], S::LK}, n0, 0, kChunk,
                                    lane);
    }
#pragma unroll
    for (int j = 0; j < NTk; ++j)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int r = m0 + (lane >> 2) + x * 8, c = n0 + 8 * j + 2 * (lane & 3);
        if (r < L) {
          const float2 G2 = ld2(&sm.G[r][c]), b2 = ld2(&sg.Bg[r][c]), k2 = ld2(&sg.Kk[r][c]);
          const float Gr[2] = {G2.x, G2.y}, bb[2] = {b2.x, b2.y}, kk[2] = {k2.x, k2.y};
#pragma unroll
          for (int y = 0; y < 2; ++y) {
            const int e = 2 * x + y;
            const float xx = t[0][j][e] * exp2_approx(Gr[y]);
            db[0][j][e] += kk[y] * xx;
            dk[0][j][e] += bb[y] * xx;
            dG[0][j][e] += bb[y] * kk[y] * xx;
          }
        }
      }
  }
  if constexpr (kTc) {
    b3_wait(&sm.bar[2]);
    tc::tmem_ld_frag<2>(tl + 384 + nn, tA[0]);
    tc::tmem_wait_ld();
    tc::tc_fence_before();  // the last TMEM read: the allocation is released after the next barrier
    acc_foreach(tA, mm, nn, lane, [&](float v, int r, int s) {
      *reinterpret_cast<__nv_bfloat16*>(p2.DA + tc::sw128_off(r, s)) =
          __float2bfloat16_rn((s < r && r < L) ? v : 0.f);
    });
    tc::fence_proxy_async();
  }
  __syncthreads();
  if constexpr (kTc) {
    // every tcgen05 product has completed and been read: release TMEM
    if (warp == 0) {
      tc::tc_fence_after();
      tc::tmem_dealloc(sm.tbase, 512);
    }
  }
  // dT = -A^T (dA A^T), strictly lower (64 x 64 x 64 products: mma.sync, also on
  // the swizzled tiles, where a tcgen05 round trip costs more than it saves)
  {
    float t[1][2][4];
    if constexpr (kTc) {
      zero_acc(t);
      warp_mma<1, 2, false, true>(t, SmemSw{p2.DA}, mm, SmemSw{sm.A}, nn, 0, kChunk, lane);
      acc_foreach(t, mm, nn, lane, [&](float v, int r, int s) {
        *reinterpret_cast<__nv_bfloat16*>(p2.X + tc::sw128_off(r, s)) = __float2bfloat16_rn(v);
      });
      __syncthreads();
      zero_acc(t);
      warp_mma<1, 2, true, false>(t, SmemSw{sm.A}, mm, SmemSw{p2.X}, nn, 0, kChunk, lane);
    } else {
      zero_acc(t);
      warp_mma<1, 2, false, true>(t, Smem{&p2.DA[0][0], S::LA}, mm, Smem{&sm.A[0][0], S::LA}, nn, 0, kChunk, lane);
      acc_foreach(t, mm, nn, lane, [&](float v, int r, int s) { p2.X[r][s] = __float2bfloat16_rn(v); });
      __syncthreads();
      zero_acc(t);
      warp_mma<1, 2, true, false>(t, Smem{&sm.A[0][0], S::LA}, mm, Smem{&p2.X[0][0], S::LA}, nn, 0, kChunk, lane);
    }
    acc_foreach(t, mm, nn, lane, [&](float v, int r, int s) {
      sm.DT[r][s] = __float2bfloat16_rn((s < r && r < L) ? -v : 0.f);
    });
  }
  __syncthreads();

  // ---- phase 3: intra-chunk VJP through the anchored scores --------------------
  // CTAs start in linear order, one per SM: the CTA pf_stride places on takes
  // this SM's slot next.  Its first operands go to L2 now, while this CTA has no
  // loads of its own in flight: one tensor prefetch each, issued by one thread.
  if (pf_stride > 0 && tid == 0) {  // the launcher passes 0 unless linear CTA ids fit 31 bits
    const uint32_t gx = gridDim.x, nxt = blockIdx.y * gx + blockIdx.x + (uint32_t)pf_stride;
    if (nxt < gx * gridDim.y) {
      const uint32_t nh = nxt / gx;
      int64_t nn, nci, nbos, nlen;
      geo.chunk(nxt - nh * gx, nn, nci);
      geo.seq(nn, nbos, nlen);
      const int tt = (int)(nbos + nci * kChunk), hh = (int)nh;
      const int hrow = (int)(((geo.chunk0(nn) + nci) * H + nh) * V);
      tc::tma_prefetch_2d(&pm.h, 0, hrow);
      tc::tma_prefetch_2d(&pm.dh, 0, hrow);
      tc::tma_prefetch_3d(&pm.dout, 0, hh, tt);
      tc::tma_prefetch_3d(&pm.vn, 0, hh, tt);
      tc::tma_prefetch_3d(&pm.dvn, 0, hh, tt);
      tc::tma_prefetch_3d(&pm.A, 0, hh, tt);
      tc::tma_prefetch_3d(&pm.G, 0, hh, tt);
    }
  }
  for (int g = tid; g < kChunk * K / 8; g += kBIntraThreads) {
    const int r = g / (K / 8), c0 = (g % (K / 8)) * 8;
    const int blk = r >> 4, a0 = blk * 16;
    float k8[8], q8[8], b8[8], Gr[8], Ga[8], o1[8], o2[8], o3[8];
    ld8(&sg.Kk[r][c0], k8);
    ld8(&sg.Q[r][c0], q8);
    ld8(&sg.Bg[r][c0], b8);
    ld8(&sm.G[r][c0], Gr);
    ld8(&sm.G[a0][c0], Ga);
    const uint2 fl2 = *reinterpret_cast<const uint2*>(&sm.flag[blk][c0]);
    const uint8_t* fl = reinterpret_cast<const uint8_t*>(&fl2);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float rowf = exp2_approx(Gr[e] - Ga[e]);
      o1[e] = q8[e] * rowf;
      o2[e] = b8[e] * k8[e] * rowf;
      o3[e] = k8[e] * (fl[e] ? 0.f : exp2_approx(Ga[e] - Gr[e]));
    }
    st8(&p3.QG[r][c0], o1);
    st8(&p3.KBG[r][c0], o2);
    st8(&p3.KN[anchor_row0(blk) + r][c0], o3);
    if (blk < 3) {
      float f[8], Gp[8];
      ld8(&sm.G[a0 + 16][c0], Ga);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = exp2_approx(Ga[e] - Gr[e]);
      for (int ai = blk + 1; ai < 4; ++ai) {
        if (ai > blk + 1) {
          ld8(&sm.G[ai * 16][c0], Ga);
          ld8(&sm.G[ai * 16 - 16][c0], Gp);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] *= exp2_approx(Ga[e] - Gp[e]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) o3[e] = k8[e] * f[e];
        st8(&p3.KN[anchor_row0(ai) + r][c0], o3);
      }
    }
  }
  __syncthreads();
  {
    // row parts: rows of block rb against columns [0, 16(rb+1))
    float r1[1][NTk][4], r2[1][NTk][4];
    zero_acc(r1);
    zero_acc(r2);
    Smem KNi{&p3.KN[anchor_row0(rb)][0], S::LK};
    warp_mma<1, NTk, false, false>(r1, Smem{&sm.DAqk[0][0], S::LA}, m0, KNi, n0, 0, 16 * (rb + 1), lane);
    warp_mma<1, NTk, false, false>(r2, Smem{&sm.DT[0][0], S::LA}, m0, KNi, n0, 0, 16 * (rb + 1), lane);
#pragma unroll
    for (int j = 0; j < NTk; ++j)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int r = m0 + (lane >> 2) + x * 8, c = n0 + 8 * j + 2 * (lane & 3);
        const float2 G2 = ld2(&sm.G[r][c]), Ga2 = ld2(&sm.G[m0][c]);
        const float2 b2 = ld2(&sg.Bg[r][c]), k2 = ld2(&sg.Kk[r][c]);
        const float2 qg2 = ld2(&p3.QG[r][c]), kbg2 = ld2(&p3.KBG[r][c]);
        const float Gr[2] = {G2.x, G2.y}, Ga[2] = {Ga2.x, Ga2.y}, bb[2] = {b2.x, b2.y}, kk[2] = {k2.x, k2.y};
        const float qg[2] = {qg2.x, qg2.y}, kbg[2] = {kbg2.x, kbg2.y};
#pragma unroll
        for (int y = 0; y < 2; ++y) {
          const int e = 2 * x + y;
          const float rowf = exp2_approx(Gr[y] - Ga[y]);
          const float rr = r2[0][j][e] * rowf;
          dq[0][j][e] += r1[0][j][e] * rowf;
          dk[0][j][e] += rr * bb[y];
          db[0][j][e] += rr * kk[y];
          // the decay-gradient pieces use the very bf16 operands the MMAs read
          // (QG = q 2^(G_r - G_a), KBG = b k 2^(G_r - G_a)), so that the row and
          // column sides below cancel exactly when summed over the chunk.
          dG[0][j][e] += qg[y] * r1[0][j][e] + kbg[y] * r2[0][j][e];
        }
      }
  }
  // column parts: this warp's rows as columns s of block rb, rows r of blocks >= rb
  for (int ib = rb; ib < 4; ++ib) {
    float cc[1][NTk][4];
    zero_acc(cc);
    warp_mma<1, NTk, true, false>(cc, Smem{&sm.DAqk[0][0], S::LA}, m0, Smem{&p3.QG[0][0], S::LK}, n0, ib * 16,
                                  ib * 16 + 16, lane);
    warp_mma<1, NTk, true, false>(cc, Smem{&sm.DT[0][0], S::LA}, m0, Smem{&p3.KBG[0][0], S::LK}, n0, ib * 16,
                                  ib * 16 + 16, lane);
#pragma unroll
    for (int j = 0; j < NTk; ++j)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int s = m0 + (lane >> 2) + x * 8, c = n0 + 8 * j + 2 * (lane & 3);
        const float2 Ga2 = ld2(&sm.G[ib * 16][c]), Gs2 = ld2(&sm.G[s][c]);
        const float2 kn2 = ld2(&p3.KN[anchor_row0(ib) + s][c]);
        const float Ga[2] = {Ga2.x, Ga2.y}, Gs[2] = {Gs2.x, Gs2.y}, kn[2] = {kn2.x, kn2.y};
        const bool own = ib == rb;
#pragma unroll
        for (int y = 0; y < 2; ++y) {
          const int e = 2 * x + y;
          float cf = exp2_approx(Ga[y] - Gs[y]);
          if (own && sm.flag[rb][c + y]) cf = 0.f;
          dk[0][j][e] += cc[0][j][e] * cf;
          // KN_ib[s] = bf16(k_s 2^(G_a - G_s)): the row side's operand
          dG[0][j][e] -= kn[y] * cc[0][j][e];
        }
      }
  }
  // exact per-pair contributions of flagged (block, channel)s
  if (sm.nflag > 0) {
#pragma unroll
    for (int j = 0; j < NTk; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = m0 + (lane >> 2) + (e >> 1) * 8, c = n0 + 8 * j + 2 * (lane & 3) + (e & 1);
        if (!sm.flag[rb][c] || r >= L) continue;
        const float Gr = sm.G[r][c], qr = qv(r, c), kr = kv(r, c), br = bv(r, c);
        float dqi = 0.f, rr = 0.f, col = 0.f;
        for (int s = m0; s <= r; ++s) {
          const float E = exp2f(Gr - sm.G[s][c]);
          const float ks = kv(s, c);
          dqi += __bfloat162float(sm.DAqk[r][s]) * ks * E;
          if (s < r) rr += __bfloat162float(sm.DT[r][s]) * ks * E;
        }
        const int rend = (m0 + 16 < L) ? m0 + 16 : L;
        for (int r2 = r; r2 < rend; ++r2) {
          const float E = exp2f(sm.G[r2][c] - Gr);
          col += (__bfloat162float(sm.DAqk[r2][r]) * qv(r2, c) +
                  __bfloat162float(sm.DT[r2][r]) * bv(r2, c) * kv(r2, c)) * E;
        }
        dq[0][j][e] += dqi;
        dk[0][j][e] += rr * br + col;
        db[0][j][e] += rr * kr;
        dG[0][j][e] += qr * dqi + kr * br * rr - kr * col;
      }
  }
  __syncthreads();  // every read of G is done: its buffer becomes dG

  // ---- phase 4: epilogue -------------------------------------------------------
  const bool l2 = a.flags & GDN2_L2NORM_QK;
  {
    float pq[2] = {0.f, 0.f}, pk[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < NTk; ++j)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int r = m0 + (lane >> 2) + x * 8, c = n0 + 8 * j + 2 * (lane & 3);
        float g0 = dG[0][j][2 * x], g1 = dG[0][j][2 * x + 1];
        if (r == L - 1) {
          const float2 l2v = ld2(&sm.last[c]);
          g0 += l2v.x;
          g1 += l2v.y;
        }
        *reinterpret_cast<float2*>(&sm.G[r][c]) = r < L ? make_float2(g0, g1) : make_float2(0.f, 0.f);
        if (l2) {
          const float2 q2 = ld2(&sg.Q[r][c]), k2 = ld2(&sg.Kk[r][c]);
          pq[x] += dq[0][j][2 * x] * q2.x + dq[0][j][2 * x + 1] * q2.y;
          pk[x] += dk[0][j][2 * x] * k2.x + dk[0][j][2 * x + 1] * k2.y;
        }
      }
    if (l2) {
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        pq[x] += __shfl_xor_sync(0xffffffffu, pq[x], 1);
        pq[x] += __shfl_xor_sync(0xffffffffu, pq[x], 2);
        pk[x] += __shfl_xor_sync(0xffffffffu, pk[x], 1);
        pk[x] += __shfl_xor_sync(0xffffffffu, pk[x], 2);
      }
      if ((lane & 3) == 0) {
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          sm.rsum[m0 + (lane >> 2) + 8 * x][ch][0] = pq[x];
          sm.rsum[m0 + (lane >> 2) + 8 * x][ch][1] = pk[x];
        }
      }
    }
  }
  __syncthreads();
  // the chunk's raw gate pre-activations (read by the dg section at the end)
  // are pulled into L2 now, so that section's loads do not wait on HBM
  constexpr int kGParts = kBIntraThreads / K, kGRows = kChunk / kGParts;
  const bool gate = a.flags & GDN2_GATE_IN_KERNEL;
  const bool g16 = a.flags & GDN2_G_BF16;
  if (gate && pf_stride > 0 && tid == 0) tc::tma_prefetch_3d(&pm.g, 0, (int)h, (int)t0);
  {
    // staged in the phase-3 operand region (dead now), written out below
    __nv_bfloat16 (*sdq)[S::LK] = reinterpret_cast<__nv_bfloat16 (*)[S::LK]>(&p3.QG[0][0]);
    __nv_bfloat16 (*sdk)[S::LK] = reinterpret_cast<__nv_bfloat16 (*)[S::LK]>(&p3.KBG[0][0]);
    TB (*sdb)[S::LB] = reinterpret_cast<TB (*)[S::LB]>(&p3.KN[0][0]);
    static_assert(kChunk * S::LB * sizeof(TB) <= sizeof(p3.KN), "staged db fits the KN operand");
    // the l2norm row factors of this lane's two rows (loaded once, not per element)
    float lq[2] = {0.f, 0.f}, lk[2] = {0.f, 0.f}, rsq[2] = {0.f, 0.f}, rsk[2] = {0.f, 0.f};
    if (l2) {
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int r = m0 + (lane >> 2) + x * 8;
        if (r < L) {
          lq[x] = ws.q_rstd[(t0 + r) * H + h];
          lk[x] = ws.k_rstd[(t0 + r) * H + h];
#pragma unroll
          for (int y = 0; y < 4; ++y) {
            rsq[x] += sm.rsum[r][y][0];
            rsk[x] += sm.rsum[r][y][1];
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < NTk; ++j)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int r = m0 + (lane >> 2) + x * 8, c = n0 + 8 * j + 2 * (lane & 3);
        float xq0 = dq[0][j][2 * x], xq1 = dq[0][j][2 * x + 1];
        float xk0 = dk[0][j][2 * x], xk1 = dk[0][j][2 * x + 1];
        if (l2 && r < L) {
          const float sq = rsq[x], sk = rsk[x], rq = lq[x], rk = lk[x];
          const float2 q2 = ld2(&sg.Q[r][c]), k2 = ld2(&sg.Kk[r][c]);
          xq0 = (xq0 - sq * q2.x) * rq;
          xq1 = (xq1 - sq * q2.y) * rq;
          xk0 = (xk0 - sk * k2.x) * rk;
          xk1 = (xk1 - sk * k2.y) * rk;
        }
        *reinterpret_cast<__nv_bfloat162*>(&sdq[r][c]) = __floats2bfloat162_rn(xq0, xq1);
        *reinterpret_cast<__nv_bfloat162*>(&sdk[r][c]) = __floats2bfloat162_rn(xk0, xk1);
        store2<TB>(&sdb[r][c], db[0][j][2 * x], db[0][j][2 * x + 1]);
      }
    __syncthreads();
    __nv_bfloat16* dqo = static_cast<__nv_bfloat16*>(gr.dq);
    __nv_bfloat16* dko = static_cast<__nv_bfloat16*>(gr.dk);
    TB* dbo = static_cast<TB*>(gr.db);
    for (int i = tid; i < L * (K / 8); i += kBIntraThreads) {
      const int r = i / (K / 8), p = (i % (K / 8)) * 8;
      const int64_t gi = tokK(r, p);
      *reinterpret_cast<uint4*>(dqo + gi) = *reinterpret_cast<const uint4*>(&sdq[r][p]);
      *reinterpret_cast<uint4*>(dko + gi) = *reinterpret_cast<const uint4*>(&sdk[r][p]);
    }
    constexpr int kBPer16 = 16 / sizeof(TB);
    for (int i = tid; i < L * (K / kBPer16); i += kBIntraThreads) {
      const int r = i / (K / kBPer16), p = (i % (K / kBPer16)) * kBPer16;
      *reinterpret_cast<uint4*>(dbo + tokK(r, p)) = *reinterpret_cast<const uint4*>(&sdb[r][p]);
    }
  }
  // dg: reverse cumsum inside the chunk, then the gate VJP.  All threads take
  // part: channel c = tid % K, row part p = tid / K (kGParts parts of the chunk).
  const bool lbnd = a.flags & GDN2_LOWER_BOUND;
  {
    constexpr int kRowsPer = kGRows;
    const int c = tid % K, p = tid / K;
    const int r_lo = p * kRowsPer, r_hi = r_lo + kRowsPer;  // rows [r_lo, r_hi)
    float part = 0.f;
    for (int r = r_lo; r < r_hi; ++r) part += sm.G[r][c];  // rows >= L hold zero
    sm.ptot[p][c] = part;
    __syncthreads();
    float acc = 0.f;
    for (int q2 = p + 1; q2 < kGParts; ++q2) acc += sm.ptot[q2][c];
    const float Aexp = gate ? __expf(a.A_log[h]) : 0.f;
    const float bias = (gate && a.dt_bias) ? a.dt_bias[h * K + c] : 0.f;
    // d(activation)/d(raw) and the A_log factor per row: independent of the
    // cumsum chain, so computed ahead of it with full ILP
    float fo[kRowsPer], fa[kRowsPer];
    if (gate) {
      float graw[kRowsPer];
      if (g16) {
        const __nv_bfloat16* gp = static_cast<const __nv_bfloat16*>(a.g);
#pragma unroll
        for (int i = 0; i < kRowsPer; ++i)
          graw[i] = (r_lo + i < L) ? __bfloat162float(gp[tokK(r_lo + i, c)]) : 0.f;
      } else {
        const float* gp = static_cast<const float*>(a.g);
#pragma unroll
        for (int i = 0; i < kRowsPer; ++i) graw[i] = (r_lo + i < L) ? gp[tokK(r_lo + i, c)] : 0.f;
      }
#pragma unroll
      for (int i = 0; i < kRowsPer; ++i) {
        const float x = graw[i] + bias;
        if (lbnd) {
          const float s2 = sigmoid_f(Aexp * x);
          fo[i] = a.lower_bound * s2 * (1.f - s2) * Aexp;
          fa[i] = fo[i] * x;
        } else {
          fo[i] = -Aexp * sigmoid_f(x);
          fa[i] = -Aexp * softplus_f(x);
        }
      }
    }
    float dA = 0.f, dbias = 0.f;
    float outv[kRowsPer];  // dg of the rows, stored after the chain
#pragma unroll
    for (int i = kRowsPer - 1; i >= 0; --i) {
      const int r = r_lo + i;
      acc += sm.G[r][c];
      float out = acc;
      if (gate) {
        out = r < L ? acc * fo[i] : 0.f;
        dA += r < L ? acc * fa[i] : 0.f;
        dbias += out;
      }
      outv[i] = out;
    }
    if (g16) {
      __nv_bfloat16* dgp = static_cast<__nv_bfloat16*>(gr.dg);
#pragma unroll
      for (int i = 0; i < kRowsPer; ++i)
        if (r_lo + i < L) dgp[tokK(r_lo + i, c)] = __float2bfloat16_rn(outv[i]);
    } else {
      float* dgp = static_cast<float*>(gr.dg);
#pragma unroll
      for (int i = 0; i < kRowsPer; ++i)
        if (r_lo + i < L) dgp[tokK(r_lo + i, c)] = outv[i];
    }
    if (gate) {
      if (a.dt_bias) atomicAdd(&gr.ddt_bias[h * K + c], dbias);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) dA += __shfl_xor_sync(0xffffffffu, dA, off);
      if (lane == 0) atomicAdd(&gr.dA_log[h], dA);
    }
  }
}

// ---------------------------------------------------------------------------
template <int K, int V>
int launch_bwd_kv(const gdn2_chunk_args& a, const gdn2_chunk_grads& g, const ChunkWs& ws, const BwdWs& bw,
                  cudaStream_t s) {
  if (scan_fwd_tc_supported(a)) {
    const int st = scan_bwd_tc_launch(a, g, ws, bw, s);
    if (st != 0) return st;
  } else {
    const size_t sm2 = sizeof(BScanSmem<K>);
    GDN2_CUDA_TRY(cudaFuncSetAttribute(chunk_scan_bwd_kernel<K, V>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sm2));
    dim3 g2((unsigned)(V / kBScanBV), (unsigned)(a.N * a.H));
    ProfScope ps(kKScanBwd, s);
    chunk_scan_bwd_kernel<K, V><<<g2, kBScanThreads, sm2, s>>>(a, g, ws, bw);
    GDN2_LAUNCH_CHECK();
  }
  if (a.flags & GDN2_BWD_STATE_ONLY) return 0;
  if (a.NT > 0) {
    const bool bwb = a.dtype_bw == GDN2_BF16;
    constexpr bool kTc = K == 128 && V == 128;  // the tcgen05 variant (1024-byte-aligned tiles)
    using S16 = std::conditional_t<kTc, BIntraSmemTc<__nv_bfloat16>, BIntraSmem<K, V, __nv_bfloat16>>;
    using S32 = std::conditional_t<kTc, BIntraSmemTc<float>, BIntraSmem<K, V, float>>;
    const size_t sm3 = (bwb ? sizeof(S16) : sizeof(S32)) + (kTc ? 1024 : 0);
    auto k3 = bwb ? chunk_bwd_intra_kernel<K, V, __nv_bfloat16> : chunk_bwd_intra_kernel<K, V, float>;
    GDN2_CUDA_TRY(cudaFuncSetAttribute(k3, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm3));
    // next-CTA L2 prefetch (0: off) when linear CTA ids, token and state-row
    // coordinates fit 31 bits and the driver accepts every map; it only warms L2
    BwdIntraPrefetch pm;
    const uint64_t tokens = (uint64_t)a.B * (uint64_t)a.T, hrows = (uint64_t)a.NT * a.H * V;
    const bool pf_ok = (uint64_t)a.NT * a.H < (1ull << 31) && tokens < (1ull << 31) && hrows < (1ull << 31) &&
                       state_rows_map(&pm.h, ws.h, K, hrows) && state_rows_map(&pm.dh, bw.dh, K, hrows) &&
                       chunk_rows_map(&pm.dout, g.dout, 2, V, a.H, tokens) &&
                       chunk_rows_map(&pm.vn, ws.v_new, 2, V, a.H, tokens) &&
                       chunk_rows_map(&pm.dvn, bw.dvn, 2, V, a.H, tokens) &&
                       chunk_rows_map(&pm.A, ws.Akk, 2, kChunk, a.H, tokens) &&
                       chunk_rows_map(&pm.G, ws.G, 4, K, a.H, tokens) &&
                       chunk_rows_map(&pm.q, ws.qn, 2, K, a.H, tokens) &&
                       chunk_rows_map(&pm.k, ws.kn, 2, K, a.H, tokens) &&
                       chunk_rows_map(&pm.b, a.b, a.dtype_bw == GDN2_BF16 ? 2 : 4, K, a.H, tokens) &&
                       chunk_rows_map(&pm.w, a.w, a.dtype_bw == GDN2_BF16 ? 2 : 4, V, a.H, tokens) &&
                       chunk_rows_map(&pm.v, a.v, 2, V, a.H, tokens) &&
                       chunk_rows_map(&pm.g, a.g, (a.flags & GDN2_G_BF16) ? 2 : 4, K, a.H, tokens);
    dim3 g3((unsigned)a.NT, (unsigned)a.H);
    ProfScope ps(kKBwdIntra, s);
    k3<<<g3, kBIntraThreads, sm3, s>>>(a, g, ws, bw, pf_ok ? sm_count() : 0, pm);
    GDN2_LAUNCH_CHECK();
  }
  return 0;
}

// Reads (and optionally clears) the fault word of the backward intra kernel.
int b3_fault_read(int clear, unsigned int* out) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_b3_fault, sizeof(v));
  if (e != cudaSuccess) return -static_cast<int>(e);
  if (clear && v) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_b3_fault, &z, sizeof(z));
    if (e != cudaSuccess) return -static_cast<int>(e);
  }
  *out = v;
  return 0;
}

int chunk_bwd_launch(const gdn2_chunk_args& a, const gdn2_chunk_grads& g, const ChunkWs& ws, const BwdWs& bw,
                     cudaStream_t s) {
  if (a.K == 128 && a.V == 128) return launch_bwd_kv<128, 128>(a, g, ws, bw, s);
  if (a.K == 128 && a.V == 64) return launch_bwd_kv<128, 64>(a, g, ws, bw, s);
  if (a.K == 64 && a.V == 128) return launch_bwd_kv<64, 128>(a, g, ws, bw, s);
  return launch_bwd_kv<64, 64>(a, g, ws, bw, s);
}

}  // namespace gdn2
