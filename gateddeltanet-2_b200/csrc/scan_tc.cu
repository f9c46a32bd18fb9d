// Forward state scan on 5th-generation tensor cores (tcgen05 + TMEM + TMA),
// for d_k = d_v = 128: chunk_gated_delta_rule_fwd_h with its fused output
// (reference: lit_gpt/gdn2_ops/chunk_kda.py:983-1335, called from
// chunk_gdn2.py:1205-1359), restated in transposed form so that every
// product has M = 128 (the state's V rows):
//
//     v_new^T = U^T - S^T Y^T                  (MMA1: S^T Y^T,   N = 64, K = 128)
//     o^T     = S^T qg^T + v_new^T Aqk^T       (MMA2 / MMA3,     N = 64, K = 128 / 64;
//                                               qg carries the output scale)
//     S^T    <- S^T Diag(2^G_last) + v_new^T kg(MMA4,            N = 128, K = 64)
//
// One CTA per (sequence, head).  S^T lives in TMEM for the whole sequence
// (lane v = state column v, TMEM column k = state row k, fp32); the products
// accumulate in TMEM; operands sit in shared memory in the 128-byte swizzled
// layout TMA writes.  MMA1 and MMA2 share A = S^T and run as one N = 128
// product over the stacked [Y; qg] tile.  Warp roles:
//   warps 0-7  state warps: TMEM lane quarter w % 4, column half w / 4.  Per
//              chunk they turn S^T into the bf16 operand (and the saved chunk
//              state h), apply the decay in TMEM, form v_new from MMA1 and U
//              (in place over the U tile) and o (into a [t][v] tile).
//   warp 8     allocates TMEM; lane 0 issues the MMAs and commits them.
//   warp 9     lane 0 loads the next chunk's tiles by TMA (and G_last by a
//              bulk copy) into the other stage.
//   warp 10    writes the chunk state h^T (a TMA store of the bf16 S^T
//              operand tile itself) and the v_new and o tiles: a TMA store per
//              full chunk, 16-byte row copies for the ragged last chunk of a
//              sequence (a tile store would run into the next sequence's rows).
// Every wait is bounded (tc::kWaitLimitNs); a wait that gives up sets
// g_tc_fault, abandons the scan and still frees TMEM before returning.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "chunk_layout.cuh"
#include "common.cuh"
#include "profile.cuh"
#include "tc.cuh"

namespace gdn2 {

__device__ unsigned int g_tc_fault;  // bit 0: a bounded wait in a tcgen05 kernel gave up

namespace {

constexpr int kTcK = 128, kTcV = 128;
constexpr int kStateThreads = 256;
constexpr int kTcThreads = kStateThreads + 96;
constexpr int kWarpMma = 8, kWarpLoad = 9, kWarpStore = 10;
constexpr uint32_t kTileBytes = 64 * 64 * 2;  // one [64 x 64] bf16 swizzled tile
constexpr uint32_t kStageTx = 9 * kTileBytes + kTcK * 4;

// TMEM columns (fp32, 128 lanes).  The per-chunk products alternate between
// two column sets by chunk parity p, so a chunk's output can still be read
// while the next chunk's products run.
constexpr uint32_t kColS = 0;  // S^T [128 x 128]
// S^T Y^T - U^T = -v_new^T [128 x 64] (forward); S^T Y^T (transition mode, U = 0)
GDN2_DEV constexpr uint32_t col_av(int p) { return 128 + 128 * p; }
// S^T qg^T + v_new^T Aqk^T = o^T [128 x 64]
GDN2_DEV constexpr uint32_t col_ao(int p) { return 192 + 128 * p; }
constexpr uint32_t kTmemCols = 512;

struct alignas(1024) TcStage {
  __nv_bfloat16 YQ[2][128 * 64];  // per 64-column block of k: rows 0-63 Y, rows 64-127 qg
  __nv_bfloat16 KG[2][64 * 64];   // [t][k]  (B operand of MMA4, N-major)
  __nv_bfloat16 U[2][64 * 64];    // [t][v]; overwritten in place by v_new
  __nv_bfloat16 Aqk[64 * 64];     // [t][s]
  float glast[kTcK];              // G of the chunk's last token (log2 units)
  float D[kTcK];                  // 2^glast, filled by the producer warp
};

struct alignas(1024) TcSmem {
  TcStage st[2];
  __nv_bfloat16 SA[2][128 * 64];  // S^T in bf16, [v][k], two 64-column blocks
  __nv_bfloat16 VN[128 * 64];     // v_new^T in bf16, [v][t]
  __nv_bfloat16 OT[2][64 * 64];   // o in bf16, [t][v], two 64-column blocks
  __nv_bfloat16 NegI[64 * 64];    // -I [t'][t] (K-major B): the first product starts from -U^T
  uint64_t full[2], empty[2], dready[2];
  uint64_t sa_ready, sa_free, mma12, vn_ready, vst_ready, mma34, o_full, ot_free;
  uint32_t tbase;
};
static_assert(sizeof(TcSmem) + 1024 <= 227 * 1024, "tcgen05 scan shared memory");
static_assert(offsetof(TcStage, glast) % 16 == 0, "bulk copy target alignment");

GDN2_DEV uint64_t kdesc(const void* p, uint32_t byte_off) {
  return tc::sdesc_sw128(tc::smem_u32(p) + byte_off, 16, 1024);
}

GDN2_DEV void fault() { atomicOr(&g_tc_fault, 1u); }

// Bounded wait whose outcome is the same on every lane of the warp (the
// warp-collective TMEM loads and stores after it must not diverge).
GDN2_DEV bool warp_wait(uint64_t* bar, uint32_t parity) {
  const bool r = tc::mbar_wait(bar, parity);
  return __all_sync(0xffffffffu, r);
}

// rows [0, L) of a [64 x 128] bf16 tile (two swizzled 64-column blocks) to
// global [tokens, H, 128] at token t0, head h; one warp, 16-byte pieces
GDN2_DEV void copy_rows_out(const __nv_bfloat16 (*tile)[64 * 64], __nv_bfloat16* dst, int64_t t0, int64_t H,
                            int64_t h, int L, int lane) {
  for (int i = lane; i < L * 16; i += 32) {
    const int t = i >> 4, piece = i & 15, b = piece >> 3, p = piece & 7;
    const uint4 val = *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(tile[b]) + t * 128 +
                                                       ((p ^ (t & 7)) << 4));
    *reinterpret_cast<uint4*>(dst + ((t0 + t) * H + h) * 128 + piece * 8) = val;
  }
}

// ---------------------------------------------------------------------------
// Segmented scans.  With few (sequence, head) pairs on the GPU, one CTA per
// pair walking its whole sequence leaves most SMs idle.  A sequence's chunks
// can then be cut into nseg segments of seg_len chunks (seg_plan).  Across a
// segment the state maps affinely, S_out = M_s S_in + h_s with
// M_s = prod_c (Diag(2^G_last) - kg^T Y) (the identity the context-parallel
// transition uses), so the forward runs
//   pass 1  segment 0 in full from the initial state, its exit state into
//           X[0]; every middle segment s twice without outputs: from the
//           identity with U = 0 (-> M[s]) and from zero (-> X[s]);
//   fold    X[s] <- M_s X[s-1] + X[s], s = 1 .. nseg-2, in fp32;
//   pass 2  segments 1 .. nseg-1 in full from X[s-1].
// The reverse scan runs the adjoint, dS_in = M_s^T dS_out + g_s, the same way
// (its passes are described at the backward kernel).  Pass 3 is the
// context-parallel transition of a whole shard: M from the identity and h_e
// from the shard's initial state, into the [K, K+V] map.
// ---------------------------------------------------------------------------
struct SegArgs {
  int nseg;      // segments per sequence
  int seg_len;   // chunks per segment
  int pass;      // 0: the whole sequence per CTA; 1, 2: the passes above; 3: CP transition;
                 // 4: CP transition in segments (every segment's M_s and h_s)
  float* X;      // [N*H, nseg, K, V] segment states (the reverse scan: cotangents)
  const float* M;  // [N*H, nseg, K, K] segment transitions
  float* P = nullptr;  // pass 4: [N*H, nseg, K, K], segment 0's transition goes to P[0]
};

enum ScanMode { kModeFull = 0, kModeTransM = 1, kModeTransH = 2 };

struct ScanJob {
  int mode;            // kModeFull: outputs; kModeTransM: identity start, U = 0; kModeTransH: no outputs
  int cb, ce;          // chunks [cb, ce) of the sequence
  const float* init;   // entering state (nullptr: zero, or the identity)
  bool init_tr;        // init stored [V][K] (row stride K), else [K][V] (row stride V)
  bool identity;
  float* exit;         // destination of the exit state, or nullptr
  int exit_ld;         // elements between its rows ([K][.] layout)
  bool exit_tr;        // store [V][K] instead
};

constexpr int64_t kKV = (int64_t)kTcK * kTcV;

GDN2_DEV ScanJob fwd_job(const gdn2_chunk_args& a, const SegArgs& sg, int64_t nh, int y, int nchunks,
                         float* maps) {
  ScanJob j{};
  const bool tr = a.flags & GDN2_TRANSPOSE_STATE;
  const float* h0 = (a.flags & GDN2_HAS_H0) ? a.h0 + nh * kKV : nullptr;
  float* ht = (a.flags & GDN2_STORE_FINAL) ? a.ht + nh * kKV : nullptr;
  j.exit_ld = kTcV;
  j.cb = 0;
  j.ce = nchunks;
  if (sg.pass == 0) {
    j.mode = kModeFull;
    j.init = h0;
    j.init_tr = tr;
    j.exit = ht;
    j.exit_tr = tr;
    return j;
  }
  if (sg.pass == 3) {
    float* mp = maps + nh * (int64_t)kTcK * (kTcK + kTcV);
    j.exit_ld = kTcK + kTcV;
    if (y == 0) {
      j.mode = kModeTransM;
      j.identity = true;
      j.exit = mp;
    } else {
      j.mode = kModeTransH;
      j.init = h0;
      j.exit = mp + kTcK;
    }
    return j;
  }
  float* X = sg.X + nh * sg.nseg * kKV;
  int seg;
  if (sg.pass == 4) {
    seg = y / 2;
    if (y & 1) {
      j.mode = kModeTransH;
      j.init = seg == 0 ? h0 : nullptr;
      j.exit = X + seg * kKV;
    } else {
      j.mode = kModeTransM;
      j.identity = true;
      j.exit = seg == 0 ? sg.P + nh * sg.nseg * kKV : const_cast<float*>(sg.M) + (nh * sg.nseg + seg) * kKV;
    }
    j.cb = seg * sg.seg_len;
    j.ce = min(j.cb + sg.seg_len, nchunks);
    return j;
  }
  if (sg.pass == 1) {
    if (y == 0) {
      seg = 0;
      j.mode = kModeFull;
      j.init = h0;
      j.init_tr = tr;
      j.exit = X;
    } else {
      seg = 1 + (y - 1) / 2;
      if ((y - 1) & 1) {
        j.mode = kModeTransH;
        j.exit = X + seg * kKV;
      } else {
        j.mode = kModeTransM;
        j.identity = true;
        j.exit = const_cast<float*>(sg.M) + (nh * sg.nseg + seg) * kKV;
      }
    }
  } else {
    seg = 1 + y;
    j.mode = kModeFull;
    j.init = X + (seg - 1) * kKV;
    if (seg == sg.nseg - 1) {
      j.exit = ht;
      j.exit_tr = tr;
    }
  }
  j.cb = seg * sg.seg_len;
  j.ce = min(j.cb + sg.seg_len, nchunks);
  return j;
}

// The job's entering state into TMEM (this thread: lane v, columns k0..k0+63)
GDN2_DEV void load_state(const ScanJob& j, uint32_t taddr, int v, int k0) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    float x[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int k = k0 + 32 * q + i;
      x[i] = j.identity ? (k == v ? 1.f : 0.f)
             : j.init   ? (j.init_tr ? j.init[(int64_t)v * kTcK + k] : j.init[(int64_t)k * kTcV + v])
                        : 0.f;
    }
    tc::tmem_st32(taddr + k0 + 32 * q, x);
  }
  tc::tmem_wait_st();
}

// The state in TMEM (lane v, columns k0..k0+63) to the job's exit destination
GDN2_DEV void store_state(const ScanJob& j, uint32_t taddr, int v, int k0) {
  if (!j.exit) return;
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    float x[32];
    tc::tmem_ld32(taddr + k0 + 32 * q, x);
    tc::tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int k = k0 + 32 * q + i;
      if (j.exit_tr) j.exit[(int64_t)v * kTcK + k] = x[i];
      else j.exit[(int64_t)k * j.exit_ld + v] = x[i];
    }
  }
}

template <bool kSave>
__global__ void __launch_bounds__(kTcThreads, 1)
chunk_scan_fwd_tc_kernel(const gdn2_chunk_args a, const ChunkWs ws, const SegArgs sg, float* maps,
                         const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmQG,
                         const __grid_constant__ CUtensorMap tmKG, const __grid_constant__ CUtensorMap tmU,
                         const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmO,
                         const __grid_constant__ CUtensorMap tmVN, const __grid_constant__ CUtensorMap tmH) {
  extern __shared__ unsigned char smem_raw[];
  TcSmem& sm = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t H = a.H;
  const int64_t nh = blockIdx.x, n = nh / H, h = nh % H;
  SeqGeom geo{a.cu_seqlens, a.chunk_index, a.chunk_offset, a.T, (a.T + kChunk - 1) / kChunk};
  int64_t bos, len;
  geo.seq(n, bos, len);
  const int nchunks = (int)((len + kChunk - 1) / kChunk);
  const int64_t c0 = geo.chunk0(n);
  const ScanJob job = fwd_job(a, sg, nh, (int)blockIdx.y, nchunks, maps);
  const int cb = job.cb, nloc = job.ce > job.cb ? job.ce - job.cb : 0;
  const bool outs = job.mode == kModeFull;     // o (and, saving, h and v_new) are written
  const bool uzero = job.mode == kModeTransM;  // U = 0: the U tiles are not loaded
  const bool save = kSave && outs;
  auto chunk_len = [&](int c) {
    const int64_t r = len - (int64_t)c * kChunk;
    return (int)(r < kChunk ? r : kChunk);
  };

  if (tid == 0) {
    tc::mbar_init(&sm.full[0], 1);
    tc::mbar_init(&sm.full[1], 1);
    // a stage is free once the MMAs' commit and (with outputs) the output warp
    // having read U have arrived.  Without outputs the output warp takes no
    // part at all: nothing would keep the state warps within one phase of
    // vst_ready for it.
    tc::mbar_init(&sm.empty[0], outs ? 2 : 1);
    tc::mbar_init(&sm.empty[1], outs ? 2 : 1);
    tc::mbar_init(&sm.dready[0], 32);  // the producer warp's lanes, D of the stage written
    tc::mbar_init(&sm.dready[1], 32);
    tc::mbar_init(&sm.sa_ready, kStateThreads);
    tc::mbar_init(&sm.sa_free, 1);
    tc::mbar_init(&sm.mma12, 1);
    tc::mbar_init(&sm.vn_ready, kStateThreads);
    tc::mbar_init(&sm.vst_ready, kStateThreads);
    tc::mbar_init(&sm.mma34, 1);
    tc::mbar_init(&sm.o_full, kStateThreads);
    tc::mbar_init(&sm.ot_free, 1);
    tc::mbar_fence_init();
  }
  for (int i = tid; i < 64 * 64; i += kTcThreads) {
    const int r = i >> 6, c = i & 63;
    *reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<char*>(sm.NegI) + tc::sw128_off(r, c)) =
        __float2bfloat16_rn(r == c ? -1.f : 0.f);
  }
  tc::fence_proxy_async();  // -I -> the tensor core
  if (warp == kWarpMma) tc::tmem_alloc(&sm.tbase, kTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tb = sm.tbase;
  bool ok = true;

  if (warp < 8) {
    // ------------------------------------------------------------ state warps
    const int qtr = warp & 3, half = warp >> 2;
    const int v = 32 * qtr + lane;
    const uint32_t tl = tb + ((uint32_t)(32 * qtr) << 16);
    const int kb0 = 64 * half;  // this thread's state rows k (entering and exit states)
    const int tb0 = 32 * half;  // this thread's tokens t (v_new, o)
    load_state(job, tl + kColS, v, kb0);
    // o of local chunk i into the [t][v] tile; runs while chunk i + 1's first
    // product executes (its accumulator columns alternate by parity)
    auto output = [&](int i) -> bool {
      float x[32];
      tc::tmem_ld32(tl + col_ao(i & 1) + tb0, x);
      tc::tmem_wait_ld();
      if (i > 0 && !warp_wait(&sm.ot_free, (i - 1) & 1)) return false;
      char* ot = reinterpret_cast<char*>(sm.OT[v >> 6]);
#pragma unroll
      for (int t = 0; t < 32; ++t)
        *reinterpret_cast<__nv_bfloat16*>(ot + tc::sw128_off(tb0 + t, v & 63)) = __float2bfloat16_rn(x[t]);
      tc::fence_proxy_async();
      tc::mbar_arrive(&sm.o_full);
      return true;
    };
    for (int it = 0; it < nloc; ++it) {
      const int s = it & 1;
      TcStage& st = sm.st[s];
      const int L = chunk_len(cb + it);
      if (!(ok = warp_wait(&sm.dready[s], (it >> 1) & 1))) break;  // the stage and its D

      // step 1: entering state -> bf16 operand rows (also the saved h^T); decay in TMEM
      if (save && it > 0 && !(ok = warp_wait(&sm.sa_free, (it - 1) & 1))) break;
      char* sarow = reinterpret_cast<char*>(sm.SA[half]) + v * 128;
      {
        float x0[32], x1[32];
        tc::tmem_ld32(tl + kColS + kb0, x0);
        tc::tmem_ld32(tl + kColS + kb0 + 32, x1);
        tc::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          *reinterpret_cast<uint4*>(sarow + ((q ^ (v & 7)) << 4)) = pack8(x0 + 8 * q);
          *reinterpret_cast<uint4*>(sarow + (((4 + q) ^ (v & 7)) << 4)) = pack8(x1 + 8 * q);
        }
        const float4* d4 = reinterpret_cast<const float4*>(st.D + kb0);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 d = d4[q], e = d4[8 + q];
          x0[4 * q + 0] *= d.x;
          x0[4 * q + 1] *= d.y;
          x0[4 * q + 2] *= d.z;
          x0[4 * q + 3] *= d.w;
          x1[4 * q + 0] *= e.x;
          x1[4 * q + 1] *= e.y;
          x1[4 * q + 2] *= e.z;
          x1[4 * q + 3] *= e.w;
        }
        tc::tmem_st32(tl + kColS + kb0, x0);
        tc::tmem_st32(tl + kColS + kb0 + 32, x1);
      }
      tc::tmem_wait_st();
      tc::fence_proxy_async();
      tc::tc_fence_before();
      tc::mbar_arrive(&sm.sa_ready);
      if (outs && it > 0 && !(ok = output(it - 1))) break;

      // step 2: v_new = U - (S^T Y^T)^T, in place over U and as the MMA operand
      if (!(ok = warp_wait(&sm.mma12, it & 1))) break;
      tc::tc_fence_after();
      {
        // -v_new^T of this thread's 32 tokens (the U^T term came in with the product)
        float x[32];
        tc::tmem_ld32(tl + col_av(it & 1) + tb0, x);
        __nv_bfloat16* ucol = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<char*>(st.U[v >> 6]) +
                                                            ((v & 7) << 1));
        const int vb = (v & 63) >> 3;
        __nv_bfloat16 u[32];
        tc::tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const __nv_bfloat16 vn = __float2bfloat16_rn(tb0 + t < L ? -x[t] : 0.f);
          u[t] = vn;
          x[t] = __bfloat162float(vn);
        }
        // the MMA operand first; the copy for the store follows off the critical path
        char* row = reinterpret_cast<char*>(sm.VN) + v * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(row + (((4 * half + q) ^ (v & 7)) << 4)) = pack8(x + 8 * q);
        tc::fence_proxy_async();
        tc::tc_fence_before();
        tc::mbar_arrive(&sm.vn_ready);
        if (save) {
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const int tt = tb0 + t;
            ucol[(tt * 128 + ((vb ^ (tt & 7)) << 4)) >> 1] = u[t];
          }
          tc::fence_proxy_async();
        }
        tc::mbar_arrive(&sm.vst_ready);  // the stage's U reads (and v_new writes) are done
      }

      // the chunk's products are complete: S is updated, o is in TMEM
      if (!(ok = warp_wait(&sm.mma34, it & 1))) break;
      tc::tc_fence_after();
    }
    if (ok && outs && nloc > 0) ok = output(nloc - 1);
    if (ok) store_state(job, tl + kColS, v, kb0);
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && nloc > 0) {
      constexpr uint32_t kId64 = tc::idesc_bf16(128, 64, 0, 0);
      constexpr uint32_t kIdS = tc::idesc_bf16(128, 128, 0, 1);
      uint64_t* last = nullptr;  // barrier of the last commit and its phase parity
      uint32_t last_par = 0;
      for (int it = 0; it < nloc; ++it) {
        const int s = it & 1;
        TcStage& st = sm.st[s];
        if (!(ok = tc::mbar_wait(&sm.full[s], (it >> 1) & 1) && tc::mbar_wait(&sm.sa_ready, it & 1))) break;
        tc::tc_fence_after();
        // S^T Y^T - U^T = -v_new^T: the U^T part as U^T (-I) (U as an M-major operand,
        // 64-row blocks 8 KB apart), then S^T Y^T onto it; S^T qg^T (o's first part)
        // into the next 64 columns (qg: rows 64-127 of each [Y; qg] block)
        constexpr uint32_t kIdU = tc::idesc_bf16(128, 64, 1, 0);
        if (!uzero) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::mma_bf16(tb + col_av(it & 1), tc::sdesc_sw128(tc::smem_u32(st.U[0]) + kk * 2048, kTileBytes, 1024),
                         kdesc(sm.NegI, kk * 32), kIdU, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc::mma_bf16(tb + col_av(it & 1), kdesc(sm.SA[kk >> 2], (kk & 3) * 32),
                       kdesc(st.YQ[kk >> 2], (kk & 3) * 32), kId64, !uzero || kk > 0);
        if (outs) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            tc::mma_bf16(tb + col_ao(it & 1), kdesc(sm.SA[kk >> 2], (kk & 3) * 32),
                         kdesc(st.YQ[kk >> 2], 64 * 128 + (kk & 3) * 32), kId64, kk > 0);
        }
        tc::mma_commit(&sm.mma12);
        last = &sm.mma12;
        last_par = it & 1;
        if (!(ok = tc::mbar_wait(&sm.vn_ready, it & 1))) break;
        tc::tc_fence_after();
        if (outs) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            tc::mma_bf16(tb + col_ao(it & 1), kdesc(sm.VN, kk * 32), kdesc(st.Aqk, kk * 32), kId64, 1);
        }
        // kg as an N-major operand: 64-column blocks 8 KB apart, 8-row groups 1 KB apart
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::mma_bf16(tb + kColS, kdesc(sm.VN, kk * 32),
                       tc::sdesc_sw128(tc::smem_u32(st.KG[0]) + kk * 2048, kTileBytes, 1024), kIdS, 1);
        tc::mma_commit(&sm.mma34);
        tc::mma_commit(&sm.empty[s]);
        last = &sm.mma34;
        last_par = it & 1;
      }
      // the MMAs issued have completed before TMEM is released
      if (last && !tc::mbar_wait(last, last_par)) ok = false;
    }
  } else if (warp == kWarpLoad) {
    // ------------------------------------------------------------ TMA producer
    // lane 0 issues the loads; once a stage has landed the whole warp turns its
    // G_last into the decay D = 2^G_last and publishes it (dready).  Without
    // outputs qg and Aqk are not loaded, and U is not loaded for the M columns.
    if (lane == 0) {
      tc::prefetch_tensormap(&tmY);
      tc::prefetch_tensormap(&tmKG);
      if (!uzero) tc::prefetch_tensormap(&tmU);
      if (outs) {
        tc::prefetch_tensormap(&tmQG);
        tc::prefetch_tensormap(&tmA);
      }
    }
    const uint32_t tx = (outs ? 9u : (uzero ? 4u : 6u)) * kTileBytes + kTcK * 4;
    int it = 0;
    for (; it < nloc; ++it) {
      const int s = it & 1;
      TcStage& st = sm.st[s];
      if (it >= 2 && !(ok = warp_wait(&sm.empty[s], ((it >> 1) - 1) & 1))) break;
      if (lane == 0) {
        const int64_t t0 = bos + (int64_t)(cb + it) * kChunk;
        const int L = chunk_len(cb + it);
        const int tt = (int)t0, hh = (int)h;
        tc::mbar_arrive_expect_tx(&sm.full[s], tx);
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          tc::tma_load_3d(st.YQ[b], &tmY, &sm.full[s], 64 * b, hh, tt);
          if (outs) tc::tma_load_3d(st.YQ[b] + 64 * 64, &tmQG, &sm.full[s], 64 * b, hh, tt);
          tc::tma_load_3d(st.KG[b], &tmKG, &sm.full[s], 64 * b, hh, tt);
          if (!uzero) tc::tma_load_3d(st.U[b], &tmU, &sm.full[s], 64 * b, hh, tt);
        }
        if (outs) tc::tma_load_3d(st.Aqk, &tmA, &sm.full[s], 0, hh, tt);
        tc::bulk_load(st.glast, ws.G + ((t0 + L - 1) * H + h) * kTcK, kTcK * 4, &sm.full[s]);
      }
      __syncwarp();
      if (!(ok = warp_wait(&sm.full[s], (it >> 1) & 1))) break;
#pragma unroll
      for (int j = 0; j < kTcK / 32; ++j) st.D[lane + 32 * j] = exp2_approx(st.glast[lane + 32 * j]);
      tc::mbar_arrive(&sm.dready[s]);
    }
    // a load in flight (only after a wait gave up) lands before the CTA exits
    if (!ok && it < nloc) tc::mbar_wait(&sm.full[it & 1], (it >> 1) & 1);
  } else if (outs) {
    // ------------------------------------------------------------ output writer
    // Per chunk: h^T (from the S^T operand tile), o of the chunk before (its
    // output step runs during this chunk), v_new (in place over the U tile),
    // then the releases.  Every release (ot_free, sa_free, the stage's empty)
    // follows this warp's wait on vst_ready, and the state warps wait for
    // ot_free (or sa_free) of chunk i before they can arrive on vst_ready for
    // chunk i + 1, which keeps them within one phase of each barrier this
    // warp waits on.
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(a.o);
    auto store_o = [&](int c) {
      const int64_t t0 = bos + (int64_t)c * kChunk;
      const int L = chunk_len(c);
      if (L == kChunk) {
        if (lane == 0) {
          tc::tma_store_3d(&tmO, sm.OT[0], 0, (int)h, (int)t0);
          tc::tma_store_3d(&tmO, sm.OT[1], 64, (int)h, (int)t0);
          tc::bulk_commit();
        }
      } else {
        copy_rows_out(sm.OT, o, t0, H, h, L, lane);
      }
    };
    for (int it = 0; it < nloc; ++it) {
      const int s = it & 1, c = cb + it;
      TcStage& st = sm.st[s];
      const int64_t t0 = bos + (int64_t)c * kChunk;
      const int L = chunk_len(c);
      if (save) {
        if (!(ok = warp_wait(&sm.sa_ready, it & 1))) break;
        if (lane == 0) {
          const int row = (int)(((c0 + c) * H + h) * kTcV);
          tc::tma_store_2d(&tmH, sm.SA[0], 0, row);
          tc::tma_store_2d(&tmH, sm.SA[1], 64, row);
          tc::bulk_commit();
        }
      }
      if (it > 0) {
        if (!(ok = warp_wait(&sm.o_full, (it - 1) & 1))) break;
        store_o(c - 1);
      }
      if (!(ok = warp_wait(&sm.vst_ready, it & 1))) break;
      if (save) {
        if (L == kChunk) {
          if (lane == 0) {
            tc::tma_store_3d(&tmVN, st.U[0], 0, (int)h, (int)t0);
            tc::tma_store_3d(&tmVN, st.U[1], 64, (int)h, (int)t0);
            tc::bulk_commit();
          }
        } else {
          copy_rows_out(st.U, ws.v_new, t0, H, h, L, lane);
        }
      }
      if (lane == 0) tc::bulk_wait_read_all();
      __syncwarp();
      if (lane == 0) {
        if (save) tc::mbar_arrive(&sm.sa_free);
        if (it > 0) tc::mbar_arrive(&sm.ot_free);
        tc::mbar_arrive(&sm.empty[s]);
      }
    }
    if (ok && nloc > 0) {
      if ((ok = warp_wait(&sm.o_full, (nloc - 1) & 1))) {
        store_o(cb + nloc - 1);
        if (lane == 0) tc::bulk_wait_read_all();
      }
    }
    if (lane == 0) tc::bulk_wait_all();
  }

  if (!ok) fault();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tb, kTmemCols);
  }
}

// ===========================================================================
// Backward state scan (reverse over chunks), transposed like the forward:
//     dh^T[c]  = dS^T                                  (stored, bf16)
//     dv^T     = do^T Aqk + dS^T kg^T                   (MMA-a: N = 64, K = 64;
//                                                        MMA-b: N = 64, K = 128)
//     dS^T    <- dS^T Diag(2^G_last) + do^T qg - dv^T Y (MMA-c, MMA-d: N = 128, K = 64)
// (reference: chunk_kda.py:1356-1669 with the dAv of :3769-3831).  do and Aqk
// enter as N-/M-major operands straight from their TMA tiles; dv^T is written
// negated as the A operand of MMA-d.  Rows of do past a ragged sequence end
// are zeroed in shared memory: TMA loads the next sequence's rows there, and
// MMA-a and MMA-c contract over tokens with no other operand zero there.
// ===========================================================================
constexpr uint32_t kColDV = 128;  // dv^T [128 x 64]; dS^T at kColS

struct alignas(1024) BtStage {
  __nv_bfloat16 DO[2][64 * 64];  // [t][v], two 64-column blocks (M-major A of MMA-a / MMA-c)
  __nv_bfloat16 KG[2][64 * 64];  // [t][k]   (K-major B of MMA-b)
  __nv_bfloat16 QG[2][64 * 64];  // [t][k]   (N-major B of MMA-c)
  __nv_bfloat16 Y[2][64 * 64];   // [t][k]   (N-major B of MMA-d)
  __nv_bfloat16 Aqk[64 * 64];    // [s][t]   (N-major B of MMA-a)
  float glast[kTcK];
  float D[kTcK];                 // 2^glast, filled by the producer warp
};

struct alignas(1024) BtSmem {
  BtStage st[2];
  __nv_bfloat16 DSA[2][128 * 64];  // dS^T in bf16, [v][k] (A of MMA-b; also the stored dh^T)
  __nv_bfloat16 DVA[128 * 64];     // -dv^T in bf16, [v][t] (A of MMA-d)
  __nv_bfloat16 DVT[2][64 * 64];   // dv in bf16, [t][v] (stored)
  uint64_t full[2], empty[2], dready[2];
  uint64_t dsa_ready, dsa_free, dv_ready, dva_ready, dvt_ready, dvt_free, ds_ready;
  uint32_t tbase;
};
static_assert(sizeof(BtSmem) + 1024 <= 227 * 1024, "tcgen05 backward scan shared memory");

// The reverse scan's jobs.  Pass 0: the whole sequence from dht (dh0 out).
// Segmented (sg.X holds the cotangents Z[nh, s]):
//   pass 1  the last segment in full from dht, its entering cotangent into
//           Z[nseg-1]; every middle segment s from zero without outputs,
//           into Z[s] (its own contribution g_s);
//   fold    Z[s] <- M_s^T Z[s+1] + Z[s], s = nseg-2 .. 1 (the forward's M_s);
//   pass 2  segments 0 .. nseg-2 in full from Z[s+1]; segment 0 writes dh0.
GDN2_DEV ScanJob bwd_job(const gdn2_chunk_args& a, const gdn2_chunk_grads& gr, const SegArgs& sg, int64_t nh,
                         int y, int nchunks) {
  ScanJob j{};
  const bool tr = a.flags & GDN2_TRANSPOSE_STATE;
  const float* dht = gr.dht ? gr.dht + nh * kKV : nullptr;
  float* dh0 = gr.dh0 ? gr.dh0 + nh * kKV : nullptr;
  j.exit_ld = kTcV;
  j.cb = 0;
  j.ce = nchunks;
  if (sg.pass == 0) {
    j.mode = kModeFull;
    j.init = dht;
    j.init_tr = tr;
    j.exit = dh0;
    j.exit_tr = tr;
    return j;
  }
  float* Z = sg.X + nh * sg.nseg * kKV;
  int seg;
  if (sg.pass == 1) {
    if (y == 0) {
      seg = sg.nseg - 1;
      j.mode = kModeFull;
      j.init = dht;
      j.init_tr = tr;
      j.exit = Z + seg * kKV;
    } else {
      seg = y;
      j.mode = kModeTransH;
      j.exit = Z + seg * kKV;
    }
  } else {
    seg = y;
    j.mode = kModeFull;
    j.init = Z + (seg + 1) * kKV;
    if (seg == 0) {
      j.exit = dh0;
      j.exit_tr = tr;
    }
  }
  j.cb = seg * sg.seg_len;
  j.ce = min(j.cb + sg.seg_len, nchunks);
  return j;
}

__global__ void __launch_bounds__(kTcThreads, 1)
chunk_scan_bwd_tc_kernel(const gdn2_chunk_args a, const gdn2_chunk_grads gr, const ChunkWs ws, const BwdWs bw,
                         const SegArgs sg, const __grid_constant__ CUtensorMap tmDO,
                         const __grid_constant__ CUtensorMap tmKG, const __grid_constant__ CUtensorMap tmQG,
                         const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmDV, const __grid_constant__ CUtensorMap tmDH) {
  extern __shared__ unsigned char smem_raw[];
  BtSmem& sm = *reinterpret_cast<BtSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t H = a.H;
  const int64_t nh = blockIdx.x, n = nh / H, h = nh % H;
  SeqGeom geo{a.cu_seqlens, a.chunk_index, a.chunk_offset, a.T, (a.T + kChunk - 1) / kChunk};
  int64_t bos, len;
  geo.seq(n, bos, len);
  const int nchunks = (int)((len + kChunk - 1) / kChunk);
  const int64_t c0 = geo.chunk0(n);
  const ScanJob job = bwd_job(a, gr, sg, nh, (int)blockIdx.y, nchunks);
  const int nloc = job.ce > job.cb ? job.ce - job.cb : 0;
  const bool outs = job.mode == kModeFull;  // dh and dv_new are written
  // iteration it handles chunk ce - 1 - it
  auto chunk_of = [&](int it) { return job.ce - 1 - it; };
  auto chunk_len = [&](int c) {
    const int64_t r = len - (int64_t)c * kChunk;
    return (int)(r < kChunk ? r : kChunk);
  };

  if (tid == 0) {
    tc::mbar_init(&sm.full[0], 1);
    tc::mbar_init(&sm.full[1], 1);
    tc::mbar_init(&sm.empty[0], 1);
    tc::mbar_init(&sm.empty[1], 1);
    tc::mbar_init(&sm.dready[0], 32);
    tc::mbar_init(&sm.dready[1], 32);
    tc::mbar_init(&sm.dsa_ready, kStateThreads);
    tc::mbar_init(&sm.dsa_free, 1);
    tc::mbar_init(&sm.dv_ready, 1);
    tc::mbar_init(&sm.dva_ready, kStateThreads);
    tc::mbar_init(&sm.dvt_ready, kStateThreads);
    tc::mbar_init(&sm.dvt_free, 1);
    tc::mbar_init(&sm.ds_ready, 1);
    tc::mbar_fence_init();
  }
  if (warp == kWarpMma) tc::tmem_alloc(&sm.tbase, 256);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tb = sm.tbase;
  bool ok = true;

  if (warp < 8) {
    // ------------------------------------------------------------ state warps
    const int qtr = warp & 3, half = warp >> 2;
    const int v = 32 * qtr + lane;
    const uint32_t tl = tb + ((uint32_t)(32 * qtr) << 16);
    const int kb0 = 64 * half, tb0 = 32 * half;
    load_state(job, tl + kColS, v, kb0);
    for (int it = 0; it < nloc; ++it) {
      const int s = it & 1, c = chunk_of(it), L = chunk_len(c);
      BtStage& st = sm.st[s];
      if (!(ok = warp_wait(&sm.dready[s], (it >> 1) & 1))) break;  // the stage and its D
      if (L < kChunk) {  // do rows past the sequence end -> 0
        for (int i = tid; i < (kChunk - L) * 16; i += kStateThreads) {
          const int t = L + i / 16, piece = i % 16;
          *reinterpret_cast<uint4*>(reinterpret_cast<char*>(st.DO[piece >> 3]) + t * 128 + ((piece & 7) << 4)) =
              make_uint4(0u, 0u, 0u, 0u);
        }
      }

      // step 1: dS^T -> bf16 operand rows (also the stored dh^T); decay in TMEM
      if (it > 0 && !(ok = warp_wait(&sm.dsa_free, (it - 1) & 1))) break;
      {
        char* row = reinterpret_cast<char*>(sm.DSA[half]) + v * 128;
        float x0[32], x1[32];
        tc::tmem_ld32(tl + kColS + kb0, x0);
        tc::tmem_ld32(tl + kColS + kb0 + 32, x1);
        tc::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          *reinterpret_cast<uint4*>(row + ((q ^ (v & 7)) << 4)) = pack8(x0 + 8 * q);
          *reinterpret_cast<uint4*>(row + (((4 + q) ^ (v & 7)) << 4)) = pack8(x1 + 8 * q);
        }
        const float4* d4 = reinterpret_cast<const float4*>(st.D + kb0);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 d = d4[q], e = d4[8 + q];
          x0[4 * q + 0] *= d.x;
          x0[4 * q + 1] *= d.y;
          x0[4 * q + 2] *= d.z;
          x0[4 * q + 3] *= d.w;
          x1[4 * q + 0] *= e.x;
          x1[4 * q + 1] *= e.y;
          x1[4 * q + 2] *= e.z;
          x1[4 * q + 3] *= e.w;
        }
        tc::tmem_st32(tl + kColS + kb0, x0);
        tc::tmem_st32(tl + kColS + kb0 + 32, x1);
      }
      tc::tmem_wait_st();
      tc::fence_proxy_async();
      tc::tc_fence_before();
      tc::mbar_arrive(&sm.dsa_ready);

      // step 2: dv -> the negated operand [v][t] (critical), then the stored tile [t][v]
      if (!(ok = warp_wait(&sm.dv_ready, it & 1))) break;
      tc::tc_fence_after();
      {
        float x[32];
        tc::tmem_ld32(tl + kColDV + tb0, x);
        tc::tmem_wait_ld();
        __nv_bfloat16 dvb[32];
        float nx[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          dvb[i] = __float2bfloat16_rn(tb0 + i < L ? x[i] : 0.f);
          nx[i] = -__bfloat162float(dvb[i]);
        }
        char* row = reinterpret_cast<char*>(sm.DVA) + v * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(row + (((4 * half + q) ^ (v & 7)) << 4)) = pack8(nx + 8 * q);
        tc::fence_proxy_async();
        tc::tc_fence_before();
        tc::mbar_arrive(&sm.dva_ready);
        if (it > 0 && !(ok = warp_wait(&sm.dvt_free, (it - 1) & 1))) break;
        if (outs) {
          char* dvt = reinterpret_cast<char*>(sm.DVT[v >> 6]);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            *reinterpret_cast<__nv_bfloat16*>(dvt + tc::sw128_off(tb0 + i, v & 63)) = dvb[i];
          tc::fence_proxy_async();
        }
        tc::mbar_arrive(&sm.dvt_ready);
      }
      if (!(ok = warp_wait(&sm.ds_ready, it & 1))) break;
      tc::tc_fence_after();
    }
    if (ok) store_state(job, tl + kColS, v, kb0);
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && nloc > 0) {
      constexpr uint32_t kIdA = tc::idesc_bf16(128, 64, 1, 1);   // M-major do, N-major Aqk
      constexpr uint32_t kIdB = tc::idesc_bf16(128, 64, 0, 0);   // dS^T, kg
      constexpr uint32_t kIdC = tc::idesc_bf16(128, 128, 1, 1);  // M-major do, N-major qg
      constexpr uint32_t kIdD = tc::idesc_bf16(128, 128, 0, 1);  // -dv^T, N-major Y
      uint64_t* last = nullptr;
      uint32_t last_par = 0;
      for (int it = 0; it < nloc; ++it) {
        const int s = it & 1;
        BtStage& st = sm.st[s];
        if (!(ok = tc::mbar_wait(&sm.full[s], (it >> 1) & 1) && tc::mbar_wait(&sm.dsa_ready, it & 1))) break;
        tc::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::mma_bf16(tb + kColDV, tc::sdesc_sw128(tc::smem_u32(st.DO[0]) + kk * 2048, kTileBytes, 1024),
                       tc::sdesc_sw128(tc::smem_u32(st.Aqk) + kk * 2048, kTileBytes, 1024), kIdA, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc::mma_bf16(tb + kColDV, kdesc(sm.DSA[kk >> 2], (kk & 3) * 32), kdesc(st.KG[kk >> 2], (kk & 3) * 32),
                       kIdB, 1);
        tc::mma_commit(&sm.dv_ready);
        last = &sm.dv_ready;
        last_par = it & 1;
        if (!(ok = tc::mbar_wait(&sm.dva_ready, it & 1))) break;
        tc::tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::mma_bf16(tb + kColS, tc::sdesc_sw128(tc::smem_u32(st.DO[0]) + kk * 2048, kTileBytes, 1024),
                       tc::sdesc_sw128(tc::smem_u32(st.QG[0]) + kk * 2048, kTileBytes, 1024), kIdC, 1);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::mma_bf16(tb + kColS, kdesc(sm.DVA, kk * 32),
                       tc::sdesc_sw128(tc::smem_u32(st.Y[0]) + kk * 2048, kTileBytes, 1024), kIdD, 1);
        tc::mma_commit(&sm.ds_ready);
        tc::mma_commit(&sm.empty[s]);
        last = &sm.ds_ready;
        last_par = it & 1;
      }
      if (last && !tc::mbar_wait(last, last_par)) ok = false;
    }
  } else if (warp == kWarpLoad) {
    // ------------------------------------------------------------ TMA producer
    // lane 0 issues the loads; once a stage has landed the whole warp writes its
    // decay D = 2^G_last and publishes it (dready)
    if (lane == 0) {
      tc::prefetch_tensormap(&tmDO);
      tc::prefetch_tensormap(&tmKG);
      tc::prefetch_tensormap(&tmQG);
      tc::prefetch_tensormap(&tmY);
      tc::prefetch_tensormap(&tmA);
    }
    int it = 0;
    for (; it < nloc; ++it) {
      const int s = it & 1, c = chunk_of(it), L = chunk_len(c);
      BtStage& st = sm.st[s];
      if (it >= 2 && !(ok = warp_wait(&sm.empty[s], ((it >> 1) - 1) & 1))) break;
      if (lane == 0) {
        const int64_t t0 = bos + (int64_t)c * kChunk;
        const int tt = (int)t0, hh = (int)h;
        tc::mbar_arrive_expect_tx(&sm.full[s], kStageTx);
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          tc::tma_load_3d(st.DO[b], &tmDO, &sm.full[s], 64 * b, hh, tt);
          tc::tma_load_3d(st.KG[b], &tmKG, &sm.full[s], 64 * b, hh, tt);
          tc::tma_load_3d(st.QG[b], &tmQG, &sm.full[s], 64 * b, hh, tt);
          tc::tma_load_3d(st.Y[b], &tmY, &sm.full[s], 64 * b, hh, tt);
        }
        tc::tma_load_3d(st.Aqk, &tmA, &sm.full[s], 0, hh, tt);
        tc::bulk_load(st.glast, ws.G + ((t0 + L - 1) * H + h) * kTcK, kTcK * 4, &sm.full[s]);
      }
      __syncwarp();
      if (!(ok = warp_wait(&sm.full[s], (it >> 1) & 1))) break;
#pragma unroll
      for (int j = 0; j < kTcK / 32; ++j) st.D[lane + 32 * j] = exp2_approx(st.glast[lane + 32 * j]);
      tc::mbar_arrive(&sm.dready[s]);
    }
    if (!ok && it < nloc) tc::mbar_wait(&sm.full[it & 1], (it >> 1) & 1);
  } else {
    // ------------------------------------------------------------ output writer
    // dh^T from the dS^T operand tile, dv from its [t][v] tile (without
    // outputs only the releases).  The state warps cannot run more than one
    // phase of dsa_ready / dvt_ready ahead of this warp (they wait for
    // dsa_free / dvt_free before refilling the tiles).
    for (int it = 0; it < nloc; ++it) {
      const int c = chunk_of(it), L = chunk_len(c);
      const int64_t t0 = bos + (int64_t)c * kChunk;
      if (!(ok = warp_wait(&sm.dsa_ready, it & 1))) break;
      if (lane == 0) {
        if (outs) {
          const int row = (int)(((c0 + c) * H + h) * kTcV);
          tc::tma_store_2d(&tmDH, sm.DSA[0], 0, row);
          tc::tma_store_2d(&tmDH, sm.DSA[1], 64, row);
          tc::bulk_commit();
          tc::bulk_wait_read_all();
        }
        tc::mbar_arrive(&sm.dsa_free);
      }
      __syncwarp();
      if (!(ok = warp_wait(&sm.dvt_ready, it & 1))) break;
      if (outs) {
        if (L == kChunk) {
          if (lane == 0) {
            tc::tma_store_3d(&tmDV, sm.DVT[0], 0, (int)h, (int)t0);
            tc::tma_store_3d(&tmDV, sm.DVT[1], 64, (int)h, (int)t0);
            tc::bulk_commit();
            tc::bulk_wait_read_all();
          }
        } else {
          copy_rows_out(sm.DVT, bw.dvn, t0, H, h, L, lane);
        }
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&sm.dvt_free);
    }
    if (lane == 0) tc::bulk_wait_all();
  }

  if (!ok) fault();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tb, 256);
  }
}

// ---------------------------------------------------------------------------
// Folds of the segment maps (fp32, CUDA cores):
//   forward   X[s] <- M_s X[s-1] + X[s],    s = 1 .. nseg-2
//   backward  Z[s] <- M_s^T Z[s+1] + Z[s],  s = nseg-2 .. 1
// The steps are serial, so each is kept short: one CTA per (sequence x head,
// 8-column slice of the state), 256 threads; thread (hf, r) sums half hf of
// the contraction for output row r in 8 independent chains, the halves meet
// in shared memory.  The next step's M (64 KB, rows padded to 132 floats) is
// copied in by cp.async and its addend rows are loaded into registers while
// this step computes.  The forward reads M by rows (float4 along x), the
// backward by columns (consecutive r across the warp).
// ---------------------------------------------------------------------------
constexpr int kFoldThreads = 2 * kTcK, kFoldBV = kTcV / kFoldCtasPerPair, kFoldLd = kTcK + 4;
constexpr int kFoldSmem = (2 * kTcK * kFoldLd + 2 * kTcK * kFoldBV) * 4;

GDN2_DEV void fold_cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(tc::smem_u32(dst)), "l"(src));
}

// nsteps folds (steps 1 .. nsteps) over buffers of nseg segments; without
// kAdd the addend is zero (X[s] <- M_s X[s-1]).  With `out` the last result is
// also written to out[nh] (rows of out_ld floats, from column out_col).
template <bool kBwd, bool kAdd>
__global__ void __launch_bounds__(kFoldThreads)
seg_fold_kernel(const float* __restrict__ M, float* __restrict__ X, int nseg, int nsteps, float* out, int out_ld,
                int out_col) {
  extern __shared__ __align__(16) float fold_smem[];
  float* const Mb0 = fold_smem;
  float* const Mb1 = fold_smem + kTcK * kFoldLd;
  float (*Ss)[kFoldBV] = reinterpret_cast<float (*)[kFoldBV]>(fold_smem + 2 * kTcK * kFoldLd);
  float (*Ps)[kFoldBV] = Ss + kTcK;  // the second half's partial sums
  const int tid = threadIdx.x, r = tid % kTcK, hf = tid / kTcK;
  const int64_t nh = blockIdx.y;
  const int v0 = blockIdx.x * kFoldBV;
  float* Xn = X + nh * nseg * kKV;
  const float* Mn = M + nh * nseg * kKV;
  auto seg_of = [&](int step) { return kBwd ? nseg - 1 - step : step; };
  auto row_of = [&](int step) { return Xn + seg_of(step) * kKV + (int64_t)r * kTcV + v0; };
  auto load_m = [&](int step, float* dst) {
    const float* src = Mn + seg_of(step) * kKV;
    for (int i = tid; i < kTcK * kTcK / 4; i += kFoldThreads) {
      const int row = i / (kTcK / 4), p = (i % (kTcK / 4)) * 4;
      fold_cp16(dst + row * kFoldLd + p, src + row * kTcK + p);
    }
    asm volatile("cp.async.commit_group;\n" ::);
  };
  if (nsteps < 1) return;
  load_m(1, Mb1);
  float4 add0 = make_float4(0.f, 0.f, 0.f, 0.f), add1 = add0;  // the next addend (half 0)
  if (hf == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(row_of(0));
    *reinterpret_cast<float4*>(&Ss[r][0]) = s4[0];
    *reinterpret_cast<float4*>(&Ss[r][4]) = s4[1];
    if (kAdd) {
      const float4* a4 = reinterpret_cast<const float4*>(row_of(1));
      add0 = a4[0];
      add1 = a4[1];
    }
  }
  for (int step = 1; step <= nsteps; ++step) {
    const float* Ms = (step & 1) ? Mb1 : Mb0;
    if (step + 1 <= nsteps) {
      load_m(step + 1, (step & 1) ? Mb0 : Mb1);
      asm volatile("cp.async.wait_group 1;\n" ::);
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::);
    }
    __syncthreads();  // this step's M has landed; the state rows are written
    float acc[kFoldBV];
    acc[0] = add0.x, acc[1] = add0.y, acc[2] = add0.z, acc[3] = add0.w;
    acc[4] = add1.x, acc[5] = add1.y, acc[6] = add1.z, acc[7] = add1.w;
    if (kAdd && hf == 0 && step + 1 <= nsteps) {  // the next step's addend, in flight during this one
      const float4* a4 = reinterpret_cast<const float4*>(row_of(step + 1));
      add0 = a4[0];
      add1 = a4[1];
    }
    const int x0 = hf * (kTcK / 2);
#pragma unroll 4
    for (int x = x0; x < x0 + kTcK / 2; x += 4) {
      float m[4];
      if (kBwd) {
#pragma unroll
        for (int j = 0; j < 4; ++j) m[j] = Ms[(x + j) * kFoldLd + r];
      } else {
        const float4 m4 = *reinterpret_cast<const float4*>(Ms + r * kFoldLd + x);
        m[0] = m4.x, m[1] = m4.y, m[2] = m4.z, m[3] = m4.w;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 s0 = *reinterpret_cast<const float4*>(&Ss[x + j][0]);
        const float4 s1 = *reinterpret_cast<const float4*>(&Ss[x + j][4]);
        acc[0] = fmaf(m[j], s0.x, acc[0]);
        acc[1] = fmaf(m[j], s0.y, acc[1]);
        acc[2] = fmaf(m[j], s0.z, acc[2]);
        acc[3] = fmaf(m[j], s0.w, acc[3]);
        acc[4] = fmaf(m[j], s1.x, acc[4]);
        acc[5] = fmaf(m[j], s1.y, acc[5]);
        acc[6] = fmaf(m[j], s1.z, acc[6]);
        acc[7] = fmaf(m[j], s1.w, acc[7]);
      }
    }
    if (hf == 1) {
      *reinterpret_cast<float4*>(&Ps[r][0]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(&Ps[r][4]) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
    __syncthreads();  // every thread has read the state rows and this step's M; partials are in Ps
    if (hf == 0) {
      const float4 p0 = *reinterpret_cast<const float4*>(&Ps[r][0]);
      const float4 p1 = *reinterpret_cast<const float4*>(&Ps[r][4]);
      const float4 o0 = make_float4(acc[0] + p0.x, acc[1] + p0.y, acc[2] + p0.z, acc[3] + p0.w);
      const float4 o1 = make_float4(acc[4] + p1.x, acc[5] + p1.y, acc[6] + p1.z, acc[7] + p1.w);
      *reinterpret_cast<float4*>(&Ss[r][0]) = o0;
      *reinterpret_cast<float4*>(&Ss[r][4]) = o1;
      float4* xp = reinterpret_cast<float4*>(row_of(step));
      xp[0] = o0;
      xp[1] = o1;
      if (out && step == nsteps) {
        float4* op = reinterpret_cast<float4*>(out + (nh * kTcK + r) * (int64_t)out_ld + out_col + v0);
        op[0] = o0;
        op[1] = o1;
      }
    }
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// [tokens, H, inner] bf16 -> tiles of 64 tokens x 64 inner of one head, swizzled 128 B
bool token_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t H, uint64_t tokens) {
  auto enc = encode_fn();
  if (!enc || !base) return false;
  cuuint64_t dims[3] = {inner, H, tokens};
  cuuint64_t strides[2] = {inner * 2, H * inner * 2};
  cuuint32_t box[3] = {64, 1, 64};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [rows, inner] bf16 -> tiles of 128 rows x 64 inner, swizzled 128 B
bool rows_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows) {
  auto enc = encode_fn();
  if (!enc || !base) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// [tokens, H, inner] of 2- or 4-byte elements -> boxes of 64 tokens x `inner` of
// one head, unswizzled: the shape of an L2 tensor prefetch of one chunk's rows
bool chunk_rows_map(CUtensorMap* m, const void* base, int elem_bytes, uint64_t inner, uint64_t H, uint64_t tokens) {
  auto enc = encode_fn();
  if (!enc || !base || inner > 256 || (elem_bytes != 2 && elem_bytes != 4)) return false;
  const uint64_t eb = (uint64_t)elem_bytes;
  cuuint64_t dims[3] = {inner, H, tokens};
  cuuint64_t strides[2] = {inner * eb, H * inner * eb};
  cuuint32_t box[3] = {(cuuint32_t)inner, 1, 64};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
             const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [rows, inner] bf16 -> unswizzled boxes of 128 rows x inner (one chunk's state of
// 128 value rows), for L2 tensor prefetches; false when rejected
bool state_rows_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows) {
  auto enc = encode_fn();
  if (!enc || !base || inner > 256) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {(cuuint32_t)inner, 128};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool scan_fwd_tc_supported(const gdn2_chunk_args& a) { return a.K == kTcK && a.V == kTcV; }

namespace {

int launch_fold(bool bwd, bool add, const float* M, float* X, int nseg, int nsteps, int64_t NH, cudaStream_t s,
                float* out = nullptr, int out_ld = 0, int out_col = 0) {
  if (nsteps < 1) return 0;
  auto k = bwd ? seg_fold_kernel<true, true> : (add ? seg_fold_kernel<false, true> : seg_fold_kernel<false, false>);
  GDN2_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kFoldSmem));
  ProfScope ps(kKSegFold, s);
  k<<<dim3(kTcV / kFoldBV, (unsigned)NH), kFoldThreads, kFoldSmem, s>>>(M, X, nseg, nsteps, out, out_ld, out_col);
  GDN2_LAUNCH_CHECK();
  return 0;
}

// Forward scan launches of one pass (0, 1, 2) or the CP transition (3).
int fwd_tc_pass(const gdn2_chunk_args& a, const ChunkWs& ws, const SegArgs& sg, float* maps, unsigned grid_y,
                cudaStream_t s) {
  const uint64_t tokens = (uint64_t)a.B * (uint64_t)a.T, H = (uint64_t)a.H;
  const bool trans = sg.pass == 3 || sg.pass == 4;  // the CP transition writes no outputs
  const bool save = (a.flags & GDN2_SAVE_FOR_BWD) && !trans;
  auto kern = save ? chunk_scan_fwd_tc_kernel<true> : chunk_scan_fwd_tc_kernel<false>;
  const int smem = (int)sizeof(TcSmem) + 1024;
  // a runtime call first: it binds this thread's context, which the driver's
  // tensor-map encoder needs (autograd runs the backward on its own threads)
  GDN2_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  CUtensorMap mY, mQG, mKG, mU, mA, mO, mVN, mH;
  if (!token_map(&mY, ws.Y, kTcK, H, tokens) || !token_map(&mQG, ws.qg, kTcK, H, tokens) ||
      !token_map(&mKG, ws.kg, kTcK, H, tokens) || !token_map(&mU, ws.U, kTcV, H, tokens) ||
      !token_map(&mA, ws.Aqk, kChunk, H, tokens))
    return GDN2_ERR_TENSOR_MAP;
  // the transition writes no o: its output maps are never used
  if (trans) mO = mY;
  else if (!token_map(&mO, a.o, kTcV, H, tokens)) return GDN2_ERR_TENSOR_MAP;
  if (save ? !token_map(&mVN, ws.v_new, kTcV, H, tokens) ||
                 !rows_map(&mH, ws.h, kTcK, (uint64_t)a.NT * H * kTcV)
           : false)
    return GDN2_ERR_TENSOR_MAP;
  if (!save) mVN = mH = mO;  // unused without SAVE_FOR_BWD
  ProfScope ps(kKScanFwdTc, s);
  kern<<<dim3((unsigned)(a.N * a.H), grid_y), kTcThreads, smem, s>>>(a, ws, sg, maps, mY, mQG, mKG, mU, mA, mO,
                                                                      mVN, mH);
  GDN2_LAUNCH_CHECK();
  return 0;
}

int bwd_tc_pass(const gdn2_chunk_args& a, const gdn2_chunk_grads& g, const ChunkWs& ws, const BwdWs& bw,
                const SegArgs& sg, unsigned grid_y, cudaStream_t s) {
  const uint64_t tokens = (uint64_t)a.B * (uint64_t)a.T, H = (uint64_t)a.H;
  const int smem = (int)sizeof(BtSmem) + 1024;
  // binds this thread's context before the driver's tensor-map encoder runs
  GDN2_CUDA_TRY(cudaFuncSetAttribute(chunk_scan_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  CUtensorMap mDO, mKG, mQG, mY, mA, mDV, mDH;
  if (!token_map(&mDO, g.dout, kTcV, H, tokens) || !token_map(&mKG, ws.kg, kTcK, H, tokens) ||
      !token_map(&mQG, ws.qg, kTcK, H, tokens) || !token_map(&mY, ws.Y, kTcK, H, tokens) ||
      !token_map(&mA, ws.Aqk, kChunk, H, tokens) || !token_map(&mDV, bw.dvn, kTcV, H, tokens) ||
      !rows_map(&mDH, bw.dh, kTcK, (uint64_t)a.NT * H * kTcV))
    return GDN2_ERR_TENSOR_MAP;
  ProfScope ps(kKScanBwdTc, s);
  chunk_scan_bwd_tc_kernel<<<dim3((unsigned)(a.N * a.H), grid_y), kTcThreads, smem, s>>>(
      a, g, ws, bw, sg, mDO, mKG, mQG, mY, mA, mDV, mDH);
  GDN2_LAUNCH_CHECK();
  return 0;
}

}  // namespace

int scan_fwd_tc_launch(const gdn2_chunk_args& a, const ChunkWs& ws, cudaStream_t s) {
  const SegPlan plan = seg_plan(a);
  if (plan.nseg <= 1) return fwd_tc_pass(a, ws, SegArgs{1, plan.seg_len, 0, nullptr, nullptr}, nullptr, 1, s);
  const int n = plan.nseg;
  int st = fwd_tc_pass(a, ws, SegArgs{n, plan.seg_len, 1, ws.segX, ws.segM}, nullptr, (unsigned)(2 * n - 3), s);
  if (st) return st;
  if ((st = launch_fold(false, true, ws.segM, ws.segX, n, n - 2, a.N * a.H, s))) return st;
  return fwd_tc_pass(a, ws, SegArgs{n, plan.seg_len, 2, ws.segX, ws.segM}, nullptr, (unsigned)(n - 1), s);
}

int scan_bwd_tc_launch(const gdn2_chunk_args& a, const gdn2_chunk_grads& g, const ChunkWs& ws, const BwdWs& bw,
                       cudaStream_t s) {
  const SegPlan plan = seg_plan(a);
  if (plan.nseg <= 1) return bwd_tc_pass(a, g, ws, bw, SegArgs{1, plan.seg_len, 0, nullptr, nullptr}, 1, s);
  const int n = plan.nseg;
  int st = bwd_tc_pass(a, g, ws, bw, SegArgs{n, plan.seg_len, 1, bw.segZ, ws.segM}, (unsigned)(n - 1), s);
  if (st) return st;
  if ((st = launch_fold(true, true, ws.segM, bw.segZ, n, n - 2, a.N * a.H, s))) return st;
  return bwd_tc_pass(a, g, ws, bw, SegArgs{n, plan.seg_len, 2, bw.segZ, ws.segM}, (unsigned)(n - 1), s);
}

int scan_trans_tc_launch(const gdn2_chunk_args& a, const ChunkWs& ws, float* maps, cudaStream_t s) {
  const SegPlan plan = trans_plan(a);
  if (plan.nseg <= 1) return fwd_tc_pass(a, ws, SegArgs{1, plan.seg_len, 3, nullptr, nullptr}, maps, 2, s);
  // every segment's M_s (segment 0's into P[0]) and h_s (segment 0's from the
  // shard's initial state), then h_e = fold of the h_s and M = P[n-1] = M_{n-1} .. M_0
  const int n = plan.nseg;
  SegArgs sg{n, plan.seg_len, 4, ws.segX, ws.segM};
  sg.P = ws.segP;
  int st = fwd_tc_pass(a, ws, sg, maps, (unsigned)(2 * n), s);
  if (st) return st;
  const int ld = kTcK + kTcV;
  if ((st = launch_fold(false, true, ws.segM, ws.segX, n, n - 1, a.N * a.H, s, maps, ld, kTcK))) return st;
  return launch_fold(false, false, ws.segM, ws.segP, n, n - 1, a.N * a.H, s, maps, ld, 0);
}

// Reads (and optionally clears) the fault word of the current device.
int tc_fault_read(int clear, unsigned int* out) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_fault, sizeof(v));
  if (e != cudaSuccess) return -static_cast<int>(e);
  if (clear && v) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_tc_fault, &z, sizeof(z));
    if (e != cudaSuccess) return -static_cast<int>(e);
  }
  *out = v;
  return 0;
}

}  // namespace gdn2
