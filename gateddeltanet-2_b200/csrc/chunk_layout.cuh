// Layout of the chunk workspace: the forward's scratch (WY factors the scan
// consumes) plus what the backward reads back.  Host and device share it.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace gdn2 {

struct ChunkWs {
  // token-major [tokens, H, *] like the inputs
  __nv_bfloat16* qn;   // normalised q (l2norm) — aliases q otherwise
  __nv_bfloat16* kn;
  float* q_rstd;       // [tokens, H]
  float* k_rstd;
  float* G;            // chunk-local cumsum of the (activated) gate, log2 units
  __nv_bfloat16* Aqk;  // [tokens, H, 64]
  __nv_bfloat16* Akk;  // (I+T)^-1, [tokens, H, 64]
  __nv_bfloat16* Y;    // A (b k 2^G)           [tokens, H, K]
  __nv_bfloat16* U;    // A (w v)               [tokens, H, V]
  __nv_bfloat16* kg;   // k 2^(G_last - G)      [tokens, H, K]
  __nv_bfloat16* qg;   // scale q 2^G           [tokens, H, K]
  __nv_bfloat16* v_new;// [tokens, H, V]
  __nv_bfloat16* h;    // per-chunk entering state, transposed: [NT, H, V, K]
  float* segX;         // segmented scan: segment states [N*H, nseg, K, V] fp32 (or nullptr)
  float* segM;         // segmented scan: segment transitions [N*H, nseg, K, K] fp32 (kept for the backward)
  float* segP;         // segmented CP transition: products of the segment transitions [N*H, nseg, K, K]
  // fp32 inputs (dtype_qkv == GDN2_F32) run the token-serial fp32 path instead:
  float* qf;           // l2-normalised q, fp32 [tokens, H, K] (with l2norm; else aliases q)
  float* kf;
  float* gf;           // activated log-decay, fp32 [tokens, H, K] (with the gate in the kernel; else aliases g)
  float* ckpt;         // state entering each chunk, fp32 [NT, H, K, V] (saved for the backward)
};

struct BwdWs {
  __nv_bfloat16* dh;   // state cotangent at the end of each chunk, transposed [NT, H, V, K]
  __nv_bfloat16* dvn;  // cotangent of v_new [tokens, H, V]
  float* segZ;         // segmented reverse scan: segment state cotangents [N*H, nseg, K, V] fp32
  // fp32 path:
  float* tok_states;   // the states entering each token of one chunk, fp32 [N*H, 64, K, V]
  float* dqf;          // cotangents of the normalised q, k and the activated gate, fp32 [tokens, H, K]
  float* dkf;          //   (with l2norm / the gate; else the outputs are written directly)
  float* dgf;
};

inline size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

// How the tcgen05 scans cut each sequence into segments (scan_tc.cu).  With
// one CTA per (sequence, head) a scan walks every chunk of its sequence in
// series, so with few pairs per GPU most SMs idle.  Cutting a sequence into
// nseg segments runs the scans in three launches (segment transitions, an
// fp32 fold, the segments from their entering states): more CTAs in flight,
// about twice the scan work.  The plan minimises a cost in microseconds
// measured on B200 (one resident scan CTA per SM, 148 SMs): a chunk step of
// a scan CTA ~3.3 us, a scan launch ~8 us of fixed cost, a serial fold step
// ~2 us per wave of fold CTAs (16 per pair) plus ~5 us per fold launch.
// Dense batches of d_k = d_v = 128 with at least 32 chunks per sequence only;
// the result depends on the arguments alone, so the forward, the backward
// and the workspace queries agree.
struct SegPlan {
  int nseg;     // segments per sequence (1: no segmentation)
  int seg_len;  // chunks per segment
};
constexpr int kPlanSms = 148;
constexpr int kSegMinChunks = 32;
constexpr int kFoldCtasPerPair = 16;

inline SegPlan seg_plan(const gdn2_chunk_args& a) {
  const int64_t nts = (a.T + 63) / 64;
  SegPlan p{1, (int)nts};
  if (a.K != 128 || a.V != 128 || a.cu_seqlens || a.N <= 0 || nts < kSegMinChunks) return p;
  const int64_t NH = a.N * a.H;
  auto waves = [](int64_t ctas) { return (double)((ctas + kPlanSms - 1) / kPlanSms); };
  constexpr double kStep = 3.3, kPass = 8.0, kFoldStep = 2.0, kFoldLaunch = 5.0;
  const double base = waves(NH) * (double)nts * kStep + kPass;
  double best = base;
  SegPlan cand = p;
  for (int64_t n = 3; n <= 64; ++n) {
    const int64_t L = (nts + n - 1) / n;
    const int64_t nn = (nts + L - 1) / L;  // segments actually formed
    if (nn < 3 || L < 2) continue;
    const double cost = (waves(NH * (2 * nn - 3)) + waves(NH * (nn - 1))) * (double)L * kStep + 2 * kPass +
                        waves(NH * kFoldCtasPerPair) * (double)(nn - 2) * kFoldStep + kFoldLaunch;
    if (cost < best) {
      best = cost;
      cand = SegPlan{(int)nn, (int)L};
    }
  }
  return best < 0.85 * base ? cand : p;
}

// The context-parallel transition of a shard ([M | h_e], gdn2_cp_transition)
// in segments: one pass computes every segment's M_s and h_s (two CTAs per
// segment), two folds compose them (no second pass).  Same cost model.
inline SegPlan trans_plan(const gdn2_chunk_args& a) {
  const int64_t nts = (a.T + 63) / 64;
  SegPlan p{1, (int)nts};
  if (a.K != 128 || a.V != 128 || a.cu_seqlens || a.N <= 0 || nts < kSegMinChunks) return p;
  const int64_t NH = a.N * a.H;
  auto waves = [](int64_t ctas) { return (double)((ctas + kPlanSms - 1) / kPlanSms); };
  constexpr double kStep = 3.3, kPass = 8.0, kFoldStep = 2.0, kFoldLaunch = 5.0;
  const double base = waves(2 * NH) * (double)nts * kStep + kPass;
  double best = base;
  SegPlan cand = p;
  for (int64_t n = 2; n <= 64; ++n) {
    const int64_t L = (nts + n - 1) / n;
    const int64_t nn = (nts + L - 1) / L;
    if (nn < 2 || L < 2) continue;
    const double cost = waves(2 * NH * nn) * (double)L * kStep + kPass +
                        2 * (waves(NH * kFoldCtasPerPair) * (double)(nn - 1) * kFoldStep + kFoldLaunch);
    if (cost < best) {
      best = cost;
      cand = SegPlan{(int)nn, (int)L};
    }
  }
  return best < 0.85 * base ? cand : p;
}

// Carves `base` (or computes the size when base == nullptr).
inline size_t chunk_ws_layout(const gdn2_chunk_args& a, void* base, ChunkWs* ws) {
  const size_t tok = (size_t)a.B * (size_t)a.T;
  const size_t H = (size_t)a.H, K = (size_t)a.K, V = (size_t)a.V;
  const bool save = a.flags & GDN2_SAVE_FOR_BWD;
  const bool l2 = a.flags & GDN2_L2NORM_QK;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align_up(off + bytes);
    return base ? (void*)((char*)base + o) : nullptr;
  };
  ChunkWs w{};
  if (a.dtype_qkv == GDN2_F32) {
    const bool gate = a.flags & GDN2_GATE_IN_KERNEL;
    w.qf = l2 ? (float*)take(tok * H * K * 4) : (float*)a.q;
    w.kf = l2 ? (float*)take(tok * H * K * 4) : (float*)a.k;
    if (l2) {
      w.q_rstd = (float*)take(tok * H * 4);
      w.k_rstd = (float*)take(tok * H * 4);
    }
    w.gf = gate ? (float*)take(tok * H * K * 4) : (float*)a.g;
    if (save) w.ckpt = (float*)take((size_t)a.NT * H * K * V * 4);
    if (ws) *ws = w;
    return off;
  }
  w.G = (float*)take(tok * H * K * 4);
  w.Aqk = (__nv_bfloat16*)take(tok * H * 64 * 2);
  w.Akk = (__nv_bfloat16*)take(tok * H * 64 * 2);
  w.Y = (__nv_bfloat16*)take(tok * H * K * 2);
  w.U = (__nv_bfloat16*)take(tok * H * V * 2);
  w.kg = (__nv_bfloat16*)take(tok * H * K * 2);
  w.qg = (__nv_bfloat16*)take(tok * H * K * 2);
  if (save) {
    w.v_new = (__nv_bfloat16*)take(tok * H * V * 2);
    w.h = (__nv_bfloat16*)take((size_t)a.NT * H * K * V * 2);
    if (l2) {
      w.qn = (__nv_bfloat16*)take(tok * H * K * 2);
      w.kn = (__nv_bfloat16*)take(tok * H * K * 2);
      w.q_rstd = (float*)take(tok * H * 4);
      w.k_rstd = (float*)take(tok * H * 4);
    }
  }
  if (!l2) {
    w.qn = (__nv_bfloat16*)a.q;
    w.kn = (__nv_bfloat16*)a.k;
  }
  const SegPlan plan = seg_plan(a), tplan = trans_plan(a);
  const int nbuf = plan.nseg > tplan.nseg ? plan.nseg : tplan.nseg;
  if (nbuf > 1) {
    const size_t nsl = (size_t)a.N * H * (size_t)nbuf;
    w.segX = (float*)take(nsl * K * V * 4);
    w.segM = (float*)take(nsl * K * K * 4);
    if (tplan.nseg > 1) w.segP = (float*)take(nsl * K * K * 4);
  }
  if (ws) *ws = w;
  return off;
}

inline size_t bwd_ws_layout(const gdn2_chunk_args& a, void* base, BwdWs* ws) {
  const size_t tok = (size_t)a.B * (size_t)a.T;
  const size_t H = (size_t)a.H, K = (size_t)a.K, V = (size_t)a.V;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align_up(off + bytes);
    return base ? (void*)((char*)base + o) : nullptr;
  };
  BwdWs w{};
  if (a.dtype_qkv == GDN2_F32) {
    w.tok_states = (float*)take((size_t)a.N * H * 64 * K * V * 4);
    if (a.flags & GDN2_L2NORM_QK) {
      w.dqf = (float*)take(tok * H * K * 4);
      w.dkf = (float*)take(tok * H * K * 4);
    }
    if (a.flags & GDN2_GATE_IN_KERNEL) w.dgf = (float*)take(tok * H * K * 4);
    if (ws) *ws = w;
    return off;
  }
  w.dh = (__nv_bfloat16*)take((size_t)a.NT * H * K * V * 2);
  w.dvn = (__nv_bfloat16*)take(tok * H * V * 2);
  const SegPlan plan = seg_plan(a);
  if (plan.nseg > 1) w.segZ = (float*)take((size_t)a.N * H * (size_t)plan.nseg * K * V * 4);
  if (ws) *ws = w;
  return off;
}

// first row of anchor i's section in the KN operand: 0, 16, 48, 96
GDN2_DEV constexpr int anchor_row0(int i) { return 8 * i * (i + 1); }

int chunk_fwd_launch(const gdn2_chunk_args& a, const ChunkWs& ws, cudaStream_t s);
// fp32 inputs: token-serial fp32 forward / backward (chunk_fp32.cu)
int chunk_fwd_fp32_launch(const gdn2_chunk_args& a, const ChunkWs& ws, cudaStream_t s);
int chunk_bwd_fp32_launch(const gdn2_chunk_args& a, const gdn2_chunk_grads& g, const ChunkWs& ws, const BwdWs& bw,
                          cudaStream_t s);
int chunk_transition_launch(const gdn2_chunk_args& a, const ChunkWs& ws, float* maps, cudaStream_t s);
int chunk_bwd_launch(const gdn2_chunk_args& a, const gdn2_chunk_grads& g, const ChunkWs& ws, const BwdWs& bw,
                     cudaStream_t s);
// Checkpoints of the token-serial kernel for the chunked fp32 path: the fp32
// state entering every 64-token chunk, [NT, H, K, V] (global chunk index from
// chunk_offset for varlen, n * chunks_per_seq + c for dense batches).
struct RecCheckpoints {
  float* states = nullptr;
  const int32_t* chunk_offset = nullptr;
  int64_t chunks_per_seq = 0;
};
int recurrent_fwd(const gdn2_recurrent_args& a, cudaStream_t s, const RecCheckpoints& ck = RecCheckpoints{});

// tcgen05 forward scan (scan_tc.cu), d_k = d_v = 128
bool scan_fwd_tc_supported(const gdn2_chunk_args& a);
int scan_fwd_tc_launch(const gdn2_chunk_args& a, const ChunkWs& ws, cudaStream_t s);
int scan_bwd_tc_launch(const gdn2_chunk_args& a, const gdn2_chunk_grads& g, const ChunkWs& ws, const BwdWs& bw,
                       cudaStream_t s);
// context-parallel transition [M | h_e] of a dense shard on the tcgen05 scan (d_k = d_v = 128)
int scan_trans_tc_launch(const gdn2_chunk_args& a, const ChunkWs& ws, float* maps, cudaStream_t s);
int tc_fault_read(int clear, unsigned int* out);
// [tokens, H, inner] (2- or 4-byte elements) -> unswizzled boxes of 64 tokens x inner of
// one head, for L2 tensor prefetches of a chunk's rows (scan_tc.cu); false when rejected
bool chunk_rows_map(CUtensorMap* m, const void* base, int elem_bytes, uint64_t inner, uint64_t H, uint64_t tokens);
// [rows, inner] bf16 -> unswizzled boxes of 128 rows x inner (L2 prefetches of a chunk's state)
bool state_rows_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows);
// fault word of the backward intra kernel (chunk_bwd.cu): bit 0 = a tcgen05 wait gave up
int b3_fault_read(int clear, unsigned int* out);
// fault word of the forward intra kernel (chunk_fwd.cu): bit 0 = its wait on the w, v copies gave up
int f1_fault_read(int clear, unsigned int* out);
// fault word of the layer kernels (layer.cu): bit 1 = a staging wait gave up
int layer_fault_read(int clear, unsigned int* out);

}  // namespace gdn2
