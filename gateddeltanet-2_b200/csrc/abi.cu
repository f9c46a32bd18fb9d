// extern "C" entry points declared in include/gdn2.h: argument validation,
// workspace carving and dispatch.  Nothing here allocates device memory.
#include "chunk_layout.cuh"
#include "common.cuh"

using namespace gdn2;

namespace {

bool dim_ok(int64_t d) { return d == 64 || d == 128; }

int check_chunk(const gdn2_chunk_args* a, bool need_ptrs = true, bool need_out = true) {
  if (!a) return GDN2_ERR_NULL_POINTER;
  if (a->B < 0 || a->T < 0 || a->H <= 0 || a->N < 0 || a->NT < 0) return GDN2_ERR_SHAPE;
  if (!dim_ok(a->K) || !dim_ok(a->V)) return GDN2_ERR_UNSUPPORTED_DIM;
  if (a->dtype_qkv == GDN2_F32) {
    // the fp32 path takes every input in fp32 and has no separate intra stage
    if (a->dtype_bw != GDN2_F32 || (a->flags & GDN2_G_BF16)) return GDN2_ERR_DTYPE;
    if (a->flags & GDN2_SKIP_INTRA) return GDN2_ERR_FLAGS;
  } else if (a->dtype_qkv != GDN2_BF16) {
    return GDN2_ERR_DTYPE;
  }
  if (a->dtype_bw != GDN2_BF16 && a->dtype_bw != GDN2_F32) return GDN2_ERR_DTYPE;
  if (a->cu_seqlens) {
    if (a->B != 1 || !a->chunk_index || !a->chunk_offset) return GDN2_ERR_SHAPE;
  } else {
    if (a->N != a->B) return GDN2_ERR_SHAPE;
    const int64_t nts = (a->T + 63) / 64;
    if (a->NT != a->B * nts) return GDN2_ERR_SHAPE;
  }
  if ((a->flags & GDN2_LOWER_BOUND) && !(a->flags & GDN2_GATE_IN_KERNEL)) return GDN2_ERR_FLAGS;
  if (!need_ptrs) return GDN2_OK;
  if (a->B * a->T > 0 && (!a->q || !a->k || !a->v || !a->g || !a->b || !a->w || (need_out && !a->o)))
    return GDN2_ERR_NULL_POINTER;
  if ((a->flags & GDN2_GATE_IN_KERNEL) && !a->A_log) return GDN2_ERR_NULL_POINTER;
  if ((a->flags & GDN2_HAS_H0) && !a->h0) return GDN2_ERR_NULL_POINTER;
  if (need_out && (a->flags & GDN2_STORE_FINAL) && !a->ht) return GDN2_ERR_NULL_POINTER;
  // 16-byte alignment of the vectorised streams
  const void* ptrs[] = {a->q, a->k, a->v, a->b, a->w, a->o, a->g};
  for (const void* p : ptrs)
    if (p && (reinterpret_cast<uintptr_t>(p) & 15)) return GDN2_ERR_ALIGNMENT;
  return GDN2_OK;
}

}  // namespace

extern "C" {

int gdn2_abi_version(void) { return 100; }

const char* gdn2_status_string(int s) {
  switch (s) {
    case GDN2_OK: return "ok";
    case GDN2_ERR_NULL_POINTER: return "a required pointer is NULL";
    case GDN2_ERR_SHAPE: return "inconsistent shapes";
    case GDN2_ERR_DTYPE: return "unsupported dtype";
    case GDN2_ERR_UNSUPPORTED_DIM: return "head dims K and V must be 64 or 128";
    case GDN2_ERR_ALIGNMENT: return "tensor base pointers must be 16-byte aligned";
    case GDN2_ERR_WORKSPACE: return "workspace missing or too small";
    case GDN2_ERR_FLAGS: return "inconsistent flags";
    case GDN2_ERR_NO_DEVICE: return "no sm_100 device";
    case GDN2_ERR_SCRATCH_LIMIT:
      return "problem needs more than the 32 MiB built-in scratch; use gdn2_chunk_fwd with a caller workspace";
    case GDN2_ERR_TENSOR_MAP: return "cuTensorMapEncodeTiled unavailable or rejected a workspace array";
    default: break;
  }
  if (s < 0) return cudaGetErrorString(static_cast<cudaError_t>(-s));
  return "unknown status";
}

int gdn2_device_fault_read(int clear, unsigned int* out) {
  if (!out) return GDN2_ERR_NULL_POINTER;
  unsigned int a = 0, b = 0, c = 0, d = 0;
  int st = gdn2::tc_fault_read(clear, &a);
  if (st == 0) st = gdn2::b3_fault_read(clear, &c);
  if (st == 0) st = gdn2::f1_fault_read(clear, &d);
  if (st == 0) st = gdn2::layer_fault_read(clear, &b);
  *out = a | b | c | d;
  return st;
}

int gdn2_device_supported(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) return 0;
  return (major == 10 && minor == 0) ? 1 : 0;
}

size_t gdn2_chunk_workspace_size(const gdn2_chunk_args* a) {
  if (check_chunk(a, false) != GDN2_OK) return 0;
  return chunk_ws_layout(*a, nullptr, nullptr);
}

size_t gdn2_chunk_workspace_offset(const gdn2_chunk_args* a, int which) {
  if (check_chunk(a, false) != GDN2_OK) return ~size_t(0);
  // carve a fake base: offsets are the pointers' distance from it
  char* const base = reinterpret_cast<char*>(size_t(1) << 40);
  ChunkWs ws;
  chunk_ws_layout(*a, base, &ws);
  switch (which) {
    case GDN2_WS_CHUNK_STATES:
      if (a->dtype_qkv == GDN2_F32)
        return ws.ckpt ? (size_t)(reinterpret_cast<char*>(ws.ckpt) - base) : ~size_t(0);
      return ws.h ? (size_t)(reinterpret_cast<char*>(ws.h) - base) : ~size_t(0);
    default: return ~size_t(0);
  }
}

size_t gdn2_chunk_bwd_workspace_size(const gdn2_chunk_args* a) {
  if (check_chunk(a, false) != GDN2_OK) return 0;
  return bwd_ws_layout(*a, nullptr, nullptr);
}

int gdn2_chunk_fwd(const gdn2_chunk_args* a, void* workspace, size_t workspace_bytes, gdn2_stream_t stream) {
  int st = check_chunk(a);
  if (st) return st;
  const size_t need = chunk_ws_layout(*a, nullptr, nullptr);
  if (need > workspace_bytes || (need > 0 && !workspace)) return GDN2_ERR_WORKSPACE;
  if (a->N == 0 || a->B * a->T == 0) return GDN2_OK;
  ChunkWs ws;
  chunk_ws_layout(*a, workspace, &ws);
  if (a->dtype_qkv == GDN2_F32) return chunk_fwd_fp32_launch(*a, ws, reinterpret_cast<cudaStream_t>(stream));
  return chunk_fwd_launch(*a, ws, reinterpret_cast<cudaStream_t>(stream));
}

int gdn2_chunk_bwd(const gdn2_chunk_args* a, const gdn2_chunk_grads* gr, const void* workspace,
                   size_t workspace_bytes, void* bwd_workspace, size_t bwd_workspace_bytes,
                   gdn2_stream_t stream) {
  int st = check_chunk(a, true, false);  // the backward reads no o / ht
  if (st) return st;
  if (!(a->flags & GDN2_SAVE_FOR_BWD)) return GDN2_ERR_FLAGS;
  const bool state_only = a->flags & GDN2_BWD_STATE_ONLY;
  if (!gr || !gr->dout) return GDN2_ERR_NULL_POINTER;
  if (state_only ? !gr->dh0 : (!gr->dq || !gr->dk || !gr->dv || !gr->dg || !gr->db || !gr->dw))
    return GDN2_ERR_NULL_POINTER;
  if ((a->flags & GDN2_HAS_H0) && !gr->dh0) return GDN2_ERR_NULL_POINTER;
  if (!state_only && (a->flags & GDN2_GATE_IN_KERNEL) && !gr->dA_log) return GDN2_ERR_NULL_POINTER;
  if (!state_only && (a->flags & GDN2_GATE_IN_KERNEL) && a->dt_bias && !gr->ddt_bias)
    return GDN2_ERR_NULL_POINTER;
  const size_t need = chunk_ws_layout(*a, nullptr, nullptr);
  if (need > workspace_bytes || (need > 0 && !workspace)) return GDN2_ERR_WORKSPACE;
  const size_t need_b = bwd_ws_layout(*a, nullptr, nullptr);
  if (need_b > bwd_workspace_bytes || (need_b > 0 && !bwd_workspace)) return GDN2_ERR_WORKSPACE;
  ChunkWs ws;
  chunk_ws_layout(*a, const_cast<void*>(workspace), &ws);
  BwdWs bw;
  bwd_ws_layout(*a, bwd_workspace, &bw);
  if (a->dtype_qkv == GDN2_F32) return chunk_bwd_fp32_launch(*a, *gr, ws, bw, reinterpret_cast<cudaStream_t>(stream));
  return chunk_bwd_launch(*a, *gr, ws, bw, reinterpret_cast<cudaStream_t>(stream));
}

int gdn2_recurrent_fwd(const gdn2_recurrent_args* a, gdn2_stream_t stream) {
  if (!a) return GDN2_ERR_NULL_POINTER;
  if (a->B < 0 || a->T < 0 || a->H <= 0 || a->HV <= 0 || a->N < 0) return GDN2_ERR_SHAPE;
  if (a->HV % a->H) return GDN2_ERR_SHAPE;
  if (!dim_ok(a->K) || !dim_ok(a->V)) return GDN2_ERR_UNSUPPORTED_DIM;
  if ((a->dtype_qkv != GDN2_BF16 && a->dtype_qkv != GDN2_F32) ||
      (a->dtype_gbw != GDN2_BF16 && a->dtype_gbw != GDN2_F32))
    return GDN2_ERR_DTYPE;
  if (a->cu_seqlens && a->B != 1) return GDN2_ERR_SHAPE;
  if (!a->cu_seqlens && a->N != a->B) return GDN2_ERR_SHAPE;
  if (a->B * a->T > 0 && (!a->q || !a->k || !a->v || !a->g || !a->b || !a->w || !a->o))
    return GDN2_ERR_NULL_POINTER;
  if ((a->flags & GDN2_GATE_IN_KERNEL) && !a->A_log) return GDN2_ERR_NULL_POINTER;
  if ((a->flags & GDN2_HAS_H0) && !a->h0) return GDN2_ERR_NULL_POINTER;
  if ((a->flags & GDN2_STORE_FINAL) && !a->ht) return GDN2_ERR_NULL_POINTER;
  if (a->ssm_state_indices && !(a->flags & GDN2_STORE_FINAL)) return GDN2_ERR_FLAGS;
  if (a->num_accepted_tokens && !a->ssm_state_indices) return GDN2_ERR_FLAGS;
  const float* sp[] = {a->h0, a->ht};
  for (const float* p : sp)
    if (p && (reinterpret_cast<uintptr_t>(p) & 15)) return GDN2_ERR_ALIGNMENT;
  if (a->N == 0 || a->B * a->T == 0) return GDN2_OK;
  return recurrent_fwd(*a, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
