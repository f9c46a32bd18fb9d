/*
 * gdn2.h — C ABI of the B200 (sm_100a) Gated Delta Rule-2 operator.
 *
 * The operator keeps a per-(sequence, head) matrix state S in R^{K x V} (fp32)
 * and, per token, applies
 *
 *     S <- Diag(exp(g_t)) S
 *     u  = w_t * v_t - S^T (b_t * k_t)
 *     S <- S + k_t u^T
 *     o_t = S^T (scale * q_t)
 *
 * Three entry points carry the hot path:
 *   gdn2_chunk_fwd      chunkwise (C = 64) forward used for training/prefill;
 *   gdn2_chunk_bwd      its backward (dq, dk, dv, dg, db, dw, dh0, dA_log, ddt_bias);
 *   gdn2_recurrent_fwd  the token-serial decode step.
 * A context-parallel long-sequence mode adds
 *   gdn2_cp_transition  a shard's boundary affine map (M, h_e);
 *   gdn2_cp_compose     the exclusive prefix of those maps over ranks.
 *
 * Conventions shared by every entry point
 *   - Pointers are device pointers unless stated otherwise.  Tensors are dense
 *     and row-major in the reference's layouts: q, k, g, b are [B, T, H, K];
 *     v, w, o are [B, T, H, V]; states are [N, H, K, V] (or [N, H, V, K] with
 *     GDN2_TRANSPOSE_STATE).  With cu_seqlens (packed varlen) B must be 1 and
 *     the N sequences are the spans [cu[i], cu[i+1]) of the T axis.
 *   - The caller allocates every buffer, including the workspaces whose sizes
 *     the *_workspace_size queries return.  No entry point allocates memory.
 *   - Work is enqueued on `stream`; nothing synchronises the host.
 *   - Return value: 0 on success, > 0 for an invalid argument (nothing was
 *     launched), < 0 for a CUDA error (-(cudaError_t)).  gdn2_status_string()
 *     names the code.
 */
#ifndef GDN2_B200_H_
#define GDN2_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* gdn2_stream_t; /* == cudaStream_t */

/* element types */
enum gdn2_dtype { GDN2_BF16 = 0, GDN2_F32 = 1 };

/* option flags */
enum gdn2_flags {
  GDN2_L2NORM_QK = 1 << 0,       /* use_qk_l2norm_in_kernel (eps 1e-6 inside the sqrt) */
  GDN2_GATE_IN_KERNEL = 1 << 1,  /* g is raw: g <- -exp(A_log) * softplus(g + dt_bias) */
  GDN2_LOWER_BOUND = 1 << 2,     /* with GATE_IN_KERNEL: g <- lower_bound * sigmoid(exp(A_log)*(g+dt_bias)) */
  GDN2_TRANSPOSE_STATE = 1 << 3, /* states stored [.., V, K] */
  GDN2_HAS_H0 = 1 << 4,          /* initial_state given */
  GDN2_STORE_FINAL = 1 << 5,     /* write the final state to `ht` */
  GDN2_SAVE_FOR_BWD = 1 << 6,    /* chunk fwd: keep what gdn2_chunk_bwd needs in the workspace */
  GDN2_BWD_STATE_ONLY = 1 << 7,  /* chunk bwd: only the state-cotangent scan (no reference counterpart):
                                    writes dh0 = d(loss)/d(initial state) for the given do and dht;
                                    dq, dk, dv, dg, db, dw may be NULL */
  GDN2_G_BF16 = 1 << 8,          /* chunk fwd/bwd: g (and dg) are bf16 instead of fp32 (the layer's
                                    gate pre-activation comes out of a bf16 GEMM) */
  GDN2_SKIP_INTRA = 1 << 9       /* chunk fwd (no reference counterpart): the workspace already holds
                                    the intra-chunk factors of these same inputs and flags, written
                                    by gdn2_cp_transition or an earlier gdn2_chunk_fwd; only the
                                    state scan runs (a context-parallel shard's forward from its
                                    composed entering state reuses its transition's factors) */
};

/* status codes (> 0: invalid argument) */
enum gdn2_status {
  GDN2_OK = 0,
  GDN2_ERR_NULL_POINTER = 1,
  GDN2_ERR_SHAPE = 2,
  GDN2_ERR_DTYPE = 3,
  GDN2_ERR_UNSUPPORTED_DIM = 4, /* K or V not in {64, 128} */
  GDN2_ERR_ALIGNMENT = 5,
  GDN2_ERR_WORKSPACE = 6,       /* workspace pointer NULL or too small */
  GDN2_ERR_FLAGS = 7,
  GDN2_ERR_NO_DEVICE = 8,
  GDN2_ERR_SCRATCH_LIMIT = 9,   /* problem larger than gdn2_chunk_fwd_static_scratch's 32 MiB */
  GDN2_ERR_TENSOR_MAP = 10      /* the driver could not describe a workspace array for TMA */
};

/* ------------------------------------------------------------------------- */
/* chunkwise forward / backward                                              */
/* ------------------------------------------------------------------------- */
/*
 * Replaces the reference's chunk_gdn2 / ChunkGDN2Function
 * (lit_gpt/gdn2_ops/chunk_gdn2.py:1363-1511 public API, :2504-2665 autograd)
 * and the pipeline behind it: chunk_gdn2_fwd (:1205-1359), chunk_gdn2_bwd
 * (:2330-2493), l2norm_fwd/bwd (:2542-2544, :2638-2640), the gate activation
 * kda_gate_chunk_cumsum (chunk_kda.py:2636-2733) and kda_gate_bwd (:2420-2555).
 */
typedef struct gdn2_chunk_args {
  int64_t B, T, H, K, V; /* q,k,g,b [B,T,H,K]; v,w,o [B,T,H,V] */
  int64_t N;             /* number of sequences: B, or len(cu_seqlens)-1 */
  int64_t NT;            /* total number of 64-token chunks over all sequences */
  const int64_t* cu_seqlens;   /* [N+1] device, or NULL for dense [B,T] */
  const int32_t* chunk_index;  /* [NT, 2] device (sequence, chunk-in-sequence) for varlen, else NULL */
  const int32_t* chunk_offset; /* [N+1] device: first global chunk of each sequence (varlen), else NULL */
  float scale;           /* attention scale (reference default K^-0.5) */
  float lower_bound;     /* used with GDN2_LOWER_BOUND */
  int32_t flags;         /* enum gdn2_flags */
  int32_t dtype_qkv;     /* q, k, v, do and o (and dq, dk, dv): GDN2_BF16, or GDN2_F32 for the
                            fp32 path (every input fp32: dtype_bw GDN2_F32, no GDN2_G_BF16),
                            which computes the recurrence token by token in fp32 */
  int32_t dtype_bw;      /* b, w (and db, dw): GDN2_BF16 or GDN2_F32 */
  const void* q;
  const void* k;
  const void* v;
  const void* g;         /* log-decay (natural log), or the raw pre-activation: fp32, or bf16 with GDN2_G_BF16 */
  const void* b;
  const void* w;
  const float* A_log;    /* [H]     with GDN2_GATE_IN_KERNEL */
  const float* dt_bias;  /* [H*K]   optional with GDN2_GATE_IN_KERNEL */
  const float* h0;       /* [N,H,K,V] fp32 with GDN2_HAS_H0 */
  float* ht;             /* [N,H,K,V] fp32 with GDN2_STORE_FINAL */
  void* o;               /* [B,T,H,V] dtype_qkv */
} gdn2_chunk_args;

typedef struct gdn2_chunk_grads {
  const void* dout;      /* [B,T,H,V] dtype_qkv: cotangent of o */
  const float* dht;      /* [N,H,K,V] fp32 cotangent of the final state, or NULL */
  void* dq;              /* [B,T,H,K] dtype_qkv */
  void* dk;              /* [B,T,H,K] dtype_qkv */
  void* dv;              /* [B,T,H,V] dtype_qkv */
  void* dg;              /* [B,T,H,K] g's dtype (w.r.t. g as passed: raw when gated in kernel) */
  void* db;              /* [B,T,H,K] dtype_bw */
  void* dw;              /* [B,T,H,V] dtype_bw */
  float* dh0;            /* [N,H,K,V] fp32 when GDN2_HAS_H0, else may be NULL */
  float* dA_log;         /* [H] fp32 with GDN2_GATE_IN_KERNEL */
  float* ddt_bias;       /* [H*K] fp32 with GDN2_GATE_IN_KERNEL and dt_bias */
} gdn2_chunk_grads;

/* Bytes of the forward->backward context: everything gdn2_chunk_fwd saves with
 * GDN2_SAVE_FOR_BWD (normalised q/k, cumulative gates, WY factors, chunk
 * states).  Without GDN2_SAVE_FOR_BWD only the forward's own scratch. */
size_t gdn2_chunk_workspace_size(const gdn2_chunk_args* a);
/* Bytes of additional scratch gdn2_chunk_bwd needs (state cotangents, dv). */
size_t gdn2_chunk_bwd_workspace_size(const gdn2_chunk_args* a);

/* Buffers of the forward workspace a caller may read after gdn2_chunk_fwd. */
enum gdn2_ws_buffer {
  GDN2_WS_CHUNK_STATES = 0 /* per-chunk entering states h, present with GDN2_SAVE_FOR_BWD:
                              bf16 transposed [NT, H, V, K] (bf16 inputs), or fp32 [NT, H, K, V]
                              (GDN2_F32 inputs) */
};
/* Byte offset of buffer `which` inside the workspace gdn2_chunk_fwd fills for
 * these arguments, or (size_t)-1 when these arguments keep no such buffer
 * (no counterpart in the reference, whose Python op returns h as a tensor
 * with return_intermediate_states, chunk_gdn2.py:1495-1511). */
size_t gdn2_chunk_workspace_offset(const gdn2_chunk_args* a, int which);

int gdn2_chunk_fwd(const gdn2_chunk_args* a, void* workspace, size_t workspace_bytes,
                   gdn2_stream_t stream);
/* `workspace` must hold what gdn2_chunk_fwd wrote with GDN2_SAVE_FOR_BWD for
 * the same arguments. */
int gdn2_chunk_bwd(const gdn2_chunk_args* a, const gdn2_chunk_grads* gr,
                   const void* workspace, size_t workspace_bytes,
                   void* bwd_workspace, size_t bwd_workspace_bytes, gdn2_stream_t stream);

/*
 * Forward without any caller workspace, for callers that cannot allocate
 * device memory (a serving engine that reserved the device up front and
 * forbids later allocations, a plugin inside a framework that owns the
 * allocator, a latency-critical loop that cannot afford an allocation's
 * implicit synchronisation).  No counterpart in the reference: it has no C
 * entry points, and its Python ops allocate through torch.
 *
 * Same arguments and results as gdn2_chunk_fwd without GDN2_SAVE_FOR_BWD
 * (that flag is rejected: a backward needs a context that outlives the call)
 * and without GDN2_SKIP_INTRA (also rejected: the shared array may hold
 * another problem's factors).
 * The scratch is one 32 MiB device array inside the library, present on every
 * GPU that loads it until the process exits; problems whose
 * gdn2_chunk_workspace_size exceeds 32 MiB return GDN2_ERR_SCRATCH_LIMIT (about
 * 1.8 KB per token-head at K = V = 128: e.g. 16 heads x 1150 tokens fit).
 * All calls share the array: calls whose kernels overlap on the GPU race, so
 * serialise them.  Nothing in it needs clearing between calls.  The first call
 * on each device resolves the array's device address (cudaGetSymbolAddress,
 * with that device current); make that first call before any stream capture.
 * The address is cached per device ordinal, i.e. for the device's primary
 * context: after cudaDeviceReset, or with another driver context current,
 * restart the process before calling again.
 * Nothing is allocated, by this call or by anything it calls.
 */
int gdn2_chunk_fwd_static_scratch(const gdn2_chunk_args* a, gdn2_stream_t stream);

/* ------------------------------------------------------------------------- */
/* token-serial recurrence (decode)                                          */
/* ------------------------------------------------------------------------- */
/*
 * Replaces fused_recurrent_gdn2 / fused_recurrent_gdn2_fwd and its kernel
 * (lit_gpt/gdn2_ops/fused_recurrent_gdn2.py:81-277 kernel, :284-395 launcher,
 * :399-492 public API), including the serving features of the kernel:
 * varlen (cu_seqlens), a paged state pool (ssm_state_indices), speculative
 * decoding (num_accepted_tokens) and grouped value heads (HV a multiple of H).
 */
typedef struct gdn2_recurrent_args {
  int64_t B, T, H, HV, K, V; /* q,k [B,T,H,K]; v,w,o [B,T,HV,V]; g,b [B,T,HV,K] */
  int64_t N;                 /* sequences */
  const int64_t* cu_seqlens; /* [N+1] or NULL */
  const int32_t* ssm_state_indices; /* [N] or [N, stride_indices_seq] pool slots, or NULL */
  const int32_t* num_accepted_tokens; /* [N] with ssm_state_indices (spec decoding), or NULL */
  int64_t stride_indices_seq;  /* row stride of ssm_state_indices */
  int64_t state_slot_stride_in;  /* elements between pool slots of h0 (default HV*K*V) */
  int64_t state_slot_stride_out; /* elements between slots of ht (default HV*K*V) */
  float scale;
  float lower_bound;
  int32_t flags;      /* GDN2_L2NORM_QK | GDN2_GATE_IN_KERNEL | GDN2_LOWER_BOUND |
                         GDN2_TRANSPOSE_STATE | GDN2_HAS_H0 | GDN2_STORE_FINAL */
  int32_t inplace;    /* with ssm_state_indices: write each token's state to its pool slot */
  int32_t dtype_qkv;  /* q, k, v, o */
  int32_t dtype_gbw;  /* g, b, w */
  const void* q;
  const void* k;
  const void* v;
  const void* g;
  const void* b;
  const void* w;
  const float* A_log;
  const float* dt_bias;
  const float* h0;    /* may alias ht (in-place update) */
  float* ht;
  void* o;
} gdn2_recurrent_args;

int gdn2_recurrent_fwd(const gdn2_recurrent_args* a, gdn2_stream_t stream);

/* ------------------------------------------------------------------------- */
/* context parallel (T sharded over ranks)                                   */
/* ------------------------------------------------------------------------- */
/*
 * A shard of a sequence maps the state it receives affinely (per head):
 *     S_out = M S_in + h_e,  M in R^{K x K}, h_e in R^{K x V}
 * gdn2_cp_transition computes [M | h_e] for each sequence of a dense shard
 * (gate activation, l2norm and the WY factors as in gdn2_chunk_fwd; h_e from
 * the given initial state, or zero), packed as maps[N, H, K, K+V] fp32 (M in
 * columns 0..K-1).  It needs the workspace gdn2_chunk_workspace_size reports
 * for the same arguments (without GDN2_SAVE_FOR_BWD).  This mirrors the KDA
 * context-parallel pre-process of the reference (chunk_kda.py:102-330,
 * :774-852), which GDN2 shares the scan kernels with but never enables
 * (chunk_gdn2.py:86-92).
 * gdn2_cp_compose folds the maps of ranks 0..rank-1, gathered as
 * [world, N, H, K, K+V], into `state` [N, H, K, V] fp32 in place: on entry the
 * sequence's initial state (or zeros), on return this rank's entering state
 * (S <- M_j S + h_j in rank order; chunk_kda.py:465-477).
 */
int gdn2_cp_transition(const gdn2_chunk_args* a, float* maps, void* workspace,
                       size_t workspace_bytes, gdn2_stream_t stream);
int gdn2_cp_compose(const float* gathered_maps, int32_t rank, int64_t N, int64_t H, int64_t K,
                    int64_t V, float* state, gdn2_stream_t stream);
/* Context-parallel backward (no reference counterpart for GDN2; the reference
 * sketches the KDA equivalent, chunk_kda.py:855-945).  Rank j's shard maps the
 * cotangent of its exit state to that of its entering state affinely,
 * dS_in = M_j^T dS_out + g_j, where g_j is gdn2_chunk_bwd's dh0 under
 * GDN2_BWD_STATE_ONLY with the shard's own do and dht.  gdn2_cp_compose_bwd
 * folds the ranks after this one: on entry `dstate` [N, H, K, V] holds this
 * rank's own dht (or zeros); on return the full cotangent of its exit state,
 * dht + dS_in(rank + 1) with dS_in(j) = M_j^T dS_in(j + 1) + g_j, dS_in(world) = 0.
 * gathered_maps: [world, N, H, K, K+V] (M in columns 0..K-1, as
 * gdn2_cp_transition writes them); gathered_g: [world, N, H, K, V]. */
int gdn2_cp_compose_bwd(const float* gathered_maps, const float* gathered_g, int32_t rank, int32_t world,
                        int64_t N, int64_t H, int64_t K, int64_t V, float* dstate, gdn2_stream_t stream);

/* ------------------------------------------------------------------------- */
/* the GatedDeltaNet2 layer around the operator (lit_gpt/gdn2.py:282-464)    */
/* ------------------------------------------------------------------------- */
/*
 * The layer's first-stage projections are one GEMM (gdn2.py:300-325) whose
 * output rows hold the sections q_raw | k_raw | v_raw | b_raw | w_raw | f0 | g0
 * (widths Dk, Dk, Dv, Dk, Dv, Dfg, Dfg) in that order.  gdn2_layer_prep_fwd
 * turns that bf16 matrix into the operator's inputs in one pass:
 *   q, k, v = SiLU(causal depthwise conv1d of q_raw | k_raw | v_raw), the fla
 *             ShortConvolution of gdn2.py:342-367, or SiLU alone when
 *             conv_size == 0 (gdn2.py:369-372);
 *   b = b_scale * sigmoid(b_raw), w = sigmoid(w_raw)  (gdn2.py:383-384, :410-412);
 *   f0, g0 copied out contiguous (inputs of the second-stage GEMMs).
 * Sequences are rows of T tokens, or given by cu_seqlens [N+1] (device int64)
 * over all rows (every sequence non-empty).  conv_state_in / conv_state_out:
 * bf16 [N, 2Dk+Dv, W] holding each sequence's last W conv inputs, newest at
 * index W-1 (fla's cache layout with the q, k, v channels concatenated); the
 * first output of a sequence reads entries 1..W-1 as its history.
 * conv_state_out may alias conv_state_in only when every sequence is one
 * token (rows == N, the decode step).
 * gdn2_layer_prep_bwd is the reverse pass: from the cotangents of q, k, v, b,
 * w, f0, g0 it writes d(proj) (every section) and the conv weight / bias
 * gradients in fp32 (reduced in a fixed order: bitwise reproducible).  The
 * conv state carries no cotangent (it is an inference cache).
 */
typedef struct gdn2_prep_args {
  int64_t rows, T, N;
  const int64_t* cu_seqlens;
  int64_t Dk, Dv, Dfg;          /* multiples of 8 */
  int64_t conv_size;            /* W: 0 (no convolution), 2, 3 or 4 */
  int64_t proj_stride;          /* elements between rows of proj, >= 3Dk+2Dv+2Dfg, multiple of 8 */
  float b_scale;                /* erase-gate ceiling (2 with allow_neg_eigval) */
  int32_t flags;                /* reserved: 0 */
  const void* proj;             /* bf16 [rows, proj_stride] */
  const float* conv_weight;     /* fp32 [2Dk+Dv, W] */
  const float* conv_bias;       /* fp32 [2Dk+Dv] or NULL */
  const void* conv_state_in;    /* bf16 [N, 2Dk+Dv, W] or NULL (zero history) */
  void* conv_state_out;         /* bf16 [N, 2Dk+Dv, W] or NULL */
  void *q, *k, *v;              /* bf16 [rows, Dk | Dk | Dv] */
  void *b, *w;                  /* bf16 [rows, Dk | Dv] */
  void *f0, *g0;                /* bf16 [rows, Dfg] each, or both NULL (not copied) */
} gdn2_prep_args;

typedef struct gdn2_prep_grads {
  const void *dq, *dk, *dv, *db, *dw;  /* bf16, shapes of q, k, v, b, w */
  const void *df0, *dg0;        /* bf16 [rows, Dfg], or NULL (zero) */
  void* dproj;                  /* bf16 [rows, proj_stride]; columns past the sections untouched */
  float* dconv_weight;          /* fp32 [2Dk+Dv, W] (overwritten) */
  float* dconv_bias;            /* fp32 [2Dk+Dv] or NULL */
} gdn2_prep_grads;

int gdn2_layer_prep_fwd(const gdn2_prep_args* a, gdn2_stream_t stream);
size_t gdn2_layer_prep_bwd_workspace_size(const gdn2_prep_args* a);
int gdn2_layer_prep_bwd(const gdn2_prep_args* a, const gdn2_prep_grads* g, void* workspace,
                        size_t workspace_bytes, gdn2_stream_t stream);

/* Gated output norm, FusedRMSNormSwishGate of gdn2.py:462 (fla
 * fused_norm_gate.py:35-104), per row of D:
 *     y = x / sqrt(mean(x^2) + eps) * weight * gate * sigmoid(gate)
 * x, gate, y: bf16 [rows, D]; weight fp32 [D]; rstd fp32 [rows] (kept for the
 * backward); D in {64, 128, 256}.  The backward writes dx, dgate (bf16) and
 * dweight (fp32 [D], overwritten, fixed reduction order) using a workspace of
 * gdn2_norm_gate_bwd_workspace_size bytes. */
int gdn2_norm_gate_fwd(const void* x, const void* gate, const float* weight, float eps, int64_t rows,
                       int64_t D, void* y, float* rstd, gdn2_stream_t stream);
size_t gdn2_norm_gate_bwd_workspace_size(int64_t rows, int64_t D);
int gdn2_norm_gate_bwd(const void* dy, const void* x, const void* gate, const float* weight,
                       const float* rstd, int64_t rows, int64_t D, void* dx, void* dgate, float* dweight,
                       void* workspace, size_t workspace_bytes, gdn2_stream_t stream);

/* ------------------------------------------------------------------------- */
/* opt-in per-kernel timing (measurement hook, no reference counterpart)     */
/* ------------------------------------------------------------------------- */
/* While enabled, every launch of the library is bracketed by CUDA events on
 * its stream.  gdn2_profile_read waits for the recorded launches, writes up
 * to max_entries {kernel name, launches, total device ms} records, clears the
 * record and returns how many it wrote (< 0: CUDA error). */
typedef struct gdn2_kernel_stat {
  const char* name;
  int64_t launches;
  double total_ms;
} gdn2_kernel_stat;
int gdn2_profile_enable(int on);
int gdn2_profile_read(gdn2_kernel_stat* out, int max_entries);

/* Fault word of the current device (no reference counterpart).  The
 * tensor-core kernels and the layer's staging kernels bound every wait on a
 * barrier; a wait that gives up abandons its work, sets a bit of this word
 * (bit 0: tensor-core scan or an intra-chunk kernel, bit 1: layer prep) and
 * returns, leaving the context usable.  Writes the word to *out (after a device sync the caller performs)
 * and clears it when clear != 0.  Returns 0 or a negative CUDA error. */
int gdn2_device_fault_read(int clear, unsigned int* out);

/* ------------------------------------------------------------------------- */
const char* gdn2_status_string(int status);
/* 1 when the library was built for the running device (sm_100a present). */
int gdn2_device_supported(int device);
/* Version of this ABI (major*100 + minor). */
int gdn2_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* GDN2_B200_H_ */
