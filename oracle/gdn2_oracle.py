"""CPU oracle for the Gated Delta Rule-2 operator (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The shipped operator
(``gateddeltanet-2_b200``) never calls into this file and raises when its CUDA
library is missing.

It restates, in float64 numpy, the per-token recurrence that the reference
implements token-serially in
``lit_gpt/gdn2_ops/fused_recurrent_gdn2.py:193-243`` and chunkwise in
``lit_gpt/gdn2_ops/chunk_gdn2.py:1205-1359`` (forward) and ``:2330-2493``
(backward).  Per token, with ``S`` the ``[K, V]`` state:

    S  <- Diag(exp(g_t)) S                       (decay, natural log gate)
    u   = w_t * v_t - S^T (b_t * k_t)            (gated read)
    S  <- S + k_t u^T                            (rank-one write)
    o_t = S^T (scale * q_t)                      (read after the update)

The backward is derived by hand (reverse-mode through the four lines above)
and is independent of the reference's chunkwise WY backward; the two agree
to rounding, which is how the chunkwise reference is checked.

Helpers that sit inside the op's math in the third-party ``fla`` package
(version 0.5.1, git bb324a32, installed in this image) are restated here too:

* ``l2norm_fwd`` / ``l2norm_bwd``: ``fla/modules/l2norm.py:42`` (rstd =
  1/sqrt(sum(x^2) + eps), eps 1e-6) and ``:73``
  (dx = dy*rstd - sum(dy*y)*y*rstd).
* the decay-gate activation ``-exp(A_log) * softplus(g + dt_bias)``
  (``chunk_kda.py:2296-2324``, ``:2676-2681``) or, with ``lower_bound``,
  ``lower_bound * sigmoid(exp(A_log) * (g + dt_bias))`` (``:2326-2338``), and
  its backward (``chunk_kda.py:2420-2555``).

Parity pin: ``tests/golden/`` holds outputs of the reference's own kernels
(run under the Triton CPU interpreter by ``tests/golden/make_golden.py``);
``tests/test_oracle.py`` checks this module against them.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

L2NORM_EPS = 1e-6


# ----------------------------------------------------------------------------
# fla helpers restated
# ----------------------------------------------------------------------------
def l2norm_fwd(x: np.ndarray, eps: float = L2NORM_EPS):
    """y = x / sqrt(sum(x^2) + eps) over the last axis; returns (y, rstd).

    Follows fla ``modules/l2norm.py:100-101`` as called from
    ``chunk_gdn2.py:2542-2544``.
    """
    x = np.asarray(x, dtype=np.float64)
    rstd = 1.0 / np.sqrt(np.sum(x * x, axis=-1) + eps)
    return x * rstd[..., None], rstd


def l2norm_bwd(y: np.ndarray, rstd: np.ndarray, dy: np.ndarray):
    """dx = dy*rstd - sum(dy*y)*y*rstd  (fla ``modules/l2norm.py:134``)."""
    y = np.asarray(y, np.float64)
    dy = np.asarray(dy, np.float64)
    r = np.asarray(rstd, np.float64)[..., None]
    return dy * r - np.sum(dy * y, axis=-1, keepdims=True) * y * r


def softplus(x: np.ndarray) -> np.ndarray:
    """log(1 + e^x), passing x through above 20 (fla ``ops/utils/softplus.py``)."""
    x = np.asarray(x, np.float64)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def sigmoid(x: np.ndarray) -> np.ndarray:
    return 1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))


def gate_fwd(g_raw, A_log, dt_bias=None, lower_bound=None):
    """Decay-gate activation on [..., H, K] (``chunk_kda.py:2676-2681``)."""
    g = np.asarray(g_raw, np.float64)
    H, K = g.shape[-2:]
    if dt_bias is not None:
        g = g + np.asarray(dt_bias, np.float64).reshape(H, K)
    a = np.exp(np.asarray(A_log, np.float64).reshape(H, 1))
    if lower_bound is None:
        return -a * softplus(g)
    return lower_bound * sigmoid(a * g)


def gate_bwd(g_raw, A_log, dyg, dt_bias=None, lower_bound=None):
    """Backward of ``gate_fwd``: (dg_raw, dA_log, d_dt_bias).

    Follows ``chunk_kda.py:2436-2470`` (kernel) and ``:2515-2555`` (sums).
    """
    g = np.asarray(g_raw, np.float64)
    dyg = np.asarray(dyg, np.float64)
    H, K = g.shape[-2:]
    if dt_bias is not None:
        g = g + np.asarray(dt_bias, np.float64).reshape(H, K)
    a = np.exp(np.asarray(A_log, np.float64).reshape(H, 1))
    if lower_bound is None:
        yg = -a * softplus(g)
        dg = -a * dyg * sigmoid(g)
        dA = np.sum((dyg * yg).reshape(-1, H, K), axis=(0, 2))
    else:
        s = sigmoid(a * g)
        dg = dyg * lower_bound * s * (1.0 - s) * a
        dA = np.sum((dg * g).reshape(-1, H, K), axis=(0, 2))
    dbias = None
    if dt_bias is not None:
        dbias = dg.reshape(-1, H * K).sum(0)
    return dg, dA.reshape(np.shape(A_log)), dbias


# ----------------------------------------------------------------------------
# the recurrence on one dense batch of sequences: arrays [B, T, H, *]
# ----------------------------------------------------------------------------
def _key_head_index(H: int, HV: int) -> np.ndarray:
    return np.arange(HV) // (HV // H)


def recurrent_fwd(q, k, v, g, b, w, scale, h0=None, keep_states=False):
    """Token-serial forward.  q,k: [B,T,H,K]; v,w: [B,T,HV,V]; g,b: [B,T,HV,K].

    Returns (o [B,T,HV,V], S_T [B,HV,K,V], states) where ``states[t]`` is the
    state before token t (only when ``keep_states``).  Mirrors
    ``fused_recurrent_gdn2.py:193-243``.
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    g = np.asarray(g, np.float64)
    b = np.asarray(b, np.float64)
    w = np.asarray(w, np.float64)
    B, T, H, K = q.shape
    HV, V = v.shape[2], v.shape[3]
    kh = _key_head_index(H, HV)
    S = np.zeros((B, HV, K, V)) if h0 is None else np.array(h0, np.float64, copy=True)
    o = np.zeros((B, T, HV, V))
    states = np.zeros((T, B, HV, K, V)) if keep_states else None
    for t in range(T):
        if keep_states:
            states[t] = S
        qt = q[:, t][:, kh] * scale
        kt = k[:, t][:, kh]
        S = S * np.exp(g[:, t])[..., None]
        bk = b[:, t] * kt
        u = w[:, t] * v[:, t] - np.einsum("bhkv,bhk->bhv", S, bk)
        S = S + kt[..., None] * u[..., None, :]
        o[:, t] = np.einsum("bhkv,bhk->bhv", S, qt)
    return o, S, states


def recurrent_bwd(q, k, v, g, b, w, scale, states, do, dht=None):
    """Hand-derived reverse-mode of ``recurrent_fwd`` (H == HV).

    Returns (dq, dk, dv, dg, db, dw, dh0); dg is w.r.t. the natural-log
    decay ``g`` fed to the recurrence.
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    g = np.asarray(g, np.float64)
    b = np.asarray(b, np.float64)
    w = np.asarray(w, np.float64)
    do = np.asarray(do, np.float64)
    B, T, H, K = q.shape
    V = v.shape[-1]
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    dg = np.zeros_like(g)
    db = np.zeros_like(b)
    dw = np.zeros_like(w)
    dS = np.zeros((B, H, K, V)) if dht is None else np.array(dht, np.float64, copy=True)
    for t in range(T - 1, -1, -1):
        S_prev = states[t]
        alpha = np.exp(g[:, t])
        Sa = S_prev * alpha[..., None]
        bk = b[:, t] * k[:, t]
        u = w[:, t] * v[:, t] - np.einsum("bhkv,bhk->bhv", Sa, bk)
        St = Sa + k[:, t][..., None] * u[..., None, :]
        qs = q[:, t] * scale
        # o_t = St^T qs
        dq[:, t] = scale * np.einsum("bhkv,bhv->bhk", St, do[:, t])
        dS = dS + qs[..., None] * do[:, t][..., None, :]
        # St = Sa + k u^T
        du = np.einsum("bhkv,bhk->bhv", dS, k[:, t])
        dk[:, t] = np.einsum("bhkv,bhv->bhk", dS, u)
        dSa = dS
        # u = w*v - Sa^T bk
        dw[:, t] = du * v[:, t]
        dv[:, t] = du * w[:, t]
        de = -du
        dSa = dSa + bk[..., None] * de[..., None, :]
        dbk = np.einsum("bhkv,bhv->bhk", Sa, de)
        db[:, t] = dbk * k[:, t]
        dk[:, t] += dbk * b[:, t]
        # Sa = Diag(alpha) S_prev
        dg[:, t] = np.sum(Sa * dSa, axis=-1)
        dS = dSa * alpha[..., None]
    return dq, dk, dv, dg, db, dw, dS


# ----------------------------------------------------------------------------
# op-level restatements with the reference's argument conventions
# ----------------------------------------------------------------------------
def _split_varlen(x, cu_seqlens):
    """[1, total, ...] -> list of [1, T_i, ...] views."""
    cu = [int(c) for c in cu_seqlens]
    return [x[:, cu[i]:cu[i + 1]] for i in range(len(cu) - 1)]


def _state_in(h0, transpose):
    if h0 is None:
        return None
    h0 = np.asarray(h0, np.float64)
    return np.swapaxes(h0, -1, -2) if transpose else h0


def _state_out(S, transpose):
    return np.swapaxes(S, -1, -2) if transpose else S


@dataclass
class ChunkResult:
    o: np.ndarray
    final_state: np.ndarray | None
    grads: dict | None


def chunk_gdn2(q, k, v, g, b, w, scale=None, initial_state=None,
               output_final_state=False, use_qk_l2norm_in_kernel=False,
               use_gate_in_kernel=False, cu_seqlens=None, lower_bound=None,
               transpose_state_layout=False, A_log=None, dt_bias=None,
               do=None, dht=None) -> ChunkResult:
    """Float64 restatement of ``chunk_gdn2`` (``chunk_gdn2.py:1363-1511``).

    Runs the forward and, when a cotangent ``do`` is given, the backward of
    ``ChunkGDN2Function`` (``:2504-2665``) with the same gradient list:
    dq, dk, dv, dg, db, dw, dA_log, dt_bias, dh0.  Sequences in a varlen
    batch (``cu_seqlens``) are processed independently.
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    K = q.shape[-1]
    if scale is None:
        scale = K ** -0.5
    g_raw = np.asarray(g, np.float64)
    if use_gate_in_kernel:
        g_act = gate_fwd(g_raw, A_log, dt_bias, lower_bound)
    else:
        g_act = g_raw
    if use_qk_l2norm_in_kernel:
        qn, q_rstd = l2norm_fwd(q)
        kn, k_rstd = l2norm_fwd(k)
    else:
        qn, kn = q, k
    h0 = _state_in(initial_state, transpose_state_layout)

    if cu_seqlens is None:
        segs = [(slice(None), slice(None))]
        B = q.shape[0]
    else:
        cu = [int(c) for c in cu_seqlens]
        segs = [(slice(0, 1), slice(cu[i], cu[i + 1])) for i in range(len(cu) - 1)]
        B = len(cu) - 1

    o = np.zeros(v.shape, np.float64)
    H, V = q.shape[2], v.shape[-1]
    ht = np.zeros((B, H, K, V))
    states_all = []
    for i, (bs, ts) in enumerate(segs):
        h0_i = None
        if h0 is not None:
            h0_i = h0 if cu_seqlens is None else h0[i:i + 1]
        o_i, S_i, st = recurrent_fwd(qn[bs, ts], kn[bs, ts], np.asarray(v, np.float64)[bs, ts],
                                      g_act[bs, ts], np.asarray(b, np.float64)[bs, ts],
                                      np.asarray(w, np.float64)[bs, ts], scale, h0_i,
                                      keep_states=do is not None)
        o[bs, ts] = o_i
        if cu_seqlens is None:
            ht = S_i
        else:
            ht[i] = S_i[0]
        states_all.append(st)
    final_state = _state_out(ht, transpose_state_layout) if output_final_state else None
    if do is None:
        return ChunkResult(o, final_state, None)

    do = np.asarray(do, np.float64)
    dht_ = _state_in(dht, transpose_state_layout)
    dq = np.zeros_like(qn)
    dk = np.zeros_like(kn)
    dv = np.zeros(v.shape)
    dga = np.zeros(g_raw.shape)
    db = np.zeros(np.shape(b))
    dw = np.zeros(np.shape(w))
    dh0 = np.zeros((B, H, K, V))
    for i, (bs, ts) in enumerate(segs):
        dht_i = None
        if dht_ is not None:
            dht_i = dht_ if cu_seqlens is None else dht_[i:i + 1]
        r = recurrent_bwd(qn[bs, ts], kn[bs, ts], np.asarray(v, np.float64)[bs, ts],
                          g_act[bs, ts], np.asarray(b, np.float64)[bs, ts],
                          np.asarray(w, np.float64)[bs, ts], scale, states_all[i],
                          do[bs, ts], dht_i)
        dq[bs, ts], dk[bs, ts], dv[bs, ts], dga[bs, ts], db[bs, ts], dw[bs, ts] = r[:6]
        if cu_seqlens is None:
            dh0 = r[6]
        else:
            dh0[i] = r[6][0]
    if use_qk_l2norm_in_kernel:
        dq = l2norm_bwd(qn, q_rstd, dq)
        dk = l2norm_bwd(kn, k_rstd, dk)
    dA_log = ddt = None
    if use_gate_in_kernel:
        dg, dA_log, ddt = gate_bwd(g_raw, A_log, dga, dt_bias, lower_bound)
    else:
        dg = dga
    grads = dict(q=dq, k=dk, v=dv, g=dg, b=db, w=dw, A_log=dA_log, dt_bias=ddt,
                 h0=_state_out(dh0, transpose_state_layout) if initial_state is not None else None)
    return ChunkResult(o, final_state, grads)


def fused_recurrent_gdn2(q, k, v, g, b, w, A_log=None, dt_bias=None, scale=None,
                         initial_state=None, output_final_state=False,
                         use_qk_l2norm_in_kernel=False, use_gate_in_kernel=False,
                         lower_bound=None, cu_seqlens=None,
                         transpose_state_layout=False):
    """Float64 restatement of ``fused_recurrent_gdn2``
    (``fused_recurrent_gdn2.py:399-492``): returns (o, final_state).

    The in-kernel l2norm (``:198-200``) and gate (``:203-214``) are applied per
    token exactly as the reference kernel does.
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    K = q.shape[-1]
    if scale is None:
        scale = K ** -0.5
    if use_qk_l2norm_in_kernel:
        q = l2norm_fwd(q)[0]
        k = l2norm_fwd(k)[0]
    g = np.asarray(g, np.float64)
    if use_gate_in_kernel:
        HV = v.shape[2]
        H = q.shape[2]
        kh = _key_head_index(H, HV)
        gg = g + (np.asarray(dt_bias, np.float64).reshape(H, K)[kh] if dt_bias is not None else 0.0)
        a = np.exp(np.asarray(A_log, np.float64).reshape(-1)[kh])[:, None]
        g = lower_bound * sigmoid(a * gg) if lower_bound is not None else -a * softplus(gg)
    h0 = _state_in(initial_state, transpose_state_layout)
    if cu_seqlens is None:
        o, S, _ = recurrent_fwd(q, k, v, g, b, w, scale, h0)
    else:
        cu = [int(c) for c in cu_seqlens]
        N = len(cu) - 1
        o = np.zeros(v.shape, np.float64)
        S = np.zeros((N, v.shape[2], K, v.shape[-1]))
        for i in range(N):
            ts = slice(cu[i], cu[i + 1])
            h0_i = None if h0 is None else h0[i:i + 1]
            o_i, S_i, _ = recurrent_fwd(q[:, ts], k[:, ts], np.asarray(v)[:, ts], g[:, ts],
                                        np.asarray(b)[:, ts], np.asarray(w)[:, ts], scale, h0_i)
            o[:, ts] = o_i
            S[i] = S_i[0]
    return o, (_state_out(S, transpose_state_layout) if output_final_state else None)


# ----------------------------------------------------------------------------
# chunkwise restatement (for kernel-level debugging of the WY pipeline)
# ----------------------------------------------------------------------------
def chunk_intermediates(q, k, v, g, b, w, scale, chunk=64):
    """Per-chunk WY quantities for one head, float64.

    q,k,g,b: [T,K]; v,w: [T,V]; g natural-log decay.  Returns a dict with
    G (chunk-local cumsum of g / ln 2, ``chunk_gdn2.py:1236-1253``), Aqk
    (scale-folded, lower incl. diagonal), A = (I+T)^-1, Y = A (b*2^G*k)
    (the reference's ``w`` buffer), U = A (w*v) (its ``u`` buffer) and
    kg = k*2^(G_last-G) (``recompute_w_u_fwd_gdn2_kernel``, ``:837-929``).
    """
    q, k, v, g, b, w = (np.asarray(x, np.float64) for x in (q, k, v, g, b, w))
    T = q.shape[0]
    out = {n: [] for n in ("G", "Aqk", "A", "Y", "U", "kg")}
    for s in range(0, T, chunk):
        e = min(s + chunk, T)
        G = np.cumsum(g[s:e], axis=0) / math.log(2.0)
        D = G[:, None, :] - G[None, :, :]            # [r, s, c]
        n = e - s
        lower = np.tril(np.ones((n, n), bool))
        E = np.where(lower[..., None], np.exp2(np.where(lower[..., None], D, 0.0)), 0.0)
        Aqk = scale * np.einsum("rc,sc,rsc->rs", q[s:e], k[s:e], E)
        Tm = np.einsum("rc,sc,rsc->rs", b[s:e] * k[s:e], k[s:e], E)
        Tm = np.tril(Tm, -1)
        A = np.linalg.inv(np.eye(n) + Tm)
        out["G"].append(G)
        out["Aqk"].append(np.tril(Aqk))
        out["A"].append(A)
        out["Y"].append(A @ (b[s:e] * np.exp2(G) * k[s:e]))
        out["U"].append(A @ (w[s:e] * v[s:e]))
        out["kg"].append(k[s:e] * np.exp2(G[-1][None, :] - G))
    return out
