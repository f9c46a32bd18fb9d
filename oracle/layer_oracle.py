"""CPU oracle for the GatedDeltaNet2 layer around the operator (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product.  Only ``tests/`` and
``bench.py``'s CPU legs may import it; the shipped layer
(``gateddeltanet-2_b200/layer.py``) runs CUDA kernels and never calls here.

It restates in float64 numpy the pieces of ``lit_gpt/gdn2.py:282-464`` that
sit around the GDN2 operator:

* the short causal depthwise convolutions with SiLU (``gdn2.py:342-367``),
  computed by fla's ``ShortConvolution`` / ``causal_conv1d`` (fla 0.5.1,
  ``fla/modules/conv/short_conv.py``, Triton kernels in
  ``fla/modules/conv/triton/kernels.py``).  Cache layout ``[N, D, W]``
  holding the last ``W`` inputs, newest at index ``W-1``; the first output of
  a sequence reads cache entries ``1..W-1`` as its history;
* the sigmoid gates ``b = b_scale * sigmoid(b_raw)``, ``w = sigmoid(w_raw)``
  (``gdn2.py:383-384``, ``:410-412``);
* the gated output norm ``FusedRMSNormSwishGate`` (``gdn2.py:462``;
  ``fla/modules/fused_norm_gate.py:35-104``):
  ``y = x / sqrt(mean(x^2) + eps) * weight * g * sigmoid(g)``.

Backward passes are derived by hand (reverse mode through the formulas
above).  Parity pin: ``tests/golden/layer_*.npz`` hold fla's own kernel
outputs (``tests/golden/make_golden_layer.py``); ``tests/test_layer_oracle.py``
checks this module against them.
"""

from __future__ import annotations

import numpy as np


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def _segments(B, T, cu_seqlens):
    """(batch row, start, end) of every sequence."""
    if cu_seqlens is None:
        return [(n, 0, T) for n in range(B)]
    cu = [int(c) for c in cu_seqlens]
    return [(0, cu[n], cu[n + 1]) for n in range(len(cu) - 1)]


def short_conv_fwd(x, weight, bias=None, initial_state=None, cu_seqlens=None, activation=True):
    """x [B, T, D], weight [D, W] -> (y [B, T, D], final_state [N, D, W], z).

    ``z`` is the pre-activation, kept for the backward."""
    x = np.asarray(x, np.float64)
    w = np.asarray(weight, np.float64)
    B, T, D = x.shape
    W = w.shape[1]
    y = np.zeros_like(x)
    z = np.zeros_like(x)
    segs = _segments(B, T, cu_seqlens)
    fs = np.zeros((len(segs), D, W))
    for n, (r, s, e) in enumerate(segs):
        hist = (np.asarray(initial_state[n], np.float64).T[1:] if initial_state is not None
                else np.zeros((W - 1, D)))
        xx = np.concatenate([hist, x[r, s:e]], 0)
        for t in range(e - s):
            zt = (xx[t:t + W] * w.T).sum(0)
            if bias is not None:
                zt = zt + np.asarray(bias, np.float64)
            z[r, s + t] = zt
        fs[n] = xx[-W:].T
    y = z * sigmoid(z) if activation else z.copy()
    return y, fs, z


def short_conv_bwd(x, weight, z, dy, initial_state=None, cu_seqlens=None, activation=True):
    """-> (dx, dweight, dbias, dinitial_state).  The final state carries no
    cotangent: the layer keeps it only as an inference cache."""
    x = np.asarray(x, np.float64)
    w = np.asarray(weight, np.float64)
    dy = np.asarray(dy, np.float64)
    B, T, D = x.shape
    W = w.shape[1]
    if activation:
        s = sigmoid(z)
        dz = dy * s * (1.0 + z * (1.0 - s))
    else:
        dz = dy
    dx = np.zeros_like(x)
    dw = np.zeros_like(w)
    segs = _segments(B, T, cu_seqlens)
    dh0 = np.zeros((len(segs), D, W))
    for n, (r, s_, e) in enumerate(segs):
        hist = (np.asarray(initial_state[n], np.float64).T[1:] if initial_state is not None
                else np.zeros((W - 1, D)))
        xx = np.concatenate([hist, x[r, s_:e]], 0)
        dxx = np.zeros_like(xx)
        for t in range(e - s_):
            dxx[t:t + W] += w.T * dz[r, s_ + t]
            dw += (xx[t:t + W] * dz[r, s_ + t]).T
        dx[r, s_:e] = dxx[W - 1:]
        dh0[n][:, 1:] = dxx[:W - 1].T
    dbias = dz.sum((0, 1))
    return dx, dw, dbias, dh0


def gates_fwd(b_raw, w_raw, b_scale=1.0):
    return b_scale * sigmoid(np.asarray(b_raw, np.float64)), sigmoid(np.asarray(w_raw, np.float64))


def gates_bwd(b_raw, w_raw, db, dw, b_scale=1.0):
    sb = sigmoid(np.asarray(b_raw, np.float64))
    sw = sigmoid(np.asarray(w_raw, np.float64))
    return db * b_scale * sb * (1 - sb), dw * sw * (1 - sw)


def norm_gate_fwd(x, gate, weight, eps):
    """Rows over the last axis.  -> (y, rstd)."""
    x = np.asarray(x, np.float64)
    g = np.asarray(gate, np.float64)
    rstd = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    y = x * rstd * np.asarray(weight, np.float64) * g * sigmoid(g)
    return y, rstd


def norm_gate_bwd(x, gate, weight, rstd, dy):
    """-> (dx, dgate, dweight)."""
    x = np.asarray(x, np.float64)
    g = np.asarray(gate, np.float64)
    w = np.asarray(weight, np.float64)
    dy = np.asarray(dy, np.float64)
    sg = sigmoid(g)
    xhat = x * rstd
    dyn = dy * g * sg
    dgate = dy * xhat * w * sg * (1.0 + g * (1.0 - sg))
    dweight = (dyn * xhat).reshape(-1, x.shape[-1]).sum(0)
    dxhat = dyn * w
    dx = rstd * (dxhat - xhat * (dxhat * xhat).mean(-1, keepdims=True))
    return dx, dgate, dweight


# ---------------------------------------------------------------------------
# the whole token mixer (gdn2.py:230-467), forward and backward
# ---------------------------------------------------------------------------
def layer_forward_backward(params, x, dout, cfg, cu_seqlens=None):
    """Float64 restatement of ``GatedDeltaNet2.forward`` in chunk mode
    (merged projections, short convs, in-operator gate activation and q/k
    l2norm, gated norm, output projection) and its backward.

    params: name -> array, the reference module's state-dict names.
    x: [B, T, hidden]; dout: cotangent of the output.
    cfg: dict(num_heads, head_dim, conv_size, use_short_conv, allow_neg_eigval, norm_eps,
    num_v_heads).  With num_v_heads > num_heads (grouped value heads, ``gdn2.py:395-399``)
    q, k, g, b and the gate parameters are repeated over each group of value heads
    before the operator and their gradients summed back over the group.
    Returns (out, grads) with grads[name] for every parameter and grads["x"].
    """
    from . import gdn2_oracle as orc

    P = {n: np.asarray(v, np.float64) for n, v in params.items()}
    x = np.asarray(x, np.float64)
    dout = np.asarray(dout, np.float64)
    B, T, hid = x.shape
    H, K = cfg["num_heads"], cfg["head_dim"]
    HV = cfg.get("num_v_heads") or H
    rep = HV // H
    V = K
    Dk, Dv = H * K, HV * V
    Dfg = V
    W = cfg["conv_size"] if cfg.get("use_short_conv", True) else 0
    bs = 2.0 if cfg.get("allow_neg_eigval", False) else 1.0
    names = ["q_proj.weight", "k_proj.weight", "v_proj.weight", "b_proj.weight", "w_proj.weight",
             "f_proj.0.weight", "g_proj.0.weight"]
    widths = [Dk, Dk, Dv, Dk, Dv, Dfg, Dfg]
    Wcat = np.concatenate([P[n] for n in names], 0)
    proj = x @ Wcat.T
    offs = np.cumsum([0] + widths)
    sec = [proj[..., offs[i]:offs[i + 1]] for i in range(7)]
    conv_w = {}
    qkv, zs = [], []
    for i, nm in enumerate(("q_conv1d", "k_conv1d", "v_conv1d")):
        if W:
            cw = P[nm + ".weight"].reshape(widths[i], W)
            cb = P.get(nm + ".bias")
            y, _, z = short_conv_fwd(sec[i], cw, cb, None, cu_seqlens)
            conv_w[nm] = (cw, cb)
        else:
            z = sec[i]
            y = z * sigmoid(z)
        qkv.append(y)
        zs.append(z)
    b, w = gates_fwd(sec[3], sec[4], bs)
    f_pre = sec[5] @ P["f_proj.1.weight"].T
    g_gate = sec[6] @ P["g_proj.1.weight"].T + P["g_proj.1.bias"]

    def heads(a, d):
        return a.reshape(B, T, -1, d)

    def kheads(a):  # key-side heads, repeated over each group of value heads
        return np.repeat(heads(a, K), rep, axis=2)

    def ungroup(a):  # gradient of a repeated key-side tensor: sum over the group
        return a.reshape(B, T, H, rep, K).sum(3).reshape(B, T, Dk)

    A_log = np.repeat(P["A_log"], rep)
    dt_bias = np.repeat(P["dt_bias"].reshape(H, K), rep, axis=0).reshape(-1)
    # the operator's backward needs d(o); run its forward first for o
    r = orc.chunk_gdn2(kheads(qkv[0]), kheads(qkv[1]), heads(qkv[2], V), kheads(f_pre), kheads(b),
                       heads(w, V), use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True, A_log=A_log,
                       dt_bias=dt_bias, cu_seqlens=cu_seqlens)
    o = r.o
    yn, rstd = norm_gate_fwd(o, heads(g_gate, V), P["o_norm.weight"], cfg.get("norm_eps", 1e-5))
    yflat = yn.reshape(B, T, Dv)
    out = yflat @ P["o_proj.weight"].T

    G = {}
    G["o_proj.weight"] = dout.reshape(-1, hid).T @ yflat.reshape(-1, Dv)
    dy = (dout @ P["o_proj.weight"]).reshape(B, T, HV, V)
    do, dgg, G["o_norm.weight"] = norm_gate_bwd(o, heads(g_gate, V), P["o_norm.weight"], rstd, dy)
    dgg = dgg.reshape(B, T, Dv)
    G["g_proj.1.weight"] = dgg.reshape(-1, Dv).T @ sec[6].reshape(-1, Dfg)
    G["g_proj.1.bias"] = dgg.reshape(-1, Dv).sum(0)
    dsec = [None] * 7
    dsec[6] = dgg @ P["g_proj.1.weight"]
    r = orc.chunk_gdn2(kheads(qkv[0]), kheads(qkv[1]), heads(qkv[2], V), kheads(f_pre), kheads(b),
                       heads(w, V), use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True, A_log=A_log,
                       dt_bias=dt_bias, cu_seqlens=cu_seqlens, do=do)
    g = dict(r.grads)
    G["A_log"] = g["A_log"].reshape(H, rep).sum(1)
    G["dt_bias"] = g["dt_bias"].reshape(H, rep, K).sum(1).reshape(-1)
    for n in ("q", "k", "g", "b"):
        g[n] = ungroup(g[n])
    dfp = g["g"].reshape(B, T, Dk)
    G["f_proj.1.weight"] = dfp.reshape(-1, Dk).T @ sec[5].reshape(-1, Dfg)
    dsec[5] = dfp @ P["f_proj.1.weight"]
    dsec[3], dsec[4] = gates_bwd(sec[3], sec[4], g["b"].reshape(B, T, Dk), g["w"].reshape(B, T, Dv), bs)
    for i, (nm, gn) in enumerate((("q_conv1d", "q"), ("k_conv1d", "k"), ("v_conv1d", "v"))):
        d = g[gn].reshape(B, T, widths[i])
        if W:
            cw, cb = conv_w[nm]
            dx_, dw_, db_, _ = short_conv_bwd(sec[i], cw, zs[i], d, None, cu_seqlens)
            G[nm + ".weight"] = dw_.reshape(widths[i], 1, W)
            if cb is not None:
                G[nm + ".bias"] = db_
            dsec[i] = dx_
        else:
            s = sigmoid(zs[i])
            dsec[i] = d * s * (1 + zs[i] * (1 - s))
    dproj = np.concatenate(dsec, -1)
    dWcat = dproj.reshape(-1, offs[-1]).T @ x.reshape(-1, hid)
    for i, n in enumerate(names):
        G[n] = dWcat[offs[i]:offs[i + 1]]
    G["x"] = dproj @ Wcat
    return out, G
