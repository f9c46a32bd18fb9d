"""Pin the CPU oracle to the reference: every golden vector in tests/golden/
(outputs of the reference's own kernels) must be reproduced by
``oracle.gdn2_oracle`` within the operator's tolerance.

Tolerance (from the operator's contract): |x - ref| <= 1e-2 + 2e-3*|ref|
elementwise, for outputs, final states and every gradient.  fp32 golden cases
are held to a much tighter bound, since both sides then compute in >= fp32.
"""

import numpy as np
import pytest

from golden_io import case_names, load_case
from oracle import gdn2_oracle as orc

RTOL, ATOL = 2e-3, 1e-2


def check(name, actual, expected, rtol=RTOL, atol=ATOL):
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    assert actual.shape == expected.shape, (name, actual.shape, expected.shape)
    err = np.abs(actual - expected)
    bound = atol + rtol * np.abs(expected)
    bad = err > bound
    assert not bad.any(), (
        f"{name}: {bad.sum()} / {bad.size} elements out of tolerance; "
        f"max abs err {err.max():.3e}, max |ref| {np.abs(expected).max():.3e}")


def _tol(meta):
    # every golden case ran the reference in fp32 (bf16 cases on bf16-valued
    # inputs), so the fp64 oracle must agree far inside the op tolerance
    return (1e-4, 1e-5)


@pytest.mark.parametrize("name", case_names("recurrent"))
def test_oracle_recurrent_matches_reference(name):
    meta, t, _ = load_case(name)
    o, ht = orc.fused_recurrent_gdn2(
        t["in_q"], t["in_k"], t["in_v"], t["in_g"], t["in_b"], t["in_w"],
        A_log=t.get("in_A_log"), dt_bias=t.get("in_dt_bias"),
        initial_state=t["in_h0"], output_final_state=True,
        use_qk_l2norm_in_kernel=meta["l2norm"], use_gate_in_kernel=meta["gate"],
        cu_seqlens=meta["cu_seqlens"], transpose_state_layout=meta["transpose"])
    rtol, atol = _tol(meta)
    check("o", o, t["out_o"], rtol, atol)
    check("ht", ht, t["out_ht"], rtol, atol)


@pytest.mark.parametrize("name", case_names("chunk"))
def test_oracle_chunk_matches_reference(name):
    meta, t, _ = load_case(name)
    r = orc.chunk_gdn2(
        t["in_q"], t["in_k"], t["in_v"], t["in_g"], t["in_b"], t["in_w"],
        initial_state=t.get("in_h0"), output_final_state=True,
        use_qk_l2norm_in_kernel=meta["l2norm"], use_gate_in_kernel=meta["gate"],
        cu_seqlens=meta["cu_seqlens"], lower_bound=meta["lower_bound"],
        transpose_state_layout=meta["transpose"],
        A_log=t.get("in_A_log"), dt_bias=t.get("in_dt_bias"),
        do=t["in_do"], dht=t.get("in_dht"))
    rtol, atol = _tol(meta)
    check("o", r.o, t["out_o"], rtol, atol)
    check("ht", r.final_state, t["out_ht"], rtol, atol)
    for g in ("q", "k", "v", "g", "b", "w", "h0", "A_log", "dt_bias"):
        key = f"grad_{g}"
        if key in t:
            check(key, r.grads[g], t[key], rtol, atol)


def test_oracle_backward_matches_finite_differences():
    """The hand-derived backward agrees with central differences (fp64)."""
    rng = np.random.default_rng(0)
    B, T, H, K, V = 1, 6, 1, 4, 3
    q = rng.standard_normal((B, T, H, K))
    k = rng.standard_normal((B, T, H, K))
    v = rng.standard_normal((B, T, H, V))
    g = -np.log1p(np.exp(rng.standard_normal((B, T, H, K)))) * 0.3
    b = 1 / (1 + np.exp(-rng.standard_normal((B, T, H, K))))
    w = 1 / (1 + np.exp(-rng.standard_normal((B, T, H, V))))
    h0 = rng.standard_normal((B, H, K, V)) * 0.1
    do = rng.standard_normal((B, T, H, V))
    dht = rng.standard_normal((B, H, K, V))
    A_log = rng.standard_normal(H) * 0.3
    dt_bias = rng.standard_normal(H * K) * 0.3
    args = dict(initial_state=h0, output_final_state=True, use_qk_l2norm_in_kernel=True,
                use_gate_in_kernel=True, A_log=A_log, dt_bias=dt_bias)

    def loss(**over):
        a = dict(q=q, k=k, v=v, g=g, b=b, w=w)
        a.update(over)
        kw = dict(args)
        for n in ("A_log", "dt_bias"):
            if n in over:
                kw[n] = over.pop(n)
        kw["initial_state"] = over.pop("h0", h0)
        r = orc.chunk_gdn2(a["q"], a["k"], a["v"], a["g"], a["b"], a["w"], **kw)
        return float(np.sum(r.o * do) + np.sum(r.final_state * dht))

    r = orc.chunk_gdn2(q, k, v, g, b, w, do=do, dht=dht, **args)
    base = dict(q=q, k=k, v=v, g=g, b=b, w=w, h0=h0, A_log=A_log, dt_bias=dt_bias)
    eps = 1e-6
    for name, x in base.items():
        num = np.zeros_like(x)
        it = np.nditer(x, flags=["multi_index"])
        for _ in it:
            idx = it.multi_index
            xp = x.copy()
            xp[idx] += eps
            xm = x.copy()
            xm[idx] -= eps
            num[idx] = (loss(**{name: xp}) - loss(**{name: xm})) / (2 * eps)
        np.testing.assert_allclose(r.grads[name], num, rtol=1e-5, atol=1e-7, err_msg=name)


def test_chunk_intermediates_reproduce_recurrence():
    """The chunkwise WY restatement (per-chunk G, Aqk, A, Y, U, kg, then the
    inter-chunk scan) reproduces the token-serial outputs."""
    rng = np.random.default_rng(1)
    T, K, V = 150, 16, 8
    q = rng.standard_normal((T, K))
    k = rng.standard_normal((T, K)) / 4
    v = rng.standard_normal((T, V))
    g = -np.log1p(np.exp(rng.standard_normal((T, K)))) * 0.2
    b = 1 / (1 + np.exp(-rng.standard_normal((T, K))))
    w = 1 / (1 + np.exp(-rng.standard_normal((T, V))))
    scale = K ** -0.5
    im = orc.chunk_intermediates(q, k, v, g, b, w, scale, chunk=64)
    S = np.zeros((K, V))
    o = []
    for c in range(len(im["G"])):
        s = c * 64
        n = im["G"][c].shape[0]
        vn = im["U"][c] - im["Y"][c] @ S
        qg = q[s:s + n] * np.exp2(im["G"][c])
        o.append(scale * qg @ S + im["Aqk"][c] @ vn)
        S = np.exp2(im["G"][c][-1])[:, None] * S + im["kg"][c].T @ vn
    o = np.concatenate(o)
    o_ref, S_ref, _ = orc.recurrent_fwd(q[None, :, None], k[None, :, None], v[None, :, None],
                                        g[None, :, None], b[None, :, None], w[None, :, None], scale)
    np.testing.assert_allclose(o, o_ref[0, :, 0], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(S, S_ref[0, 0], rtol=1e-10, atol=1e-12)
