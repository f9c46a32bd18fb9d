"""Chunkwise forward + backward (gdn2_chunk_fwd / gdn2_chunk_bwd through
chunk_gdn2) against the reference's golden vectors and the fp64 oracle."""

import numpy as np
import pytest
import torch

from golden_io import case_names, load_case
from oracle import gdn2_oracle as orc
from tolerance import assert_close, assert_close_reduced, gate_param_masses

pytestmark = pytest.mark.gpu

# dA_log and ddt_bias are sums of B*T*K (resp. B*T) per-token terms, each
# carrying the bf16 roundings of the op's inputs and intermediates (bf16
# epsilon 2^-8); their bound is relative to the summed magnitude of the terms:
# |x - ref| <= 1e-2 + RTOL_SUM * sum|terms|.
RTOL_SUM = 1e-2


def _t(x, dtype=torch.float32, grad=False):
    t = torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)
    return t.requires_grad_(grad)


def _run_case(gdn2, name, backward=True):
    meta, t, _ = load_case(name)
    qd = torch.bfloat16 if meta["qkv_dtype"] == "bfloat16" else torch.float32
    leaves = {n: _t(t[f"in_{n}"], qd if n in "qkv" else torch.float32, grad=backward)
              for n in ("q", "k", "v", "g", "b", "w")}
    if "in_h0" in t:
        leaves["h0"] = _t(t["in_h0"], grad=backward)
    kw = {}
    if meta["gate"]:
        leaves["A_log"] = _t(t["in_A_log"], grad=backward)
        leaves["dt_bias"] = _t(t["in_dt_bias"], grad=backward)
        kw = dict(A_log=leaves["A_log"], dt_bias=leaves["dt_bias"])
    cu = None if meta["cu_seqlens"] is None else torch.tensor(meta["cu_seqlens"], device="cuda")
    o, ht = gdn2.chunk_gdn2(
        leaves["q"], leaves["k"], leaves["v"], leaves["g"], leaves["b"], leaves["w"],
        initial_state=leaves.get("h0"), output_final_state=True,
        use_qk_l2norm_in_kernel=meta["l2norm"], use_gate_in_kernel=meta["gate"],
        cu_seqlens=cu, lower_bound=meta["lower_bound"],
        transpose_state_layout=meta["transpose"], **kw)
    if backward:
        do = _t(t["in_do"], qd)
        dht = _t(t["in_dht"]) if "in_dht" in t else torch.zeros_like(ht)
        torch.autograd.backward([o, ht], [do, dht])
    torch.cuda.synchronize()
    return meta, t, o, ht, leaves


# fp32 inputs take the fp32 path (the recurrence in fp32, like the reference's
# fp32 path, which is within ~5e-7 of the naive fp32 recurrence): those cases
# are held to 1e-4 absolute + 1e-4 relative instead of the bf16 bound.
FP32_TOL = dict(rtol=1e-4, atol=1e-4)


def _tol(meta):
    return FP32_TOL if meta["qkv_dtype"] == "float32" else {}


@pytest.mark.parametrize("name", case_names("chunk"))
def test_chunk_forward_matches_reference_golden(gdn2, name):
    meta, t, o, ht, _ = _run_case(gdn2, name, backward=False)
    assert_close(o, t["out_o"], "o", **_tol(meta))
    assert_close(ht, t["out_ht"], "ht", **_tol(meta))


@pytest.mark.parametrize("name", case_names("chunk"))
def test_chunk_backward_matches_reference_golden(gdn2, name):
    meta, t, o, ht, leaves = _run_case(gdn2, name, backward=True)
    tol = _tol(meta)
    assert_close(o, t["out_o"], "o", **tol)
    assert_close(ht, t["out_ht"], "ht", **tol)
    masses = {}
    if meta["gate"]:
        mA, mdt = gate_param_masses(t["in_g"], t["in_dt_bias"], t["grad_g"], meta["H"])
        masses = {"A_log": mA, "dt_bias": mdt}
    for n, leaf in leaves.items():
        if n in masses:
            assert_close_reduced(leaf.grad, t[f"grad_{n}"], masses[n], f"d{n}",
                                 rtol=tol.get("rtol", RTOL_SUM))
        else:
            assert_close(leaf.grad, t[f"grad_{n}"], f"d{n}", **tol)


def test_config1_fp32_matches_reference_golden_at_fp32_bound(gdn2):
    """BASELINE config 1 exactly (fp32, B=1, H=2, T=256, d=64, chunk 64): the
    reference's own chunk op output and all six gradients to 1e-4."""
    meta, t, o, ht, leaves = _run_case(gdn2, "chunk_c1_fp32", backward=True)
    assert (meta["B"], meta["H"], meta["T"], meta["K"], meta["V"]) == (1, 2, 256, 64, 64)
    assert o.dtype == torch.float32
    assert_close(o, t["out_o"], "o", **FP32_TOL)
    for n in "qkvgbw":
        assert_close(leaves[n].grad, t[f"grad_{n}"], f"d{n}", **FP32_TOL)


def _inputs(seed, B, T, H, K, V, gate_scale=0.1, bw=torch.float32):
    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=g), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=g), dim=-1).bfloat16()
    v = torch.randn(B, T, H, V, generator=g).bfloat16()
    gg = -torch.nn.functional.softplus(torch.randn(B, T, H, K, generator=g)) * gate_scale
    b = torch.sigmoid(torch.randn(B, T, H, K, generator=g)).to(bw)
    w = torch.sigmoid(torch.randn(B, T, H, V, generator=g)).to(bw)
    return q, k, v, gg, b, w


@pytest.mark.parametrize("B,T,H,K,V", [(2, 200, 2, 128, 128), (1, 64, 3, 64, 128),
                                       (1, 130, 2, 128, 64), (1, 33, 1, 64, 64),
                                       (1, 777, 3, 128, 128), (3, 64, 2, 128, 128)])
def test_chunk_forward_matches_oracle(gdn2, B, T, H, K, V):
    q, k, v, gg, b, w = _inputs(B * T + H, B, T, H, K, V)
    h0 = torch.randn(B, H, K, V) * 0.1
    o, ht = gdn2.chunk_gdn2(q.cuda(), k.cuda(), v.cuda(), gg.cuda(), b.cuda(), w.cuda(),
                            initial_state=h0.cuda(), output_final_state=True)
    r = orc.chunk_gdn2(*(x.float().numpy() for x in (q, k, v, gg, b, w)),
                       initial_state=h0.numpy(), output_final_state=True)
    assert_close(o, r.o, "o")
    assert_close(ht, r.final_state, "ht")


def test_chunk_forward_extreme_decay_is_exact(gdn2):
    """Channels that forget almost instantly (log-decay -60 per token) push
    the anchored exponents out of range; the exact per-pair path must keep
    the scores (and the outputs) right."""
    B, T, H, K, V = 1, 128, 1, 128, 128
    q, k, v, gg, b, w = _inputs(3, B, T, H, K, V)
    gg[..., :8] = -60.0          # instant-forget channels
    gg[:, 40:44, :, 8:16] = -30.0  # a burst inside one block
    o, ht = gdn2.chunk_gdn2(q.cuda(), k.cuda(), v.cuda(), gg.cuda(), b.cuda(), w.cuda(),
                            output_final_state=True)
    r = orc.chunk_gdn2(*(x.float().numpy() for x in (q, k, v, gg, b, w)), output_final_state=True)
    assert_close(o, r.o, "o")
    assert_close(ht, r.final_state, "ht")


def _bwd_vs_oracle(gdn2, q, k, v, gg, b, w, h0=None, dht=True, gate=None, l2=False, seed=0):
    B, T, H, K = q.shape
    V = v.shape[-1]
    gen = torch.Generator().manual_seed(seed + 99)
    do = torch.randn(B, T, H, V, generator=gen).bfloat16()
    dht_t = torch.randn(B, H, K, V, generator=gen) * 0.1 if dht else None
    leaves = [x.cuda().requires_grad_(True) for x in (q, k, v, gg, b, w)]
    h0_d = h0.cuda().requires_grad_(True) if h0 is not None else None
    kw = {}
    if gate is not None:
        A_log, dt_bias = (x.cuda().requires_grad_(True) for x in gate)
        kw = dict(A_log=A_log, dt_bias=dt_bias)
    o, ht = gdn2.chunk_gdn2(*leaves, initial_state=h0_d, output_final_state=True,
                            use_qk_l2norm_in_kernel=l2, use_gate_in_kernel=gate is not None, **kw)
    torch.autograd.backward([o, ht], [do.cuda(), dht_t.cuda() if dht else torch.zeros_like(ht)])
    torch.cuda.synchronize()
    r = orc.chunk_gdn2(*(x.float().numpy() for x in (q, k, v, gg, b, w)),
                       initial_state=None if h0 is None else h0.numpy(), output_final_state=True,
                       use_qk_l2norm_in_kernel=l2, use_gate_in_kernel=gate is not None,
                       A_log=None if gate is None else gate[0].numpy(),
                       dt_bias=None if gate is None else gate[1].numpy(),
                       do=do.float().numpy(), dht=None if dht_t is None else dht_t.numpy())
    assert_close(o, r.o, "o")
    assert_close(ht, r.final_state, "ht")
    for n, leaf in zip("qkvgbw", leaves):
        assert_close(leaf.grad, r.grads[n], f"d{n}")
    if h0 is not None:
        assert_close(h0_d.grad, r.grads["h0"], "dh0")
    if gate is not None:
        mA, mdt = gate_param_masses(gg, gate[1], r.grads["g"], H)
        assert_close_reduced(kw["A_log"].grad, r.grads["A_log"], mA, "dA_log", rtol=RTOL_SUM)
        assert_close_reduced(kw["dt_bias"].grad, r.grads["dt_bias"], mdt, "ddt_bias", rtol=RTOL_SUM)
        # the reductions themselves are exact: they must equal the sums over the
        # kernel's own dg, through dg_raw = dyg * d(g_act)/d(g_raw)
        dg_k = leaves[3].grad.double().cpu().numpy()
        x = gg.double().numpy() + gate[1].double().numpy().reshape(H, K)
        sp, sg = np.log1p(np.exp(x)), 1.0 / (1.0 + np.exp(-x))
        own_A = (dg_k * sp / sg).reshape(-1, H, K).sum((0, 2))
        own_dt = dg_k.reshape(-1, H * K).sum(0)
        # (exact up to fp32 summation; with a bf16 dg the kernel reduced the
        # unrounded values, so one bf16 rounding of each term separates them)
        rt = 2.0 ** -8 if gg.dtype == torch.bfloat16 else 1e-5
        assert_close_reduced(kw["A_log"].grad, own_A, mA, "dA_log vs own dg", rtol=rt, atol=1e-6)
        assert_close_reduced(kw["dt_bias"].grad, own_dt, mdt, "ddt_bias vs own dg", rtol=rt, atol=1e-6)


@pytest.mark.parametrize("B,T,H,K,V,bw", [(2, 200, 2, 128, 128, torch.float32),
                                          (1, 64, 2, 64, 128, torch.bfloat16),
                                          (1, 130, 1, 128, 64, torch.float32),
                                          (1, 33, 1, 64, 64, torch.bfloat16)])
def test_chunk_backward_matches_oracle(gdn2, B, T, H, K, V, bw):
    q, k, v, gg, b, w = _inputs(B * T + H + 1, B, T, H, K, V, bw=bw)
    h0 = torch.randn(B, H, K, V) * 0.1
    _bwd_vs_oracle(gdn2, q, k, v, gg, b, w, h0=h0, seed=T)


@pytest.mark.parametrize("gdtype,bwdtype", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16)])
def test_chunk_backward_gate_and_l2norm_match_oracle(gdn2, gdtype, bwdtype):
    """Gate activation and q/k l2norm in the kernel; the bf16 case is the
    layer's call (bf16 raw gate pre-activation read as is, dg written in bf16,
    bf16 b and w)."""
    B, T, H, K, V = 1, 192, 2, 128, 128
    q, k, v, gg, b, w = _inputs(11, B, T, H, K, V, bw=bwdtype)
    g2 = torch.Generator().manual_seed(5)
    graw = torch.randn(B, T, H, K, generator=g2).to(gdtype)
    A_log = torch.rand(H, generator=g2) * 2.0
    dt_bias = torch.randn(H * K, generator=g2) * 0.5
    q = (q.float() * 3).bfloat16()
    _bwd_vs_oracle(gdn2, q, k, v, graw, b, w, gate=(A_log, dt_bias), l2=True, seed=3)


def test_chunk_backward_extreme_decay_is_exact(gdn2):
    B, T, H, K, V = 1, 128, 1, 128, 128
    q, k, v, gg, b, w = _inputs(13, B, T, H, K, V)
    gg[..., :8] = -60.0
    gg[:, 40:44, :, 8:16] = -30.0
    _bwd_vs_oracle(gdn2, q, k, v, gg, b, w, seed=4)


def test_chunk_backward_varlen_matches_oracle(gdn2):
    cu = [0, 50, 179, 180, 300]
    T, H, K, V = cu[-1], 2, 128, 128
    q, k, v, gg, b, w = _inputs(21, 1, T, H, K, V)
    gen = torch.Generator().manual_seed(8)
    h0 = torch.randn(len(cu) - 1, H, K, V, generator=gen) * 0.1
    do = torch.randn(1, T, H, V, generator=gen).bfloat16()
    dht = torch.randn(len(cu) - 1, H, K, V, generator=gen) * 0.1
    leaves = [x.cuda().requires_grad_(True) for x in (q, k, v, gg, b, w)]
    h0_d = h0.cuda().requires_grad_(True)
    o, ht = gdn2.chunk_gdn2(*leaves, initial_state=h0_d, output_final_state=True,
                            cu_seqlens=torch.tensor(cu, device="cuda"))
    torch.autograd.backward([o, ht], [do.cuda(), dht.cuda()])
    r = orc.chunk_gdn2(*(x.float().numpy() for x in (q, k, v, gg, b, w)), initial_state=h0.numpy(),
                       output_final_state=True, cu_seqlens=cu, do=do.float().numpy(), dht=dht.numpy())
    assert_close(o, r.o, "o")
    assert_close(ht, r.final_state, "ht")
    for n, leaf in zip("qkvgbw", leaves):
        assert_close(leaf.grad, r.grads[n], f"d{n}")
    assert_close(h0_d.grad, r.grads["h0"], "dh0")


@pytest.mark.parametrize("K,V,transpose", [(128, 128, False), (128, 128, True), (64, 64, False)])
def test_intermediate_states_match_oracle_prefix_states(gdn2, K, V, transpose):
    """return_intermediate_states: h[c] is the state entering chunk c, i.e. the
    state after the first 64 c tokens (stored in bf16, like the reference's h:
    the bound adds bf16's relative step, 2^-8)."""
    B, T, H = 1, 200, 2
    q, k, v, gg, b, w = _inputs(11, B, T, H, K, V)
    h0 = torch.randn(B, H, K, V) * 0.1
    with torch.inference_mode():
        _, _, hs = gdn2.chunk_gdn2(q.cuda(), k.cuda(), v.cuda(), gg.cuda(), b.cuda(), w.cuda(),
                                   initial_state=(h0.transpose(-1, -2) if transpose else h0).contiguous().cuda(),
                                   output_final_state=True, return_intermediate_states=True,
                                   transpose_state_layout=transpose)
    torch.cuda.synchronize()
    assert hs.shape == (B, (T + 63) // 64, H) + ((V, K) if transpose else (K, V))
    x = [t.float().numpy() for t in (q, k, v, gg, b, w)]
    for c in range(hs.shape[1]):
        if c == 0:
            ref = h0.numpy()
        else:
            _, ref, _ = orc.recurrent_fwd(*(t[:, :64 * c] for t in x), K ** -0.5, h0.numpy())
        got = hs[:, c].float().cpu().numpy()
        if transpose:
            got = got.swapaxes(-1, -2)
        np.testing.assert_allclose(got, ref, rtol=2e-3 + 2 ** -8, atol=1e-2, err_msg=f"h[{c}]")


@pytest.mark.parametrize("K,V,gate,l2", [(128, 128, True, True), (64, 128, False, False),
                                         (128, 64, False, True), (64, 64, True, False)])
def test_fp32_path_matches_oracle_at_fp32_bound(gdn2, K, V, gate, l2):
    """fp32 inputs: forward, final state and every gradient (with h0, dht,
    the gate and l2norm in the kernel) against the fp64 oracle to 1e-4."""
    B, T, H = 2, 150, 2
    g = torch.Generator().manual_seed(K + V + gate)
    q = torch.randn(B, T, H, K, generator=g) * (3.0 if l2 else 1.0)
    k = torch.randn(B, T, H, K, generator=g)
    if not l2:
        q, k = (torch.nn.functional.normalize(x, dim=-1) for x in (q, k))
    v = torch.randn(B, T, H, V, generator=g)
    graw = torch.randn(B, T, H, K, generator=g) if gate else -torch.nn.functional.softplus(
        torch.randn(B, T, H, K, generator=g)) * 0.1
    b = torch.sigmoid(torch.randn(B, T, H, K, generator=g))
    w = torch.sigmoid(torch.randn(B, T, H, V, generator=g))
    h0 = torch.randn(B, H, K, V, generator=g) * 0.1
    do = torch.randn(B, T, H, V, generator=g)
    dht = torch.randn(B, H, K, V, generator=g) * 0.1
    A_log = torch.rand(H, generator=g) * 2.0
    dt_bias = torch.randn(H * K, generator=g) * 0.5
    leaves = [x.cuda().requires_grad_(True) for x in (q, k, v, graw, b, w)]
    h0_d = h0.cuda().requires_grad_(True)
    kw = {}
    if gate:
        A_d, dt_d = A_log.cuda().requires_grad_(True), dt_bias.cuda().requires_grad_(True)
        kw = dict(A_log=A_d, dt_bias=dt_d)
    o, ht = gdn2.chunk_gdn2(*leaves, initial_state=h0_d, output_final_state=True,
                            use_qk_l2norm_in_kernel=l2, use_gate_in_kernel=gate, **kw)
    assert o.dtype == torch.float32
    torch.autograd.backward([o, ht], [do.cuda(), dht.cuda()])
    torch.cuda.synchronize()
    r = orc.chunk_gdn2(*(x.double().numpy() for x in (q, k, v, graw, b, w)), initial_state=h0.double().numpy(),
                       output_final_state=True, use_qk_l2norm_in_kernel=l2, use_gate_in_kernel=gate,
                       A_log=A_log.double().numpy() if gate else None,
                       dt_bias=dt_bias.double().numpy() if gate else None,
                       do=do.double().numpy(), dht=dht.double().numpy())
    assert_close(o, r.o, "o", **FP32_TOL)
    assert_close(ht, r.final_state, "ht", **FP32_TOL)
    for n, leaf in zip("qkvgbw", leaves):
        assert_close(leaf.grad, r.grads[n], f"d{n}", **FP32_TOL)
    assert_close(h0_d.grad, r.grads["h0"], "dh0", **FP32_TOL)
    if gate:
        mA, mdt = gate_param_masses(graw, dt_bias, r.grads["g"], H)
        assert_close_reduced(A_d.grad, r.grads["A_log"], mA, "dA_log", rtol=1e-5, atol=1e-4)
        assert_close_reduced(dt_d.grad, r.grads["dt_bias"], mdt, "ddt_bias", rtol=1e-5, atol=1e-4)


def test_fp32_intermediate_states_and_varlen(gdn2):
    """fp32 chunk states (return_intermediate_states, kept in fp32) and a
    packed batch with a transposed state layout on the fp32 path."""
    cu = [0, 70, 71, 200]
    T, H, K, V = cu[-1], 2, 64, 128
    g = torch.Generator().manual_seed(12)
    q, k = (torch.nn.functional.normalize(torch.randn(1, T, H, K, generator=g), dim=-1) for _ in range(2))
    v = torch.randn(1, T, H, V, generator=g)
    gg = -torch.nn.functional.softplus(torch.randn(1, T, H, K, generator=g)) * 0.1
    b = torch.sigmoid(torch.randn(1, T, H, K, generator=g))
    w = torch.sigmoid(torch.randn(1, T, H, V, generator=g))
    h0 = torch.randn(3, H, K, V, generator=g) * 0.1
    with torch.inference_mode():
        o, htT, hs = gdn2.chunk_gdn2(*(x.cuda() for x in (q, k, v, gg, b, w)),
                                     initial_state=h0.transpose(-1, -2).contiguous().cuda(),
                                     output_final_state=True, cu_seqlens=torch.tensor(cu, device="cuda"),
                                     return_intermediate_states=True, transpose_state_layout=True)
    torch.cuda.synchronize()
    assert hs.dtype == torch.float32 and hs.shape == (1, 6, H, V, K)
    r = orc.chunk_gdn2(*(x.double().numpy() for x in (q, k, v, gg, b, w)), initial_state=h0.double().numpy(),
                       output_final_state=True, cu_seqlens=cu)
    assert_close(o, r.o, "o", **FP32_TOL)
    assert_close(htT.transpose(-1, -2), r.final_state, "ht", **FP32_TOL)
    x = [t.double().numpy() for t in (q, k, v, gg, b, w)]
    # chunk c enters after the tokens [bos, t_end) of its sequence: seq 0 (70 tokens) has
    # chunks 0, 1; seq 1 (1 token) chunk 2; seq 2 (129 tokens) chunks 3, 4, 5
    starts = {0: (0, 0), 1: (0, 64), 2: (1, 70), 3: (2, 71), 4: (2, 135), 5: (2, 199)}
    for c, (n, t_end) in starts.items():
        bos = cu[n]
        if t_end == bos:
            ref = h0.double().numpy()[n]
        else:
            _, ref, _ = orc.recurrent_fwd(*(t[:, bos:t_end] for t in x), K ** -0.5, h0.double().numpy()[n:n + 1])
            ref = ref[0]
        np.testing.assert_allclose(hs[0, c].transpose(-1, -2).double().cpu().numpy(), ref, rtol=1e-4, atol=1e-4,
                                   err_msg=f"h[{c}]")


# Segmented scans (few (sequence, head) pairs, at least 32 chunks per sequence):
# the workspace plan cuts each sequence into segments, the scans run as
# segment transitions + an fp32 fold + the segments from their entering
# states.  B=1, H=2, T=2100 gives 11 segments of 3 chunks (the last chunk
# holds 52 tokens).
@pytest.mark.parametrize("B,T,H", [(1, 2100, 2), (2, 2048, 1)])
def test_segmented_scan_matches_oracle(gdn2, B, T, H):
    K = V = 128
    q, k, v, gg, b, w = _inputs(T + H, B, T, H, K, V)
    h0 = torch.randn(B, H, K, V, generator=torch.Generator().manual_seed(T)) * 0.1
    _bwd_vs_oracle(gdn2, q, k, v, gg, b, w, h0=h0, seed=T)


def test_segmented_scan_extreme_decay_is_exact(gdn2):
    """The segmented scans with channels that forget almost instantly (log-decay
    -60 per token) and a burst inside one block: the segment maps carry decays
    that underflow to zero and the fp32 folds compose them with the surviving
    channels; forward, final state and every gradient must still match.  B=1,
    H=2, T=2100 runs in 11 segments."""
    B, T, H, K, V = 1, 2100, 2, 128, 128
    q, k, v, gg, b, w = _inputs(23, B, T, H, K, V)
    gg[..., :8] = -60.0
    gg[:, 1000:1004, :, 8:16] = -30.0
    h0 = torch.randn(B, H, K, V, generator=torch.Generator().manual_seed(23)) * 0.1
    _bwd_vs_oracle(gdn2, q, k, v, gg, b, w, h0=h0, seed=23)


def test_segmented_scan_gate_l2norm_transposed_state(gdn2):
    """Segments with the gate and l2norm in the kernel and [V, K] states."""
    B, T, H, K, V = 1, 2300, 1, 128, 128
    q, k, v, gg, b, w = _inputs(31, B, T, H, K, V, bw=torch.bfloat16)
    g2 = torch.Generator().manual_seed(6)
    graw = torch.randn(B, T, H, K, generator=g2)
    A_log = torch.rand(H, generator=g2) * 2.0
    dt_bias = torch.randn(H * K, generator=g2) * 0.5
    h0 = torch.randn(B, H, K, V, generator=g2) * 0.1
    do = torch.randn(B, T, H, V, generator=g2).bfloat16()
    dht = torch.randn(B, H, K, V, generator=g2) * 0.1
    leaves = [x.cuda().requires_grad_(True) for x in (q, k, v, graw, b, w)]
    h0T = h0.transpose(-1, -2).contiguous().cuda().requires_grad_(True)
    A_d, dt_d = A_log.cuda().requires_grad_(True), dt_bias.cuda().requires_grad_(True)
    o, htT = gdn2.chunk_gdn2(*leaves, initial_state=h0T, output_final_state=True,
                             use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True,
                             transpose_state_layout=True, A_log=A_d, dt_bias=dt_d)
    torch.autograd.backward([o, htT], [do.cuda(), dht.transpose(-1, -2).contiguous().cuda()])
    torch.cuda.synchronize()
    r = orc.chunk_gdn2(*(x.float().numpy() for x in (q, k, v, graw, b, w)), initial_state=h0.numpy(),
                       output_final_state=True, use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True,
                       A_log=A_log.numpy(), dt_bias=dt_bias.numpy(), do=do.float().numpy(), dht=dht.numpy())
    assert_close(o, r.o, "o")
    assert_close(htT.transpose(-1, -2), r.final_state, "ht")
    for n, leaf in zip("qkvgbw", leaves):
        assert_close(leaf.grad, r.grads[n], f"d{n}")
    assert_close(h0T.grad.transpose(-1, -2), r.grads["h0"], "dh0")
    mA, mdt = gate_param_masses(graw, dt_bias, r.grads["g"], H)
    assert_close_reduced(A_d.grad, r.grads["A_log"], mA, "dA_log", rtol=RTOL_SUM)
    assert_close_reduced(dt_d.grad, r.grads["dt_bias"], mdt, "ddt_bias", rtol=RTOL_SUM)


def test_segmented_intermediate_states(gdn2):
    """return_intermediate_states when the forward scan runs in segments: the
    chunk states come from the segment passes."""
    B, T, H, K, V = 1, 2100, 1, 128, 128
    q, k, v, gg, b, w = _inputs(17, B, T, H, K, V)
    with torch.inference_mode():
        _, _, hs = gdn2.chunk_gdn2(q.cuda(), k.cuda(), v.cuda(), gg.cuda(), b.cuda(), w.cuda(),
                                   output_final_state=True, return_intermediate_states=True)
    torch.cuda.synchronize()
    x = [t.float().numpy() for t in (q, k, v, gg, b, w)]
    for c in (1, 2, 3, 4, 6, 17, 29, 30, 31, 32):  # around segment boundaries (3 chunks each)
        _, ref, _ = orc.recurrent_fwd(*(t[:, :64 * c] for t in x), K ** -0.5)
        np.testing.assert_allclose(hs[:, c].float().cpu().numpy(), ref, rtol=2e-3 + 2 ** -8, atol=1e-2,
                                   err_msg=f"h[{c}]")


def test_no_bounded_wait_gave_up(gdn2):
    """The tensor-core kernels run above bound every barrier wait; none of
    them may have given up (that would mean invalid results above)."""
    assert gdn2._lib.device_fault_read(clear=True) == 0
