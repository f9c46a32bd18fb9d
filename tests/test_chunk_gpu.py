"""Chunkwise forward + backward (gdn2_chunk_fwd / gdn2_chunk_bwd through
chunk_gdn2) against the reference's golden vectors and the fp64 oracle."""

import numpy as np
import pytest
import torch

from golden_io import case_names, load_case
from oracle import gdn2_oracle as orc
from tolerance import assert_close

pytestmark = pytest.mark.gpu


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


@pytest.mark.parametrize("name", case_names("chunk"))
def test_chunk_forward_matches_reference_golden(gdn2, name):
    _, t, o, ht, _ = _run_case(gdn2, name, backward=False)
    assert_close(o, t["out_o"], "o")
    assert_close(ht, t["out_ht"], "ht")


@pytest.mark.parametrize("name", case_names("chunk"))
def test_chunk_backward_matches_reference_golden(gdn2, name):
    _, t, o, ht, leaves = _run_case(gdn2, name, backward=True)
    assert_close(o, t["out_o"], "o")
    assert_close(ht, t["out_ht"], "ht")
    for n, leaf in leaves.items():
        assert_close(leaf.grad, t[f"grad_{n}"], f"d{n}")


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
                                       (1, 130, 2, 128, 64), (1, 33, 1, 64, 64)])
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
