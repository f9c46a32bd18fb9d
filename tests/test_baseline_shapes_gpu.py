"""Parity at the BASELINE.json shapes the numbers are quoted on.

* config 2: B=4, H=16, T=4096, d_k=d_v=128, bf16 q, k, v, fp32 gates: the whole
  fwd+bwd on the GPU, compared with the fp64 oracle on four sampled
  (sequence, head) pairs (outputs, final states, all six gradients);
* config 3: N=256 sequences x 16 heads, fp32 128x128 states updated in place,
  four decode steps, every sequence compared;
* config 5: one T=131072 sequence, T split over 8 context-parallel ranks
  emulated in this process (transition maps, fold, shard forwards), compared
  with the oracle on two sampled heads and with the single-GPU forward;
* also the strong-split shard of config 2 at 8 GPUs (4 sequences x 2 heads),
  where the scans run in segments.

Config 1 (fp32, B=1, H=2, T=256, d=64) is pinned against the reference's own
output at the fp32 bound in test_chunk_gpu.py."""

import importlib

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import gdn2_oracle as orc
from tolerance import assert_close

pytestmark = pytest.mark.gpu


def _config2_inputs(seed, B, T, H, K=128, V=128):
    g = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(B, T, H, K, generator=g), dim=-1).bfloat16()
    k = F.normalize(torch.randn(B, T, H, K, generator=g), dim=-1).bfloat16()
    v = torch.randn(B, T, H, V, generator=g).bfloat16()
    gg = -F.softplus(torch.randn(B, T, H, K, generator=g)) * 0.1
    b = torch.sigmoid(torch.randn(B, T, H, K, generator=g))
    w = torch.sigmoid(torch.randn(B, T, H, V, generator=g))
    do = torch.randn(B, T, H, V, generator=g).bfloat16()
    return q, k, v, gg, b, w, do


def _fwd_bwd_vs_oracle(gdn2, seed, B, T, H, pairs):
    q, k, v, gg, b, w, do = _config2_inputs(seed, B, T, H)
    leaves = [x.cuda().requires_grad_(True) for x in (q, k, v, gg, b, w)]
    o, ht = gdn2.chunk_gdn2(*leaves, output_final_state=True)
    torch.autograd.backward([o], [do.cuda()])
    torch.cuda.synchronize()
    # the sampled pairs as one oracle batch of single-head sequences
    bs, hs = [p[0] for p in pairs], [p[1] for p in pairs]
    pick = lambda x: x[bs, :, hs].unsqueeze(2).float().numpy()  # noqa: E731  [P, T, 1, D]
    r = orc.chunk_gdn2(*(pick(x) for x in (q, k, v, gg, b, w)), output_final_state=True, do=pick(do))
    got = lambda x: x.detach()[bs, :, hs].unsqueeze(2)  # noqa: E731
    assert_close(got(o), r.o, "o")
    assert_close(ht.detach()[bs, hs].unsqueeze(1), r.final_state, "ht")
    for n, leaf in zip("qkvgbw", leaves):
        assert_close(got(leaf.grad), r.grads[n], f"d{n}")


def test_config2_full_shape_sampled_pairs(gdn2):
    _fwd_bwd_vs_oracle(gdn2, 2024, 4, 4096, 16, [(0, 0), (1, 7), (2, 11), (3, 15)])


def test_config2_eight_gpu_shard(gdn2):
    """The per-GPU shard of config 2 split over 8 GPUs: 4 sequences x 2 heads,
    where the state scans run in segments."""
    _fwd_bwd_vs_oracle(gdn2, 2025, 4, 4096, 2, [(0, 0), (3, 1)])


def test_config3_decode_full_shape(gdn2):
    N, H, K, V, steps = 256, 16, 128, 128, 4
    g = torch.Generator().manual_seed(3)
    S0 = torch.randn(N, H, K, V, generator=g) * 0.02
    toks = [(F.normalize(torch.randn(N, 1, H, K, generator=g), dim=-1).bfloat16(),
             F.normalize(torch.randn(N, 1, H, K, generator=g), dim=-1).bfloat16(),
             torch.randn(N, 1, H, V, generator=g).bfloat16(),
             -F.softplus(torch.randn(N, 1, H, K, generator=g)) * 0.1,
             torch.sigmoid(torch.randn(N, 1, H, K, generator=g)),
             torch.sigmoid(torch.randn(N, 1, H, V, generator=g))) for _ in range(steps)]
    S = S0.cuda()
    outs = []
    for x in toks:
        o, _ = gdn2.fused_recurrent_gdn2_fwd(*(t.cuda() for t in x), initial_state=S, inplace_final_state=True)
        outs.append(o)
    torch.cuda.synchronize()
    Sr = S0.double().numpy()
    for i, x in enumerate(toks):
        o_ref, Sr, _ = orc.recurrent_fwd(*(t.double().numpy() for t in x), K ** -0.5, Sr)
        assert_close(outs[i], o_ref, f"o step {i}")
    assert_close(S, Sr, "state after 4 in-place steps")


def test_config5_context_parallel_sampled_heads(gdn2):
    cp = importlib.import_module("gateddeltanet-2_b200.cp")
    be = cp.CudaBackend()
    T, H, K, V, world = 131072, 16, 128, 128, 8
    q, k, v, gg, b, w, _ = _config2_inputs(5, 1, T, H)
    q, k, v, gg, b, w = (x.cuda() for x in (q, k, v, gg, b, w))
    Ts = T // world
    kw = dict(scale=K ** -0.5, use_qk_l2norm_in_kernel=False, use_gate_in_kernel=False, A_log=None,
              dt_bias=None, lower_bound=None)
    shards = [[x[:, r * Ts:(r + 1) * Ts] for x in (q, k, v, gg, b, w)] for r in range(world)]
    gathered = torch.stack([be.transition(*s, **kw) for s in shards])
    zero = torch.zeros(1, H, K, V, device="cuda")
    outs = []
    for r in range(world):
        S_in = be.compose(gathered, r, zero)
        outs.append(be.forward(*shards[r], initial_state=S_in, scale=K ** -0.5))
    o = torch.cat([x[0] for x in outs], dim=1)
    ht = outs[-1][1]
    with torch.no_grad():
        o_full, ht_full = gdn2.chunk_gdn2(q, k, v, gg, b, w, output_final_state=True)
    torch.cuda.synchronize()
    heads = [0, 9]
    x = [t[:, :, heads].float().cpu().numpy() for t in (q, k, v, gg, b, w)]
    o_ref, S_ref, _ = orc.recurrent_fwd(*x, K ** -0.5)
    assert_close(o[:, :, heads], o_ref, "o (8 emulated CP ranks)")
    assert_close(ht[:, heads], S_ref, "final state (8 emulated CP ranks)")
    assert_close(o_full[:, :, heads], o_ref, "o (one GPU)")
    assert_close(ht_full[:, heads], S_ref, "final state (one GPU)")
    assert_close(o, o_full, "o (CP vs one GPU)")
