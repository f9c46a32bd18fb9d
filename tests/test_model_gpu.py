"""GPU checks of the config-4 hybrid model (GDN2 + sliding-window attention)
built on the B200 layer: the attention wiring against a plain PyTorch
restatement, end-to-end training on a small model, and data-parallel
gradients over NCCL (2 GPUs) against one process on the whole batch."""

import importlib
import os
import socket
import subprocess
import sys

import pytest
import torch
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _mod():
    importlib.import_module("gateddeltanet-2_b200")
    from gdn2_b200 import model
    return model


def small_config(m):
    return m.HybridConfig(vocab_size=512, n_layer=2, n_embd=256, n_head=2, intermediate_size=512,
                          local_window=64, block_size=256)


def test_sliding_window_attention_matches_sdpa(gdn2):
    """Per-head (q, k, v) split, RoPE and the (window-1, 0) window against SDPA
    with the same band mask, in fp32 on bf16 inputs."""
    m = _mod()
    cfg = small_config(m)
    torch.manual_seed(0)
    attn = m.CausalSelfAttention(cfg).cuda().to(torch.bfloat16)
    B, T = 2, 200
    x = torch.randn(B, T, cfg.n_embd, device="cuda", dtype=torch.bfloat16)
    rope = m.build_rope_cache(T, cfg.head_size, "cuda")
    with torch.no_grad():
        got = attn(x, rope).float()
        qkv = (x.float() @ attn.attn.weight.float().t()).view(B, T, cfg.n_head, 3, cfg.head_size)
        q, k, v = qkv.unbind(3)
        q = m.apply_rope(q.bfloat16(), *rope).float()
        k = m.apply_rope(k.bfloat16(), *rope).float()
        v = v.bfloat16().float()
        i = torch.arange(T, device="cuda")
        band = (i[None, :] <= i[:, None]) & (i[:, None] - i[None, :] < cfg.local_window)
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           attn_mask=band).transpose(1, 2).reshape(B, T, -1)
        ref = o @ attn.proj.weight.float().t()
    err = (got - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item(), err


def test_small_model_trains(gdn2):
    """Every parameter gets a gradient and the loss falls on a repeated batch."""
    m = _mod()
    cfg = small_config(m)
    torch.manual_seed(1)
    model = m.GPT(cfg).cuda()
    model.init_weights()
    opt = torch.optim.AdamW(model.parameters(), lr=2e-3, fused=True)
    idx = torch.randint(0, cfg.vocab_size, (2, 256), device="cuda")
    tgt = torch.randint(0, cfg.vocab_size, (2, 256), device="cuda")
    losses = []
    for step in range(40):
        losses.append(float(m.train_step(model, opt, idx, tgt)))
        if step == 0:
            for n, p in model.named_parameters():
                assert p.grad is not None and torch.isfinite(p.grad).all(), n
                assert p.grad.abs().max() > 0, f"{n}: zero gradient"
    assert all(map(lambda v: v == v, losses)), losses
    assert losses[-1] < 0.5 * losses[0], losses


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_model_ddp_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = os.path.join(ROOT, "tests", "model_ddp_check.py")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), script]
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "DDP_OK" in r.stdout
