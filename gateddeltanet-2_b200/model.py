"""Hybrid GDN2 / sliding-window-attention language model on the B200 operator.

The config-4 workload: a ~1.3B decoder whose token mixers alternate between
``GatedDeltaNet2`` (this package's layer, CUDA kernels end to end) and causal
sliding-window attention, with pre-norm residual blocks, SwiGLU MLPs and
RMSNorm.  Structure, parameter names and initialisation follow the
reference's ``lit_gpt/model.py``: ``GPT`` (``:27-153``: ``wte`` -> blocks ->
``ln_f`` -> ``lm_head``), ``Block`` (``:206-247``: every ``gdn2_per_layer``-th
block mixes with ``GatedDeltaNet2``), ``CausalSelfAttention`` (``:250-334``:
fused per-head qkv projection, RoPE on q and k in fp32, flash attention with
window ``(local_window - 1, 0)``) and ``SwiGLU`` (``:401-412``), so a
reference state dict for the same shape loads unchanged.

Only the GDN2 mixers are this build's kernels.  Attention runs flash_attn's
library kernel (``flash_attn_func`` with a window, as the reference does);
the GEMMs run cuBLAS; RMSNorm, RoPE, SwiGLU's gate and the loss are torch.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .layer import GatedDeltaNet2


@dataclass
class HybridConfig:
    """Config 4: d_model 2048, 24 layers alternating GDN2 (16 heads, d_k = d_v
    = 128) and 2048-window attention, SwiGLU, RMSNorm, vocab 32000, seq 4096.
    intermediate_size 4608 puts the model at 1.33B parameters."""
    vocab_size: int = 32000
    padding_multiple: int = 64
    n_layer: int = 24
    n_embd: int = 2048
    n_head: int = 16
    intermediate_size: int = 4608
    gdn2_per_layer: int = 2
    local_window: int = 2048
    norm_eps: float = 1e-5
    block_size: int = 4096
    rope_base: int = 10000
    mamba_init: bool = True

    @property
    def head_size(self) -> int:
        return self.n_embd // self.n_head

    @property
    def padded_vocab_size(self) -> int:
        m = self.padding_multiple
        return ((self.vocab_size + m - 1) // m) * m


class RMSNorm(nn.Module):
    """y = x / sqrt(mean(x^2) + eps) * weight (the reference's FusedRMSNorm)."""

    def __init__(self, size: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(size))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.rms_norm(x, (x.shape[-1],), self.weight, self.eps)


def build_rope_cache(seq_len: int, n_elem: int, device, base: int = 10000):
    """cos, sin [seq_len, n_elem / 2] (``lit_gpt/model.py:374-398``)."""
    theta = 1.0 / (base ** (torch.arange(0, n_elem, 2, device=device, dtype=torch.float32) / n_elem))
    idx_theta = torch.outer(torch.arange(seq_len, device=device, dtype=torch.float32), theta)
    return torch.cos(idx_theta), torch.sin(idx_theta)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate the two halves of each head (non-interleaved), in fp32; x [B, T, H, D]."""
    xf = x.float()
    half = xf.shape[-1] // 2
    x1, x2 = xf[..., :half], xf[..., half:]
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1).to(x.dtype)


class CausalSelfAttention(nn.Module):
    """Sliding-window causal attention with RoPE (``lit_gpt/model.py:250-334``)."""

    def __init__(self, config: HybridConfig):
        super().__init__()
        self.n_head, self.head_size = config.n_head, config.head_size
        self.attn = nn.Linear(config.n_embd, 3 * config.n_embd, bias=False)
        self.proj = nn.Linear(config.n_embd, config.n_embd, bias=False)
        self.window = config.local_window

    def forward(self, x: torch.Tensor, rope) -> torch.Tensor:
        from flash_attn import flash_attn_func
        B, T, C = x.shape
        # per head: (q, k, v) consecutive, as the reference's grouped layout with one query per group
        qkv = self.attn(x).view(B, T, self.n_head, 3, self.head_size)
        q, k, v = qkv.unbind(dim=3)
        cos, sin = rope
        q, k = apply_rope(q, cos[:T], sin[:T]), apply_rope(k, cos[:T], sin[:T])
        o = flash_attn_func(q, k, v.contiguous(), causal=True,
                            window_size=(-1, -1) if self.window is None else (self.window - 1, 0))
        return self.proj(o.reshape(B, T, C))


class SwiGLU(nn.Module):
    def __init__(self, in_features: int, hidden_features: int):
        super().__init__()
        self.w1 = nn.Linear(in_features, hidden_features, bias=False)
        self.w2 = nn.Linear(in_features, hidden_features, bias=False)
        self.w3 = nn.Linear(hidden_features, in_features, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.w3(F.silu(self.w1(x)) * self.w2(x))


class LLaMAMLP(nn.Module):
    def __init__(self, config: HybridConfig):
        super().__init__()
        self.swiglu = SwiGLU(config.n_embd, config.intermediate_size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.swiglu(x)


class Block(nn.Module):
    """Pre-norm residual block (``lit_gpt/model.py:206-247``)."""

    def __init__(self, config: HybridConfig, layer_idx: int, gdn2_cls=None):
        super().__init__()
        self.norm_1 = RMSNorm(config.n_embd, eps=config.norm_eps)
        self.use_gdn2 = config.gdn2_per_layer > 0 and layer_idx % config.gdn2_per_layer == 0
        if self.use_gdn2:
            self.attn = (gdn2_cls or GatedDeltaNet2)(hidden_size=config.n_embd, head_dim=config.head_size,
                                                     num_heads=config.n_head, layer_idx=layer_idx)
        else:
            self.attn = CausalSelfAttention(config)
        self.norm_2 = RMSNorm(config.n_embd, eps=config.norm_eps)
        self.mlp = LLaMAMLP(config)

    def forward(self, x: torch.Tensor, rope) -> torch.Tensor:
        n_1 = self.norm_1(x)
        h = self.attn(n_1)[0] if self.use_gdn2 else self.attn(n_1, rope)
        x = x + h
        return x + self.mlp(self.norm_2(x))


class GPT(nn.Module):
    """``lit_gpt/model.py:27-153`` for training (no KV cache).  ``gdn2_cls``
    swaps the GDN2 mixer class (same constructor and state dict), e.g. for
    timing the reference's own layer in the same model."""

    def __init__(self, config: HybridConfig, gdn2_cls=None):
        super().__init__()
        self.config = config
        self.lm_head = nn.Linear(config.n_embd, config.padded_vocab_size, bias=False)
        self.transformer = nn.ModuleDict(dict(
            wte=nn.Embedding(config.padded_vocab_size, config.n_embd),
            h=nn.ModuleList(Block(config, i, gdn2_cls) for i in range(config.n_layer)),
            ln_f=RMSNorm(config.n_embd, eps=config.norm_eps),
        ))
        self.rope_cache = None

    def init_weights(self) -> None:
        """The reference's ``_init_weights`` with ``mamba_init`` (``lit_gpt/model.py:47-78``):
        embedding N(0, 0.02), biases zero (except GDN2's), residual output projections
        kaiming-uniform / sqrt(2 n_layer); the GDN2 layers keep their own init."""
        n_layer = self.config.n_layer
        for module in self.modules():
            if isinstance(module, nn.Embedding):
                nn.init.normal_(module.weight, std=0.02)
        for blk in self.transformer.h:
            outs = [blk.mlp.swiglu.w3.weight]
            if not blk.use_gdn2:
                outs.append(blk.attn.proj.weight)
            for p in outs:
                nn.init.kaiming_uniform_(p, a=math.sqrt(5))
                with torch.no_grad():
                    p /= math.sqrt(2 * n_layer)

    def forward(self, idx: torch.Tensor) -> torch.Tensor:
        B, T = idx.shape
        if self.rope_cache is None or self.rope_cache[0].shape[0] < T or self.rope_cache[0].device != idx.device:
            self.rope_cache = build_rope_cache(max(T, self.config.block_size), self.config.head_size,
                                               idx.device, self.config.rope_base)
        x = self.transformer.wte(idx)
        for blk in self.transformer.h:
            x = blk(x, self.rope_cache)
        return self.lm_head(self.transformer.ln_f(x))


def num_parameters(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())


def train_step(model: nn.Module, optimizer, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """One training step: bf16 autocast forward, cross-entropy, backward, optimizer
    step (gradients all-reduced by DDP when ``model`` is wrapped).  Returns the loss."""
    optimizer.zero_grad(set_to_none=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits = model(idx)
    loss = F.cross_entropy(logits.float().view(-1, logits.shape[-1]), targets.view(-1))
    loss.backward()
    optimizer.step()
    return loss.detach()
