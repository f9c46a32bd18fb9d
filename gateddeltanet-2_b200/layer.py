"""GatedDeltaNet2 token mixer on the B200 operator.

Drop-in for ``lit_gpt/gdn2.py:GatedDeltaNet2`` (constructor ``:95-228``,
forward ``:230-467``): the same constructor arguments, parameter names and
shapes (a reference state dict loads unchanged), the same forward signature
and return value ``(o, None, past_key_values)``.

What runs where:

* the seven first-stage projections: one GEMM over the concatenated weights
  (``gdn2.py:300-325``; cuBLAS through ``F.linear``);
* ``layer_prep_fwd_kernel`` (``gdn2_layer_prep_fwd``): the short convolutions
  with SiLU on q, k, v, the sigmoid gates b, w (times 2 with
  ``allow_neg_eigval``) and contiguous copies of the two second-stage GEMM
  inputs, in one pass over the projection output.  Its backward
  (``gdn2_layer_prep_bwd``) writes the projection cotangent in one pass and
  the conv weight gradients;
* the second-stage f / g GEMMs (cuBLAS);
* ``chunk_gdn2`` (training / prefill; gate activation and q/k l2norm fused
  into the operator) or ``fused_recurrent_gdn2`` (decode of <= 64 tokens
  outside training), both this package's CUDA operators;
* ``norm_gate_fwd/bwd_kernel`` (``gdn2_norm_gate_fwd/bwd``): the SiLU-gated
  RMSNorm, then the output GEMM (cuBLAS).

The reference's environment switches (``GDN2_FUSED_PROJ``,
``GDN2_GATE_IN_KERNEL``, ``GDN2_GATE_MIN_DECAY``, ``GDN2_BETA_MAX``) are not
read: the projections are always merged and the gate runs inside the
operator whenever the reference's default would (chunk mode, no grouped
value heads).
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .chunk import chunk_gdn2
from .recurrent import fused_recurrent_gdn2


# ---------------------------------------------------------------------------
# autograd functions over the layer kernels
# ---------------------------------------------------------------------------
def _prep_args(proj, T, N, cu, Dk, Dv, Dfg, conv_size, b_scale, conv_w, conv_b, state_in, state_out, outs):
    q, k, v, b, w, f0, g0 = outs
    return _lib.PrepArgs(
        rows=proj.shape[0], T=T, N=N, cu_seqlens=_lib.ptr(cu), Dk=Dk, Dv=Dv, Dfg=Dfg,
        conv_size=conv_size, proj_stride=proj.stride(0), b_scale=b_scale, flags=0,
        proj=proj.data_ptr(), conv_weight=_lib.ptr(conv_w), conv_bias=_lib.ptr(conv_b),
        conv_state_in=_lib.ptr(state_in), conv_state_out=_lib.ptr(state_out),
        q=_lib.ptr(q), k=_lib.ptr(k), v=_lib.ptr(v), b=_lib.ptr(b), w=_lib.ptr(w),
        f0=_lib.ptr(f0), g0=_lib.ptr(g0))


class LayerPrepFunction(torch.autograd.Function):
    """proj [rows, 3Dk+2Dv+2Dfg] bf16 -> q, k, v, b, w, f0, g0 (bf16, contiguous)
    and the final conv state (inference cache, no gradient)."""

    @staticmethod
    def forward(ctx, proj, conv_w, conv_b, Dk, Dv, Dfg, T, N, cu, conv_size, b_scale, state_in, want_state):
        _lib.require_device(proj)
        assert proj.dtype == torch.bfloat16 and proj.stride(1) == 1
        rows, dev = proj.shape[0], proj.device
        outs = [torch.empty(rows, d, device=dev, dtype=torch.bfloat16) for d in (Dk, Dk, Dv, Dk, Dv, Dfg, Dfg)]
        C = 2 * Dk + Dv
        state_out = (torch.empty(N, C, conv_size, device=dev, dtype=torch.bfloat16)
                     if (want_state and conv_size > 0) else None)
        cw = conv_w.detach().to(torch.float32).contiguous() if conv_w is not None else None
        cb = conv_b.detach().to(torch.float32).contiguous() if conv_b is not None else None
        sin = state_in.to(torch.bfloat16).contiguous() if state_in is not None else None
        args = _prep_args(proj, T, N, cu, Dk, Dv, Dfg, conv_size, b_scale, cw, cb, sin, state_out, outs)
        _lib.check(_lib.load().gdn2_layer_prep_fwd(args, _lib.stream_ptr(dev)), "gdn2_layer_prep_fwd")
        ctx.save_for_backward(proj, cw, cb, sin, cu)
        ctx.meta = (Dk, Dv, Dfg, T, N, conv_size, b_scale, conv_w is not None and conv_w.dtype,
                    conv_b is not None and conv_b.dtype)
        ctx.mark_non_differentiable(*([state_out] if state_out is not None else []))
        return (*outs, state_out)

    @staticmethod
    def backward(ctx, dq, dk, dv, db, dw, df0, dg0, _dstate):
        proj, cw, cb, sin, cu = ctx.saved_tensors
        Dk, Dv, Dfg, T, N, conv_size, b_scale, cw_dtype, cb_dtype = ctx.meta
        dev, rows = proj.device, proj.shape[0]

        def bf(t, d):
            if t is None:
                return torch.zeros(rows, d, device=dev, dtype=torch.bfloat16)
            return t.to(torch.bfloat16).contiguous()

        grads = [bf(dq, Dk), bf(dk, Dk), bf(dv, Dv), bf(db, Dk), bf(dw, Dv)]
        gf0 = df0.to(torch.bfloat16).contiguous() if df0 is not None else None
        gg0 = dg0.to(torch.bfloat16).contiguous() if dg0 is not None else None
        if (gf0 is None) != (gg0 is None):
            gf0 = gf0 if gf0 is not None else torch.zeros(rows, Dfg, device=dev, dtype=torch.bfloat16)
            gg0 = gg0 if gg0 is not None else torch.zeros(rows, Dfg, device=dev, dtype=torch.bfloat16)
        # same row stride as proj: the kernel addresses both with it
        dproj = torch.empty(rows, proj.stride(0), device=dev, dtype=torch.bfloat16)[:, :proj.shape[1]]
        C = 2 * Dk + Dv
        dcw = torch.empty(C, conv_size, device=dev, dtype=torch.float32) if conv_size > 0 else None
        dcb = torch.empty(C, device=dev, dtype=torch.float32) if (cb is not None and conv_size > 0) else None
        f0_dummy = proj if Dfg > 0 else None  # non-NULL f0 / g0 select the copy sections
        args = _prep_args(proj, T, N, cu, Dk, Dv, Dfg, conv_size, b_scale, cw, cb, sin, None,
                          [proj, proj, proj, proj, proj, f0_dummy, f0_dummy])
        gr = _lib.PrepGrads(dq=grads[0].data_ptr(), dk=grads[1].data_ptr(), dv=grads[2].data_ptr(),
                            db=grads[3].data_ptr(), dw=grads[4].data_ptr(), df0=_lib.ptr(gf0),
                            dg0=_lib.ptr(gg0), dproj=dproj.data_ptr(), dconv_weight=_lib.ptr(dcw),
                            dconv_bias=_lib.ptr(dcb))
        lib = _lib.load()
        ws_bytes = lib.gdn2_layer_prep_bwd_workspace_size(args)
        ws = torch.empty(max(ws_bytes, 1), device=dev, dtype=torch.uint8)
        _lib.check(lib.gdn2_layer_prep_bwd(args, gr, ws.data_ptr(), ws_bytes, _lib.stream_ptr(dev)),
                   "gdn2_layer_prep_bwd")
        if dproj.shape[1] > 3 * Dk + 2 * Dv + 2 * Dfg:
            dproj[:, 3 * Dk + 2 * Dv + 2 * Dfg:] = 0
        dcw_out = dcw.to(cw_dtype) if (dcw is not None and ctx.needs_input_grad[1]) else None
        dcb_out = dcb.to(cb_dtype) if (dcb is not None and ctx.needs_input_grad[2]) else None
        return (dproj, dcw_out, dcb_out) + (None,) * 10


class NormGateFunction(torch.autograd.Function):
    """y = x / sqrt(mean(x^2) + eps) * weight * gate * sigmoid(gate) over rows of D."""

    @staticmethod
    def forward(ctx, x, gate, weight, eps):
        _lib.require_device(x)
        D = x.shape[-1]
        xs = x.to(torch.bfloat16).reshape(-1, D).contiguous()
        gs = gate.to(torch.bfloat16).reshape(-1, D).contiguous()
        wf = weight.detach().to(torch.float32).contiguous()
        rows = xs.shape[0]
        y = torch.empty_like(xs)
        rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
        _lib.check(_lib.load().gdn2_norm_gate_fwd(xs.data_ptr(), gs.data_ptr(), wf.data_ptr(), float(eps), rows, D,
                                                  y.data_ptr(), rstd.data_ptr(), _lib.stream_ptr(x.device)),
                   "gdn2_norm_gate_fwd")
        ctx.save_for_backward(xs, gs, wf, rstd)
        ctx.meta = (x.shape, x.dtype, gate.shape, gate.dtype, weight.dtype)
        return y.view(x.shape).to(x.dtype)

    @staticmethod
    def backward(ctx, dy):
        xs, gs, wf, rstd = ctx.saved_tensors
        xshape, xdtype, gshape, gdtype, wdtype = ctx.meta
        rows, D = xs.shape
        dys = dy.to(torch.bfloat16).reshape(rows, D).contiguous()
        dx = torch.empty_like(xs)
        dg = torch.empty_like(gs)
        dwt = torch.empty(D, device=xs.device, dtype=torch.float32)
        lib = _lib.load()
        ws_bytes = lib.gdn2_norm_gate_bwd_workspace_size(rows, D)
        ws = torch.empty(max(ws_bytes, 1), device=xs.device, dtype=torch.uint8)
        _lib.check(lib.gdn2_norm_gate_bwd(dys.data_ptr(), xs.data_ptr(), gs.data_ptr(), wf.data_ptr(),
                                          rstd.data_ptr(), rows, D, dx.data_ptr(), dg.data_ptr(), dwt.data_ptr(),
                                          ws.data_ptr(), ws_bytes, _lib.stream_ptr(xs.device)),
                   "gdn2_norm_gate_bwd")
        return dx.view(xshape).to(xdtype), dg.view(gshape).to(gdtype), dwt.to(wdtype), None


# ---------------------------------------------------------------------------
# modules (parameter names and shapes of the reference's fla modules)
# ---------------------------------------------------------------------------
class ShortConvolution(nn.Conv1d):
    """Parameter holder with fla ShortConvolution's layout (weight [D, 1, W],
    optional bias [D]); the convolution itself runs inside the layer's prep
    kernel, fused with its neighbours."""

    def __init__(self, hidden_size: int, kernel_size: int, bias: bool = False, activation: str | None = "silu",
                 **kwargs):
        super().__init__(hidden_size, hidden_size, kernel_size, groups=hidden_size, bias=bias,
                         padding=kernel_size - 1)
        if activation not in ("silu", "swish"):
            raise ValueError(f"Activation `{activation}` not supported: the fused prep kernel applies SiLU.")
        self.hidden_size = hidden_size
        self.activation = activation

    def forward(self, *args, **kwargs):
        raise RuntimeError("ShortConvolution runs inside GatedDeltaNet2's fused prep kernel")


class FusedRMSNormSwishGate(nn.Module):
    """fla FusedRMSNormSwishGate (weight [hidden_size], ones) on the CUDA norm kernels."""

    def __init__(self, hidden_size: int, elementwise_affine: bool = True, eps: float = 1e-5, **kwargs):
        super().__init__()
        if not elementwise_affine:
            raise ValueError("FusedRMSNormSwishGate here keeps its weight (elementwise_affine=True)")
        if hidden_size not in (64, 128, 256):
            raise ValueError(f"gated norm width must be 64, 128 or 256, got {hidden_size}")
        self.hidden_size = hidden_size
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
        return NormGateFunction.apply(x, g, self.weight, self.eps)


class LayerCache:
    """Minimal per-layer state cache with fla's ``Cache`` access pattern
    (``len``, ``[layer_idx]``, ``update(layer_idx=..., recurrent_state=...,
    conv_state=..., offset=...)``)."""

    def __init__(self):
        self.states: list[dict] = []
        self.seen_tokens = 0

    def __len__(self):
        return len(self.states)

    def __getitem__(self, i):
        return self.states[i]

    def update(self, layer_idx: int, recurrent_state=None, conv_state=None, offset: int = 1, **kwargs):
        while len(self.states) <= layer_idx:
            self.states.append(dict(recurrent_state=None, conv_state=None))
        st = self.states[layer_idx]
        if recurrent_state is not None:
            st["recurrent_state"] = recurrent_state
        if conv_state is not None:
            st["conv_state"] = conv_state
        if layer_idx == 0:
            self.seen_tokens += offset
        return st


def _unpad(attention_mask: torch.Tensor):
    """(indices of kept tokens, cu_seqlens int64) of a [B, T] 0/1 mask."""
    lens = attention_mask.sum(-1, dtype=torch.int64)
    indices = torch.nonzero(attention_mask.flatten(), as_tuple=False).flatten()
    cu = F.pad(lens.cumsum(0), (1, 0))
    return indices, cu


class GatedDeltaNet2(nn.Module):
    """Gated DeltaNet 2 token mixer (``lit_gpt/gdn2.py:49-467``) on B200 kernels.

    S_t = (I - k_t (b_t * k_t)^T) Diag(exp(g_t)) S_{t-1} + k_t (w_t * v_t)^T
    """

    def __init__(
        self,
        hidden_size: int = 2048,
        expand_v: float = 1,
        head_dim: int = 128,
        num_heads: int = 16,
        num_v_heads: int | None = None,
        mode: str = "chunk",
        use_short_conv: bool = True,
        allow_neg_eigval: bool = False,
        conv_size: int = 4,
        conv_bias: bool = False,
        layer_idx: int | None = None,
        norm_eps: float = 1e-5,
        **kwargs,
    ):
        super().__init__()
        self.mode = mode
        self.allow_neg_eigval = allow_neg_eigval
        self.hidden_size = hidden_size
        self.expand_v = expand_v
        self.use_short_conv = use_short_conv
        self.conv_size = conv_size
        self.conv_bias = conv_bias
        self.head_dim = head_dim
        self.num_heads = num_heads
        self.num_v_heads = num_v_heads if num_v_heads is not None else num_heads
        self.head_k_dim = head_dim
        self.head_v_dim = int(self.head_dim * self.expand_v)
        self.key_dim = int(self.num_heads * self.head_k_dim)
        self.value_dim = int(self.num_v_heads * self.head_v_dim)
        self.layer_idx = layer_idx

        if not math.isclose(self.num_v_heads * self.head_dim * expand_v, self.value_dim, rel_tol=1e-5):
            raise ValueError(
                f"expand_v={expand_v} does not produce an integer value when multiplied by key_dim={self.key_dim}. "
                f"Resulting value_dim would be {self.num_v_heads * self.head_dim * expand_v}, which is invalid "
                "for nn.Linear.")
        if self.num_v_heads > self.num_heads and self.num_v_heads % self.num_heads != 0:
            raise ValueError(f"num_v_heads={self.num_v_heads} must be divisible by num_heads={self.num_heads}.")
        if not math.isclose(head_dim * expand_v, self.head_v_dim, rel_tol=1e-5):
            raise ValueError(
                f"expand_v={expand_v} does not produce an integer value when multiplied by head_dim={head_dim}. "
                f"Resulting head_v_dim would be {head_dim * expand_v}, which is invalid for FusedRMSNormSwishGate.")
        assert mode in ["chunk", "fused_recurrent"], f"Not supported mode `{mode}`."
        if use_short_conv and conv_size not in (2, 3, 4):
            raise ValueError(f"conv_size must be 2, 3 or 4 for the fused prep kernel, got {conv_size}")

        self.q_proj = nn.Linear(hidden_size, self.key_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, self.key_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, self.value_dim, bias=False)
        if use_short_conv:
            self.q_conv1d = ShortConvolution(self.key_dim, conv_size, bias=conv_bias, activation="silu")
            self.k_conv1d = ShortConvolution(self.key_dim, conv_size, bias=conv_bias, activation="silu")
            self.v_conv1d = ShortConvolution(self.value_dim, conv_size, bias=conv_bias, activation="silu")
        self.f_proj = nn.Sequential(
            nn.Linear(hidden_size, self.head_v_dim, bias=False),
            nn.Linear(self.head_v_dim, self.key_dim, bias=False),
        )
        self.b_proj = nn.Linear(hidden_size, self.key_dim, bias=False)
        self.w_proj = nn.Linear(hidden_size, self.value_dim, bias=False)
        self.A_log = nn.Parameter(torch.log(torch.empty(self.num_heads, dtype=torch.float32).uniform_(1, 16)))
        self.A_log._no_weight_decay = True
        dt = torch.exp(
            torch.rand(self.key_dim, dtype=torch.float32) * (math.log(0.1) - math.log(0.001)) + math.log(0.001)
        ).clamp(min=1e-4)
        inv_dt = dt + torch.log(-torch.expm1(-dt))
        self.dt_bias = nn.Parameter(inv_dt)
        self.dt_bias._no_weight_decay = True
        self.g_proj = nn.Sequential(
            nn.Linear(hidden_size, self.head_v_dim, bias=False),
            nn.Linear(self.head_v_dim, self.value_dim, bias=True),
        )
        self.o_norm = FusedRMSNormSwishGate(self.head_v_dim, eps=norm_eps)
        self.o_proj = nn.Linear(self.value_dim, hidden_size, bias=False)
        self.apply(self._initialize_weights)

    def _initialize_weights(self, module: nn.Module):
        if getattr(module, "_is_hf_initialized", False):
            return
        if isinstance(module, nn.Linear):
            nn.init.xavier_uniform_(module.weight, gain=2 ** -2.5)
            if module.bias is not None:
                nn.init.zeros_(module.bias)
        module._is_hf_initialized = True

    # the three conv weights as one [2Dk+Dv, W] matrix (and bias), in the
    # prep kernel's channel order q | k | v
    def _conv_params(self):
        if not self.use_short_conv:
            return None, None
        W = self.conv_size
        convs = (self.q_conv1d, self.k_conv1d, self.v_conv1d)
        w = torch.cat([c.weight.reshape(c.hidden_size, W) for c in convs], 0)
        b = torch.cat([c.bias for c in convs], 0) if self.conv_bias else None
        return w, b

    def forward(self, hidden_states, attention_mask=None, past_key_values=None, use_cache=False,
                output_attentions=False, **kwargs):
        if attention_mask is not None:
            assert len(attention_mask.shape) == 2, (
                "Expected attention_mask as a 0-1 matrix with shape [batch_size, seq_len] "
                "for padding purposes (0 indicating padding). "
                "Arbitrary attention masks of shape [batch_size, seq_len, seq_len] are not allowed.")
        batch_size, q_len, _ = hidden_states.shape
        mode = "fused_recurrent" if (q_len <= 64 and not self.training) else self.mode
        if self.training:
            assert mode == "chunk", "Only chunk mode is supported in training."

        last_state = None
        if past_key_values is not None:
            if self.layer_idx is None:
                raise ValueError("a layer_idx is required to use a cache")
            if len(past_key_values) > self.layer_idx:
                last_state = past_key_values[self.layer_idx]

        cu_seqlens = kwargs.get("cu_seqlens")
        indices = None
        if attention_mask is not None:
            indices, cu_seqlens = _unpad(attention_mask[:, -q_len:])
            hidden_states = hidden_states.reshape(-1, hidden_states.shape[-1]).index_select(0, indices).unsqueeze(0)
        if cu_seqlens is not None:
            cu_seqlens = cu_seqlens.to(device=hidden_states.device, dtype=torch.int64)
        B, T = hidden_states.shape[:2]
        N = B if cu_seqlens is None else len(cu_seqlens) - 1

        w_cat = torch.cat((self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self.b_proj.weight,
                           self.w_proj.weight, self.f_proj[0].weight, self.g_proj[0].weight), dim=0)
        fused = F.linear(hidden_states, w_cat)
        proj = fused.reshape(B * T, fused.shape[-1])
        if proj.dtype != torch.bfloat16:
            proj = proj.to(torch.bfloat16)

        conv_in = None
        if self.use_short_conv and last_state is not None and last_state.get("conv_state") is not None:
            conv_in = torch.cat(tuple(last_state["conv_state"]), 1)
        conv_w, conv_b = self._conv_params()
        Dk, Dv, Dfg = self.key_dim, self.value_dim, self.head_v_dim
        b_scale = 2.0 if self.allow_neg_eigval else 1.0
        q, k, v, b, w, f0, g0, conv_out = LayerPrepFunction.apply(
            proj, conv_w, conv_b, Dk, Dv, Dfg, T, N, cu_seqlens, self.conv_size if self.use_short_conv else 0,
            b_scale, conv_in, bool(use_cache))
        f_pre = self.f_proj[1](f0)
        g_gate = self.g_proj[1](g0)

        H, HV, K, V = self.num_heads, self.num_v_heads, self.head_k_dim, self.head_v_dim
        gate_in_kernel = mode == "chunk" and HV == H
        if gate_in_kernel:
            g = f_pre
        else:
            g = -self.A_log.float().exp().repeat_interleave(K) * F.softplus(f_pre.float() + self.dt_bias)
        q, k, g, b = (x.reshape(B, T, H, K) for x in (q, k, g, b))
        v, w = v.reshape(B, T, HV, V), w.reshape(B, T, HV, V)
        if HV > H:
            q, k, g, b = (x.repeat_interleave(HV // H, dim=2) for x in (q, k, g, b))

        recurrent_state = last_state["recurrent_state"] if last_state is not None else None
        if mode == "chunk":
            o, recurrent_state = chunk_gdn2(
                q=q, k=k, v=v, g=g, b=b, w=w, A_log=self.A_log, dt_bias=self.dt_bias,
                initial_state=recurrent_state, output_final_state=use_cache, use_qk_l2norm_in_kernel=True,
                use_gate_in_kernel=gate_in_kernel, cu_seqlens=cu_seqlens)
        else:
            o, recurrent_state = fused_recurrent_gdn2(
                q=q, k=k, v=v, g=g, b=b, w=w, A_log=self.A_log, dt_bias=self.dt_bias,
                initial_state=recurrent_state, output_final_state=use_cache, use_qk_l2norm_in_kernel=True,
                use_gate_in_kernel=False, cu_seqlens=cu_seqlens)

        if past_key_values is not None:
            conv_state = None
            if conv_out is not None:
                conv_state = (conv_out[:, :Dk], conv_out[:, Dk:2 * Dk], conv_out[:, 2 * Dk:])
            past_key_values.update(layer_idx=self.layer_idx, recurrent_state=recurrent_state,
                                   conv_state=conv_state, offset=q_len)

        o = self.o_norm(o, g_gate.reshape(B, T, HV, V))
        o = self.o_proj(o.reshape(B, T, HV * V))
        if attention_mask is not None:
            out = o.new_zeros(batch_size * q_len, o.shape[-1])
            out.index_copy_(0, indices, o.squeeze(0))
            o = out.view(batch_size, q_len, -1)
        return o, None, past_key_values
