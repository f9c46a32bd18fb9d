"""Generate golden vectors for the GatedDeltaNet2 layer's elementwise pieces.

The reference layer (``lit_gpt/gdn2.py``) wraps the GDN2 operator with two
third-party ``fla`` modules (fla 0.5.1, git bb324a32, installed in this
image; the reference pins no version):

* ``ShortConvolution`` (``gdn2.py:342-367``): a causal depthwise conv1d of
  kernel size 4 with SiLU, run by ``fla.modules.conv.triton.ops``
  ``causal_conv1d_fwd`` / ``causal_conv1d_bwd`` (varlen, initial state,
  final state);
* ``FusedRMSNormSwishGate`` (``gdn2.py:462``): ``rms_norm_gated`` from
  ``fla.modules.fused_norm_gate`` with the swish gate.

Their Triton kernels run here on the CPU through the Triton interpreter.
Shims (fla itself is untouched): ``custom_device_ctx`` -> nullcontext,
autotuner timings -> constants, and ``get_multiprocessor_count`` -> 4 in
``fla.modules.fused_norm_gate`` (the interpreter has no driver to ask).
All cases run in fp32.  No case feeds a cotangent of the final conv state:
the layer keeps that state only as an inference cache, and fla's backward
drops the cotangent of its oldest column.

``layer_full_fp32`` runs the reference's whole ``GatedDeltaNet2`` layer
(``lit_gpt/gdn2.py``, training mode, chunk path) forward and backward on a
small fp32 case, importing it from a temporary copy of ``lit_gpt`` built by
``make_golden.py``'s shims (plus ``gdn2.py`` itself, unmodified).  That case
needs the reference checkout (``--ref``, default the build container's path);
the other cases need only fla.

Run: ``python tests/golden/make_golden_layer.py [--ref /path/to/reference]``.
"""

from __future__ import annotations

import contextlib
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _shims():
    os.environ["TRITON_INTERPRET"] = "1"
    import warnings
    warnings.filterwarnings("ignore")
    import fla.utils as fu
    fu.custom_device_ctx = lambda index: contextlib.nullcontext()
    import triton.runtime.autotuner as at
    at.Autotuner._bench = lambda self, *a, **k: [1.0, 1.0, 1.0]
    import fla.modules.fused_norm_gate as fng
    fng.get_multiprocessor_count = lambda *a, **k: 4


def _save(name, meta, arrays):
    rec = {k: (None if v is None else v.detach().cpu().numpy().astype(np.float32)) for k, v in arrays.items()}
    rec["meta"] = np.array(repr(meta))
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **{k: v for k, v in rec.items() if v is not None})
    print("wrote", name)


def conv_case(name, seed, B, T, D, W, cu_seqlens=None, h0=False, bias=False, dht=False):
    import torch
    from fla.modules.conv.triton.ops import causal_conv1d_bwd, causal_conv1d_fwd
    g = torch.Generator().manual_seed(seed)
    N = B if cu_seqlens is None else len(cu_seqlens) - 1
    cu = None if cu_seqlens is None else torch.tensor(cu_seqlens, dtype=torch.long)
    x = torch.randn(B, T, D, generator=g)
    w = torch.randn(D, W, generator=g) * 0.5
    bb = torch.randn(D, generator=g) * 0.1 if bias else None
    s0 = torch.randn(N, D, W, generator=g) if h0 else None
    y, fs = causal_conv1d_fwd(x=x, weight=w, bias=bb, residual=None, initial_state=s0,
                              output_final_state=True, activation="silu", cu_seqlens=cu)
    dy = torch.randn(y.shape, generator=g)
    dfs = torch.randn(fs.shape, generator=g) if dht else None
    dx, dw, dbias, _, dh0 = causal_conv1d_bwd(x=x, dy=dy, dht=dfs, weight=w, bias=bb, residual=None,
                                               initial_state=s0, activation="silu", cu_seqlens=cu)
    meta = dict(kind="conv", B=B, T=T, D=D, W=W, cu_seqlens=cu_seqlens, h0=h0, bias=bias, dht=dht)
    _save(name, meta, dict(x=x, weight=w, bias=bb, h0=s0, y=y, final_state=fs, dy=dy, dht=dfs,
                           dx=dx, dweight=dw, dbias=dbias if bias else None, dh0=dh0 if h0 else None))


def norm_case(name, seed, R, V, eps):
    import torch
    from fla.modules.fused_norm_gate import rms_norm_gated
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(R, V, generator=g).requires_grad_()
    gate = (torch.randn(R, V, generator=g) * 2).requires_grad_()
    w = (1 + 0.1 * torch.randn(V, generator=g)).requires_grad_()
    y = rms_norm_gated(x, gate, w, None, "swish", eps=eps)
    dy = torch.randn(y.shape, generator=g)
    y.backward(dy)
    meta = dict(kind="norm_gate", R=R, V=V, eps=eps)
    _save(name, meta, dict(x=x, gate=gate, weight=w, y=y, dy=dy, dx=x.grad, dgate=gate.grad, dweight=w.grad))


def layer_case(name, seed, ref_root, hidden, H, head_dim, T, num_v_heads=None):
    import shutil
    import sys

    import torch
    sys.path.insert(0, HERE)
    import make_golden
    _, _, pkg_root = make_golden._install_shims(ref_root)  # fla shims, patched op copies in refpkg
    shutil.copy(os.path.join(ref_root, "lit_gpt", "gdn2.py"), os.path.join(pkg_root, "refpkg", "gdn2.py"))
    import importlib
    ref = importlib.import_module("refpkg.gdn2")
    torch.manual_seed(seed)
    layer = ref.GatedDeltaNet2(hidden_size=hidden, head_dim=head_dim, num_heads=H, num_v_heads=num_v_heads,
                               conv_bias=True, allow_neg_eigval=True, layer_idx=0)
    with torch.no_grad():  # move the ones / zeros initialisations off their defaults
        layer.o_norm.weight.add_(0.1 * torch.randn_like(layer.o_norm.weight))
        layer.g_proj[1].bias.add_(0.1 * torch.randn_like(layer.g_proj[1].bias))
        for c in (layer.q_conv1d, layer.k_conv1d, layer.v_conv1d):
            c.bias.add_(0.1 * torch.randn_like(c.bias))
    layer.train()
    params = {n: p.detach().clone() for n, p in layer.named_parameters()}
    x = torch.randn(1, T, hidden).requires_grad_()
    out = layer(x)[0]
    dout = torch.randn_like(out)
    out.backward(dout)
    arrays = {"x": x, "dout": dout, "out": out, "dx": x.grad}
    for n, p in layer.named_parameters():
        arrays["p:" + n] = params[n]
        arrays["g:" + n] = p.grad
    meta = dict(kind="layer", hidden=hidden, num_heads=H, num_v_heads=num_v_heads or H, head_dim=head_dim, T=T,
                conv_size=4,
                conv_bias=True, allow_neg_eigval=True, norm_eps=1e-5)
    _save(name, meta, arrays)


def main():
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("GDN2_REFERENCE_ROOT"),
                    help="checkout of the reference repository (or set GDN2_REFERENCE_ROOT); "
                         "without it only the fla conv / norm cases are made")
    args = ap.parse_args()
    _shims()
    conv_case("layer_conv_varlen_h0", 0, 1, 100, 64, 4, cu_seqlens=[0, 2, 7, 39, 100], h0=True)
    conv_case("layer_conv_batch_bias", 1, 2, 70, 32, 4, bias=True)
    conv_case("layer_conv_k3", 2, 1, 40, 16, 3, cu_seqlens=[0, 17, 40], h0=True)
    norm_case("layer_norm_gate_v128", 3, 96, 128, 1e-5)
    norm_case("layer_norm_gate_v64", 4, 40, 64, 1e-6)
    if args.ref and os.path.isdir(args.ref):
        layer_case("layer_full_fp32", 5, args.ref, hidden=64, H=2, head_dim=64, T=100)
        # grouped value heads: 2 value heads share each key head (the gate runs in torch there)
        layer_case("layer_gva_fp32", 6, args.ref, hidden=64, H=1, head_dim=64, T=100, num_v_heads=2)


if __name__ == "__main__":
    main()
