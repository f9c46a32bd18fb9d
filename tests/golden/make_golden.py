"""Generate the golden vectors in this folder from the reference's own kernels.

The reference (chutesai/GatedDeltaNet-2) ships no tests and no fixtures, so
its outputs are produced here by running its unmodified Triton kernels on the
CPU through the Triton interpreter (``TRITON_INTERPRET=1``).  This script only
runs where the reference checkout is present (the build container); the
``.npz`` files it writes are committed and are what the tests read.

Harness-side shims (the reference files themselves are never edited):

1. ``fla.utils.custom_device_ctx`` -> ``nullcontext``: ``input_guard`` calls
   ``torch.cpu.device``, which does not exist.
2. ``triton.runtime.autotuner.Autotuner._bench`` -> constant timings: there is
   no GPU to benchmark configurations on, so the first config is taken.
3. ``fla.utils.IS_GATHER_SUPPORTED = False``: the interpreter cannot run fla's
   ``gather``; the reference's non-gather branch is taken instead.
4. The reference modules are imported from a temporary copy in which the
   loop-index casts ``i_t.to(tl.int64)`` (``chunk_kda.py:1092``, ``:1457``,
   ``:3884``; ``chunk_gdn2.py:1593``) read ``tl.cast(i_t, tl.int64)``; the
   interpreter hands those loops a Python int, which has no ``.to``.
5. ``GDN2_FUSE_O=1``: with the installed fla 0.5.1, the non-fused output path
   (``chunk_gdn2.py:1331-1342``) passes a keyword fla no longer accepts.
6. bf16 cases run the reference's fp32 path on bf16-valued inputs.  The
   Triton 3.6 interpreter keeps bf16 tiles as raw uint16 bits and applies
   numpy arithmetic (``np.multiply``, ``np.matmul``) to those bits unconverted
   (``triton/runtime/interpreter.py`` ``binary_op``/``create_dot``), so no
   bf16 arithmetic inside a reference kernel is meaningful under it.  q, k, v
   are therefore drawn, rounded to bf16 (that is what the fixture stores and
   what the GPU tests feed the CUDA path) and handed to the reference as fp32.
   The reference then skips its own bf16 roundings of intermediates; the
   tolerance (2e-3 relative / 1e-2 absolute) covers that difference.

Run: ``python tests/golden/make_golden.py [--ref /path/to/reference]``.
"""

from __future__ import annotations

import argparse
import contextlib
import importlib
import os
import shutil
import sys
import tempfile
import time
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _install_shims(ref_root: str):
    os.environ["TRITON_INTERPRET"] = "1"
    os.environ["GDN2_FUSE_O"] = "1"
    import warnings
    warnings.filterwarnings("ignore")
    import fla.utils as fu
    fu.custom_device_ctx = lambda index: contextlib.nullcontext()
    fu.IS_GATHER_SUPPORTED = False
    import triton.runtime.autotuner as at
    at.Autotuner._bench = lambda self, *a, **k: [1.0, 1.0, 1.0]

    tmp = tempfile.mkdtemp(prefix="gdn2_ref_")
    pkg = os.path.join(tmp, "refpkg")
    os.makedirs(os.path.join(pkg, "gdn2_ops"))
    open(os.path.join(pkg, "__init__.py"), "w").close()
    src_dir = os.path.join(ref_root, "lit_gpt", "gdn2_ops")
    for name in ("chunk_gdn2.py", "chunk_kda.py", "fused_recurrent_gdn2.py"):
        with open(os.path.join(src_dir, name)) as f:
            text = f.read()
        text = text.replace("i_t.to(tl.int64)", "tl.cast(i_t, tl.int64)")
        with open(os.path.join(pkg, "gdn2_ops", name), "w") as f:
            f.write(text)
    with open(os.path.join(pkg, "gdn2_ops", "__init__.py"), "w") as f:
        f.write("")
    sys.path.insert(0, tmp)
    chunk = importlib.import_module("refpkg.gdn2_ops.chunk_gdn2")
    rec = importlib.import_module("refpkg.gdn2_ops.fused_recurrent_gdn2")
    return chunk, rec, tmp


def _bits(x):
    """Store bf16 tensors as raw uint16 bits, others as float32."""
    import torch
    if x is None:
        return None
    x = x.detach().cpu()
    if x.dtype == torch.bfloat16:
        return x.view(torch.int16).numpy().view(np.uint16)
    return x.float().numpy()


def make_inputs(seed, B, T, H, K, V, qkv_dtype, normalize_qk=True, h0=False,
                gate_raw=False, bw_dtype=None):
    """Seeded inputs drawn as the configs describe: q,k ~ N(0,1) (then
    L2-normalised per head unless the op normalises), v ~ N(0,1),
    b = sigmoid(N(0,1)) [..,K], w = sigmoid(N(0,1)) [..,V],
    log alpha = -softplus(N(0,1)) * 0.1 (or the raw pre-activation)."""
    import torch
    import torch.nn.functional as F
    gen = torch.Generator().manual_seed(seed)
    bwd_t = bw_dtype or torch.float32
    q = torch.randn(B, T, H, K, generator=gen)
    k = torch.randn(B, T, H, K, generator=gen)
    if normalize_qk:
        q = F.normalize(q, p=2, dim=-1)
        k = F.normalize(k, p=2, dim=-1)
    v = torch.randn(B, T, H, V, generator=gen)
    b = torch.sigmoid(torch.randn(B, T, H, K, generator=gen))
    w = torch.sigmoid(torch.randn(B, T, H, V, generator=gen))
    graw = torch.randn(B, T, H, K, generator=gen)
    g = graw if gate_raw else -F.softplus(graw) * 0.1
    out = dict(q=q.to(qkv_dtype), k=k.to(qkv_dtype), v=v.to(qkv_dtype),
               g=g.float(), b=b.to(bwd_t), w=w.to(bwd_t))
    # bf16-valued inputs travel to the reference as fp32 (see note 6 above);
    # the fixture keeps the bf16 bits.
    out = {n: t.float() for n, t in out.items()}
    if h0:
        out["h0"] = torch.randn(B, H, K, V, generator=gen) * 0.1
    return out, gen


def run_chunk_case(chunk_mod, name, seed, B, T, H, K, V, qkv_dtype, *,
                   l2norm=False, gate=False, h0=False, dht=False,
                   cu_seqlens=None, lower_bound=None, transpose=False):
    import torch
    inp, gen = make_inputs(seed, B, T, H, K, V, qkv_dtype, normalize_qk=not l2norm,
                           h0=h0, gate_raw=gate)
    extra = {}
    if gate:
        extra["A_log"] = (torch.rand(H, generator=gen) * 2.0).float()
        extra["dt_bias"] = (torch.randn(H * K, generator=gen) * 0.5).float()
    N = B if cu_seqlens is None else len(cu_seqlens) - 1
    if h0 and cu_seqlens is not None:
        inp["h0"] = torch.randn(N, H, K, V, generator=gen) * 0.1
    if h0 and transpose:
        inp["h0"] = inp["h0"].transpose(-1, -2).contiguous()
    do = torch.randn(B, T, H, V, generator=gen).to(qkv_dtype).float()
    dht_t = None
    if dht:
        shp = (N, H, V, K) if transpose else (N, H, K, V)
        dht_t = torch.randn(*shp, generator=gen) * 0.1

    leaves = {n: t.clone().requires_grad_(True) for n, t in inp.items()}
    for n, t in extra.items():
        leaves[n] = t.clone().requires_grad_(True)
    cu = None if cu_seqlens is None else torch.tensor(cu_seqlens, dtype=torch.long)
    t0 = time.time()
    o, ht = chunk_mod.chunk_gdn2(
        leaves["q"], leaves["k"], leaves["v"], leaves["g"], leaves["b"], leaves["w"],
        initial_state=leaves.get("h0"), output_final_state=True,
        use_qk_l2norm_in_kernel=l2norm, use_gate_in_kernel=gate,
        cu_seqlens=cu, lower_bound=lower_bound,
        transpose_state_layout=transpose,
        **({"A_log": leaves["A_log"], "dt_bias": leaves["dt_bias"]} if gate else {}))
    t1 = time.time()
    grads = [do] + ([dht_t] if dht_t is not None else [torch.zeros_like(ht)])
    torch.autograd.backward([o, ht], grads)
    t2 = time.time()
    rec = {f"in_{n}": _bits(t.to(qkv_dtype) if n in "qkv" else t) for n, t in inp.items()}
    rec.update({f"in_{n}": _bits(t) for n, t in extra.items()})
    rec["in_do"] = _bits(do.to(qkv_dtype))
    if dht_t is not None:
        rec["in_dht"] = _bits(dht_t)
    rec["out_o"] = _bits(o)
    rec["out_ht"] = _bits(ht)
    for n, t in leaves.items():
        rec[f"grad_{n}"] = _bits(t.grad)
    meta = dict(kind="chunk", B=B, T=T, H=H, K=K, V=V, l2norm=l2norm, gate=gate,
                h0=h0, dht=dht, transpose=transpose,
                qkv_dtype=str(qkv_dtype).replace("torch.", ""),
                lower_bound=lower_bound, seed=seed,
                cu_seqlens=list(cu_seqlens) if cu_seqlens is not None else None)
    rec["meta"] = np.array(repr(meta))
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **{k: v for k, v in rec.items() if v is not None})
    print(f"{name}: fwd {t1 - t0:.1f}s bwd {t2 - t1:.1f}s -> {path}", flush=True)


def run_recurrent_case(rec_mod, name, seed, B, T, H, K, V, qkv_dtype, *,
                       l2norm=False, gate=False, cu_seqlens=None, transpose=False):
    import torch
    inp, gen = make_inputs(seed, B, T, H, K, V, qkv_dtype, normalize_qk=not l2norm,
                           gate_raw=gate)
    N = B if cu_seqlens is None else len(cu_seqlens) - 1
    h0 = torch.randn(N, H, K, V, generator=gen) * 0.02
    if transpose:
        h0 = h0.transpose(-1, -2).contiguous()
    extra = {}
    if gate:
        extra["A_log"] = (torch.rand(H, generator=gen) * 2.0).float()
        extra["dt_bias"] = (torch.randn(H * K, generator=gen) * 0.5).float()
    cu = None if cu_seqlens is None else torch.tensor(cu_seqlens, dtype=torch.long)
    t0 = time.time()
    o, ht = rec_mod.fused_recurrent_gdn2(
        inp["q"], inp["k"], inp["v"], inp["g"], inp["b"], inp["w"],
        initial_state=h0, output_final_state=True,
        use_qk_l2norm_in_kernel=l2norm, use_gate_in_kernel=gate,
        cu_seqlens=cu, transpose_state_layout=transpose, **extra)
    t1 = time.time()
    rec = {f"in_{n}": _bits(t.to(qkv_dtype) if n in "qkv" else t) for n, t in inp.items()}
    rec.update({f"in_{n}": _bits(t) for n, t in extra.items()})
    rec["in_h0"] = _bits(h0)
    rec["out_o"] = _bits(o)
    rec["out_ht"] = _bits(ht)
    meta = dict(kind="recurrent", B=B, T=T, H=H, K=K, V=V, l2norm=l2norm, gate=gate,
                transpose=transpose, qkv_dtype=str(qkv_dtype).replace("torch.", ""),
                seed=seed, cu_seqlens=list(cu_seqlens) if cu_seqlens is not None else None)
    rec["meta"] = np.array(repr(meta))
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **rec)
    print(f"{name}: fwd {t1 - t0:.1f}s -> {path}", flush=True)


CHUNK_CASES = {
    # config 1: B=1, H=2, T=256, d=64, fp32, zero initial state
    "chunk_c1_fp32": dict(seed=0, B=1, T=256, H=2, K=64, V=64, qkv="float32"),
    # bf16 training dtypes at d=128, ragged T (two full chunks + a 32-token tail),
    # random h0 and final-state cotangent, l2norm inside the op
    "chunk_bf16_d128_ragged": dict(seed=1, B=1, T=160, H=2, K=128, V=128, qkv="bfloat16",
                                   l2norm=True, h0=True, dht=True),
    # gate activation inside the op (A_log, dt_bias), as the layer calls it
    "chunk_bf16_gate": dict(seed=2, B=1, T=128, H=2, K=128, V=128, qkv="bfloat16",
                            l2norm=True, gate=True),
    # packed variable-length batch with per-sequence initial states
    "chunk_fp32_varlen": dict(seed=3, B=1, T=200, H=2, K=64, V=64, qkv="float32",
                              h0=True, dht=True, cu_seqlens=[0, 70, 134, 200]),
    # transposed state layout
    "chunk_fp32_transpose": dict(seed=4, B=1, T=96, H=1, K=64, V=64, qkv="float32",
                                 h0=True, dht=True, transpose=True),
}

RECURRENT_CASES = {
    "rec_bf16_decode": dict(seed=10, B=4, T=1, H=2, K=128, V=128, qkv="bfloat16", l2norm=True),
    "rec_bf16_multi": dict(seed=11, B=2, T=9, H=2, K=128, V=128, qkv="bfloat16"),
    "rec_fp32_gate": dict(seed=12, B=2, T=5, H=2, K=64, V=64, qkv="float32",
                          l2norm=True, gate=True),
    "rec_fp32_varlen_t": dict(seed=13, B=1, T=12, H=2, K=64, V=64, qkv="float32",
                              cu_seqlens=[0, 5, 12], transpose=True),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("GDN2_REFERENCE_ROOT"),
                    help="checkout of the reference repository (or set GDN2_REFERENCE_ROOT)")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    if not args.ref:
        ap.error("give the reference checkout with --ref or GDN2_REFERENCE_ROOT")
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    chunk_mod, rec_mod, tmp = _install_shims(args.ref)
    try:
        for name, c in RECURRENT_CASES.items():
            if args.only and args.only not in name:
                continue
            c = dict(c)
            dt = getattr(torch, c.pop("qkv"))
            run_recurrent_case(rec_mod, name, c.pop("seed"), c.pop("B"), c.pop("T"), c.pop("H"),
                               c.pop("K"), c.pop("V"), dt, **c)
        for name, c in CHUNK_CASES.items():
            if args.only and args.only not in name:
                continue
            c = dict(c)
            dt = getattr(torch, c.pop("qkv"))
            run_chunk_case(chunk_mod, name, c.pop("seed"), c.pop("B"), c.pop("T"), c.pop("H"),
                           c.pop("K"), c.pop("V"), dt, **c)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


if __name__ == "__main__":
    main()
