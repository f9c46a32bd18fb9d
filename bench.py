#!/usr/bin/env python
"""Benchmark of the GDN2 operator on B200 (the headline metric of this build).

Metric: "GDN2 op fwd+bwd tokens/s (H16,d128,T4K) & decode-step state HBM GB/s".

One step = forward + backward of ``chunk_gdn2`` on config 2 (B=4, H=16,
T=4096, d_k=d_v=128, chunk 64; q,k,v bf16 with q,k L2-normalised, b,w =
sigmoid(N(0,1)) fp32, log-decay = -softplus(N(0,1))*0.1 fp32), synthetic
data.  Every rank processes its own independent batch of config-2 sequences
(the (batch x head) units shard over GPUs with no communication), so the
per-GPU work is fixed and ``scaling`` is "weak".  The decode step (config 3:
N=256 sequences, H=16, 128x128 fp32 state, updated in place) is measured in
the same run and reported under ``decode``.

``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]``
(multi-GPU through ``torch.distributed.run``; one rank per GPU).
``--batch`` / ``--decode-seqs`` shrink the two workloads for ncu captures; a
line measured with either changed is not a config-2 / config-3 number.
``--impl reference`` times the reference's algorithm on the host cores (the
oracle port: the reference has no CPU implementation of its own and its
kernels are Triton/sm_120 CUDA); it runs on rank 0 only.

``--impl reference-triton`` times the reference's own Triton op on the GPU
(the unmodified ``lit_gpt/gdn2_ops`` installed under ``baseline/_ref``) on
config 2 and config 3, next to this build's op on identical inputs, and
prints one extra JSON line (``"impl": "reference-triton"``).  Both arms get
bf16 b, w there: the reference's backward rejects fp32 ``w`` with bf16 ``v``.

``--model`` measures the config-4 training step: the 1.33B hybrid LM
(24 layers alternating GatedDeltaNet2 and 2048-window attention, SwiGLU,
RMSNorm, vocab 32000) on uniform-random token ids, seq 4096, micro-batch 4
per GPU, bf16 autocast, fused AdamW step, gradients all-reduced by DDP over
NCCL when launched with one rank per GPU.

``--cp`` measures config 5: a B=1, H=16, T=131072 prefill (forward) whose T axis
is split into equal contiguous shards over the ranks (one boundary-map
all_gather, prefix composition, shard forward from the composed state); the
whole sequence is fixed, so ``scaling`` is "strong".  Every rank also runs the
single-GPU forward of the whole sequence and reports how far its shard is from it.

``--layer`` measures instead the whole GatedDeltaNet2 token mixer
(``lit_gpt/gdn2.py``) at the config-4 layer shape (d_model 2048, 16 heads,
d=128, T=4096, micro-batch 4 per GPU), forward + backward under bf16
autocast with fp32 parameters (the reference trains ``bf16-mixed``), and
prints its own JSON line with the layer kernels' rooflines.
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GDN2 op fwd+bwd tokens/s (H16,d128,T4K) & decode-step state HBM GB/s"
B, T, H, K, V = 4, 4096, 16, 128, 128
DEC_N = 256
FALLBACK_HBM_GBS = 6650.0

# Algorithmic bytes per token-head of each kernel's interface (every input read
# once, every output written once), config-2 dtypes, no l2norm in the op.
KERNEL_BYTES_PER_TOKEN_HEAD = {
    # reads q,k,v bf16 + g,b,w fp32; writes G fp32, Aqk, A, Y, U, kg, qg bf16
    "chunk_intra_kernel": 3 * 2 * 128 + 3 * 4 * 128 + 4 * 128 + 2 * 2 * 64 + 4 * 2 * 128,
    # reads Y, qg, kg, U, Aqk; writes o, v_new and the chunk states h (K*V bf16 / 64 tokens)
    "chunk_scan_fwd_kernel": 4 * 2 * 128 + 2 * 64 + 2 * 2 * 128 + (128 * 128 * 2) // 64,
    # the same interface, on tcgen05 tensor cores (d_k = d_v = 128)
    "chunk_scan_fwd_tc_kernel": 4 * 2 * 128 + 2 * 64 + 2 * 2 * 128 + (128 * 128 * 2) // 64,
    # reads Y, qg, kg, Aqk, do; writes dh (K*V bf16 / 64 tokens) and dv_new
    "chunk_scan_bwd_kernel": 3 * 2 * 128 + 2 * 64 + 2 * 128 + (128 * 128 * 2) // 64 + 2 * 128,
    "chunk_scan_bwd_tc_kernel": 3 * 2 * 128 + 2 * 64 + 2 * 128 + (128 * 128 * 2) // 64 + 2 * 128,
    # reads h, dh, do, v_new, dv_new, A, G, q, k, b, w, v; writes dq, dk, dv, dg, db, dw
    "chunk_bwd_intra_kernel": 2 * (128 * 128 * 2) // 64 + 3 * 2 * 128 + 2 * 64 + 4 * 128
    + 2 * 2 * 128 + 2 * 4 * 128 + 2 * 128 + 3 * 2 * 128 + 3 * 4 * 128,
}
# decode: fp32 state read + write per (sequence, head) plus per-token vectors
def decode_bytes_per_step(n):
    return 2 * n * H * K * V * 4 + n * H * (3 * 2 * 128 + 3 * 4 * 128) + n * H * V * 2


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-triton"])
    ap.add_argument("--decode-steps", type=int, default=1024)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=B,
                    help="sequences per GPU (config 2 is 4; smaller values are for ncu captures)")
    ap.add_argument("--decode-seqs", type=int, default=DEC_N,
                    help="decode sequences per GPU (config 3 is 256; smaller for ncu captures)")
    ap.add_argument("--layer", action="store_true",
                    help="measure the GatedDeltaNet2 layer (config-4 layer shape) instead of the op")
    ap.add_argument("--cp", action="store_true",
                    help="measure config-5 context-parallel prefill (T=131072 split over the ranks)")
    ap.add_argument("--model", action="store_true",
                    help="measure the config-4 hybrid LM training step (1.33B, DDP over the ranks)")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


TRAFFIC_FILE = os.path.join(ROOT, "profiles", "dram_traffic_per_launch_config2_config3.txt")


def traffic_table():
    """DRAM bytes (read + write) per launch at the full config-2 / config-3
    sizes, from the committed ncu summary: lines ``traffic <kernel> <bytes>``."""
    out = {}
    try:
        with open(TRAFFIC_FILE) as f:
            for ln in f:
                parts = ln.split()
                if len(parts) == 3 and parts[0] == "traffic":
                    out[parts[1]] = int(parts[2])
    except OSError:
        pass
    return out


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# reference arm: the reference's algorithm on the host cores
# ---------------------------------------------------------------------------
def run_reference(args, world):
    from oracle.parallel import OraclePool, synthetic
    pool = OraclePool()
    # size a step so that warmup + steps stay within ~3 minutes
    calib = synthetic(1, 64, H, K, V, seed=1)
    pool.fwd_bwd(*calib)
    t64 = min(pool.fwd_bwd(*calib) for _ in range(2))
    budget = 150.0 / max(1, args.steps + args.warmup)
    Ts = int(max(64, min(T, 64 * math.floor(budget / max(t64, 1e-3)))))
    x = synthetic(1, Ts, H, K, V, seed=2)
    for _ in range(args.warmup):
        pool.fwd_bwd(*x)
    tot = 0.0
    for _ in range(args.steps):
        tot += pool.fwd_bwd(*x)
    pool.close()
    tps = Ts * args.steps / tot
    sample = f"one sequence of T={Ts} tokens x H=16 heads (d=128) per step, fp64 oracle port"
    line = {
        "metric": METRIC, "value": tps, "unit": "tokens/s", "impl": "reference",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * tot / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "config2 GDN2 op fwd+bwd (H16, d128), sampled on host cores",
                   "seq_len_sample": Ts, "heads": H, "head_dim": K},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": pool.nproc, "kind": "port",
                         "sample": sample},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_ours():
    """Bounded sample of config 2 through the oracle on the host cores."""
    from oracle.parallel import OraclePool, synthetic
    pool = OraclePool()
    x = synthetic(1, 1024, H, K, V, seed=3)
    pool.fwd_bwd(*synthetic(1, 64, H, K, V, seed=4))
    t = pool.fwd_bwd(*x)
    pool.close()
    return {"value": 1024 / t, "unit": "tokens/s", "cores": pool.nproc, "kind": "port",
            "sample": "one sequence of T=1024 tokens x H=16 heads (d=128), fwd+bwd, fp64 oracle "
                      f"over {pool.nproc} processes, {t:.1f} s"}


# ---------------------------------------------------------------------------
# the reference's own Triton op on the GPU (baseline/_ref)
# ---------------------------------------------------------------------------
def load_reference_triton():
    """``lit_gpt.gdn2_ops`` from ``baseline/_ref`` (unmodified files), imported
    under a bare parent package: ``lit_gpt/__init__.py`` needs Lightning, which
    the op does not use."""
    import types
    base = os.path.join(ROOT, "baseline", "_ref", "lit_gpt")
    if not os.path.isdir(os.path.join(base, "gdn2_ops")):
        raise ImportError("baseline/_ref/lit_gpt/gdn2_ops is not installed")
    if "lit_gpt" not in sys.modules:
        pkg = types.ModuleType("lit_gpt")
        pkg.__path__ = [base]
        sys.modules["lit_gpt"] = pkg
    chunk = importlib.import_module("lit_gpt.gdn2_ops.chunk_gdn2")
    rec = importlib.import_module("lit_gpt.gdn2_ops.fused_recurrent_gdn2")
    return chunk, rec


def load_reference_layer():
    """The reference's ``GatedDeltaNet2`` (``lit_gpt/gdn2.py``, fla's Triton short
    convolutions and gated norm, the reference's Triton op) from ``baseline/_ref``."""
    load_reference_triton()
    return importlib.import_module("lit_gpt.gdn2").GatedDeltaNet2


def run_reference_triton(args, world, rank, local):
    if rank != 0:
        return
    try:
        ref_chunk, ref_rec = load_reference_triton()
        ref_layer = load_reference_layer() if (args.layer or args.model) else None
    except Exception as e:  # noqa: BLE001
        print(json.dumps({"impl": "reference-triton", "unavailable": f"{type(e).__name__}: {e}"}), flush=True)
        return
    if args.layer:
        run_layer(args, 1, 0, local, layer_cls=ref_layer, impl="reference-triton")
        return
    if args.model:
        run_model(args, 1, 0, local, gdn2_cls=ref_layer, impl="reference-triton")
        return
    import torch
    import torch.nn.functional as F
    gdn2 = importlib.import_module("gateddeltanet-2_b200")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev).manual_seed(1234)
    nb, nd = args.batch, args.decode_seqs

    def rnd(*shape):
        return torch.randn(*shape, device=dev, generator=gen)

    q = F.normalize(rnd(nb, T, H, K), dim=-1).bfloat16()
    k = F.normalize(rnd(nb, T, H, K), dim=-1).bfloat16()
    v = rnd(nb, T, H, V).bfloat16()
    g = -F.softplus(rnd(nb, T, H, K)) * 0.1
    b = torch.sigmoid(rnd(nb, T, H, K)).bfloat16()
    w = torch.sigmoid(rnd(nb, T, H, V)).bfloat16()
    do = rnd(nb, T, H, V).bfloat16()
    leaves = [x.requires_grad_(True) for x in (q, k, v, g, b, w)]

    def fwd_bwd(fn):
        def step():
            o, _ = fn(*leaves)
            return torch.autograd.grad(o, leaves, do)
        return step

    def timed(fn, n):
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(n):
            fn()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e)

    arms = {"reference": fwd_bwd(ref_chunk.chunk_gdn2), "ours": fwd_bwd(gdn2.chunk_gdn2)}
    # parity of the two arms on these inputs (max |diff| relative to max |o|)
    with torch.no_grad():
        o_r, _ = ref_chunk.chunk_gdn2(q, k, v, g, b, w)
        o_o, _ = gdn2.chunk_gdn2(q, k, v, g, b, w)
        rel = float((o_r.float() - o_o.float()).abs().max() / o_r.float().abs().max())
    res = {}
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(vis.split(",")[local] if vis else local)
    clocks.start()
    for name, fn in arms.items():
        for _ in range(max(3, args.warmup)):
            fn()
        ms = timed(fn, args.steps)
        res[name] = {"ms_per_step": ms / args.steps, "tokens_per_s": nb * T * args.steps / (ms / 1e3)}

    # decode, config 3: in-place state, one token per sequence
    S_r = rnd(nd, H, K, V) * 0.02
    S_o = S_r.clone()
    xs = (F.normalize(rnd(nd, 1, H, K), dim=-1).bfloat16(), F.normalize(rnd(nd, 1, H, K), dim=-1).bfloat16(),
          rnd(nd, 1, H, V).bfloat16(), -F.softplus(rnd(nd, 1, H, K)) * 0.1,
          torch.sigmoid(rnd(nd, 1, H, K)), torch.sigmoid(rnd(nd, 1, H, V)))
    dec = {}
    for name, fn in (("reference", lambda: ref_rec.fused_recurrent_gdn2_fwd(*xs, initial_state=S_r,
                                                                           inplace_final_state=True)),
                     ("ours", lambda: gdn2.fused_recurrent_gdn2_fwd(*xs, initial_state=S_o,
                                                                   inplace_final_state=True))):
        for _ in range(10):
            fn()
        ms = timed(fn, args.decode_steps)
        us = 1e3 * ms / args.decode_steps
        dec[name] = {"us_per_step": us, "state_GBps": decode_bytes_per_step(nd) / (us * 1e-6) / 1e9}
    clk = clocks.stop()
    line = {
        "metric": METRIC, "impl": "reference-triton", "value": res["reference"]["tokens_per_s"],
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": res["reference"]["ms_per_step"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"config2: GDN2 op fwd+bwd, B={nb} H=16 T=4096 dk=dv=128; "
                               f"config3 decode N={nd}", "gates": "b, w bf16; log-decay fp32"},
        "source": "lit_gpt/gdn2_ops from baseline/_ref (the reference's Triton path on sm_100)",
        "fwd_bwd": res, "speedup_ours_over_reference": res["ours"]["tokens_per_s"] / res["reference"]["tokens_per_s"],
        "decode": dec, "decode_speedup": dec["reference"]["us_per_step"] / dec["ours"]["us_per_step"],
        "o_max_rel_diff": rel, "clocks": clk,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# the GatedDeltaNet2 layer (config-4 layer shape)
# ---------------------------------------------------------------------------
D_MODEL = 2048


def layer_kernel_bytes_per_token(Dk, Dv, Dfg, H, V):
    """Algorithmic bytes per token of the layer kernels (each tensor of the
    kernel's interface read or written once; bf16 activations)."""
    sec = 2 * (2 * Dk + Dv + Dk + Dv)  # q, k, v, b, w sections
    fg = 2 * 2 * Dfg
    return {
        "layer_prep_fwd_kernel": 2 * (sec + fg),                 # read proj sections, write outputs
        "layer_prep_bwd_kernel": sec + sec + fg + (sec + fg),    # read proj + cotangents, write dproj
        "norm_gate_fwd_kernel": 3 * 2 * H * V + 4 * H,           # read x, gate; write y, rstd
        "norm_gate_bwd_kernel": 5 * 2 * H * V + 4 * H,           # read dy, x, gate, rstd; write dx, dgate
    }


def run_layer(args, world, rank, local, layer_cls=None, impl="ours"):
    import torch
    import torch.distributed as dist
    layer_mod = importlib.import_module("gateddeltanet-2_b200.layer")
    from gdn2_b200 import _lib

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    nb = args.batch
    torch.manual_seed(1234 + rank)
    m = (layer_cls or layer_mod.GatedDeltaNet2)(hidden_size=D_MODEL, head_dim=K, num_heads=H,
                                                layer_idx=0).to(dev).train()
    x = torch.randn(nb, T, D_MODEL, device=dev, dtype=torch.bfloat16).requires_grad_(True)
    dout = torch.randn(nb, T, D_MODEL, device=dev, dtype=torch.bfloat16)
    params = list(m.parameters())

    def step():
        for p in params:
            p.grad = None
        x.grad = None
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = m(x)[0]
        torch.autograd.backward(out, dout)

    def timed(fn, n):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(n):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = torch.tensor([s.elapsed_time(e)], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            dist.barrier()
        return float(ms.item())

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(vis.split(",")[local] if vis else local)
    clocks.start()
    _lib.profile_enable(True)
    ms = timed(step, args.steps)
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    clk = clocks.stop()
    peak, peak_kind = peaks()
    tok = nb * T
    bpt = layer_kernel_bytes_per_token(m.key_dim, m.value_dim, m.head_v_dim, H, V) if impl == "ours" else {}
    kernels = {}
    for name, (n, tms) in sorted(prof.items(), key=lambda kv: -kv[1][1]):
        ent = {"launches": n, "ms_per_step": tms / args.steps, "us_per_launch": 1e3 * tms / max(n, 1)}
        if name in bpt:
            achieved = bpt[name] * tok / (tms / max(n, 1) / 1e3) / 1e9
            ent.update(roofline={"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                                 "frac": achieved / peak, "peak_source": peak_kind,
                                 "algorithmic_bytes_per_launch": bpt[name] * tok})
        kernels[name] = ent
    ours_ms = sum(t for _, t in prof.values()) / args.steps
    step_ms = ms / args.steps
    if rank == 0:
        line = {
            "metric": "GatedDeltaNet2 layer fwd+bwd tokens/s (d2048, H16, d128, T4K)", "impl": impl,
            "value": world * tok * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic, random-init layer",
            "config": {"workload": f"config-4 layer: GatedDeltaNet2 fwd+bwd, B={nb} T={T} d_model={D_MODEL} "
                                   "H=16 d=128 conv 4, bf16 autocast, fp32 params",
                       "global_batch": nb * world, "seq_len": T,
                       "parallelism": f"data parallel replicas, {world} GPU(s), no gradient all-reduce"},
            "clocks": clk, "gpu_launches": sum(n for n, _ in prof.values()),
            "kernels": kernels,
            "time_split_ms": {"our_kernels": ours_ms, "gemms_and_torch_ops": step_ms - ours_ms},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# config 5: context-parallel prefill
# ---------------------------------------------------------------------------
CP_T = 131072


def run_cp(args, world, rank, local):
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F
    gdn2 = importlib.import_module("gateddeltanet-2_b200")
    from gdn2_b200 import cp

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    gen = torch.Generator(device=dev).manual_seed(5)  # the same sequence on every rank

    def rnd(*shape):
        return torch.randn(*shape, device=dev, generator=gen)

    q = F.normalize(rnd(1, CP_T, H, K), dim=-1).bfloat16()
    k = F.normalize(rnd(1, CP_T, H, K), dim=-1).bfloat16()
    v = rnd(1, CP_T, H, V).bfloat16()
    g = -F.softplus(rnd(1, CP_T, H, K)) * 0.1
    b = torch.sigmoid(rnd(1, CP_T, H, K))
    w = torch.sigmoid(rnd(1, CP_T, H, V))
    Ts = CP_T // world
    shard = [x[:, rank * Ts:(rank + 1) * Ts].contiguous() for x in (q, k, v, g, b, w)]

    def step():
        with torch.no_grad():
            return cp.chunk_gdn2_cp(*shard) if world > 1 else gdn2.chunk_gdn2(*shard, output_final_state=True)

    def timed(fn, n):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(n):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = torch.tensor([s.elapsed_time(e)], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            dist.barrier()
        return float(ms.item())

    for _ in range(max(3, args.warmup)):
        step()
    ms = timed(step, args.steps)
    o, ht = step()
    with torch.no_grad():
        o_ref, ht_ref = gdn2.chunk_gdn2(q, k, v, g, b, w, output_final_state=True)
    err = float((o.float() - o_ref[:, rank * Ts:(rank + 1) * Ts].float()).abs().max())
    err_t = torch.tensor([err], device=dev)
    if world > 1:
        dist.all_reduce(err_t, op=dist.ReduceOp.MAX)
    st_err = float((ht - ht_ref).abs().max()) if rank == world - 1 else 0.0
    st_t = torch.tensor([st_err], device=dev)
    if world > 1:
        dist.all_reduce(st_t, op=dist.ReduceOp.MAX)
    if rank == 0:
        line = {
            "metric": "config-5 context-parallel prefill tokens/s (B=1, H16, d128, T=131072)",
            "value": CP_T * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "config5: chunk_gdn2 forward of one T=131072 sequence, T split into "
                                   f"{world} contiguous shard(s), boundary maps all-gathered over NCCL",
                       "global_batch": 1, "seq_len": CP_T, "heads": H, "head_dim": K,
                       "parallelism": f"cp{world}"},
            "o_max_abs_diff_vs_single_gpu": float(err_t.item()),
            "final_state_max_abs_diff_vs_single_gpu": float(st_t.item()),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# config 4: the hybrid LM training step
# ---------------------------------------------------------------------------
def run_model(args, world, rank, local, gdn2_cls=None, impl="ours"):
    import torch
    import torch.distributed as dist
    importlib.import_module("gateddeltanet-2_b200")
    from gdn2_b200 import _lib
    from gdn2_b200 import model as hm

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    nb = args.batch
    cfg = hm.HybridConfig()
    torch.manual_seed(1234)  # the same initial weights on every rank
    net = hm.GPT(cfg, gdn2_cls=gdn2_cls).to(dev)
    net.init_weights()
    nparams = hm.num_parameters(net)
    model = net
    if world > 1:
        model = torch.nn.parallel.DistributedDataParallel(net, device_ids=[local], gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(net.parameters(), lr=4e-4, betas=(0.9, 0.95), weight_decay=0.1, fused=True)
    gen = torch.Generator(device=dev).manual_seed(99 + rank)
    tokens = torch.randint(0, cfg.vocab_size, (nb, T + 1), device=dev, generator=gen)
    idx, tgt = tokens[:, :-1].contiguous(), tokens[:, 1:].contiguous()

    def step():
        return hm.train_step(model, opt, idx, tgt)

    def timed(fn, n):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(n):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = torch.tensor([s.elapsed_time(e)], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            dist.barrier()
        return float(ms.item())

    for _ in range(max(3, args.warmup)):
        loss0 = step()
    torch.cuda.synchronize()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(vis.split(",")[local] if vis else local)
    clocks.start()
    _lib.profile_enable(True)
    ms = timed(step, args.steps)
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    clk = clocks.stop()
    loss = float(step())
    step_ms = ms / args.steps
    ours_ms = sum(t for _, t in prof.values()) / args.steps
    if rank == 0:
        line = {
            "metric": "config-4 hybrid LM training tokens/s (1.33B, GDN2 + 2048-window attention, seq 4096)",
            "impl": impl,
            "value": world * nb * T * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: uniform-random token ids, random-init weights",
            "config": {"workload": f"config4: {nparams / 1e9:.2f}B hybrid LM, 24 layers (12 GatedDeltaNet2, 12 "
                                   "sliding-window attention), d_model 2048, SwiGLU 4608, vocab 32000; fwd + "
                                   "loss + bwd + fused AdamW step",
                       "global_batch": nb * world, "seq_len": T, "micro_batch": nb,
                       "parallelism": f"dp{world} (DistributedDataParallel over NCCL)" if world > 1 else "dp1",
                       "params": nparams},
            "clocks": clk, "gpu_launches": sum(n for n, _ in prof.values()),
            "gdn2_kernels_ms_per_step": ours_ms,
            "gdn2_kernels": {n: round(1e3 * t / max(c, 1), 1) for n, (c, t) in prof.items()},
            "loss_after": loss, "loss_first_warmup": float(loss0),
            "peak_mem_gb": torch.cuda.max_memory_allocated(dev) / 1e9,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
def main():
    args = parse()
    nb, nd = args.batch, args.decode_seqs
    dec_bytes = decode_bytes_per_step(nd)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            run_reference(args, world)
        return
    if args.impl == "reference-triton":
        run_reference_triton(args, world, rank, local)
        return
    if args.layer:
        run_layer(args, world, rank, local)
        return
    if args.model:
        run_model(args, world, rank, local)
        return
    if args.cp:
        run_cp(args, world, rank, local)
        return

    cpu_base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_base = cpu_baseline_ours()  # before any GPU work (spawned pool)

    import torch
    import torch.distributed as dist
    import torch.nn.functional as F
    gdn2 = importlib.import_module("gateddeltanet-2_b200")
    from gdn2_b200 import _lib

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    gen = torch.Generator(device=dev).manual_seed(1234 + rank)

    def rnd(*shape):
        return torch.randn(*shape, device=dev, generator=gen)

    q = F.normalize(rnd(nb, T, H, K), dim=-1).bfloat16()
    k = F.normalize(rnd(nb, T, H, K), dim=-1).bfloat16()
    v = rnd(nb, T, H, V).bfloat16()
    g = -F.softplus(rnd(nb, T, H, K)) * 0.1
    b = torch.sigmoid(rnd(nb, T, H, K))
    w = torch.sigmoid(rnd(nb, T, H, V))
    do = rnd(nb, T, H, V).bfloat16()
    leaves = [x.requires_grad_(True) for x in (q, k, v, g, b, w)]

    def step():
        o, _ = gdn2.chunk_gdn2(*leaves)
        return torch.autograd.grad(o, leaves, do)

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(fn, n):
        barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(n):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = torch.tensor([s.elapsed_time(e)], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        barrier()
        return float(ms.item())

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()

    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(vis.split(",")[local] if vis else local)
    clocks.start()
    _lib.profile_enable(True)
    ms = timed(step, args.steps)
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    clk = clocks.stop()
    gpu_launches = sum(n for n, _ in prof.values())
    tok_per_step = world * nb * T
    value = tok_per_step * args.steps / (ms / 1e3)

    # ---- end to end through the public API: pinned host inputs -> device ----
    # Every step copies its own inputs and cotangent from pinned host memory
    # inside the timed region.  Two device buffer sets: step i+1's copy runs on
    # a second stream while step i computes (what a data loader with prefetch
    # does); a step waits only for its own copy.
    host = [x.detach().cpu().pin_memory() for x in (q, k, v, g, b, w, do)]
    sets = [[torch.empty_like(x) for x in (q, k, v, g, b, w, do)] for _ in range(2)]
    copy_stream = torch.cuda.Stream(device=dev)
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    for ev in consumed:
        ev.record()
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()

    def issue_copy(i):
        sl = i % 2
        copy_stream.wait_event(consumed[sl])  # the step that last used this set is done with it
        with torch.cuda.stream(copy_stream):
            for d, hsrc in zip(sets[sl], host):
                d.copy_(hsrc, non_blocking=True)
            copied[sl].record(copy_stream)

    def e2e_run(n):
        copy_stream.wait_stream(torch.cuda.current_stream())  # copies start inside the timed region
        issue_copy(0)
        for i in range(n):
            if i + 1 < n:
                issue_copy(i + 1)
            sl = i % 2
            torch.cuda.current_stream().wait_event(copied[sl])
            bufs = sets[sl]
            ins = [x.requires_grad_(True) for x in bufs[:6]]
            o, _ = gdn2.chunk_gdn2(*ins)
            torch.autograd.grad(o, ins, bufs[6])
            loss = (o.float() * bufs[6].float()).sum()
            loss_host.copy_(loss, non_blocking=True)
            consumed[sl].record()
            for d in bufs[:6]:
                d.requires_grad_(False)

    n_e2e = max(3, min(args.steps, 20))
    e2e_run(2)
    e2e_ms = timed(lambda: e2e_run(n_e2e), 1)
    h2d = sum(x.numel() * x.element_size() for x in host)
    e2e = {"value": tok_per_step * n_e2e / (e2e_ms / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4, "steps": n_e2e,
           "path": "chunk_gdn2 fwd+bwd; each step's inputs and cotangent copied from pinned host "
                   "memory inside the timed region (double-buffered: the next step's copy overlaps "
                   "this step's compute), loss scalar read back"}

    # ---- decode (config 3): in-place state update, 1 token per sequence --------
    S = rnd(nd, H, K, V) * 0.02
    ring = []
    for i in range(4):
        ring.append((F.normalize(rnd(nd, 1, H, K), dim=-1).bfloat16(),
                     F.normalize(rnd(nd, 1, H, K), dim=-1).bfloat16(),
                     rnd(nd, 1, H, V).bfloat16(), -F.softplus(rnd(nd, 1, H, K)) * 0.1,
                     torch.sigmoid(rnd(nd, 1, H, K)), torch.sigmoid(rnd(nd, 1, H, V))))
    it = [0]

    def dec_step():
        x = ring[it[0] & 3]
        it[0] += 1
        gdn2.fused_recurrent_gdn2_fwd(*x, initial_state=S, inplace_final_state=True)

    for _ in range(10):
        dec_step()
    _lib.profile_enable(True)
    dec_ms = timed(dec_step, args.decode_steps)
    dprof = _lib.profile_read()
    _lib.profile_enable(False)
    peak, peak_kind = peaks()
    dec_us = 1e3 * dec_ms / args.decode_steps
    dec_gbs = dec_bytes / (dec_us * 1e-6) / 1e9
    dk = dprof.get("recurrent_kernel", (1, dec_ms))
    dk_us = 1e3 * dk[1] / max(dk[0], 1)
    decode = {"metric": "decode-step state HBM GB/s", "value": world * dec_gbs, "unit": "GB/s",
              "us_per_step": dec_us, "tokens_per_s": world * nd / (dec_us * 1e-6),
              "config": {"workload": "config3 decode step", "sequences_per_gpu": nd, "heads": H,
                         "state": f"fp32 [{nd},16,128,128] in place", "steps": args.decode_steps},
              "roofline": {"bound": "hbm", "achieved": dec_bytes / (dk_us * 1e-6) / 1e9,
                           "peak": peak, "unit": "GB/s",
                           "frac": dec_bytes / (dk_us * 1e-6) / 1e9 / peak,
                           "peak_source": peak_kind, "kernel": "recurrent_kernel",
                           "us_per_launch": dk_us,
                           "traffic": traffic_table().get("recurrent_kernel") if nd == DEC_N else None}}

    # ---- roofline of the dominant kernel of the fwd+bwd step ------------------
    dom = max(prof.items(), key=lambda kv: kv[1][1])
    name, (nl, tms) = dom
    per_launch_s = tms / nl / 1e3
    alg = KERNEL_BYTES_PER_TOKEN_HEAD[name] * nb * T * H
    achieved = alg / per_launch_s / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": peak_kind,
                "traffic": traffic_table().get(name) if nb == B else None, "kernel": name,
                "algorithmic_bytes_per_launch": alg, "us_per_launch": per_launch_s * 1e6,
                "kernel_shares": {n: round(t / sum(x[1] for x in prof.values()), 4)
                                  for n, (c, t) in prof.items()}}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": f"config2: GDN2 op fwd+bwd, B={nb} H=16 T=4096 dk=dv=128 chunk 64 per GPU",
                       "global_batch": nb * world, "seq_len": T, "heads": H, "head_dim": K,
                       "parallelism": f"(batch x head) shards, {world} GPU(s), no collectives",
                       "l2": f"inputs {0.15 * nb:.2f} GB per GPU per step (> 126 MB L2), no flush needed",
                       "gates": "b, w, log-decay fp32; q, k, v bf16"},
            "clocks": clk, "e2e": e2e, "gpu_launches": gpu_launches, "roofline": roofline,
            "decode": decode,
        }
        if cpu_base is not None:
            line["cpu_baseline"] = cpu_base
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
