#!/usr/bin/env python
"""Benchmark of the GDN2 operator on B200 (the headline metric of this build).

Metric: "GDN2 op fwd+bwd tokens/s (H16,d128,T4K) & decode-step state HBM GB/s".

One step = forward + backward of ``chunk_gdn2`` on config 2 (B=4, H=16,
T=4096, d_k=d_v=128, chunk 64; q,k,v bf16 with q,k L2-normalised, b,w =
sigmoid(N(0,1)) fp32, log-decay = -softplus(N(0,1))*0.1 fp32), synthetic
data.  The 64 (sequence, head) pairs of that fixed workload are split over
the ranks (rank r takes heads [r 16/N, (r+1) 16/N) of all four sequences; no
communication), so ``value`` is the whole job's tokens/s with strong
scaling: 64, 32, 16, 8 pairs per GPU at N = 1, 2, 4, 8.  With few pairs per
GPU the library cuts the state scans into segments to keep the SMs busy.

The same JSON line carries, as extra keys:
  ``weak``      config 2 with B=4 x 16 heads on every rank (N > 1);
  ``e2e``       the strong-split step through ``chunk_gdn2`` with every step's
                inputs copied from pinned host memory (each rank its own heads);
  ``decode``    config 3: 256 sequences x 16 heads, fp32 128x128 states updated in
                place, split over the ranks by sequence (strong), 1024 steps;
  ``cp``        config 5: one T=131072 sequence, forward, T split over the ranks
                (one all_gather of boundary maps over NCCL; N=1 is the
                single-GPU forward), each shard checked against the single-GPU result;
  ``model``     config 4: the 1.33B hybrid LM training step, micro-batch 4 per GPU,
                DistributedDataParallel over NCCL for N > 1;
  ``reference_triton`` (N=1) the reference's own Triton op on the same GPU and inputs,
                configs 2 and 3 (``lit_gpt/gdn2_ops`` from ``baseline/_ref``);
  ``cpu_baseline`` / ``cpu_baselines`` (N=1) the host cores: the fp64 oracle port
                of the algorithm, the naive fp32 torch recurrence with autograd
                (config 1, and config 2 per token-head) and the naive torch decode
                step (config 3).

``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]``
(multi-GPU through ``torch.distributed.run``; one rank per GPU).
``--batch`` / ``--decode-seqs`` / ``--heads`` shrink the two workloads for ncu
captures; a line measured with any of them changed is not a config-2 /
config-3 number.
``--impl reference`` times the reference's algorithm on the host cores (the
oracle port: the reference has no CPU implementation of its own and its
kernels are Triton/sm_120 CUDA); it runs on rank 0 only.
``--impl reference-triton`` prints the reference-Triton comparison alone
(bf16 b, w in both arms: the reference's backward rejects fp32 ``w`` with
bf16 ``v``); with ``--layer`` / ``--model`` the reference's whole layer.
``--cp``, ``--model`` and ``--layer`` print the config-5, config-4 and
GatedDeltaNet2-layer (config-4 layer shape) measurements as lines of their own.
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
    ap.add_argument("--no-reference-triton", action="store_true",
                    help="skip the reference Triton op in the default N=1 line (its autotuning takes minutes)")
    ap.add_argument("--batch", type=int, default=B,
                    help="sequences per GPU (config 2 is 4; smaller values are for ncu captures)")
    ap.add_argument("--heads", type=int, default=None,
                    help="heads per GPU; default 16/N (the strong split).  Set on one GPU it runs the shard one "
                         "rank of a 16/heads-GPU split runs (for ncu captures of the segmented scans)")
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
# ranks and device timing
# ---------------------------------------------------------------------------
class Ranks:
    """World, rank and device of this process, with max-over-ranks timing."""

    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dev = None
        self.dist = None

    def init_gpu(self, timeout_s=180):
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.dist = dist
        if self.world > 1 and not dist.is_initialized():
            from datetime import timedelta
            dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s), device_id=self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, x: float) -> float:
        import torch
        if self.world == 1:
            return float(x)
        t = torch.tensor([float(x)], device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def timed(self, fn, n) -> float:
        """ms for n calls of fn on this rank's current stream, max over ranks;
        a barrier and a device synchronize on both sides."""
        import torch
        self.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(n):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = self.max(s.elapsed_time(e))
        self.barrier()
        return ms

    def clocks(self):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        return ClockSampler(vis.split(",")[self.local] if vis else self.local)

    def close(self):
        if self.world > 1 and self.dist is not None and self.dist.is_initialized():
            self.dist.destroy_process_group()

    def solo(self):
        """This process alone (rank 0 of an arm that runs without the others):
        no process group, no collectives."""
        r = Ranks()
        r.world, r.rank, r.local = 1, 0, self.local
        return r


def config2_inputs(dev, nb, heads, seed, bf16_gates=False):
    """Config-2 inputs of nb sequences x `heads` heads, generated on the device."""
    import torch
    import torch.nn.functional as F
    gen = torch.Generator(device=dev).manual_seed(seed)

    def rnd(*shape):
        return torch.randn(*shape, device=dev, generator=gen)

    gd = torch.bfloat16 if bf16_gates else torch.float32
    q = F.normalize(rnd(nb, T, heads, K), dim=-1).bfloat16()
    k = F.normalize(rnd(nb, T, heads, K), dim=-1).bfloat16()
    v = rnd(nb, T, heads, V).bfloat16()
    g = -F.softplus(rnd(nb, T, heads, K)) * 0.1
    b = torch.sigmoid(rnd(nb, T, heads, K)).to(gd)
    w = torch.sigmoid(rnd(nb, T, heads, V)).to(gd)
    do = rnd(nb, T, heads, V).bfloat16()
    return q, k, v, g, b, w, do


def decode_inputs(dev, nd, seed):
    import torch
    import torch.nn.functional as F
    gen = torch.Generator(device=dev).manual_seed(seed)

    def rnd(*shape):
        return torch.randn(*shape, device=dev, generator=gen)

    S = rnd(nd, H, K, V) * 0.02
    ring = [(F.normalize(rnd(nd, 1, H, K), dim=-1).bfloat16(), F.normalize(rnd(nd, 1, H, K), dim=-1).bfloat16(),
             rnd(nd, 1, H, V).bfloat16(), -F.softplus(rnd(nd, 1, H, K)) * 0.1,
             torch.sigmoid(rnd(nd, 1, H, K)), torch.sigmoid(rnd(nd, 1, H, V))) for _ in range(4)]
    return S, ring


# ---------------------------------------------------------------------------
# host-core baselines
# ---------------------------------------------------------------------------
def run_reference(args, world):
    """--impl reference: the reference's algorithm (the fp64 oracle port) on
    all host cores.  A step is the whole config-2 workload (B=4 sequences of
    T=4096 x 16 heads) when warmup + steps fit in about four minutes, else a
    shorter T per sequence, stated in the line."""
    from oracle.parallel import OraclePool, synthetic
    pool = OraclePool()
    calib = synthetic(1, 256, H, K, V, seed=1)
    pool.fwd_bwd(*calib)
    t256 = min(pool.fwd_bwd(*calib) for _ in range(2))
    per_token = t256 / 256
    n = max(1, args.steps + args.warmup)
    budget = 240.0 / n
    Ts = T if B * T * per_token <= budget else int(max(256, min(T, 256 * math.floor(budget / (B * t256)))))
    x = synthetic(B, Ts, H, K, V, seed=2)
    for _ in range(args.warmup):
        pool.fwd_bwd(*x)
    tot = 0.0
    for _ in range(args.steps):
        tot += pool.fwd_bwd(*x)
    pool.close()
    tps = B * Ts * args.steps / tot
    sample = (f"{B} sequences of T={Ts} tokens x H=16 heads (d=128) per step"
              f"{' (the whole config-2 workload)' if Ts == T else ''}, fp64 oracle port, heads over "
              f"{pool.nproc} processes")
    line = {
        "metric": METRIC, "value": tps, "unit": "tokens/s", "impl": "reference",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * tot / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": f"config2 GDN2 op fwd+bwd, B={B} H=16 T={Ts} dk=dv=128, on host cores",
                   "global_batch": B, "seq_len": Ts, "heads": H, "head_dim": K},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": pool.nproc, "kind": "port",
                         "sample": sample},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline_ours():
    """The fp64 oracle port on a bounded sample of config 2 (all host cores)."""
    from oracle.parallel import OraclePool, synthetic
    pool = OraclePool()
    pool.fwd_bwd(*synthetic(1, 64, H, K, V, seed=4))
    x = synthetic(1, 512, H, K, V, seed=3)
    tot, n = 0.0, 0
    while tot < 8.0 and n < 40:
        tot += pool.fwd_bwd(*x)
        n += 1
    pool.close()
    return {"value": 512 * n / tot, "unit": "tokens/s", "cores": pool.nproc, "kind": "port",
            "sample": f"{n} x one sequence of T=512 tokens x H=16 heads (d=128), fwd+bwd, fp64 oracle "
                      f"over {pool.nproc} processes, {tot:.1f} s"}


def naive_torch_recurrence(q, k, v, g, b, w, scale):
    """The Gated Delta Rule-2 recurrence token by token in fp32 torch, as the
    reference's naive form (fused_recurrent_gdn2.py:193-243): autograd gives
    the backward."""
    import torch
    Bn, Tn, Hn, Kn = q.shape
    S = q.new_zeros(Bn, Hn, Kn, v.shape[-1])
    outs = []
    for t in range(Tn):
        S = S * torch.exp(g[:, t])[..., None]
        u = w[:, t] * v[:, t] - torch.einsum("bhkv,bhk->bhv", S, b[:, t] * k[:, t])
        S = S + k[:, t][..., None] * u[:, :, None, :]
        outs.append(torch.einsum("bhkv,bhk->bhv", S, q[:, t] * scale))
    return torch.stack(outs, 1), S


def cpu_baselines_torch():
    """BASELINE B2 (naive fp32 torch recurrence with autograd, config 1 and
    config 2 per token-head) and B4 (naive torch decode step, config 3) on
    every host core; each sample runs for at least 5 s and reports its median
    call."""
    import torch
    import torch.nn.functional as F
    ncores = os.cpu_count() or 1
    torch.set_num_threads(ncores)
    gen = torch.Generator().manual_seed(0)

    def mk(Bn, Tn, Hn, d):
        q = F.normalize(torch.randn(Bn, Tn, Hn, d, generator=gen), dim=-1)
        k = F.normalize(torch.randn(Bn, Tn, Hn, d, generator=gen), dim=-1)
        v = torch.randn(Bn, Tn, Hn, d, generator=gen)
        b = torch.sigmoid(torch.randn(Bn, Tn, Hn, d, generator=gen))
        w = torch.sigmoid(torch.randn(Bn, Tn, Hn, d, generator=gen))
        g = -F.softplus(torch.randn(Bn, Tn, Hn, d, generator=gen)) * 0.1
        do = torch.randn(Bn, Tn, Hn, d, generator=gen)
        return [x.requires_grad_(True) for x in (q, k, v, g, b, w)], do

    def median(xs):
        xs = sorted(xs)
        m = len(xs) // 2
        return xs[m] if len(xs) % 2 else 0.5 * (xs[m - 1] + xs[m])

    # every sample: two untimed calls (allocator and thread-pool warm-up), then
    # calls for at least 5 s; the median call (host noise on tiny per-token ops
    # moves the mean by >10% between runs)
    def time_fwd_bwd(Bn, Tn, Hn, d, min_s=5.0):
        leaves, do = mk(Bn, Tn, Hn, d)

        def call():
            o, _ = naive_torch_recurrence(*leaves, d ** -0.5)
            torch.autograd.grad(o, leaves, do)

        call()
        call()
        ts = []
        while sum(ts) < min_s:
            t0 = time.perf_counter()
            call()
            ts.append(time.perf_counter() - t0)
        return median(ts), len(ts)

    out = {"cores": ncores, "cpu": cpu_model(), "torch_threads": torch.get_num_threads()}
    t1, n1 = time_fwd_bwd(1, 256, 2, 64)
    out["b2_config1"] = {"value": 256 / t1, "unit": "tokens/s", "ms_per_step": 1e3 * t1, "repeats": n1,
                         "sample": "config 1: B=1 H=2 T=256 d=64, naive fp32 torch recurrence, fwd + autograd bwd"}
    t2, n2 = time_fwd_bwd(1, 256, 1, 128)
    per_token_head = t2 / 256
    out["b2_config2"] = {"value": 1.0 / (per_token_head * H), "unit": "tokens/s", "repeats": n2,
                         "sample": "config 2 per token-head: B=1 H=1 T=256 d=128, naive fp32 torch, fwd + "
                                   "autograd bwd, scaled to 16 heads per token"}
    # B4: the config-3 decode step, in place on fp32 S [256, 16, 128, 128]
    with torch.no_grad():
        S = torch.randn(DEC_N, H, K, V, generator=gen) * 0.02
        q = F.normalize(torch.randn(DEC_N, H, K, generator=gen), dim=-1)
        k = F.normalize(torch.randn(DEC_N, H, K, generator=gen), dim=-1)
        v = torch.randn(DEC_N, H, V, generator=gen)
        b = torch.sigmoid(torch.randn(DEC_N, H, K, generator=gen))
        w = torch.sigmoid(torch.randn(DEC_N, H, V, generator=gen))
        g = -F.softplus(torch.randn(DEC_N, H, K, generator=gen)) * 0.1
        def step():
            S.mul_(torch.exp(g)[..., None])
            u = w * v - torch.einsum("nhkv,nhk->nhv", S, b * k)
            S.add_(k[..., None] * u[:, :, None, :])
            torch.einsum("nhkv,nhk->nhv", S, q * K ** -0.5)

        step()
        step()
        ts = []
        while sum(ts) < 5.0:
            t0 = time.perf_counter()
            step()
            ts.append(time.perf_counter() - t0)
        n = len(ts)
    us = 1e6 * median(ts)
    out["b4_decode"] = {"value": decode_bytes_per_step(DEC_N) / (us * 1e-6) / 1e9, "unit": "GB/s",
                        "us_per_step": us, "repeats": n,
                        "sample": "config 3 decode step: naive torch on fp32 S [256,16,128,128] in place"}
    return out


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


def measure_reference_triton(rk, steps, warmup, nb=B, nd=DEC_N):
    """The reference's Triton op and this build's op on identical inputs on
    this GPU: config-2 fwd+bwd and the config-3 decode step."""
    import torch
    ref_chunk, ref_rec = load_reference_triton()
    gdn2 = importlib.import_module("gateddeltanet-2_b200")
    q, k, v, g, b, w, do = config2_inputs(rk.dev, nb, H, 1234, bf16_gates=True)
    leaves = [x.requires_grad_(True) for x in (q, k, v, g, b, w)]

    def fwd_bwd(fn):
        def step():
            o, _ = fn(*leaves)
            return torch.autograd.grad(o, leaves, do)
        return step

    arms = {"reference": fwd_bwd(ref_chunk.chunk_gdn2), "ours": fwd_bwd(gdn2.chunk_gdn2)}
    with torch.no_grad():
        o_r, _ = ref_chunk.chunk_gdn2(q, k, v, g, b, w)
        o_o, _ = gdn2.chunk_gdn2(q, k, v, g, b, w)
        rel = float((o_r.float() - o_o.float()).abs().max() / o_r.float().abs().max())
    res = {}
    for name, fn in arms.items():
        # the reference's Triton autotuner benchmarks its configurations during
        # the first calls (minutes on a fresh box), and later calls can still
        # tune a kernel they reach for the first time: warm up until three
        # consecutive steps agree within 5% (at least five steps), and keep the
        # warm-up trace in the line
        trace = []
        while len(trace) < 80:
            trace.append(rk.timed(fn, 1))
            last = trace[-3:]
            if len(trace) >= max(5, warmup) and max(last) <= 1.05 * min(last):
                break
        # then every step timed on its own: a late one-off compile or tuning call
        # shows as one outlier instead of inflating the mean; the median is the
        # steady-state step, the mean and the list stay in the line
        per = sorted(rk.timed(fn, 1) for _ in range(steps))
        med = per[len(per) // 2] if len(per) % 2 else 0.5 * (per[len(per) // 2 - 1] + per[len(per) // 2])
        res[name] = {"ms_per_step": med, "tokens_per_s": nb * T / (med / 1e3),
                     "mean_ms_per_step": sum(per) / len(per), "max_ms_per_step": per[-1],
                     "timed_steps_ms_sorted": [round(t, 3) for t in per],
                     "warmup_steps_ms": [round(t, 3) for t in trace], "settled": len(trace) < 80}
    S_r, ring = decode_inputs(rk.dev, nd, 77)
    S_o = S_r.clone()
    xs = ring[0]
    dec = {}
    for name, fn in (("reference", lambda: ref_rec.fused_recurrent_gdn2_fwd(*xs, initial_state=S_r,
                                                                           inplace_final_state=True)),
                     ("ours", lambda: gdn2.fused_recurrent_gdn2_fwd(*xs, initial_state=S_o,
                                                                   inplace_final_state=True))):
        for _ in range(10):
            fn()
        ms = rk.timed(fn, 1024)
        us = 1e3 * ms / 1024
        dec[name] = {"us_per_step": us, "state_GBps": decode_bytes_per_step(nd) / (us * 1e-6) / 1e9}
    return {
        "source": "lit_gpt/gdn2_ops from baseline/_ref (the reference's Triton path on sm_100, unmodified)",
        "config": f"config2 fwd+bwd B={nb} H=16 T=4096 d=128 (b, w bf16 in both arms); config3 decode N={nd}",
        "fwd_bwd": res, "speedup_ours_over_reference": res["ours"]["tokens_per_s"] / res["reference"]["tokens_per_s"],
        "decode": dec, "decode_speedup": dec["reference"]["us_per_step"] / dec["ours"]["us_per_step"],
        "o_max_rel_diff": rel,
    }


def run_reference_triton(args, rk):
    if rk.rank != 0:
        return
    rk = rk.solo()
    try:
        load_reference_triton()
        ref_layer = load_reference_layer() if (args.layer or args.model) else None
    except Exception as e:  # noqa: BLE001
        print(json.dumps({"impl": "reference-triton", "unavailable": f"{type(e).__name__}: {e}"}), flush=True)
        return
    if args.layer:
        run_layer(args, 1, 0, rk.local, layer_cls=ref_layer, impl="reference-triton")
        return
    if args.model:
        rk.init_gpu()
        print(json.dumps(measure_model(rk, args.batch, args.steps, args.warmup, gdn2_cls=ref_layer,
                                       impl="reference-triton")), flush=True)
        return
    rk.init_gpu()
    clocks = rk.clocks()
    clocks.start()
    r = measure_reference_triton(rk, args.steps, args.warmup, args.batch, args.decode_seqs)
    line = {"metric": METRIC, "impl": "reference-triton", "value": r["fwd_bwd"]["reference"]["tokens_per_s"],
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
            "ms_per_step": r["fwd_bwd"]["reference"]["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "clocks": clocks.stop(), **r}
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


def measure_cp(rk, steps, warmup):
    """Forward of one T=131072 sequence, T split over the ranks (N=1: the
    single-GPU forward).  Every rank also runs the single-GPU forward of the
    whole sequence and reports how far its shard is from it."""
    import torch
    import torch.nn.functional as F
    gdn2 = importlib.import_module("gateddeltanet-2_b200")
    from gdn2_b200 import cp
    world, rank = rk.world, rk.rank
    gen = torch.Generator(device=rk.dev).manual_seed(5)  # the same sequence on every rank

    def rnd(*shape):
        return torch.randn(*shape, device=rk.dev, generator=gen)

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

    for _ in range(max(3, warmup)):
        step()
    ms = rk.timed(step, steps)
    o, ht = step()
    with torch.no_grad():
        o_ref, ht_ref = gdn2.chunk_gdn2(q, k, v, g, b, w, output_final_state=True)
    err = rk.max(float((o.float() - o_ref[:, rank * Ts:(rank + 1) * Ts].float()).abs().max()))
    st_err = rk.max(float((ht - ht_ref).abs().max()) if rank == world - 1 else 0.0)
    del q, k, v, g, b, w, shard, o_ref
    return {
        "metric": "config-5 context-parallel prefill tokens/s (B=1, H16, d128, T=131072)",
        "value": CP_T * steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "ms_per_step": ms / steps, "scaling": "strong",
        "workload": f"config5: forward of one T={CP_T} sequence (H=16, d=128), T split into {world} contiguous "
                    "shard(s)" + (", boundary maps all-gathered over NCCL" if world > 1 else ""),
        "parallelism": f"cp{world}",
        "o_max_abs_diff_vs_single_gpu": err, "final_state_max_abs_diff_vs_single_gpu": st_err,
    }


def run_cp(args, rk):
    rk.init_gpu(120)
    r = measure_cp(rk, args.steps, args.warmup)
    if rk.rank == 0:
        line = {"metric": r["metric"], "value": r["value"], "unit": "tokens/s", "n_gpus": rk.world,
                "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": r["ms_per_step"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic",
                "config": {"workload": r["workload"], "global_batch": 1, "seq_len": CP_T, "heads": H,
                           "head_dim": K, "parallelism": r["parallelism"]},
                "o_max_abs_diff_vs_single_gpu": r["o_max_abs_diff_vs_single_gpu"],
                "final_state_max_abs_diff_vs_single_gpu": r["final_state_max_abs_diff_vs_single_gpu"]}
        print(json.dumps(line), flush=True)
    rk.close()


# ---------------------------------------------------------------------------
# config 4: the hybrid LM training step
# ---------------------------------------------------------------------------
def measure_model(rk, nb, steps, warmup, gdn2_cls=None, impl="ours"):
    import torch
    importlib.import_module("gateddeltanet-2_b200")
    from gdn2_b200 import _lib
    from gdn2_b200 import model as hm
    world = rk.world if impl == "ours" else 1
    cfg = hm.HybridConfig()
    torch.manual_seed(1234)  # the same initial weights on every rank
    net = hm.GPT(cfg, gdn2_cls=gdn2_cls).to(rk.dev)
    net.init_weights()
    nparams = hm.num_parameters(net)
    model = net
    if world > 1:
        model = torch.nn.parallel.DistributedDataParallel(net, device_ids=[rk.local], gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(net.parameters(), lr=4e-4, betas=(0.9, 0.95), weight_decay=0.1, fused=True)
    gen = torch.Generator(device=rk.dev).manual_seed(99 + rk.rank)
    tokens = torch.randint(0, cfg.vocab_size, (nb, T + 1), device=rk.dev, generator=gen)
    idx, tgt = tokens[:, :-1].contiguous(), tokens[:, 1:].contiguous()

    def step():
        return hm.train_step(model, opt, idx, tgt)

    torch.cuda.reset_peak_memory_stats(rk.dev)
    for _ in range(max(3, warmup)):
        loss0 = step()
    torch.cuda.synchronize()
    _lib.profile_enable(True)
    ms = rk.timed(step, steps) if world > 1 else rk.solo().timed(step, steps)
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    loss = float(step())
    out = {
        "metric": "config-4 hybrid LM training tokens/s (1.33B, GDN2 + 2048-window attention, seq 4096)",
        "impl": impl, "value": world * nb * T * steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": max(3, warmup), "ms_per_step": ms / steps, "scaling": "weak",
        "workload": f"config4: {nparams / 1e9:.2f}B hybrid LM, 24 layers (12 GatedDeltaNet2, 12 sliding-window "
                    "attention), d_model 2048, SwiGLU 4608, vocab 32000; fwd + loss + bwd + fused AdamW step",
        "global_batch": nb * world, "seq_len": T, "micro_batch": nb,
        "parallelism": f"dp{world} (DistributedDataParallel over NCCL)" if world > 1 else "dp1", "params": nparams,
        "gpu_launches": sum(n for n, _ in prof.values()),
        "gdn2_kernels_ms_per_step": sum(t for _, t in prof.values()) / steps,
        "gdn2_kernels_us_per_launch": {n: round(1e3 * t / max(c, 1), 1) for n, (c, t) in prof.items()},
        "loss_after": loss, "loss_first_warmup": float(loss0),
        "peak_mem_gb": torch.cuda.max_memory_allocated(rk.dev) / 1e9,
    }
    del model, net, opt
    return out


def run_model(args, rk):
    rk.init_gpu(180)
    clocks = rk.clocks()
    clocks.start()
    r = measure_model(rk, args.batch, args.steps, args.warmup)
    clk = clocks.stop()
    if rk.rank == 0:
        line = {"metric": r["metric"], "impl": "ours", "value": r["value"], "unit": "tokens/s",
                "n_gpus": rk.world, "steps": args.steps, "warmup": r["warmup"], "ms_per_step": r["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic: uniform-random token ids, random-init weights",
                "config": {k: r[k] for k in ("workload", "global_batch", "seq_len", "micro_batch", "parallelism",
                                             "params")},
                "clocks": clk, **{k: r[k] for k in ("gpu_launches", "gdn2_kernels_ms_per_step",
                                                    "gdn2_kernels_us_per_launch", "loss_after",
                                                    "loss_first_warmup", "peak_mem_gb")}}
        print(json.dumps(line), flush=True)
    rk.close()


# ---------------------------------------------------------------------------
# config 2: the operator's fwd+bwd step
# ---------------------------------------------------------------------------
def op_step(gdn2, leaves, do):
    o, _ = gdn2.chunk_gdn2(*leaves)
    return torch_grad(o, leaves, do)


def torch_grad(o, leaves, do):
    import torch
    return torch.autograd.grad(o, leaves, do)


def measure_op(rk, nb, heads, steps, warmup, seed, profile=True):
    """fwd+bwd of chunk_gdn2 on nb sequences x `heads` heads per rank; returns
    (ms for `steps` steps (max over ranks), per-kernel profile, inputs)."""
    import torch
    gdn2 = importlib.import_module("gateddeltanet-2_b200")
    from gdn2_b200 import _lib
    q, k, v, g, b, w, do = config2_inputs(rk.dev, nb, heads, seed)
    leaves = [x.requires_grad_(True) for x in (q, k, v, g, b, w)]

    def step():
        return op_step(gdn2, leaves, do)

    for _ in range(max(3, warmup)):
        step()
    torch.cuda.synchronize()
    if profile:
        _lib.profile_enable(True)
    ms = rk.timed(step, steps)
    prof = _lib.profile_read() if profile else {}
    if profile:
        _lib.profile_enable(False)
    return ms, prof, (q, k, v, g, b, w, do)


def measure_e2e(rk, tensors, tok_per_step, steps):
    """The strong-split step through chunk_gdn2 with this rank's inputs and
    cotangent copied from pinned host memory inside the timed region (two
    device buffer sets: step i+1's copy runs on a second stream while step i
    computes) and the loss scalar read back."""
    import torch
    gdn2 = importlib.import_module("gateddeltanet-2_b200")
    host = [x.detach().cpu().pin_memory() for x in tensors]
    sets = [[torch.empty_like(x) for x in tensors] for _ in range(2)]
    copy_stream = torch.cuda.Stream(device=rk.dev)
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

    def run(n):
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

    n = max(3, min(steps, 20))
    run(2)
    ms = rk.timed(lambda: run(n), 1)
    h2d = sum(x.numel() * x.element_size() for x in host)
    return {"value": tok_per_step * n / (ms / 1e3), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d * rk.world, "d2h_bytes_per_step": 4 * rk.world, "steps": n,
            "path": "chunk_gdn2 fwd+bwd of each rank's heads; every step's inputs and cotangent copied from "
                    "pinned host memory inside the timed region (double-buffered: the next step's copy overlaps "
                    "this step's compute), loss scalar read back; bytes summed over the ranks"}


def measure_decode(rk, nd, steps):
    gdn2 = importlib.import_module("gateddeltanet-2_b200")
    from gdn2_b200 import _lib
    S, ring = decode_inputs(rk.dev, nd, 4321 + rk.rank)
    it = [0]

    def dec_step():
        x = ring[it[0] & 3]
        it[0] += 1
        gdn2.fused_recurrent_gdn2_fwd(*x, initial_state=S, inplace_final_state=True)

    for _ in range(10):
        dec_step()
    _lib.profile_enable(True)
    ms = rk.timed(dec_step, steps)
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    return ms, prof


_T0 = time.perf_counter()


def note(msg):
    """Progress of the run on stderr (section and elapsed seconds)."""
    print(f"[bench {time.perf_counter() - _T0:7.1f} s] {msg}", file=sys.stderr, flush=True)


def dominant(prof):
    """The kernel with the largest device time among those with known bytes."""
    known = {n: v for n, v in prof.items() if n in KERNEL_BYTES_PER_TOKEN_HEAD}
    return max(known.items(), key=lambda kv: kv[1][1]) if known else None


def main():
    args = parse()
    rk = Ranks()
    if args.impl == "reference":
        if rk.rank == 0:
            run_reference(args, rk.world)
        return
    if args.impl == "reference-triton":
        run_reference_triton(args, rk)
        return
    if args.layer:
        run_layer(args, rk.world, rk.rank, rk.local)
        return
    if args.model:
        run_model(args, rk)
        return
    if args.cp:
        run_cp(args, rk)
        return

    world, rank = rk.world, rk.rank
    nb, nd_total = args.batch, args.decode_seqs
    full = nb == B and nd_total == DEC_N and args.heads is None
    cpu_base = cpu_torch = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        note("cpu baseline: oracle port")
        cpu_base = cpu_baseline_ours()  # before any GPU work (spawned pool)
        note("cpu baselines: naive torch")
        cpu_torch = cpu_baselines_torch()

    import torch
    rk.init_gpu(180)
    peak, peak_kind = peaks()

    # ---- config 2, strong split of the 64 (sequence, head) pairs ----------------
    note("config 2")
    strong = H % world == 0
    heads = H // world if strong else H
    if args.heads is not None:
        heads = args.heads
    clocks = rk.clocks()
    clocks.start()
    ms, prof, tensors = measure_op(rk, nb, heads, args.steps, args.warmup, 1234 + rank)
    clk = clocks.stop()
    tok_per_step = nb * T if strong else world * nb * T
    value = tok_per_step * args.steps / (ms / 1e3)
    gpu_launches = sum(n for n, _ in prof.values())

    dom = dominant(prof)
    roofline = None
    if dom is not None:
        name, (nl, tms) = dom
        per_launch_s = tms / nl / 1e3
        alg = KERNEL_BYTES_PER_TOKEN_HEAD[name] * nb * T * heads
        achieved = alg / per_launch_s / 1e9
        tot_ms = sum(x[1] for x in prof.values())
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "peak_source": peak_kind,
                    "traffic": traffic_table().get(name) if (full and world == 1) else None, "kernel": name,
                    "algorithmic_bytes_per_launch": alg, "us_per_launch": per_launch_s * 1e6,
                    "kernel_shares": {n: round(t / tot_ms, 4) for n, (c, t) in prof.items()},
                    "kernel_us_per_step": {n: round(1e3 * t / args.steps, 1) for n, (c, t) in prof.items()}}
    # op level: SURVEY's 7,456 algorithmic bytes per token-head for fwd+bwd
    op_bytes = 7456 * H * tok_per_step
    op_achieved = op_bytes * args.steps / (ms / 1e3) / 1e9
    op_roofline = {"bound": "hbm", "achieved": op_achieved, "peak": peak * world, "unit": "GB/s",
                   "frac": op_achieved / (peak * world), "peak_source": peak_kind,
                   "algorithmic_bytes_per_step": op_bytes,
                   "note": "whole op (all kernels), 7456 B per token-head fwd+bwd, peak summed over the GPUs"}

    weak = None
    if world > 1:
        wms, _, _ = measure_op(rk, B, H, args.steps, args.warmup, 999 + rank, profile=False)
        weak = {"value": world * B * T * args.steps / (wms / 1e3), "unit": "tokens/s",
                "ms_per_step": wms / args.steps, "global_batch": B * world, "scaling": "weak",
                "workload": f"config2 with B=4 x 16 heads on each of the {world} ranks"}

    note("config 2 end to end")
    e2e = measure_e2e(rk, tensors, tok_per_step, args.steps)
    del tensors

    # ---- config 3 decode, split by sequence ------------------------------------
    note("config 3")
    nd = nd_total // world if nd_total % world == 0 else nd_total
    dec_ms, dprof = measure_decode(rk, nd, args.decode_steps)
    dec_us = 1e3 * dec_ms / args.decode_steps
    dec_total = nd * world
    dec_gbs = decode_bytes_per_step(dec_total) / (dec_us * 1e-6) / 1e9
    dk = dprof.get("recurrent_kernel", (1, dec_ms))
    dk_us = 1e3 * dk[1] / max(dk[0], 1)
    decode = {"metric": "decode-step state HBM GB/s", "value": dec_gbs, "unit": "GB/s",
              "us_per_step": dec_us, "tokens_per_s": dec_total / (dec_us * 1e-6),
              "scaling": "strong" if nd * world == nd_total else "weak",
              "config": {"workload": "config3 decode step", "sequences": dec_total, "sequences_per_gpu": nd,
                         "heads": H, "state": f"fp32 [{dec_total},16,128,128] in place", "steps": args.decode_steps},
              "roofline": {"bound": "hbm", "achieved": decode_bytes_per_step(nd) / (dk_us * 1e-6) / 1e9,
                           "peak": peak, "unit": "GB/s",
                           "frac": decode_bytes_per_step(nd) / (dk_us * 1e-6) / 1e9 / peak,
                           "peak_source": peak_kind, "kernel": "recurrent_kernel", "us_per_launch": dk_us,
                           "traffic": traffic_table().get("recurrent_kernel") if (nd == DEC_N) else None}}
    if cpu_torch is not None:
        decode["cpu_baseline"] = {"value": cpu_torch["b4_decode"]["value"], "unit": "GB/s",
                                  "cores": cpu_torch["cores"], "kind": "port",
                                  "sample": cpu_torch["b4_decode"]["sample"]}
    torch.cuda.empty_cache()

    # ---- config 5 (CP prefill) and config 4 (model) --------------------------
    extras = {}
    if full:
        note("config 5")
        try:
            extras["cp"] = measure_cp(rk, 5, 3)
        except Exception as e:  # noqa: BLE001
            extras["cp"] = {"error": f"{type(e).__name__}: {e}"}
        torch.cuda.empty_cache()
        note("config 4")
        try:
            extras["model"] = measure_model(rk, 4, 5, 3)
        except Exception as e:  # noqa: BLE001
            extras["model"] = {"error": f"{type(e).__name__}: {e}"}
        torch.cuda.empty_cache()
        if world == 1 and not args.no_reference_triton:
            note("reference Triton op")
            try:
                extras["reference_triton"] = measure_reference_triton(rk, min(args.steps, 20), args.warmup)
                torch.cuda.empty_cache()
            except Exception as e:  # noqa: BLE001
                extras["reference_triton"] = {"unavailable": f"{type(e).__name__}: {e}"}

    note("done")
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"config2: GDN2 op fwd+bwd, B={nb} H=16 T=4096 dk=dv=128 chunk 64, "
                                   + (f"the 64 (sequence, head) pairs split over {world} GPU(s), "
                                      f"{nb * heads} per GPU" if strong else f"B={nb} x 16 heads per GPU"),
                       "global_batch": nb, "seq_len": T, "heads": H, "head_dim": K,
                       "heads_per_gpu": heads,
                       "parallelism": f"(batch x head) shards over {world} GPU(s), no collectives",
                       "l2": f"inputs {0.15 * nb * heads / H:.2f} GB per GPU per step "
                             f"({'>' if 0.15 * nb * heads / H > 0.126 else '<'} 126 MB L2), no flush",
                       "gates": "b, w, log-decay fp32; q, k, v bf16"},
            "clocks": clk, "e2e": e2e, "gpu_launches": gpu_launches, "roofline": roofline,
            "op_roofline": op_roofline, "decode": decode,
        }
        if weak is not None:
            line["weak"] = weak
        line.update(extras)
        if cpu_base is not None:
            line["cpu_baseline"] = cpu_base
        if cpu_torch is not None:
            line["cpu_baselines"] = cpu_torch
        print(json.dumps(line), flush=True)
    rk.close()


if __name__ == "__main__":
    main()
