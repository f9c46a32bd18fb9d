"""Context-parallel prefill (T sharded over ranks).

* CPU, gloo, world size 2: the protocol of ``cp.chunk_gdn2_cp`` (transition
  maps -> all_gather -> compose -> forward) with the steps computed by the
  fp64 oracle, against the oracle on the whole sequence; the backward
  protocol (state cotangent -> all_gather -> reverse compose -> shard
  backward) against the oracle's gradients of the whole sequence; and a rank
  that fails before the collective, which the surviving rank must see as an
  error.
* GPU, one device: the CUDA steps with the ranks emulated in one process,
  forward and backward.
* GPU, two devices: the real NCCL path, forward and backward (skipped with
  fewer devices).
"""

import os
import socket
import subprocess
import sys
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import gdn2_oracle as orc
from tolerance import assert_close

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class OracleBackend:
    """The protocol's three steps computed by the CPU oracle (fp64)."""

    def transition(self, q, k, v, g, b, w, *, scale, use_qk_l2norm_in_kernel, use_gate_in_kernel,
                   A_log, dt_bias, lower_bound):
        q, k, v, g, b, w = (x.double().numpy() for x in (q, k, v, g, b, w))
        if use_qk_l2norm_in_kernel:
            q, k = orc.l2norm_fwd(q)[0], orc.l2norm_fwd(k)[0]
        if use_gate_in_kernel:
            g = orc.gate_fwd(g, A_log.double().numpy(), None if dt_bias is None else dt_bias.double().numpy(),
                             lower_bound)
        B, T, H, K = q.shape
        _, h_e, _ = orc.recurrent_fwd(q, k, v, g, b, w, scale)
        eye = np.broadcast_to(np.eye(K), (B, H, K, K)).copy()
        _, M, _ = orc.recurrent_fwd(q, k, np.zeros((B, T, H, K)), g, b, np.ones((B, T, H, K)), scale, eye)
        return torch.from_numpy(np.concatenate([M, h_e], axis=-1))

    def compose(self, gathered, rank, state):
        K = state.shape[-2]
        S = state.double()
        for j in range(rank):
            S = gathered[j, ..., :K].double() @ S + gathered[j, ..., K:].double()
        return S

    def forward(self, q, k, v, g, b, w, *, initial_state, scale, use_qk_l2norm_in_kernel,
                use_gate_in_kernel, lower_bound, A_log=None, dt_bias=None):
        r = orc.chunk_gdn2(*(x.double().numpy() for x in (q, k, v, g, b, w)), scale=scale,
                           initial_state=initial_state.numpy(), output_final_state=True,
                           use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel,
                           use_gate_in_kernel=use_gate_in_kernel, lower_bound=lower_bound,
                           A_log=None if A_log is None else A_log.double().numpy(),
                           dt_bias=None if dt_bias is None else dt_bias.double().numpy())
        return torch.from_numpy(r.o), torch.from_numpy(r.final_state)

    # ---- training pieces (fp64) --------------------------------------------
    def forward_train(self, q, k, v, g, b, w, *, initial_state, scale, use_qk_l2norm_in_kernel,
                      use_gate_in_kernel, A_log, dt_bias, lower_bound):
        x = [t.detach().double().numpy() for t in (q, k, v, g, b, w)]
        kw = dict(scale=scale, use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel,
                  use_gate_in_kernel=use_gate_in_kernel, lower_bound=lower_bound,
                  A_log=None if A_log is None else A_log.detach().double().numpy(),
                  dt_bias=None if dt_bias is None else dt_bias.detach().double().numpy())
        S = initial_state.detach().double().numpy()
        r = orc.chunk_gdn2(*x, initial_state=S, output_final_state=True, **kw)
        return torch.from_numpy(r.o), torch.from_numpy(r.final_state), (x, S, kw)

    def state_cotangent(self, data, do, dht):
        x, S, kw = data
        r = orc.chunk_gdn2(*x, initial_state=S, output_final_state=True, do=do.double().numpy(),
                           dht=dht.double().numpy(), **kw)
        return torch.from_numpy(r.grads["h0"])

    def compose_bwd(self, gathered_maps, gathered_g, rank, dht):
        K = gathered_maps.shape[-2]
        X = torch.zeros(dht.shape, dtype=torch.float64)
        for j in range(gathered_maps.shape[0] - 1, rank, -1):
            X = gathered_maps[j, ..., :K].double().transpose(-1, -2) @ X + gathered_g[j].double()
        return dht.double() + X

    def backward(self, data, do, dS_out):
        x, S, kw = data
        r = orc.chunk_gdn2(*x, initial_state=S, output_final_state=True, do=do.double().numpy(),
                           dht=dS_out.double().numpy(), **kw)
        t = lambda a: None if a is None else torch.from_numpy(a)  # noqa: E731
        gr = r.grads
        return tuple(t(gr[n]) for n in ("q", "k", "v", "g", "b", "w", "A_log", "dt_bias", "h0"))


def _problem(T=96, H=2, K=16, V=8, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, T, H, K, generator=g)
    k = torch.randn(1, T, H, K, generator=g)
    v = torch.randn(1, T, H, V, generator=g)
    graw = torch.randn(1, T, H, K, generator=g)
    b = torch.sigmoid(torch.randn(1, T, H, K, generator=g))
    w = torch.sigmoid(torch.randn(1, T, H, V, generator=g))
    h0 = torch.randn(1, H, K, V, generator=g) * 0.1
    A_log = torch.rand(H, generator=g)
    dt = torch.randn(H * K, generator=g) * 0.3
    return q, k, v, graw, b, w, h0, A_log, dt


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cp_worker(rank, world, port, out_dir, fail_rank):
    import importlib
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    cp = importlib.import_module("gateddeltanet-2_b200.cp")
    q, k, v, graw, b, w, h0, A_log, dt = _problem()
    Ts = q.shape[1] // world
    sl = slice(rank * Ts, (rank + 1) * Ts)
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        o, ht = cp.chunk_gdn2_cp(q[:, sl], k[:, sl], v[:, sl], graw[:, sl], b[:, sl], w[:, sl],
                                 initial_state=h0, use_qk_l2norm_in_kernel=True,
                                 use_gate_in_kernel=True, A_log=A_log, dt_bias=dt,
                                 backend=OracleBackend())
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), o=o.numpy(), ht=ht.numpy())
    except Exception as e:  # record what this rank saw
        with open(os.path.join(out_dir, f"rank{rank}.err"), "w") as f:
            f.write(repr(e))
    finally:
        if rank != fail_rank:
            dist.destroy_process_group()


def test_cp_protocol_gloo_two_ranks():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_cp_worker, args=(world, _free_port(), d, -1), nprocs=world,
                           start_method="spawn")
        q, k, v, graw, b, w, h0, A_log, dt = _problem()
        r = orc.chunk_gdn2(*(x.double().numpy() for x in (q, k, v, graw, b, w)), initial_state=h0.numpy(),
                           output_final_state=True, use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True,
                           A_log=A_log.numpy(), dt_bias=dt.numpy())
        outs = [np.load(os.path.join(d, f"rank{i}.npz")) for i in range(world)]
        o = np.concatenate([x["o"] for x in outs], axis=1)
        np.testing.assert_allclose(o, r.o, rtol=1e-9, atol=1e-11)
        np.testing.assert_allclose(outs[-1]["ht"], r.final_state, rtol=1e-9, atol=1e-11)


def test_cp_rank_failure_is_reported_not_hung():
    """Rank 1 dies before the all_gather; rank 0's collective must end with an
    error (gloo timeout / peer loss) instead of waiting forever."""
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_cp_worker, args=(world, _free_port(), d, 1), nprocs=world,
                           start_method="spawn")
        assert os.path.exists(os.path.join(d, "rank1.err"))
        assert os.path.exists(os.path.join(d, "rank0.err")), "surviving rank did not report the failure"


def _cp_train_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    import importlib
    cp = importlib.import_module("gateddeltanet-2_b200.cp")
    q, k, v, graw, b, w, h0, A_log, dt = _problem()
    gen = torch.Generator().manual_seed(7)
    do = torch.randn(q.shape[:3] + (v.shape[-1],), generator=gen, dtype=torch.float64)
    dht = torch.randn(h0.shape, generator=gen, dtype=torch.float64)
    Ts = q.shape[1] // world
    sl = slice(rank * Ts, (rank + 1) * Ts)
    leaves = [x[:, sl].double().clone().requires_grad_(True) for x in (q, k, v, graw, b, w)]
    A = A_log.double().clone().requires_grad_(True)
    dtb = dt.double().clone().requires_grad_(True)
    h = h0.double().clone().requires_grad_(True)
    o, ht = cp.chunk_gdn2_cp(*leaves, initial_state=h, use_qk_l2norm_in_kernel=True,
                             use_gate_in_kernel=True, A_log=A, dt_bias=dtb, backend=OracleBackend())
    loss = (o * do[:, sl]).sum() + ((ht * dht).sum() if rank == world - 1 else 0.0)
    loss.backward()
    # gate parameters are shared by all shards: their gradients add up
    for p in (A, dtb):
        dist.all_reduce(p.grad)
    np.savez(os.path.join(out_dir, f"grads{rank}.npz"),
             **{n: x.grad.numpy() for n, x in zip("qkvgbw", leaves)},
             A_log=A.grad.numpy(), dt_bias=dtb.grad.numpy(), h0=h.grad.numpy(),
             do=do.numpy(), dht=dht.numpy())
    dist.destroy_process_group()


def test_cp_backward_protocol_gloo_two_ranks():
    """Per-shard gradients of the context-parallel op (fp64 oracle steps)
    against the oracle's gradients of the whole sequence."""
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_cp_train_worker, args=(world, _free_port(), d), nprocs=world,
                           start_method="spawn")
        outs = [np.load(os.path.join(d, f"grads{i}.npz")) for i in range(world)]
    q, k, v, graw, b, w, h0, A_log, dt = _problem()
    r = orc.chunk_gdn2(*(x.double().numpy() for x in (q, k, v, graw, b, w)), initial_state=h0.double().numpy(),
                       output_final_state=True, use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True,
                       A_log=A_log.double().numpy(), dt_bias=dt.double().numpy(), do=outs[0]["do"],
                       dht=outs[0]["dht"])
    for n in "qkvgbw":
        got = np.concatenate([x[n] for x in outs], axis=1)
        np.testing.assert_allclose(got, r.grads[n], rtol=1e-8, atol=1e-10, err_msg=f"d{n}")
    for n in ("A_log", "dt_bias"):
        np.testing.assert_allclose(outs[0][n], r.grads[n], rtol=1e-8, atol=1e-10, err_msg=f"d{n}")
    np.testing.assert_allclose(outs[0]["h0"], r.grads["h0"], rtol=1e-8, atol=1e-10, err_msg="dh0 (rank 0)")
    assert np.abs(outs[1]["h0"]).max() == 0.0  # only rank 0 carries the initial state's gradient


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_cp_emulated_ranks_backward_match_full_sequence(gdn2, world):
    """The CUDA backward pieces with the ranks emulated in one process (state
    cotangents, reverse compose, shard backward) against the single-GPU
    backward of the whole sequence and the oracle."""
    cp = __import__("importlib").import_module("gateddeltanet-2_b200.cp")
    be = cp.CudaBackend()
    T, H, K, V = 512, 2, 128, 128
    gen = torch.Generator().manual_seed(10 + world)
    q = torch.nn.functional.normalize(torch.randn(1, T, H, K, generator=gen), dim=-1).bfloat16().cuda()
    k = torch.nn.functional.normalize(torch.randn(1, T, H, K, generator=gen), dim=-1).bfloat16().cuda()
    v = torch.randn(1, T, H, V, generator=gen).bfloat16().cuda()
    g = (-torch.nn.functional.softplus(torch.randn(1, T, H, K, generator=gen)) * 0.1).cuda()
    b = torch.sigmoid(torch.randn(1, T, H, K, generator=gen)).cuda()
    w = torch.sigmoid(torch.randn(1, T, H, V, generator=gen)).cuda()
    h0 = (torch.randn(1, H, K, V, generator=gen) * 0.1).cuda()
    do = torch.randn(1, T, H, V, generator=gen).bfloat16().cuda()
    dht = (torch.randn(1, H, K, V, generator=gen) * 0.1).cuda()  # dh is kept in bf16: see tolerance.py
    Ts = T // world
    kw = dict(scale=K ** -0.5, use_qk_l2norm_in_kernel=False, use_gate_in_kernel=False, A_log=None,
              dt_bias=None, lower_bound=None)
    shards = [[x[:, r * Ts:(r + 1) * Ts] for x in (q, k, v, g, b, w)] for r in range(world)]
    gathered = torch.stack([be.transition(*s, **kw) for s in shards])
    data = []
    for r in range(world):
        S_in = be.compose(gathered, r, h0)
        data.append(be.forward_train(*shards[r], initial_state=S_in, **kw)[2])
    zero = torch.zeros_like(dht)
    own = [dht if r == world - 1 else zero for r in range(world)]
    dos = [do[:, r * Ts:(r + 1) * Ts] for r in range(world)]
    gp = torch.stack([be.state_cotangent(data[r], dos[r], own[r]) for r in range(world)])
    grads = []
    for r in range(world):
        dS_out = be.compose_bwd(gathered, gp, r, own[r])
        grads.append(be.backward(data[r], dos[r], dS_out))
    torch.cuda.synchronize()
    leaves = [x.clone().requires_grad_(True) for x in (q, k, v, g, b, w)]
    h0l = h0.clone().requires_grad_(True)
    o, ht = gdn2.chunk_gdn2(*leaves, initial_state=h0l, output_final_state=True)
    torch.autograd.backward([o, ht], [do, dht])
    ref = orc.chunk_gdn2(*(x.float().cpu().numpy() for x in (q, k, v, g, b, w)),
                         initial_state=h0.cpu().numpy(), output_final_state=True,
                         do=do.float().cpu().numpy(), dht=dht.cpu().numpy())
    for i, n in enumerate("qkvgbw"):
        got = torch.cat([gr[i] for gr in grads], dim=1)
        assert_close(got, ref.grads[n], f"d{n} (cp)")
        assert_close(got, leaves[i].grad, f"d{n} (cp vs single)")
    assert_close(grads[0][8], ref.grads["h0"], "dh0 (cp)")


@pytest.mark.gpu
@pytest.mark.parametrize("world,T", [(2, 512), (4, 512), (2, 4096)])
def test_cp_emulated_ranks_match_full_sequence(gdn2, world, T):
    """T = 4096 over 2 ranks: 32 chunks per shard, so each shard's transition
    runs in segments (every segment's M_s and h_s, then two folds)."""
    cp = __import__("importlib").import_module("gateddeltanet-2_b200.cp")
    be = cp.CudaBackend()
    H, K, V = 2, 128, 128
    gen = torch.Generator().manual_seed(world)
    q = torch.nn.functional.normalize(torch.randn(1, T, H, K, generator=gen), dim=-1).bfloat16().cuda()
    k = torch.nn.functional.normalize(torch.randn(1, T, H, K, generator=gen), dim=-1).bfloat16().cuda()
    v = torch.randn(1, T, H, V, generator=gen).bfloat16().cuda()
    g = (-torch.nn.functional.softplus(torch.randn(1, T, H, K, generator=gen)) * 0.1).cuda()
    b = torch.sigmoid(torch.randn(1, T, H, K, generator=gen)).cuda()
    w = torch.sigmoid(torch.randn(1, T, H, V, generator=gen)).cuda()
    h0 = (torch.randn(1, H, K, V, generator=gen) * 0.1).cuda()
    Ts = T // world
    kw = dict(scale=K ** -0.5, use_qk_l2norm_in_kernel=False, use_gate_in_kernel=False, A_log=None,
              dt_bias=None, lower_bound=None)
    shards = [[x[:, r * Ts:(r + 1) * Ts] for x in (q, k, v, g, b, w)] for r in range(world)]
    gathered = torch.stack([be.transition(*s, **kw) for s in shards])
    outs = []
    for r in range(world):
        S = be.compose(gathered, r, h0)
        outs.append(be.forward(*shards[r], initial_state=S, scale=K ** -0.5))
    o = torch.cat([x[0] for x in outs], dim=1)
    with torch.no_grad():
        o_full, ht_full = gdn2.chunk_gdn2(q, k, v, g, b, w, initial_state=h0, output_final_state=True)
    torch.cuda.synchronize()
    ref = orc.chunk_gdn2(*(x.float().cpu().numpy() for x in (q, k, v, g, b, w)),
                         initial_state=h0.cpu().numpy(), output_final_state=True)
    assert_close(o, ref.o, "o (cp)")
    assert_close(outs[-1][1], ref.final_state, "final state (cp)")
    assert_close(o, o_full, "o (cp vs single)")


@pytest.mark.gpu
def test_cp_nccl_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    script = os.path.join(ROOT, "tests", "cp_nccl_check.py")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), script]
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "CP_OK" in r.stdout


def test_factor_reuse_key_tracks_every_dependency(gdn2):
    """The CUDA backend reuses a transition's intra-chunk factors only for the
    very tensors it saw, unmodified, with the same gate parameters and flags."""
    key = gdn2.cp._reuse_key
    L = gdn2._lib
    t = [torch.zeros(2) for _ in range(8)]
    flags = L.GATE_IN_KERNEL | L.LOWER_BOUND
    base = key(t, flags, 0.1, -1.0)
    assert key(t, flags, 0.1, -1.0) == base
    assert key(t, flags, 0.1, -2.0) != base           # another lower bound
    assert key(t, flags, 0.2, -1.0) != base           # another scale
    assert key(t, L.GATE_IN_KERNEL, 0.1, -1.0) != base
    other = list(t)
    other[6] = torch.zeros(2)                          # another A_log tensor
    assert key(other, flags, 0.1, -1.0) != base
    t[7].add_(1.0)                                     # dt_bias edited in place
    assert key(t, flags, 0.1, -1.0) != base
    # without LOWER_BOUND the bound's value is irrelevant
    assert key(t, 0, 0.1, -1.0) == key(t, 0, 0.1, -3.0)
