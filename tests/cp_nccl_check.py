"""Run under torch.distributed.run with one rank per GPU: context-parallel
forward over NCCL against the single-GPU forward of the whole sequence.
Prints CP_OK on rank 0 when every rank's shard matches."""

import importlib
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    gdn2 = importlib.import_module("gateddeltanet-2_b200")
    from gdn2_b200 import cp
    from tolerance import assert_close
    T, H, K, V = 1024 * world, 4, 128, 128
    gen = torch.Generator().manual_seed(0)
    q = torch.nn.functional.normalize(torch.randn(1, T, H, K, generator=gen), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(1, T, H, K, generator=gen), dim=-1).bfloat16()
    v = torch.randn(1, T, H, V, generator=gen).bfloat16()
    g = -torch.nn.functional.softplus(torch.randn(1, T, H, K, generator=gen)) * 0.1
    b = torch.sigmoid(torch.randn(1, T, H, K, generator=gen))
    w = torch.sigmoid(torch.randn(1, T, H, V, generator=gen))
    h0 = torch.randn(1, H, K, V, generator=gen) * 0.1
    full = [x.to(dev) for x in (q, k, v, g, b, w)]
    Ts = T // world
    shard = [x[:, rank * Ts:(rank + 1) * Ts] for x in full]
    o, ht = cp.chunk_gdn2_cp(*shard, initial_state=h0.to(dev))
    with torch.no_grad():
        o_ref, ht_ref = gdn2.chunk_gdn2(*full, initial_state=h0.to(dev), output_final_state=True)
    torch.cuda.synchronize()
    assert_close(o, o_ref[:, rank * Ts:(rank + 1) * Ts], f"o rank {rank}")
    if rank == world - 1:
        assert_close(ht, ht_ref, "final state")
    # backward: per-shard gradients against the single-GPU backward of the sequence
    do = (torch.randn(1, T, H, V, generator=gen) * 0.5).bfloat16().to(dev)
    dht = (torch.randn(1, H, K, V, generator=gen) * 0.1).to(dev)
    leaves = [x.clone().requires_grad_(True) for x in shard]
    h0l = h0.to(dev).clone().requires_grad_(True)
    o, ht = cp.chunk_gdn2_cp(*leaves, initial_state=h0l)
    cot_ht = dht if rank == world - 1 else torch.zeros_like(dht)
    torch.autograd.backward([o, ht], [do[:, rank * Ts:(rank + 1) * Ts], cot_ht])
    full_l = [x.clone().requires_grad_(True) for x in full]
    h0f = h0.to(dev).clone().requires_grad_(True)
    o_f, ht_f = gdn2.chunk_gdn2(*full_l, initial_state=h0f, output_final_state=True)
    torch.autograd.backward([o_f, ht_f], [do, dht])
    torch.cuda.synchronize()
    for n, lf, ls in zip("qkvgbw", full_l, leaves):
        assert_close(ls.grad, lf.grad[:, rank * Ts:(rank + 1) * Ts], f"d{n} rank {rank}")
    if rank == 0:
        assert_close(h0l.grad, h0f.grad, "dh0")
    ok = torch.ones(1, device=dev)
    dist.all_reduce(ok)
    if rank == 0 and int(ok.item()) == world:
        print("CP_OK", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
