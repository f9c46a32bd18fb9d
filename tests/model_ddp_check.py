"""Run under torch.distributed.run with one rank per GPU: a small hybrid model
wrapped in DistributedDataParallel (NCCL gradient all-reduce) against the
same model on one process over the concatenated batch.  Prints DDP_OK on
rank 0 when every rank's averaged gradients match."""

import importlib
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    importlib.import_module("gateddeltanet-2_b200")
    from gdn2_b200 import model as m
    cfg = m.HybridConfig(vocab_size=512, n_layer=2, n_embd=256, n_head=2, intermediate_size=512,
                         local_window=64, block_size=256)
    torch.manual_seed(3)
    ref = m.GPT(cfg).to(dev)
    ref.init_weights()
    net = m.GPT(cfg).to(dev)
    net.load_state_dict(ref.state_dict())
    ddp = torch.nn.parallel.DistributedDataParallel(net, device_ids=[dev.index])
    gen = torch.Generator().manual_seed(7)
    idx = torch.randint(0, cfg.vocab_size, (2 * world, 256), generator=gen).to(dev)
    tgt = torch.randint(0, cfg.vocab_size, (2 * world, 256), generator=gen).to(dev)

    def loss_of(model, i, t):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = model(i)
        return F.cross_entropy(logits.float().view(-1, logits.shape[-1]), t.view(-1))

    loss_of(ddp, idx[2 * rank:2 * rank + 2], tgt[2 * rank:2 * rank + 2]).backward()  # DDP averages over ranks
    loss_of(ref, idx, tgt).backward()  # the whole batch on one process
    bad = []
    for (n, p), q in zip(net.named_parameters(), ref.parameters()):
        scale = q.grad.abs().max().item() + 1e-12
        err = (p.grad - q.grad).abs().max().item()
        if err > 3e-2 * scale:
            bad.append((n, err, scale))
    # every rank holds the same averaged gradients
    flat = torch.cat([p.grad.flatten() for p in net.parameters()])
    other = flat.clone()
    dist.broadcast(other, 0)
    same = torch.equal(flat, other)
    ok = torch.tensor([1 if (not bad and same) else 0], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if rank == 0:
        print("mismatches:", bad[:5], "identical across ranks:", same)
        if ok.item() == 1:
            print("DDP_OK")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
