"""2+ ranks: DDP with the tnccl comm hook produces the same gradients and the
same parameters after an optimizer step as DDP with its built-in NCCL
all-reduce. Prints PASS on rank 0."""
import datetime
import os
import sys

import torch
import torch.distributed as dist
from torch.nn.parallel import DistributedDataParallel as DDP

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    import tiny_nccl_b200 as tn
    from tiny_nccl_b200.models import GPT2, GPT2Config

    comm = tn.init_from_torch_distributed(device=rank)
    cfg = GPT2Config(n_layer=2, n_head=4, n_embd=256, vocab_size=2048, block_size=128)
    torch.manual_seed(0)
    base = GPT2(cfg, impl="fused").to(dev)
    m1 = GPT2(cfg, impl="fused").to(dev)
    m2 = GPT2(cfg, impl="fused").to(dev)
    m1.load_state_dict(base.state_dict())
    m2.load_state_dict(base.state_dict())
    d1 = DDP(m1, device_ids=[rank], bucket_cap_mb=1, gradient_as_bucket_view=True)
    d2 = DDP(m2, device_ids=[rank], bucket_cap_mb=1, gradient_as_bucket_view=True)
    state = tn.register_tnccl_hook(d1, comm)
    g = torch.Generator(device="cpu")
    g.manual_seed(100 + rank)
    idx = torch.randint(0, 2048, (2, 129), generator=g).to(dev)
    for d in (d1, d2):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = d(idx[:, :-1], idx[:, 1:])
        loss.backward()
    torch.cuda.synchronize()
    worst = 0.0
    for (n, a), (_, b) in zip(m1.named_parameters(), m2.named_parameters()):
        err = (a.grad - b.grad).abs().max().item()
        scale = b.grad.abs().max().item() + 1e-12
        worst = max(worst, err / scale)
    ok = worst < 1e-5 and state.buckets >= 1 and comm.async_error() == 0
    flag = torch.tensor([1.0 if ok else 0.0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(f"buckets={state.buckets} worst_rel_grad_diff={worst:.3e}")
        print("PASS" if flag.item() == 1.0 else "FAIL")
    torch.cuda.synchronize()
    comm.destroy()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
