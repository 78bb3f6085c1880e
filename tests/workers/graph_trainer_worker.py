"""2+ ranks: DataParallelTrainer with the flat gradient buffer and the whole
step captured in a CUDA graph (reducer="flat", cuda_graph=True; the bucket
all-reduces are tnccl kernels inside the graph, replayed every step) trains
GPT-2 (small config) in step with the eager DDP + tnccl-hook trainer from the
same weights: losses and parameters agree after 8 steps, and the graph
trainer's replays relaunch this library's kernels. Prints PASS on rank 0."""
import datetime
import math
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    import tiny_nccl_b200 as tn
    from tiny_nccl_b200.models import GPT2, GPT2Config
    from tiny_nccl_b200.parallel import DataParallelTrainer

    cfg = GPT2Config(n_layer=2, n_head=4, n_embd=256, vocab_size=2048, block_size=128)
    torch.manual_seed(1)
    a = GPT2(cfg, impl="fused").to(dev)
    b = GPT2(cfg, impl="fused").to(dev)
    b.load_state_dict(a.state_dict())
    ca = tn.init_from_torch_distributed(device=rank)
    cb = tn.init_from_torch_distributed(device=rank)
    # Small buckets, so that every step has several bucket all-reduces.
    ta = DataParallelTrainer(a, ca, reducer="flat", cuda_graph=True, bucket_cap_mb=1)
    tb = DataParallelTrainer(b, cb, reducer="ddp", bucket_cap_mb=1)
    g = torch.Generator(device="cpu")
    ok, worst = True, 0.0
    for step in range(8):
        g.manual_seed(1000 * step + rank)
        idx = torch.randint(0, 2048, (2, 129), generator=g).to(dev)
        la = ta.step(idx[:, :-1], idx[:, 1:]).item()
        lb = tb.step(idx[:, :-1], idx[:, 1:]).item()
        worst = max(worst, abs(la - lb))
        ok = ok and math.isfinite(la) and abs(la - lb) < 2e-2
    pd = max((x - y).abs().max().item() for x, y in zip(a.parameters(), b.parameters()))
    replays = ta.replayed_launches
    ok = ok and pd < 1e-2 and replays > 0 and ca.async_error() == 0 and cb.async_error() == 0
    torch.cuda.synchronize()
    ta.close()
    tb.close()
    flag = torch.tensor([1.0 if ok else 0.0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(f"worst loss diff {worst:.3e}, param diff after 8 steps {pd:.3e}, "
              f"kernels launched by replays {replays}")
        print("PASS" if flag.item() == 1.0 else "FAIL")
    torch.cuda.synchronize()
    ca.destroy()
    cb.destroy()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
