"""2 gloo ranks on CPU: FlatGradReducer (flat gradient buffer, buckets
all-reduced in order from post-accumulate-grad hooks) gives the same
gradients and parameters as DistributedDataParallel over three SGD steps,
with tiny buckets (many of them), odd parameter sizes (16-byte padding) and a
parameter that gets no gradient (its bucket is launched by finish()); and
SGD applied per bucket from the on_reduced callback during backward gives
bit-identical parameters to SGD after backward. Prints PASS on rank 0."""
import copy
import datetime
import os
import sys

import torch
import torch.distributed as dist
from torch.nn.parallel import DistributedDataParallel as DDP

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


class Net(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.a = torch.nn.Linear(16, 33)
        self.b = torch.nn.Linear(33, 5)
        self.unused = torch.nn.Parameter(torch.randn(7))

    def forward(self, x):
        return self.b(torch.nn.functional.gelu(self.a(x)))


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    from tiny_nccl_b200.parallel.reducer import FlatGradReducer

    torch.manual_seed(0)
    net_a = Net()
    net_b = copy.deepcopy(net_a)
    net_c = copy.deepcopy(net_a)
    ddp = DDP(net_b, find_unused_parameters=True)

    def avg(t):
        dist.all_reduce(t)
        t.div_(world)

    red = FlatGradReducer(net_a.parameters(), avg, bucket_bytes=256)

    def sgd(params):
        with torch.no_grad():
            for p in params:
                p -= 0.1 * p.grad

    red_c = FlatGradReducer(net_c.parameters(), avg, bucket_bytes=256, on_reduced=sgd)
    ok = len(red.buckets) >= 3
    ok = ok and all((s * 4) % 16 == 0 and (e * 4) % 16 == 0 for s, e in red.buckets)
    g = torch.Generator()
    for step in range(3):
        g.manual_seed(100 * step + rank)
        x = torch.randn(8, 16, generator=g)
        net_a(x).pow(2).mean().backward()
        red.finish()
        # After every backward each .grad is its slice of the flat buffer
        # (zero_grad unsets them; the gradients land in the slices again).
        ptr = red.flat.data_ptr()
        ok = ok and all(p.grad is not None and ptr <= p.grad.data_ptr() < ptr + red.flat.numel() * 4
                        for p in net_a.parameters())
        ddp(x).pow(2).mean().backward()
        net_c(x).pow(2).mean().backward()  # updated bucket by bucket inside backward
        red_c.finish()
        red_c.zero_grad()
        for (n, pa), (_, pb) in zip(net_a.named_parameters(), net_b.named_parameters()):
            gb = pb.grad if pb.grad is not None else torch.zeros_like(pb)
            if not torch.allclose(pa.grad, gb, rtol=1e-6, atol=1e-7):
                ok = False
                print(f"rank {rank} step {step}: grad of {n} differs", flush=True)
        with torch.no_grad():
            for pa, pb in zip(net_a.parameters(), net_b.parameters()):
                pa -= 0.1 * pa.grad
                if pb.grad is not None:
                    pb -= 0.1 * pb.grad
        red.zero_grad()
        net_b.zero_grad(set_to_none=True)
    ok = ok and red.launched == 3 * len(red.buckets)
    for pa, pb in zip(net_a.parameters(), net_b.parameters()):
        ok = ok and torch.allclose(pa, pb, rtol=1e-6, atol=1e-7)
    for pa, pc in zip(net_a.parameters(), net_c.parameters()):
        if not torch.equal(pa, pc):
            ok = False
            print(f"rank {rank}: per-bucket update differs", flush=True)
    flag = torch.tensor([1.0 if ok else 0.0])
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(f"buckets={len(red.buckets)} launched={red.launched}")
        print("PASS" if flag.item() == 1.0 else "FAIL")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
