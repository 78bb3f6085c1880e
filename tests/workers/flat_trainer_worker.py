"""2+ ranks: gradients through FlatGradReducer on a flat buffer registered
with the communicator (zero-copy NVLS when TNCCL_NVLS_ZERO_COPY=1) match DDP
with the tnccl hook, and DataParallelTrainer(reducer="flat", registered=True)
trains GPT-2 (small config) in step with reducer="ddp", also with AdamW
overlapped with backward (overlap_optimizer=True). Prints PASS on rank 0."""
import datetime
import math
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
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    import tiny_nccl_b200 as tn
    from tiny_nccl_b200.models import GPT2, GPT2Config
    from tiny_nccl_b200.parallel import DataParallelTrainer, FlatGradReducer, empty_registrable

    comm = tn.init_from_torch_distributed(device=rank)
    nvls = comm.info()["nvls"]
    cfg = GPT2Config(n_layer=2, n_head=4, n_embd=256, vocab_size=2048, block_size=128)
    torch.manual_seed(0)
    base = GPT2(cfg, impl="fused").to(dev)
    m1 = GPT2(cfg, impl="fused").to(dev)
    m2 = GPT2(cfg, impl="fused").to(dev)
    m1.load_state_dict(base.state_dict())
    m2.load_state_dict(base.state_dict())
    side = comm.side_stream()
    red = FlatGradReducer(m1.parameters(), lambda t: comm.all_reduce(t, op="avg"),
                          bucket_bytes=1 << 20,
                          alloc=(lambda n, dt, d: empty_registrable(n, dt, d)) if nvls else None,
                          stream=side)
    handle = comm.register(red.flat) if nvls else None
    d2 = DDP(m2, device_ids=[rank], bucket_cap_mb=1, gradient_as_bucket_view=True)
    tn.register_tnccl_hook(d2, comm)
    g = torch.Generator(device="cpu")
    g.manual_seed(100 + rank)
    idx = torch.randint(0, 2048, (2, 129), generator=g).to(dev)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss1 = m1(idx[:, :-1], idx[:, 1:])
    loss1.backward()
    red.finish()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss2 = d2(idx[:, :-1], idx[:, 1:])
    loss2.backward()
    torch.cuda.synchronize()
    worst = 0.0
    for (n, a), (_, b) in zip(m1.named_parameters(), m2.named_parameters()):
        err = (a.grad - b.grad).abs().max().item()
        worst = max(worst, err / (b.grad.abs().max().item() + 1e-12))
    ok = worst < 1e-5 and red.launched == len(red.buckets)
    if handle is not None:
        comm.deregister(handle)
    red.remove()

    # Whole trainer, both reducers, three steps from the same weights.
    torch.manual_seed(1)
    a = GPT2(cfg, impl="fused").to(dev)
    b = GPT2(cfg, impl="fused").to(dev)
    b.load_state_dict(a.state_dict())
    c = GPT2(cfg, impl="fused").to(dev)
    c.load_state_dict(a.state_dict())
    ta = DataParallelTrainer(a, comm, reducer="flat", registered=True)
    tb = DataParallelTrainer(b, comm, reducer="ddp")
    # AdamW applied bucket by bucket on the comm stream during backward.
    tc = DataParallelTrainer(c, comm, reducer="flat", registered=True, overlap_optimizer=True)
    for step in range(3):
        g.manual_seed(1000 * step + rank)
        idx = torch.randint(0, 2048, (2, 129), generator=g).to(dev)
        la = ta.step(idx[:, :-1], idx[:, 1:]).item()
        lb = tb.step(idx[:, :-1], idx[:, 1:]).item()
        lc = tc.step(idx[:, :-1], idx[:, 1:]).item()
        ok = ok and math.isfinite(la) and abs(la - lb) < 1e-2 and abs(la - lc) < 1e-4
    pd = max((x - y).abs().max().item() for x, y in zip(a.parameters(), b.parameters()))
    pc = max((x - y).abs().max().item() for x, y in zip(a.parameters(), c.parameters()))
    ok = ok and pd < 5e-3 and pc < 1e-5 and comm.async_error() == 0
    ta.close()
    tc.close()
    flag = torch.tensor([1.0 if ok else 0.0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(f"nvls={nvls} buckets={len(red.buckets)} worst_rel_grad_diff={worst:.3e} "
              f"param_diff_after_3_steps={pd:.3e} overlapped_optimizer_diff={pc:.3e}")
        print("PASS" if flag.item() == 1.0 else "FAIL")
    torch.cuda.synchronize()
    comm.destroy()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
