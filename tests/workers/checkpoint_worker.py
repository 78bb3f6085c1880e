"""Checkpoint / resume of the data-parallel GPT-2 trainer: train 3 steps,
save model + optimizer + step to a file, train 2 more steps; a fresh trainer
loaded from the file must reproduce those 2 losses."""
import datetime
import os
import sys
import tempfile

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


def make_trainer(comm, dev):
    from tiny_nccl_b200.models import GPT2, GPT2Config
    from tiny_nccl_b200.parallel import DataParallelTrainer
    torch.manual_seed(7)
    cfg = GPT2Config(n_layer=2, n_head=4, n_embd=256, vocab_size=1000, block_size=128)
    model = GPT2(cfg, impl="fused").to(dev)
    return DataParallelTrainer(model, comm, lr=1e-3)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    import tiny_nccl_b200 as tn

    comm = tn.init_from_torch_distributed(device=rank)
    g = torch.Generator(device="cpu").manual_seed(100 + rank)
    batches = [torch.randint(0, 1000, (2, 129), generator=g).to(dev) for _ in range(5)]

    def run(tr, bs):
        out = []
        for b in bs:
            out.append(float(tr.step(b[:, :-1], b[:, 1:])))
        return out

    tr = make_trainer(comm, dev)
    run(tr, batches[:3])
    path = os.path.join(tempfile.gettempdir(), f"tnccl_ckpt_{os.getpid()}.pt")
    torch.save(tr.state_dict(), path)
    after = run(tr, batches[3:])

    tr2 = make_trainer(comm, dev)
    tr2.load_state_dict(torch.load(path, map_location=dev))
    os.remove(path)
    resumed = run(tr2, batches[3:])
    ok = all(abs(a - b) <= 1e-3 * max(1.0, abs(a)) for a, b in zip(after, resumed))
    ok = ok and tr2.opt._step == 5 and comm.async_error() == 0
    flag = torch.tensor([1.0 if ok else 0.0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        print("losses", after, resumed)
        print("PASS" if flag.item() == 1.0 else "FAIL")
    torch.cuda.synchronize()
    comm.destroy()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
