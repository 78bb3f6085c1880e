"""2+ ranks: every algorithm at sizes that fill its last tile partially (and
odd counts) leaves the guard lines after each mailbox area intact; a guard
line overwritten from the host is reported by Communicator.validate."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    import tiny_nccl_b200 as tn

    comm = tn.init_from_torch_distributed(device=rank)
    stream = torch.cuda.Stream(device=dev)
    algos = ["oneshot", "twoshot", "ring"] + (["nvls"] if comm.info()["nvls"] else [])
    ok = True
    with torch.cuda.stream(stream):
        for algo in algos:
            for n in (1, 4097, 1_000_003, 9_000_001):
                for dtype in (torch.float32, torch.bfloat16):
                    x = torch.ones(n, device=dev, dtype=dtype)
                    comm.all_reduce(x, algo=algo)
    torch.cuda.synchronize()
    ok = ok and comm.validate() == 0 and comm.async_error() == 0
    dist.barrier()
    if rank == 0:
        comm._c.diag_corrupt_canary(2)
    bad = comm.validate()
    ok = ok and bad == (1 if rank == 0 else 0)
    flag = torch.tensor([1.0 if ok else 0.0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        print("PASS" if flag.item() == 1.0 else "FAIL")
    torch.cuda.synchronize()
    comm.destroy()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
