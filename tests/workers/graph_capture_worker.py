"""2+ ranks: tnccl all-reduces captured in a CUDA graph replay correctly (the
FIFO sequence numbers live in device memory and advance on every replay),
interleaved with eager collectives on the same communicator."""
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
    sizes = [1000, 1 << 16, 3 << 20]
    algos = ["oneshot", "twoshot", "ring"] + (["nvls"] if comm.info()["nvls"] else [])
    xs = [torch.zeros(n, device=dev) for n in sizes]
    ys = [torch.zeros(n, device=dev) for n in sizes]
    ok = True
    with torch.cuda.stream(stream):
        for x, y in zip(xs, ys):  # eager warm-up binds the stream
            comm.all_reduce(x, y)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for x, y, a in zip(xs, ys, algos * 2):
            comm.all_reduce(x, y, algo=a)
    for it in range(4):
        with torch.cuda.stream(stream):
            for i, x in enumerate(xs):
                x.fill_(float(rank + 1 + it + i))
            graph.replay()
            # an eager collective between replays must also line up
            e = torch.full((777,), float(rank), device=dev)
            comm.all_reduce(e)
        torch.cuda.synchronize()
        for i, y in enumerate(ys):
            want = sum(float(r + 1 + it + i) for r in range(world))
            ok = ok and bool(torch.all(y == want).item())
        ok = ok and bool(torch.all(e == sum(range(world))).item())
    ok = ok and comm.async_error() == 0
    flag = torch.tensor([1.0 if ok else 0.0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        print("PASS" if flag.item() == 1.0 else "FAIL")
    del graph
    torch.cuda.synchronize()
    comm.destroy()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
