"""Configuration sweep for the tnccl all-reduce kernels (channels, threads,
chunk sizes), one communicator per configuration inside one job.

Every rank sets the same TNCCL_* environment before creating each
communicator (the bootstrap rejects ranks whose configurations differ).
Timing as in allreduce_sweep.py: CUDA events around K launches on the bound
stream, max over ranks.
"""
from __future__ import annotations

import argparse
import datetime
import itertools
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--algo", default="twoshot")
    ap.add_argument("--dtype", default="fp32")
    ap.add_argument("--sizes", default="1M,16M,256M")
    ap.add_argument("--grid", default='{"TNCCL_NCHANNELS": [32, 64, 128], "TNCCL_NTHREADS": [256, 512]}')
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--out", default="")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    import tiny_nccl_b200 as tn

    dtype = {"fp32": torch.float32, "bf16": torch.bfloat16}[args.dtype]
    es = torch.empty((), dtype=dtype).element_size()
    mult = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}
    sizes = [int(s[:-1]) * mult[s[-1]] for s in args.sizes.split(",")]
    grid = json.loads(args.grid)
    keys = list(grid)
    x = torch.randn(max(sizes) // es, device=dev).to(dtype)
    y = torch.empty_like(x)
    stream = torch.cuda.Stream(device=dev)
    out = open(args.out, "a") if (args.out and rank == 0) else None
    for n_cfg, values in enumerate(itertools.product(*[grid[k] for k in keys])):
        cfg = dict(zip(keys, values))
        for k, v in cfg.items():
            os.environ[k] = str(v)
        comm = tn.init_from_torch_distributed(key=f"tnccl/tune{n_cfg}", device=local)
        for size in sizes:
            n = size // es
            with torch.cuda.stream(stream):
                for _ in range(3):
                    comm.all_reduce(x[:n], y[:n], algo=args.algo)
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            k = args.iters if size <= (64 << 20) else max(3, args.iters // 4)
            with torch.cuda.stream(stream):
                e0.record()
                for _ in range(k):
                    comm.all_reduce(x[:n], y[:n], algo=args.algo)
                e1.record()
            torch.cuda.synchronize()
            ms = torch.tensor([e0.elapsed_time(e1) / k], device=dev)
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            t = ms.item() * 1e-3
            bus = size / t / 1e9 * (2 * (world - 1) / world)
            rec = {"algo": args.algo, "cfg": cfg, "bytes": size, "us": t * 1e6, "busbw_gbs": bus,
                   "n_gpus": world, "err": comm.async_error()}
            if rank == 0:
                print(json.dumps(rec), flush=True)
                if out:
                    out.write(json.dumps(rec) + "\n")
        torch.cuda.synchronize()
        comm.destroy()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
