"""Runs one multi-rank all-reduce algorithm with emulated ranks on a single
GPU (one cooperative launch), for ncu profiles of the collective kernels and
single-GPU timing of their data movement.

    python benchmarks/emulated_kernel.py --algo twoshot --ranks 2 --bytes 64M --iters 3
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--algo", default="twoshot")
    ap.add_argument("--ranks", type=int, default=2)
    ap.add_argument("--bytes", default="64M")
    ap.add_argument("--dtype", default="fp32")
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    import tiny_nccl_b200 as tn

    mult = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}
    size = int(args.bytes[:-1]) * mult[args.bytes[-1]]
    dtype = {"fp32": torch.float32, "bf16": torch.bfloat16}[args.dtype]
    n = size // torch.empty((), dtype=dtype).element_size()
    emu = tn.load().Emulator(args.ranks)
    xs = [torch.randn(n, device="cuda").to(dtype) for _ in range(args.ranks)]
    ys = [torch.empty_like(x) for x in xs]
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    emu.all_reduce(xs, ys, algo=args.algo)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(args.iters):
        emu.all_reduce(xs, ys, algo=args.algo)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.iters
    print(f"{args.algo} ranks={args.ranks} bytes={size} ms={ms:.3f} "
          f"per-rank algbw={size / ms / 1e6:.1f} GB/s err={emu.async_error()}")
    assert emu.async_error() == 0
    emu.destroy()


if __name__ == "__main__":
    main()
