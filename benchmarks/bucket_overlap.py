"""Fused gradient all-reduce benchmark: bucketed bf16 gradients with the
1/world pre-scale and fp32 accumulation fused into the all-reduce kernel,
alone and overlapped with a dummy compute stream.

Config: NB buckets of BUCKET_MB MiB of bf16 (default 20 x 25 MiB), values
Normal(0, 1e-3) seeded per rank. For each implementation:
  * comm alone: the NB bucket all-reduces back to back on the comm stream;
  * overlapped: the same all-reduces on the comm stream while the compute
    stream runs a fixed bf16 GEMM loop; reported are the comm time, the
    compute time, and the compute slowdown against the GEMM loop alone.
Implementations: tnccl (tncclAllReduceEx with op=avg: pre-scale in the
kernel, fp32 accumulate, bf16 on the wire) and NCCL (torch.distributed
all_reduce with ReduceOp.AVG on the same bf16 buffers). Device time with CUDA
events on each stream, max over ranks.

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        benchmarks/bucket_overlap.py --out bucket.jsonl

``--registered`` puts the buckets (and their outputs) in two tncclMemAlloc
regions registered with the communicator; every tnccl bucket all-reduce that
AUTO sends through NVLS (on 8 ranks from 16 MiB) is then the zero-copy
kernel (TNCCL_NVLS_ZERO_COPY=0 turns that off).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def max_over_ranks(v: float, dev) -> float:
    t = torch.tensor([v], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--buckets", type=int, default=20)
    ap.add_argument("--bucket-mb", type=float, default=25.0)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--gemm", type=int, default=8192, help="square bf16 GEMM size of the compute loop")
    ap.add_argument("--gemm-iters", type=int, default=40)
    ap.add_argument("--channels", type=int, default=32, help="tnccl CTA cap while overlapping")
    ap.add_argument("--out", default="")
    ap.add_argument("--registered", action="store_true",
                    help="buckets in tncclMemAlloc memory registered with the communicator")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    import tiny_nccl_b200 as tn

    comm = tn.init_from_torch_distributed(device=local)
    n = int(args.bucket_mb * (1 << 20)) // 2
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    buckets = [(torch.randn(n, device=dev, generator=g) * 1e-3).to(torch.bfloat16)
               for _ in range(args.buckets)]
    outs = [torch.empty_like(b) for b in buckets]
    handles = []
    if args.registered and comm.info()["nvls"]:
        from tiny_nccl_b200.parallel import empty_registrable
        src = empty_registrable(n * args.buckets, torch.bfloat16, dev)
        dst = empty_registrable(n * args.buckets, torch.bfloat16, dev)
        for k, b in enumerate(buckets):
            src[k * n:(k + 1) * n].copy_(b)
        buckets = [src[k * n:(k + 1) * n] for k in range(args.buckets)]
        outs = [dst[k * n:(k + 1) * n] for k in range(args.buckets)]
        handles = [comm.register(src), comm.register(dst)]
    a = torch.randn(args.gemm, args.gemm, device=dev, dtype=torch.bfloat16)
    bm = torch.randn(args.gemm, args.gemm, device=dev, dtype=torch.bfloat16)
    cm = torch.empty_like(a)
    comm_stream = torch.cuda.Stream(dev)
    comp_stream = torch.cuda.Stream(dev)

    def run_comm(impl):
        with torch.cuda.stream(comm_stream):
            for b, o in zip(buckets, outs):
                if impl == "tnccl":
                    comm.all_reduce(b, o, op="avg")
                else:
                    o.copy_(b)
                    dist.all_reduce(o, op=dist.ReduceOp.AVG)

    def run_compute():
        with torch.cuda.stream(comp_stream):
            for _ in range(args.gemm_iters):
                torch.matmul(a, bm, out=cm)

    def timed(fn_comm, fn_comp):
        ev = {k: torch.cuda.Event(enable_timing=True) for k in ("c0", "c1", "g0", "g1")}
        torch.cuda.synchronize()
        dist.barrier()
        if fn_comm:
            ev["c0"].record(comm_stream)
        if fn_comp:
            ev["g0"].record(comp_stream)
        if fn_comp:
            fn_comp()
        if fn_comm:
            fn_comm()
        if fn_comm:
            ev["c1"].record(comm_stream)
        if fn_comp:
            ev["g1"].record(comp_stream)
        torch.cuda.synchronize()
        tc = ev["c0"].elapsed_time(ev["c1"]) if fn_comm else 0.0
        tg = ev["g0"].elapsed_time(ev["g1"]) if fn_comp else 0.0
        return tc, tg

    # Compute alone (reference for the slowdown).
    for _ in range(2):
        timed(None, run_compute)
    comp_alone = min(timed(None, run_compute)[1] for _ in range(args.iters))
    comp_alone = max_over_ranks(comp_alone, dev)
    total_bytes = args.buckets * n * 2
    results = []
    for impl in ("tnccl", "nccl"):
        for overlap in (False, True):
            if impl == "tnccl":
                comm.set_max_channels(args.channels if overlap else 0)
            for _ in range(2):
                timed(lambda: run_comm(impl), run_compute if overlap else None)
            tcs, tgs = [], []
            for _ in range(args.iters):
                tc, tg = timed(lambda: run_comm(impl), run_compute if overlap else None)
                tcs.append(tc)
                tgs.append(tg)
            tc = max_over_ranks(min(tcs), dev)
            tg = max_over_ranks(min(tgs), dev) if overlap else 0.0
            per_bucket = tc / args.buckets
            bus = n * 2 / (per_bucket * 1e-3) / 1e9 * (2 * (world - 1) / world)
            rec = {"impl": impl, "overlap": overlap, "n_gpus": world, "buckets": args.buckets,
                   "bucket_mb": args.bucket_mb, "dtype": "bf16", "op": "avg (pre-scale fused)",
                   "comm_ms": tc, "per_bucket_us": per_bucket * 1e3, "busbw_gbs": bus,
                   "total_bytes": total_bytes,
                   "registered": bool(handles) and impl == "tnccl",
                   "zero_copy": bool(handles) and impl == "tnccl"
                   and os.environ.get("TNCCL_NVLS_ZERO_COPY") == "1"}
            if overlap:
                rec.update({"compute_ms": tg, "compute_alone_ms": comp_alone,
                            "compute_slowdown": tg / comp_alone,
                            "tnccl_channels": args.channels if impl == "tnccl" else None})
            results.append(rec)
            if rank == 0:
                print(json.dumps(rec), flush=True)
    # Numerics: the tnccl average against NCCL's on the last bucket.
    comm.set_max_channels(0)
    ref = buckets[-1].clone()
    dist.all_reduce(ref, op=dist.ReduceOp.AVG)
    torch.cuda.synchronize()
    with torch.cuda.stream(comm_stream):  # the stream the communicator is bound to
        comm.all_reduce(buckets[-1], outs[-1], op="avg")
    torch.cuda.synchronize()
    diff = (outs[-1].float() - ref.float()).abs().max().item()
    if rank == 0:
        print(json.dumps({"check": "tnccl avg vs NCCL avg, bf16", "max_abs_diff": diff}))
        if args.out:
            with open(args.out, "a") as f:
                for r in results:
                    f.write(json.dumps(r) + "\n")
    torch.cuda.synchronize()
    for h in handles:
        comm.deregister(h)
    comm.destroy()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
