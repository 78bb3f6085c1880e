"""All-reduce bus-bandwidth sweep: tnccl algorithms vs NCCL (and the tiny-nccl
reference build when it is installed), one process per GPU.

Launch (one node):
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \
        --master-addr 127.0.0.1 --master-port 29511 benchmarks/allreduce_sweep.py \
        --dtype fp32 --min-bytes 4K --max-bytes 4G --impls oneshot,twoshot,ring,nvls,auto,nccl \
        --out sweep.jsonl

For every size and implementation: W untimed warm-up all-reduces, then K
all-reduces between two CUDA events on the launching stream, bracketed by a
barrier and a device synchronize. The time of one all-reduce is the MAX over
ranks of (elapsed / K). Bus bandwidth follows the nccl-tests convention
busBW = bytes / t * 2(P-1)/P. Buffers are Normal(0,1) seeded per rank and
are much larger than L2 from 256 MiB up; smaller sizes run L2-resident, as
they do in nccl-tests. Each line of the output file is one JSON record.

``--impls nvls_zc`` runs the NVLS algorithm on buffers from tncclMemAlloc
registered with the communicator: the zero-copy kernel (no copy through the
communicator's multicast region), or the staged one with
TNCCL_NVLS_ZERO_COPY=0 in the environment.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

LINK_GBS = 770.0  # measured peer copy per direction on this pool


def parse_size(s: str) -> int:
    s = s.strip().upper()
    mult = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}
    if s[-1] in mult:
        return int(float(s[:-1]) * mult[s[-1]])
    return int(s)


class UniqueId(ctypes.Structure):
    """tncclUniqueId: a 128-byte struct passed by value."""
    _fields_ = [("bytes", ctypes.c_ubyte * 128)]


class RefLib:
    """The unmodified tiny-nccl reference, built from its own CMake project."""

    def __init__(self, path: str):
        self.lib = ctypes.CDLL(path)
        self.lib.tncclGetUniqueId.argtypes = [ctypes.c_void_p]
        self.lib.tncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                                               UniqueId, ctypes.c_int]
        self.lib.tncclAllReduceSumF32.argtypes = [ctypes.c_void_p, ctypes.c_void_p,
                                                  ctypes.c_size_t, ctypes.c_void_p,
                                                  ctypes.c_void_p]
        self.lib.tncclCommDestroy.argtypes = [ctypes.c_void_p]
        self.comm = ctypes.c_void_p()

    def init(self, rank: int, world: int):
        uid = UniqueId()
        if rank == 0:
            assert self.lib.tncclGetUniqueId(ctypes.byref(uid)) == 0
            obj = [bytes(uid)]
        else:
            obj = [None]
        dist.broadcast_object_list(obj, src=0)
        ctypes.memmove(ctypes.byref(uid), obj[0], 128)
        rc = self.lib.tncclCommInitRank(ctypes.byref(self.comm), world, uid, rank)
        if rc != 0:
            raise RuntimeError(f"reference tncclCommInitRank failed: {rc}")

    def all_reduce(self, send, recv, count, stream):
        rc = self.lib.tncclAllReduceSumF32(ctypes.c_void_p(send), ctypes.c_void_p(recv),
                                           ctypes.c_size_t(count), self.comm,
                                           ctypes.c_void_p(stream))
        if rc != 0:
            raise RuntimeError(f"reference all-reduce failed: {rc}")

    def destroy(self):
        self.lib.tncclCommDestroy(self.comm)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--dtype", default="fp32", choices=["fp32", "bf16", "fp16"])
    ap.add_argument("--min-bytes", default="4K")
    ap.add_argument("--max-bytes", default="1G")
    ap.add_argument("--impls", default="oneshot,twoshot,ring,nvls,auto,nccl")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("--ref-max-bytes", default="1G",
                    help="largest size run for the reference ring (~2 GB/s: 4 GiB takes seconds "
                         "per call)")
    ap.add_argument("--max-seconds-per-point", type=float, default=1.5,
                    help="caps K for large sizes (time-bounded sweeps)")
    ap.add_argument("--out", default="")
    ap.add_argument("--check", action="store_true", help="verify results against NCCL")
    args = ap.parse_args()

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))

    import tiny_nccl_b200 as tn

    dtype = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}[args.dtype]
    es = torch.empty((), dtype=dtype).element_size()
    impls = [s for s in args.impls.split(",") if s]
    stream = torch.cuda.Stream(device=dev)
    comm = tn.init_from_torch_distributed(device=local)
    info = comm.info()
    for name in ("nvls", "nvls_zc"):
        if name in impls and not info["nvls"]:
            impls.remove(name)
    ref = None
    if "ref" in impls:
        path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                            "baseline", "_ref", "lib", "libtiny_nccl_ref.so")
        if dtype != torch.float32 or not os.path.exists(path):
            impls.remove("ref")
        else:
            ref = RefLib(path)
            ref.init(rank, world)

    sizes = []
    s = parse_size(args.min_bytes)
    while s <= parse_size(args.max_bytes):
        sizes.append(s)
        s *= 2
    maxn = sizes[-1] // es
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    src = torch.randn(maxn, dtype=torch.float32, device=dev, generator=gen).to(dtype)
    dst = torch.empty_like(src)
    # nvls_zc: the NVLS kernel on buffers registered with the communicator
    # (zero-copy unless TNCCL_NVLS_ZERO_COPY=0, then the staged kernel).
    reg = None
    if "nvls_zc" in impls:
        from tiny_nccl_b200.parallel import empty_registrable
        rsrc = empty_registrable(maxn, dtype, dev)
        rdst = empty_registrable(maxn, dtype, dev)
        rsrc.copy_(src)
        reg = (rsrc, rdst, comm.register(rsrc), comm.register(rdst))
    out = open(args.out, "a") if (args.out and rank == 0) else None
    results = []
    for size in sizes:
        n = size // es
        x = src[:n]
        y = dst[:n]
        for impl in impls:
            zc0 = comm.info()["zero_copy_launches"]
            if impl == "ref" and size > parse_size(args.ref_max_bytes):
                continue

            def op():
                if impl == "nccl":
                    dist.all_reduce(y)  # in place, like NCCL's own bench
                elif impl == "ref":
                    ref.all_reduce(x.data_ptr(), y.data_ptr(), n, stream.cuda_stream)
                elif impl == "nvls_zc":
                    comm.all_reduce(reg[0][:n], reg[1][:n], algo="nvls")
                else:
                    comm.all_reduce(x, y, algo=impl)

            with torch.cuda.stream(stream):
                if impl == "nccl":
                    y.copy_(x)
                for _ in range(args.warmup):
                    op()
            torch.cuda.synchronize()
            # Calibrate K so that one point stays within the time cap.
            with torch.cuda.stream(stream):
                e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
                e0.record()
                op()
                e1.record()
            torch.cuda.synchronize()
            t1 = torch.tensor([e0.elapsed_time(e1)], device=dev)
            dist.all_reduce(t1, op=dist.ReduceOp.MAX)
            k = max(5, min(args.iters, int(args.max_seconds_per_point * 1e3 / max(t1.item(), 1e-3))))
            dist.barrier()
            torch.cuda.synchronize()
            with torch.cuda.stream(stream):
                e0.record()
                for _ in range(k):
                    op()
                e1.record()
            torch.cuda.synchronize()
            ms = torch.tensor([e0.elapsed_time(e1) / k], device=dev)
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            t = ms.item() * 1e-3
            algbw = size / t / 1e9
            busbw = algbw * 2 * (world - 1) / world if world > 1 else algbw
            rec = {"impl": impl, "bytes": size, "dtype": args.dtype, "n_gpus": world,
                   "us": t * 1e6, "algbw_gbs": algbw, "busbw_gbs": busbw, "iters": k,
                   "chosen": comm.select_algo(n, dtype) if impl == "auto" else impl,
                   "frac_link": busbw / LINK_GBS}
            if impl == "nvls_zc":  # did the zero-copy kernel run?
                rec["zero_copy"] = comm.info()["zero_copy_launches"] > zc0
            if args.check and impl != "nccl":
                ref_y = x.clone()
                with torch.cuda.stream(stream):
                    dist.all_reduce(ref_y)
                    op()
                torch.cuda.synchronize()
                got = reg[1][:n] if impl == "nvls_zc" else y
                err = (got.float() - ref_y.float()).abs().max().item()
                rec["max_abs_err_vs_nccl"] = err
            results.append(rec)
            if rank == 0:
                print(json.dumps(rec), flush=True)
                if out:
                    out.write(json.dumps(rec) + "\n")
                    out.flush()
    if comm.async_error():
        print(f"rank {rank}: tnccl async error {comm.async_error()}", flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    if ref is not None:
        ref.destroy()
    if reg is not None:
        comm.deregister(reg[2])
        comm.deregister(reg[3])
    comm.destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
