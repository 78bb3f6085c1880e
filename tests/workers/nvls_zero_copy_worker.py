"""2+ ranks: the zero-copy NVLS all-reduce over registered buffers
(tncclMemAlloc + tncclCommRegister, TNCCL_NVLS_ZERO_COPY=1) gives the exact
sums of integer-valued inputs (fp32 and bf16, in and out of place, pre-scale
1/W), over many back-to-back launches interleaved with staged launches on
unregistered buffers; replays zero-copy launches captured in a CUDA graph;
then deregisters and destroys. Prints the time per
launch of the zero-copy and the staged NVLS kernel at 256 MiB, and PASS on
rank 0 (SKIP when the communicator has no NVLS)."""
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
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    import tiny_nccl_b200 as tn
    from tiny_nccl_b200.parallel import empty_registrable

    comm = tn.init_from_torch_distributed(device=rank)
    if not comm.info()["nvls"]:
        if rank == 0:
            print("SKIP: no NVLS on this communicator")
        comm.destroy()
        dist.destroy_process_group()
        return
    ok = True
    g = torch.Generator(device="cpu")
    g.manual_seed(1234 + rank)
    live = []  # (handle, tensor): registrations kept across iterations
    for dtype in (torch.float32, torch.bfloat16):
        for n in (1 << 22, 8 * 1000 + 8, 1 << 12):
            x = empty_registrable(n, dtype, dev)
            y = empty_registrable(n, dtype, dev)
            hx, hy = comm.register(x), comm.register(y)
            plain = torch.empty(n, dtype=dtype, device=dev)  # caching allocator: staged path
            for it in range(10):
                src = torch.randint(-8, 9, (n,), generator=g).to(dtype).to(dev)
                want = src.float().clone()  # .float() of fp32 is src itself
                dist.all_reduce(want)
                avg = it % 3 == 2
                if avg:
                    want = want / world
                want = want.to(dtype)
                x.copy_(src)
                if it % 2:
                    comm.all_reduce(x, None, op="avg" if avg else "sum", algo="nvls")
                    got = x
                else:
                    comm.all_reduce(x, y, op="avg" if avg else "sum", algo="nvls")
                    got = y
                plain.copy_(src)
                comm.all_reduce(plain, algo="nvls")  # staged kernel in between
                torch.cuda.synchronize()
                if avg:  # sum * (1/W) against sum / W
                    tol = 1e-2 if dtype == torch.bfloat16 else 1e-6
                    good = torch.allclose(got.float(), want.float(), rtol=tol, atol=tol)
                else:
                    good = torch.equal(got, want)
                if not good:
                    ok = False
                    d = (got.float() - want.float()).abs()
                    bad = (d > (1e-2 if avg else 0)).nonzero().flatten()
                    i0, i1 = int(bad[0]), int(bad[-1])
                    half = (n + world - 1) // world  # rank r reduces about [r*half, (r+1)*half)
                    print(f"rank {rank}: {dtype} n={n} it={it} inplace={it % 2} avg={avg} "
                          f"max diff {d.max().item()} bad {bad.numel()} first {i0} last {i1} "
                          f"(shards of ~{half}) got {got[i0].item()} want {want[i0].item()} "
                          f"x {src[i0].item()}", flush=True)
            comm.deregister(hx)
            live.append((hy, y))
    for h, _ in live:
        comm.deregister(h)
    live.clear()
    # CUDA graph: zero-copy launches captured once and replayed (their barrier
    # counters live in device memory), on a second communicator bound to a
    # side stream.
    comm2 = tn.init_from_torch_distributed(device=rank)
    stream = torch.cuda.Stream(device=dev)
    xg = empty_registrable(1 << 20, torch.float32, dev)
    hg = comm2.register(xg)
    with torch.cuda.stream(stream):
        xg.fill_(1.0)
        comm2.all_reduce(xg, algo="nvls")  # eager: binds the stream
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        comm2.all_reduce(xg, algo="nvls", op="avg")
        comm2.all_reduce(xg, algo="nvls")
    for it in range(3):
        with torch.cuda.stream(stream):
            xg.fill_(float(rank + 1 + it))
            graph.replay()
        torch.cuda.synchronize()
        want = float(sum(r + 1 + it for r in range(world)))
        if not torch.allclose(xg, torch.full_like(xg, want), rtol=1e-6):
            ok = False
            print(f"rank {rank}: graph replay {it} wrong", flush=True)
    del graph
    torch.cuda.synchronize()
    comm2.deregister(hg)
    ok = ok and comm2.async_error() == 0
    comm2.destroy()
    # Time per launch at 256 MiB fp32: zero-copy vs staged NVLS.
    n = 64 << 20
    x = empty_registrable(n, torch.float32, dev)
    h = comm.register(x)
    x.normal_()
    plain = torch.randn(n, device=dev)
    times = {}
    for name, buf in (("zero-copy", x), ("staged", plain)):
        for _ in range(3):
            comm.all_reduce(buf, algo="nvls", op="avg")
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize()
        start.record()
        for _ in range(10):
            comm.all_reduce(buf, algo="nvls", op="avg")
        end.record()
        torch.cuda.synchronize()
        t = torch.tensor([start.elapsed_time(end) / 10], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times[name] = t.item()
    comm.deregister(h)
    info = comm.info()
    ok = ok and comm.async_error() == 0 and info["registrations"] == 0
    if os.environ.get("TNCCL_NVLS_ZERO_COPY") == "1":
        ok = ok and info["zero_copy_launches"] > 0
    flag = torch.tensor([1.0 if ok else 0.0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        bus = lambda ms: n * 4 / (ms * 1e-3) * 2 * (world - 1) / world / 1e9
        for name, ms in times.items():
            print(f"{name}: {ms:.3f} ms per 256 MiB fp32 all-reduce = {bus(ms):.1f} GB/s bus")
        print(f"zero-copy launches on rank 0: {info['zero_copy_launches']}")
        print("PASS" if flag.item() == 1.0 else "FAIL")
    torch.cuda.synchronize()
    comm.destroy()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
