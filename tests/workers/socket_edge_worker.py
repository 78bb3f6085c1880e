"""Socket ring edges on GPUs (2+ ranks, one process per GPU).

argv[1] selects the set-up:
  force  TNCCL_NET=force on one host: every ring edge is a socket edge while
         the peers stay mapped (the all-peer algorithms still run over NVLink).
  hosts  every rank claims its own host (TNCCL_HOST_ID=<rank>) and rank 0's id
         is a TCP rendezvous (TNCCL_BOOTSTRAP_ADDR): no peer is mapped and the
         communicator runs the ring over sockets only, as across nodes.
  fail   as force; after a completed step rank 1 leaves without destroying
         its communicator (nothing in flight). Rank 0's proxy sees the
         connections end without close frames, records the failure in the
         status block, and rank 0's next collective is refused.

The checks: ring all-reduce against a host reference for fp32 and bf16,
several sizes (not multiples of the vector width too), in place and out of
place, many collectives in a row and a CUDA-graph replay; inputs are small
integers, so every sum is exact in both types.
"""
import datetime
import os
import socket
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def check_sizes(comm, dev, rank, world):
    ok = True
    for dtype in (torch.float32, torch.bfloat16):
        for n in (1, 7, 4096 + 3, (1 << 20) + 5, 8 << 20):
            idx = torch.arange(n, device=dev)
            x = ((idx % 5) + rank).to(dtype)
            want = sum(((idx % 5) + r).float() for r in range(world)).to(dtype)
            out = torch.empty_like(x)
            comm.all_reduce(x, out=out)
            comm.all_reduce(x)  # in place
            torch.cuda.synchronize()
            good = torch.equal(out, want) and torch.equal(x, want)
            if not good:
                print(f"rank {rank}: {dtype} n={n} mismatch")
            ok = ok and good
    return ok


def check_graph(comm, stream, dev, rank, world):
    x = torch.full((1 << 16,), float(rank + 1), device=dev)
    g = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=stream):
        comm.all_reduce(x)
    with torch.cuda.stream(stream):
        x.fill_(float(rank + 1))
        for _ in range(3):
            g.replay()
    torch.cuda.synchronize()
    want = float(sum(range(1, world + 1))) * world ** 2
    ok = bool((x == want).all())
    del g
    return ok


def main():
    mode = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    store = dist.distributed_c10d._get_default_store()
    if mode == "hosts":
        os.environ["TNCCL_HOST_ID"] = f"host{rank}"
        if rank == 0:
            os.environ["TNCCL_BOOTSTRAP_ADDR"] = f"127.0.0.1:{free_port()}"
    else:
        assert os.environ.get("TNCCL_NET") == "force"
    import tiny_nccl_b200 as tn

    comm = tn.init_from_torch_distributed(device=rank)
    stream = torch.cuda.Stream(device=dev)  # every collective runs here
    torch.cuda.set_stream(stream)
    info = comm.info()
    ok = info["socket_send_edge"] and info["socket_recv_edge"] and info["socket_channels"] > 0
    if mode == "hosts":
        ok = ok and comm.select_algo(1 << 20, torch.float32) == "ring"
        try:
            comm.all_reduce(torch.ones(16, device=dev), algo="twoshot")
            torch.cuda.synchronize()
            ok = False  # the all-peer algorithms need mapped peers
        except RuntimeError:
            pass
    if mode in ("force", "hosts"):
        ok = ok and check_sizes(comm, dev, rank, world)
        for _ in range(20):
            y = torch.full((12345,), 2.0, device=dev)
            comm.all_reduce(y)
        torch.cuda.synchronize()
        ok = ok and bool((y == 2.0 * world).all()) and comm.async_error() == 0
        ok = ok and check_graph(comm, stream, dev, rank, world)
        st = comm.net_stats()
        ok = ok and st["frames_sent"] > 0 and st["frames_received"] > 0 and st["failed"] == 0
        flag = torch.tensor([1.0 if ok else 0.0])
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if rank == 0:
            print("PASS" if flag.item() == 1.0 else "FAIL")
        torch.cuda.synchronize()
        comm.destroy()
        dist.barrier()
        dist.destroy_process_group()
        return

    # fail: one completed step, then rank 1 leaves between steps.
    x = torch.ones(1 << 16, device=dev)
    comm.all_reduce(x)
    torch.cuda.synchronize()
    ok = bool((x == world).all())
    store.set(f"tnccl_test/step_done/{rank}", "1")
    if rank == 1:
        store.get("tnccl_test/step_done/0")
        os._exit(0)  # no destroy: its sockets close without close frames
    store.get("tnccl_test/step_done/1")
    t0 = time.time()
    while comm.async_error() == 0 and time.time() - t0 < 10:
        time.sleep(0.01)
    err = comm.async_error()
    refused = False
    try:
        comm.all_reduce(x)
    except RuntimeError:
        refused = True
    print(f"rank0: proxy failure after {time.time() - t0:.2f}s async_error={err} refused={refused}")
    print("PASS" if ok and err != 0 and refused else "FAIL")
    try:
        comm.destroy()  # its barriers time out (TNCCL_BOOTSTRAP_TIMEOUT_MS)
    except RuntimeError:
        pass
    os._exit(0)


if __name__ == "__main__":
    main()
