"""2 ranks, failure detection without a GPU fault: rank 0 launches an
all-reduce that rank 1 never joins. Rank 0's bounded device waits give up
after TNCCL_TIMEOUT_MS, the kernel returns, TNCCL_TIMEOUT is reported and
further collectives are refused. Rank 1 only sits between steps (nothing in
flight) and learns of the failure on the host through the store. Run with
NVLS off (TNCCL_NVLS_ENABLE=0, NCCL_NVLS_ENABLE=0)."""
import datetime
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    import tiny_nccl_b200 as tn

    assert os.environ.get("TNCCL_NVLS_ENABLE") == "0"
    comm = tn.init_from_torch_distributed(device=rank)
    store = dist.distributed_c10d._get_default_store()
    x = torch.ones(1 << 16, device=dev)
    ok = True
    if rank == 0:
        t0 = time.time()
        comm.all_reduce(x, algo="twoshot")  # rank 1 never joins
        torch.cuda.synchronize()  # returns: the kernel gave up on its own
        waited = time.time() - t0
        err = comm.async_error()
        refused = False
        try:
            comm.all_reduce(x)
        except RuntimeError:
            refused = True
        ok = err == 5 and refused and 0.5 < waited < 30
        print(f"rank0: waited {waited:.2f}s async_error={err} refused={refused}")
        store.set("tnccl_test/rank0_status", "timeout" if err == 5 else f"err{err}")
    else:
        status = store.get("tnccl_test/rank0_status").decode()
        ok = status == "timeout"
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
