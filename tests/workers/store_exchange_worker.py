"""CPU ranks (gloo): the unique id travels through the torch.distributed
store; without a GPU every rank's communicator creation fails promptly with a
CUDA error instead of hanging in the bootstrap."""
import datetime
import os
import sys
import time

import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


def main():
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    rank = dist.get_rank()
    import tiny_nccl_b200 as tn

    store = dist.distributed_c10d._get_default_store()
    if rank == 0:
        store.set("tnccl/uid", tn.get_unique_id())
    uid = bytes(store.get("tnccl/uid"))
    assert len(uid) == 128
    t0 = time.time()
    try:
        tn.Communicator(uid, dist.get_world_size(), rank)
        outcome = "created"
    except RuntimeError as e:
        outcome = "CUDA error" if "CUDA error" in str(e) else str(e)
    elapsed = time.time() - t0
    res = [None] * dist.get_world_size()
    dist.all_gather_object(res, (outcome, elapsed))
    if rank == 0:
        ok = all(o == "CUDA error" and t < 10 for o, t in res)
        print(res)
        print("PASS" if ok else "FAIL")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
