"""NVLink primitive micro-benchmark (push stores, pull loads, push with a
release flag per chunk, local copy, the copy and reduce mixes of the
collectives, and push throughput while another warp issues ordering
operations) across CTA counts, thread counts and accesses in flight. Used to
size the collective kernels.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
        benchmarks/p2p_microbench.py --out p2p.jsonl
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--bytes", type=int, default=64 << 20)
    ap.add_argument("--out", default="")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=60))
    os.environ.setdefault("TNCCL_NCHANNELS", "128")
    os.environ.setdefault("TNCCL_CHUNK_BYTES", str(1 << 20))  # large ring area as scratch
    import tiny_nccl_b200 as tn
    comm = tn.init_from_torch_distributed(device=local)
    out = open(args.out, "a") if (args.out and rank == 0) else None
    modes = {0: "push", 1: "pull", 2: "push+flag", 3: "local", 4: "local->peer copy",
             5: "reduce mix (2 local loads -> local + peer store)",
             6: "push with a concurrent ordering op in warp 0",
             7: "TMA-staged local->peer", 8: "TMA-staged local->local",
             9: "TMA-staged local->peer, 8 copies per stage",
             10: "NVLS ld_reduce (share)", 11: "NVLS multimem.st", 12: "NVLS ld_reduce+st (share)"}
    only = [int(m) for m in os.environ.get("P2P_MODES", "0,1,3,2,4,5").split(",")]
    for mode in only:
        for ctas in (1, 8, 32, 64, 128):
            for threads in ((128, 256) if mode in (7, 8, 9) else (256, 512)):
                for unroll in ((4, 8, 16) if mode >= 10 else
                               (2, 4, 8) if mode not in (2, 7, 8, 9) else
                               (1,) if mode == 2 else (2, 3)):
                    chunks = ((16 << 10, 64 << 10, 256 << 10) if mode == 2 else
                              (0, 1, 2, 3) if mode == 6 else
                              (8192, 32768, 65536) if mode in (7, 8, 9) else (0,))
                    for chunk in chunks:
                        dist.barrier()
                        ms = comm._c.diag_bench(mode, args.bytes, ctas, threads, unroll, chunk, 5)
                        t = torch.tensor([ms], device="cuda")
                        dist.all_reduce(t, op=dist.ReduceOp.MAX)
                        gbs = args.bytes / (t.item() * 1e-3) / 1e9
                        rec = {"mode": modes[mode], "ctas": ctas, "threads": threads,
                               "unroll": unroll, "chunk": chunk, "GBps": gbs,
                               "GBps_per_cta": gbs / ctas}
                        if rank == 0:
                            print(json.dumps(rec), flush=True)
                            if out:
                                out.write(json.dumps(rec) + "\n")
    comm.destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
