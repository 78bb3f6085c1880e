#!/usr/bin/env python
"""Flagship benchmark: GPT-2 small data-parallel training throughput (tokens/s).

    python bench.py --gpus 1 --steps K --warmup W
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W [--impl reference]

Workload: GPT-2 small (12 layers, d_model 768, 12 heads,
vocabulary 50257, context 1024), micro-batch 8 per GPU, bf16 autocast, AdamW,
random initialisation, synthetic token ids Uniform[0, 50257) seeded per rank.
Weak scaling: every GPU processes 8 x 1024 tokens per step.

--impl tnccl (default): the framework's GPT-2 (fused sm_100a LayerNorm /
  cross-entropy / AdamW kernels) in DataParallelTrainer: gradients in one
  flat buffer whose ~25 MB buckets are all-reduced by tnccl kernels over
  NVLink on a side stream as backward produces them, and the whole step
  (forward, backward with those all-reduces, AdamW) captured once in a CUDA
  graph and replayed (TNCCL_DP_REDUCER=ddp: DDP with the tnccl comm hook,
  eager).
--impl reference: the unmodified tiny-nccl reference (baseline/_ref, built by
  baseline/build_reference.sh) all-reduces the gradient buckets through its
  public tncclAllReduceSumF32, inside stock PyTorch: Hugging Face GPT2LMHeadModel,
  torch.optim.AdamW, DistributedDataParallel.
--impl nccl-ddp: the NCCL-DDP baseline, the same stock PyTorch stack with
  DDP's own NCCL all-reduce.

Timing: W untimed warm-up steps (continued until at least --min-warmup-s
seconds of warm-up; the JSON reports the count as warmup_steps_run); then K
steps bracketed by a barrier and
torch.cuda.synchronize(), timed with CUDA events on the training stream; the
step time is the max over ranks. A second timed loop of K steps measures the
same metric end to end (pinned-host token copy in, loss read back each step).
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import socket
import subprocess
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GPT-2 small DP training tokens/s"
REF_LIB = os.path.join(ROOT, "baseline", "_ref", "lib", "libtiny_nccl_ref.so")


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def setup_dist():
    if "RANK" not in os.environ:
        os.environ.update({"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0",
                           "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(free_port())})
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))
    return rank, world, local, dev


def max_over_ranks(x: float, dev) -> float:
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


class UniqueId(ctypes.Structure):
    """tncclUniqueId: a 128-byte struct passed by value."""
    _fields_ = [("bytes", ctypes.c_ubyte * 128)]


class ReferenceComm:
    """ctypes handle on the reference library (tiny-nccl public API)."""

    def __init__(self, rank: int, world: int):
        lib = ctypes.CDLL(REF_LIB)
        lib.tncclGetUniqueId.argtypes = [ctypes.c_void_p]
        lib.tncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                                          UniqueId, ctypes.c_int]
        lib.tncclAllReduceSumF32.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                             ctypes.c_void_p, ctypes.c_void_p]
        lib.tncclCommDestroy.argtypes = [ctypes.c_void_p]
        self.lib = lib
        uid = UniqueId()
        obj = [None]
        if rank == 0:
            if lib.tncclGetUniqueId(ctypes.byref(uid)) != 0:
                raise RuntimeError("reference tncclGetUniqueId failed")
            obj = [bytes(uid)]
        dist.broadcast_object_list(obj, src=0)
        ctypes.memmove(ctypes.byref(uid), obj[0], 128)
        self.comm = ctypes.c_void_p()
        rc = lib.tncclCommInitRank(ctypes.byref(self.comm), world, uid, rank)
        if rc != 0:
            raise RuntimeError(f"reference tncclCommInitRank failed ({rc})")
        self.world = world

    def all_reduce_(self, t: torch.Tensor, stream: torch.cuda.Stream):
        rc = self.lib.tncclAllReduceSumF32(ctypes.c_void_p(t.data_ptr()),
                                           ctypes.c_void_p(t.data_ptr()),
                                           ctypes.c_size_t(t.numel()), self.comm,
                                           ctypes.c_void_p(stream.cuda_stream))
        if rc != 0:
            raise RuntimeError(f"reference tncclAllReduceSumF32 failed ({rc})")

    def destroy(self):
        self.lib.tncclCommDestroy(self.comm)


def build_reference_trainer(args, rank, world, dev):
    """Stock PyTorch GPT-2 (Hugging Face) + DDP whose gradient buckets go
    through the reference's tncclAllReduceSumF32 (fp32, then / world)."""
    from torch.nn.parallel import DistributedDataParallel as DDP
    from transformers import GPT2Config as HFConfig, GPT2LMHeadModel

    cfg = HFConfig(n_layer=12, n_head=12, n_embd=768, vocab_size=50257, n_positions=1024,
                   resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0)
    torch.manual_seed(1234)
    model = GPT2LMHeadModel(cfg).to(dev)
    ref = ReferenceComm(rank, world)
    side = torch.cuda.Stream(device=dev)

    def hook(state, bucket):
        buf = bucket.buffer()
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            ref.all_reduce_(buf, side)
            buf.div_(world)
            buf.record_stream(side)
            fut = torch.futures.Future(devices=[dev])
            fut.set_result(buf)
        return fut

    ddp = DDP(model, device_ids=[dev.index], bucket_cap_mb=25, gradient_as_bucket_view=True,
              static_graph=True, broadcast_buffers=False)
    ddp.register_comm_hook(None, hook)
    decay = [p for p in model.parameters() if p.dim() >= 2]
    no_decay = [p for p in model.parameters() if p.dim() < 2]
    opt = torch.optim.AdamW([{"params": decay, "weight_decay": 0.1},
                             {"params": no_decay, "weight_decay": 0.0}], lr=6e-4,
                            betas=(0.9, 0.95), fused=True)

    def step(idx, tgt):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = ddp(input_ids=idx, labels=idx)
        out.loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=False)
        return out.loss.detach()

    def launches():
        return 0  # the reference path launches no kernel of this repository

    return step, launches, ref.destroy


def build_nccl_ddp_trainer(args, rank, world, dev):
    """The NCCL-DDP baseline: stock PyTorch GPT-2 (Hugging Face), stock DDP
    (NCCL all-reduce of fp32 gradient buckets), torch fused AdamW."""
    from torch.nn.parallel import DistributedDataParallel as DDP
    from transformers import GPT2Config as HFConfig, GPT2LMHeadModel

    cfg = HFConfig(n_layer=12, n_head=12, n_embd=768, vocab_size=50257, n_positions=1024,
                   resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0)
    torch.manual_seed(1234)
    model = GPT2LMHeadModel(cfg).to(dev)
    ddp = DDP(model, device_ids=[dev.index], bucket_cap_mb=25, gradient_as_bucket_view=True,
              static_graph=True, broadcast_buffers=False)
    decay = [p for p in model.parameters() if p.dim() >= 2]
    no_decay = [p for p in model.parameters() if p.dim() < 2]
    opt = torch.optim.AdamW([{"params": decay, "weight_decay": 0.1},
                             {"params": no_decay, "weight_decay": 0.0}], lr=6e-4,
                            betas=(0.9, 0.95), fused=True)

    def step(idx, tgt):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = ddp(input_ids=idx, labels=idx)
        out.loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return out.loss.detach()

    return step, (lambda: 0), (lambda: None)


def build_tnccl_trainer(args, rank, world, dev):
    import tiny_nccl_b200 as tn
    from tiny_nccl_b200.models import GPT2, GPT2Config
    from tiny_nccl_b200.parallel import DataParallelTrainer

    comm = tn.init_from_torch_distributed(device=dev.index)
    torch.manual_seed(1234)
    model = GPT2(GPT2Config(), impl="fused").to(dev)
    trainer = DataParallelTrainer(model, comm, algo=args.algo)

    def launches():
        # API launches, plus this library's kernel nodes that CUDA-graph
        # replays of the training step launched.
        return tn.launch_count() + tn.load().ops.launch_count() + trainer.replayed_launches

    def close():
        torch.cuda.synchronize()
        trainer.close()
        comm.destroy()

    close.describe = trainer.describe
    return trainer.step, launches, close


def make_record(impl, world, B, T, steps, warmup, ms_max, clocks, launches, e2e, loss,
                grad_reducer="ddp"):
    """The one JSON line bench.py prints (rank 0): whole-job tokens/s from the
    device step time (max over ranks), plus the end-to-end number, clocks and
    the kernel-launch count of this repository's kernels."""
    from tiny_nccl_b200.models import GPT2Config
    tokens_per_s = world * B * T / (ms_max * 1e-3)
    flops = GPT2Config().flops_per_token(T) * tokens_per_s / world
    return {"metric": METRIC, "value": tokens_per_s, "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": ms_max,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic token ids Uniform[0,50257) seeded per rank; "
                                     "random-init weights",
            "impl": impl,
            "config": {"model": "GPT-2 small (124M): 12 layers, d_model 768, 12 heads, vocab 50257",
                       "global_batch": B * world, "micro_batch_per_gpu": B, "seq_len": T,
                       "parallelism": f"dp{world}", "optimizer": "AdamW", "amp": "bf16 autocast",
                       "grad_reducer": grad_reducer,
                       "l2": "no flush: one step touches several GB (activations, 124M-param "
                             "weights/grads/optimizer state), far above the 126 MB L2"},
            "clocks": clocks, "gpu_launches": launches, "e2e": e2e,
            "model_tflops_per_gpu": flops / 1e12, "loss": loss}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="tnccl", choices=["tnccl", "reference", "nccl-ddp"])
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=1024)
    ap.add_argument("--algo", default="auto")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--min-warmup-s", type=float, default=1.0,
                    help="untimed warm-up continues past --warmup steps until this long")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference" and not os.path.exists(REF_LIB):
        # baseline/build_reference.sh installs it (build() in __graft_entry__
        # runs it); TNCCL_REFERENCE_SRC, else a `reference` directory beside
        # this repository, names the reference source to build it from here.
        script = os.path.join(ROOT, "baseline", "build_reference.sh")
        src = os.environ.get("TNCCL_REFERENCE_SRC") or os.path.join(os.path.dirname(ROOT),
                                                                    "reference")
        if src and os.path.isdir(src):
            subprocess.run(["bash", script, src], stdout=subprocess.DEVNULL,
                           stderr=subprocess.DEVNULL, check=False)
        if not os.path.exists(REF_LIB):
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "baseline/_ref is not built and the reference source is absent"}))
            return

    rank, world, local, dev = setup_dist()
    B, T = args.batch, args.seq
    if args.impl == "reference":
        step, launches, close = build_reference_trainer(args, rank, world, dev)
    elif args.impl == "nccl-ddp":
        step, launches, close = build_nccl_ddp_trainer(args, rank, world, dev)
    else:
        step, launches, close = build_tnccl_trainer(args, rank, world, dev)

    # Synthetic data: a pool of distinct seeded batches per rank.
    gen = torch.Generator(device="cpu")
    gen.manual_seed(4242 + rank)
    pool = 4
    host = torch.randint(0, 50257, (pool, B, T + 1), generator=gen, dtype=torch.int64)
    host = host.pin_memory()
    dev_batches = host.to(dev)

    def run(i):
        b = dev_batches[i % pool]
        return step(b[:, :T], b[:, 1:])

    # Warm-up: the requested W steps, continued (untimed) until at least
    # --min-warmup-s seconds have passed after the first step (which loads
    # kernels and builds plans). A cold process can step ~30 % slower for its
    # next ~0.5 s (per-step times on one B200: 20 ms for steps 2-20, 14.5 ms
    # from step 21 on). Rank 0 decides when to stop, so every rank runs the
    # same number of steps (their DDP collectives stay in step).
    run(0)
    torch.cuda.synchronize()
    t_warm = time.perf_counter()
    warm = 1
    while True:
        if warm >= args.warmup:
            torch.cuda.synchronize()
            more = time.perf_counter() - t_warm < args.min_warmup_s and warm < 500
            flag = torch.tensor([1.0 if more else 0.0], device=dev)
            dist.broadcast(flag, 0)
            if flag.item() == 0.0:
                break
        run(warm)
        warm += 1
    torch.cuda.synchronize()
    dist.barrier()

    from tiny_nccl_b200.utils import ClockSampler
    sampler = ClockSampler(gpu_index=None).start() if rank == 0 else None
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    dist.barrier()
    l0 = launches()
    e0.record(stream)
    for i in range(args.steps):
        loss = run(i)
    e1.record(stream)
    torch.cuda.synchronize()
    l1 = launches()
    dist.barrier()
    clocks = sampler.stop() if sampler else {}
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = max_over_ranks(ms, dev)
    last_loss = float(loss.item())

    e2e = None
    if not args.no_e2e:
        # Every step copies its token batch host -> device (pinned, on a copy
        # stream, double-buffered) and reads its loss device -> host (into
        # pinned memory); the host reads step i's loss after launching step
        # i + 1, so the device never waits for the host.
        bufs = [torch.empty((B, T + 1), dtype=torch.int64, device=dev) for _ in range(2)]
        ready = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        loss_host = torch.empty(args.steps, dtype=torch.float32).pin_memory()
        loss_ev = [torch.cuda.Event() for _ in range(args.steps)]
        copy_stream = torch.cuda.Stream(dev)
        losses = []

        def fetch(i):
            j = i % 2
            if i >= 2:
                copy_stream.wait_event(done[j])  # step i - 2 finished reading bufs[j]
            with torch.cuda.stream(copy_stream):
                bufs[j].copy_(host[i % pool], non_blocking=True)
                ready[j].record(copy_stream)

        torch.cuda.synchronize()
        dist.barrier()
        t0 = time.perf_counter()
        fetch(0)
        for i in range(args.steps):
            if i + 1 < args.steps:
                fetch(i + 1)
            j = i % 2
            stream.wait_event(ready[j])
            l = step(bufs[j][:, :T], bufs[j][:, 1:])
            done[j].record(stream)
            loss_host[i].copy_(l.float(), non_blocking=True)  # device -> host
            loss_ev[i].record(stream)
            if i >= 1:
                loss_ev[i - 1].synchronize()
                losses.append(float(loss_host[i - 1]))
        loss_ev[args.steps - 1].synchronize()
        losses.append(float(loss_host[args.steps - 1]))
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        wall_max = max_over_ranks(wall, dev)
        e2e = {"value": world * B * T * args.steps / wall_max, "unit": "tokens/s",
               "h2d_bytes_per_step": B * (T + 1) * 8, "d2h_bytes_per_step": 4,
               "ms_per_step": wall_max * 1e3 / args.steps, "timing": "host wall clock, max over ranks"}

    if rank == 0:
        desc = getattr(close, "describe", None)
        rec = make_record(args.impl, world, B, T, args.steps, args.warmup, ms_max, clocks,
                          int(l1 - l0), e2e, last_loss, desc() if desc else "ddp")
        rec["warmup_steps_run"] = warm
        print(json.dumps(rec), flush=True)
    close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
