"""Data-parallel training step of the fused GPT-2: gradients averaged over
the ranks by tnccl kernels while backward runs, then the fused AdamW.

Default (``reducer="flat"``): :class:`FlatGradReducer` keeps every ``.grad``
in one flat buffer cut into ~25 MB buckets and all-reduces each bucket on the
communicator's side stream as soon as backward has produced it (1/world
fused into the kernel). The buffer is tncclMemAlloc memory registered with
the communicator (``registered``, ``TNCCL_DP_REGISTERED=0`` turns it off), so
on 8 ranks AUTO sends its buckets through the zero-copy NVLS kernel (the
switch reduces straight from every GPU's buffer). The whole step (forward,
backward with the bucket all-reduces, AdamW, gradient zeroing) is captured
in one CUDA graph after three eager warm-up steps and replayed for every
later step (``cuda_graph``, ``TNCCL_CUDA_GRAPH=0`` turns it off): the ~500
kernel launches of a GPT-2 small step then cost one graph launch instead of
more host time than the GPU needs for the step. Inputs are copied into
static buffers first, and the optimizer reads its step count from device
memory. AdamW also writes the bf16 copies of the weights that the next
forward's GEMMs read.

``overlap_optimizer=True`` (``TNCCL_DP_OVERLAP_OPT=1``) runs AdamW on each
bucket's parameters on the communication stream right after its all-reduce.

``reducer="ddp"`` (``TNCCL_DP_REDUCER=ddp``): DistributedDataParallel with
the tnccl comm hook, eager (DDP's reducer runs host logic during backward
that a graph replay would skip). ``reducer="nccl-ddp"``: the same with DDP's
own NCCL all-reduce, the control that isolates the collective.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist
from torch.nn.parallel import DistributedDataParallel as DDP

from ..ops.optim import AdamW, gpt2_param_groups
from .comm import Communicator, empty_registrable
from .ddp import register_tnccl_hook
from .reducer import FlatGradReducer


class DataParallelTrainer:
    def __init__(self, model: torch.nn.Module, comm: Communicator, lr: float = 6e-4,
                 weight_decay: float = 0.1, betas=(0.9, 0.95), bucket_cap_mb: int = 25,
                 algo: str = "auto", wire_dtype: torch.dtype | None = None,
                 amp_dtype: torch.dtype = torch.bfloat16, max_channels: int | None = None,
                 reducer: str | None = None, registered: bool | None = None,
                 overlap_optimizer: bool | None = None, cuda_graph: bool | None = None):
        if not dist.is_initialized():
            raise RuntimeError("DataParallelTrainer needs torch.distributed initialised")
        self.comm = comm
        # Gradient all-reduces run concurrently with backward kernels: cap
        # their CTAs so compute keeps most SMs (TNCCL_DDP_CHANNELS, default 32).
        if max_channels is None:
            max_channels = int(os.environ.get("TNCCL_DDP_CHANNELS", "32"))
        comm.set_max_channels(max_channels)
        self.model = model
        self.amp_dtype = amp_dtype
        dev = comm.device
        if reducer is None:
            reducer = os.environ.get("TNCCL_DP_REDUCER", "flat")
        if registered is None:
            # On by default: with NVLS, AUTO sends the large buckets of a
            # registered buffer through the zero-copy kernel (8 ranks: from
            # 16 MiB); TNCCL_DP_REGISTERED=0 keeps the buffer unregistered.
            registered = os.environ.get("TNCCL_DP_REGISTERED", "1") == "1"
        if overlap_optimizer is None:
            overlap_optimizer = os.environ.get("TNCCL_DP_OVERLAP_OPT", "0") == "1"
        if cuda_graph is None:
            # On by default with the flat reducer (DDP cannot be replayed).
            cuda_graph = os.environ.get("TNCCL_CUDA_GRAPH", "1") == "1" and reducer == "flat"
        if cuda_graph and reducer != "flat":
            raise ValueError("cuda_graph needs reducer='flat' (DDP's reducer runs host "
                             "logic during backward that a graph replay would skip)")
        self.cuda_graph = cuda_graph
        self._graph = None
        self._eager_steps = 0
        self._graph_kernels = 0  # this library's kernels in the captured step
        self.replayed_launches = 0  # of those, launched by graph replays so far
        self._graph_stream = torch.cuda.Stream(device=dev) if cuda_graph else None
        self.overlap_optimizer = overlap_optimizer and reducer == "flat"
        self.opt = AdamW(gpt2_param_groups(model, weight_decay), lr=lr, betas=betas)
        self.opt.device_step = cuda_graph
        # AdamW also writes the bf16 copies the next forward's GEMMs read.
        self.opt.bf16_copies = True
        self.reducer = None
        self.registration = None
        if reducer == "flat":
            if wire_dtype is not None:
                raise ValueError("wire_dtype is an option of reducer='ddp'")
            # DDP would broadcast rank 0's parameters; do the same once.
            with torch.no_grad():
                for t in list(model.parameters()) + list(model.buffers()):
                    dist.broadcast(t, 0)
            # Registration is collective and refused on every rank alike when
            # the communicator has no NVLS; the buffer then stays unregistered.
            alloc = ((lambda n, dt, d: empty_registrable(n, dt, d)) if registered
                     and comm.size > 1 and comm.info()["nvls"] else None)
            # The last bucket (the token embedding, tied to the LM head: its
            # gradient is complete only after the last backward node) overlaps
            # nothing, so it takes every channel (TNCCL_DP_TAIL_CHANNELS; 0 =
            # the communicator's configured count).
            tail = int(os.environ.get("TNCCL_DP_TAIL_CHANNELS", "0"))

            def last_all_reduce(t):
                comm.set_max_channels(tail)
                comm.all_reduce(t, op="avg", algo=algo)
                comm.set_max_channels(max_channels)

            self.reducer = FlatGradReducer(
                model.parameters(), lambda t: comm.all_reduce(t, op="avg", algo=algo),
                bucket_bytes=bucket_cap_mb << 20, alloc=alloc, stream=comm.side_stream(),
                on_reduced=self.opt.step_params if self.overlap_optimizer else None,
                last_all_reduce=last_all_reduce)
            if alloc is not None:
                self.registration = comm.register(self.reducer.flat)
            # TNCCL_DP_SPLIT_LAST=0: AdamW waits for every bucket (A/B switch).
            self._split_last = os.environ.get("TNCCL_DP_SPLIT_LAST", "1") == "1"
            last = {id(p) for p in self.reducer.bucket_params[-1]}
            self._before_last_params = [p for p in self.reducer.params if id(p) not in last]
            self.ddp = model
            self.hook_state = None
        elif reducer in ("ddp", "nccl-ddp"):
            self.ddp = DDP(model, device_ids=[dev.index], output_device=dev.index,
                           bucket_cap_mb=bucket_cap_mb, gradient_as_bucket_view=True,
                           static_graph=True, broadcast_buffers=False)
            # "nccl-ddp" keeps DDP's own NCCL all-reduce: the control that
            # isolates the collective (same model, same buckets, same steps).
            self.hook_state = (register_tnccl_hook(self.ddp, comm, algo=algo,
                                                   wire_dtype=wire_dtype)
                               if reducer == "ddp" else None)
        else:
            raise ValueError(f"reducer must be 'flat', 'ddp' or 'nccl-ddp', not {reducer!r}")
        self.reducer_name = reducer

    def step(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """One optimizer step; returns the (device) loss without synchronizing."""
        if not self.cuda_graph:
            return self._step_eager(idx, targets)
        cur = torch.cuda.current_stream(idx.device)
        if self._graph is None and self._eager_steps < 3:
            # Warm-up outside the capture (kernel loading, cuBLAS / cuDNN
            # plans, optimizer state), on the stream the capture will use.
            self._eager_steps += 1
            self._graph_stream.wait_stream(cur)
            with torch.cuda.stream(self._graph_stream):
                loss = self._step_eager(idx, targets)
            cur.wait_stream(self._graph_stream)
            return loss
        if self._graph is None:
            self._capture(idx, targets)
        self._static_idx.copy_(idx)
        self._static_tgt.copy_(targets)
        self._graph.replay()
        self.replayed_launches += self._graph_kernels
        return self._static_loss.clone()

    def _capture(self, idx: torch.Tensor, targets: torch.Tensor) -> None:
        self._static_idx = idx.clone()
        self._static_tgt = targets.clone()
        torch.cuda.synchronize(idx.device)
        from .. import launch_count
        from .._native import load
        before = launch_count() + load().ops.launch_count()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self._graph_stream):
            self._static_loss = self._step_eager(self._static_idx, self._static_tgt)
        # Every launch through the library during the capture is a kernel
        # node of the graph, launched again by each replay.
        self._graph_kernels = launch_count() + load().ops.launch_count() - before
        self._graph = graph

    def _step_eager(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        if self.overlap_optimizer:
            self.opt.begin_step()  # the buckets' hooks apply it during backward
        # Autocast's weight-cast cache is off under graph capture: cached
        # casts would be freed at the end of the region inside the capture.
        with torch.autocast("cuda", dtype=self.amp_dtype, cache_enabled=not self.cuda_graph):
            loss = self.ddp(idx, targets)
        loss.backward()
        if self.reducer is not None:
            if self.overlap_optimizer or not self._split_last:
                self.reducer.finish()
                if not self.overlap_optimizer:
                    self.opt.step()
            else:
                # AdamW updates every other bucket's parameters while the last
                # bucket (the token embedding, complete only at the end of
                # backward) is still being reduced, then that bucket's.
                self.reducer.finish(split_last=True)
                self.opt.begin_step()
                self.opt.step_params(self._before_last_params)
                self.reducer.wait_last()
                self.opt.step_params(self.reducer.bucket_params[-1])
            self.reducer.zero_grad()
        else:
            self.opt.step()
            self.opt.zero_grad(set_to_none=True)
        return loss.detach()

    def close(self) -> None:
        """Deregisters the flat gradient buffer (collective); call before the
        communicator is destroyed."""
        if self._graph is not None:
            torch.cuda.synchronize()
            self._graph = None  # releases the captured collectives' graph
        if self.registration is not None:
            self.comm.deregister(self.registration)
            self.registration = None

    def state_dict(self) -> dict:
        return {"model": self.model.state_dict(), "opt": self.opt.state_dict(),
                "step": self.opt._step}

    def describe(self) -> str:
        """The gradient path and step execution in use, e.g. 'flat+cuda-graph'."""
        d = "flat" if self.reducer is not None else self.reducer_name
        if self.registration is not None:
            d += "+registered"
        if self.overlap_optimizer:
            d += "+overlapped-adamw"
        if self.registration is not None and self.comm.info().get("zero_copy_launches", 0) > 0:
            d += "+nvls-zero-copy"  # some bucket all-reduces took the zero-copy kernel
        if self.cuda_graph:
            d += "+cuda-graph"
        return d

    def load_state_dict(self, sd: dict) -> None:
        self.model.load_state_dict(sd["model"])
        self.opt.load_state_dict(sd["opt"])
        self.opt.set_step(sd["step"])
        # The loaded optimizer state lives in new tensors: capture again
        # (after fresh warm-up steps) instead of replaying the old graph.
        if self._graph is not None:
            torch.cuda.synchronize()
            self._graph = None
        self._eager_steps = 0
