"""DDP communication hook that all-reduces gradient buckets with tnccl.

``DistributedDataParallel`` calls the hook once per gradient bucket as soon as
the bucket is ready during backward. The hook makes a side stream (the stream
the communicator is bound to) wait for the default stream, enqueues one
all-reduce on it with the 1/world_size averaging fused into the kernel as a
pre-scale, and returns a CUDA-aware future: DDP's final wait becomes a stream
dependency, not a host synchronization, so bucket communication overlaps with
the rest of backward.

Optionally the bucket is sent as bf16 (``wire_dtype=torch.bfloat16``): the
fp32 gradients are cast, reduced with fp32 accumulation, and cast back.
"""

import torch

from .comm import Communicator


class TncclHookState:
    def __init__(self, comm: Communicator, stream: torch.cuda.Stream | None = None,
                 algo: str = "auto", wire_dtype: torch.dtype | None = None):
        self.comm = comm
        # Collectives of a communicator run on the one stream it is bound to,
        # so every hook on the same communicator shares its side stream.
        self.stream = stream if stream is not None else comm.side_stream()
        self.algo = algo
        self.wire_dtype = wire_dtype
        self.buckets = 0

    def __setstate__(self, state):  # DDP may pickle hook states; keep it explicit
        self.__dict__.update(state)


def tnccl_allreduce_hook(state: TncclHookState, bucket) -> torch.futures.Future[torch.Tensor]:
    buf = bucket.buffer()
    producer = torch.cuda.current_stream(buf.device)
    side = state.stream
    side.wait_stream(producer)
    with torch.cuda.stream(side):
        if state.wire_dtype is not None and state.wire_dtype != buf.dtype:
            wire = buf.to(state.wire_dtype)
            state.comm.all_reduce(wire, op="avg", algo=state.algo)
            buf.copy_(wire)
            wire.record_stream(side)
        else:
            state.comm.all_reduce(buf, op="avg", algo=state.algo)
        buf.record_stream(side)
        fut = torch.futures.Future(devices=[buf.device])
        fut.set_result(buf)
    state.buckets += 1
    return fut


def register_tnccl_hook(ddp_model, comm: Communicator, **kwargs) -> TncclHookState:
    """Registers the hook on a DistributedDataParallel model."""
    state = TncclHookState(comm, **kwargs)
    ddp_model.register_comm_hook(state, tnccl_allreduce_hook)
    return state
