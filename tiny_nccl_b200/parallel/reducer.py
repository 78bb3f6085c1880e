"""Data-parallel gradient reduction over one flat gradient buffer.

An alternative to ``DistributedDataParallel`` + the tnccl comm hook
(:mod:`.ddp`). Every parameter's ``.grad`` is a view into one flat buffer,
cut into buckets of about ``bucket_bytes``; a post-accumulate-grad hook per
parameter counts the bucket's gradients as backward produces them, and a
bucket is all-reduced (on a side stream, averaged over ranks) as soon as it is
complete. Buckets are launched strictly in index order, so every rank issues
the same collectives in the same order whatever order its hooks fire in
(collectives of one communicator must match across ranks).

What the flat buffer adds over DDP's own buckets is where it lives: with
``alloc=empty_registrable`` it is tncclMemAlloc memory that the communicator
can register, so every bucket all-reduce that AUTO sends through NVLS (8
ranks, buckets from 16 MiB) is the zero-copy kernel (the NVSwitch reduces; the kernel only issues
multimem loads and stores, so it needs few SMs while backward runs). Bucket
boundaries and parameter offsets are multiples of 16 bytes, as that kernel
requires, and they are the same on every rank because every rank builds the
layout from the same parameter list.

``on_reduced(params)``, when given, is called right after a bucket's
all-reduce is enqueued, on the same stream, with the bucket's parameters: an
optimizer can update them there (``AdamW.step_params``) while backward
still runs for the layers below, instead of after the whole backward. That
is safe because a parameter's gradient hook fires only after the backward
node that read the parameter has been enqueued, and the side stream waits
for everything enqueued before the hook.

tiny-nccl has no trainer; the bucketing follows DDP's (reverse registration
order, ~25 MB buckets, launch in bucket order).
"""
from __future__ import annotations

from typing import Callable, Iterable

import torch


class FlatGradReducer:
    """Owns the gradients of ``params``.

    ``all_reduce(t)`` must average ``t`` in place over the ranks (it is called
    on ``stream`` when one is given). Call :meth:`finish` after every
    backward and before the optimizer step, and :meth:`zero_grad` after the
    step: it unsets every ``.grad``, and the next backward puts each one back
    as its slice of the flat buffer (written there directly by the fused
    backward kernels, copied there from any other op).
    """

    def __init__(self, params: Iterable[torch.nn.Parameter],
                 all_reduce: Callable[[torch.Tensor], None], *,
                 bucket_bytes: int = 25 << 20,
                 alloc: Callable[..., torch.Tensor] | None = None,
                 stream: torch.cuda.Stream | None = None,
                 on_reduced: Callable[[list], None] | None = None,
                 last_all_reduce: Callable[[torch.Tensor], None] | None = None):
        params = [p for p in params if p.requires_grad]
        if not params:
            raise ValueError("FlatGradReducer: no parameter requires a gradient")
        dtype, device = params[0].dtype, params[0].device
        if any(p.dtype != dtype or p.device != device for p in params):
            raise ValueError("FlatGradReducer: parameters must share one dtype and device")
        es = torch.empty((), dtype=dtype).element_size()
        align = max(1, 16 // es)  # 16-byte offsets and bucket ends
        cap = max(align, bucket_bytes // es)
        # Backward produces gradients roughly in reverse registration order.
        order = list(reversed(params))
        offsets, buckets, bucket_of = [], [], []
        off = start = 0
        for p in order:
            n = p.numel()
            if off > start and off + n - start > cap:
                buckets.append((start, off))
                start = off
            offsets.append(off)
            bucket_of.append(len(buckets))
            off += -(-n // align) * align
        buckets.append((start, off))
        self.total = off
        self.flat = (alloc(off, dtype, device) if alloc is not None
                     else torch.empty(off, dtype=dtype, device=device))
        self.flat.zero_()
        self.buckets = buckets
        self.params = order
        self._bucket_of = {}
        self._views = {}
        self._need = [0] * len(buckets)
        for p, o, b in zip(order, offsets, bucket_of):
            view = self.flat[o:o + p.numel()].view_as(p)
            p.grad = view
            # The fused backward kernels write p's gradient straight into
            # this slice while p.grad is unset (ops.fused.grad_destination).
            p._tn_grad_dest = view
            self._views[id(p)] = view
            self._bucket_of[id(p)] = b
            self._need[b] += 1
        self.bucket_params = [[] for _ in buckets]
        for p, b in zip(order, bucket_of):
            self.bucket_params[b].append(p)
        self._all_reduce = all_reduce
        # The last bucket (the first parameters registered, e.g. the token
        # embedding, whose gradient is complete only at the end of backward)
        # may be reduced differently: nothing is left to overlap with it.
        self._last_all_reduce = last_all_reduce or all_reduce
        self._on_reduced = on_reduced
        self._stream = stream
        self._pending = list(self._need)
        self._next = 0  # first bucket not launched yet
        self._fired = set()
        self.launched = 0
        # Recorded on the side stream after the next-to-last bucket's
        # all-reduce: finish(split_last=True) lets the caller start on every
        # other bucket while the last one is still being reduced.
        self._before_last = torch.cuda.Event() if stream is not None else None
        self._hooks = [p.register_post_accumulate_grad_hook(self._ready) for p in order]

    # -- hooks ----------------------------------------------------------------
    def _ready(self, p: torch.Tensor) -> None:
        # After zero_grad() the gradient arrives in one of two ways: written
        # into p's slice by a fused backward kernel (adopted as it is), or as
        # a new tensor from any other op, which goes into the slice here.
        view = self._views[id(p)]
        g = p.grad
        if g.data_ptr() != view.data_ptr() or g.stride() != view.stride():
            view.copy_(g)
            p.grad = view
        self._fired.add(id(p))
        b = self._bucket_of[id(p)]
        self._pending[b] -= 1
        while self._next < len(self.buckets) and self._pending[self._next] == 0:
            self._launch(self._next)
            self._next += 1

    def _launch(self, b: int) -> None:
        s, e = self.buckets[b]
        chunk = self.flat[s:e]
        reduce = self._last_all_reduce if b == len(self.buckets) - 1 else self._all_reduce
        if self._stream is None:
            reduce(chunk)
            if self._on_reduced is not None:
                self._on_reduced(self.bucket_params[b])
        else:
            self._stream.wait_stream(torch.cuda.current_stream(self.flat.device))
            with torch.cuda.stream(self._stream):
                reduce(chunk)
                if self._on_reduced is not None:
                    self._on_reduced(self.bucket_params[b])
                if b == len(self.buckets) - 2:
                    self._before_last.record(self._stream)
        self.launched += 1

    # -- per step ---------------------------------------------------------------
    def finish(self, split_last: bool = False) -> None:
        """Launches the buckets still waiting (parameters that got no gradient
        this step), makes the current stream wait for every all-reduce and
        re-arms the counters for the next backward. With ``split_last`` the
        current stream waits only for the buckets before the last one; call
        :meth:`wait_last` before using the last bucket's gradients."""
        for p in self.params:  # no gradient this step: its slice holds zeros
            if id(p) not in self._fired:
                view = self._views[id(p)]
                view.zero_()
                p.grad = view
        while self._next < len(self.buckets):
            self._launch(self._next)
            self._next += 1
        if self._stream is not None:
            cur = torch.cuda.current_stream(self.flat.device)
            if split_last and len(self.buckets) >= 2:
                cur.wait_event(self._before_last)
            else:
                cur.wait_stream(self._stream)
        self._pending = list(self._need)
        self._next = 0
        self._fired = set()

    def wait_last(self) -> None:
        """After ``finish(split_last=True)``: the current stream waits for the
        last bucket's all-reduce too."""
        if self._stream is not None:
            torch.cuda.current_stream(self.flat.device).wait_stream(self._stream)

    def zero_grad(self) -> None:
        """Unsets every ``.grad`` (no kernel): the next backward writes each
        gradient into its slice of the flat buffer instead of adding it to
        a zeroed one."""
        for p in self.params:
            p.grad = None

    def remove(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []
        for p in self.params:
            if getattr(p, "_tn_grad_dest", None) is self._views[id(p)]:
                del p._tn_grad_dest
