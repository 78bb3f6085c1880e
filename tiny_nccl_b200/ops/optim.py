"""AdamW on the multi-tensor sm_100a kernel (csrc/ops/adamw.cu).

Semantics of torch.optim.AdamW (decoupled weight decay, bias correction).
Parameters are grouped by weight decay: 2-D weights decay, biases, LayerNorm
gains and embeddings tables of positions follow the usual GPT-2 recipe via
the `no_decay` predicate.
"""
from __future__ import annotations

import torch

from .._native import load


class AdamW(torch.optim.Optimizer):
    def __init__(self, params, lr=6e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1):
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        super().__init__(params, defaults)
        self._step = 0
        # With device_step, the step count also lives in device memory and the
        # kernel reads it when it runs, so a step captured in a CUDA graph
        # uses the right bias correction on every replay.
        self.device_step = False
        self._step_t = None
        # With bf16_copies, every update also writes a bf16 copy of the
        # parameter (same kernel pass); the fused linear layers use it instead
        # of casting the fp32 parameter again in the next forward
        # (tiny_nccl_b200.ops.fused.bf16_weight).
        self.bf16_copies = False
        # Kept outside self.state: Optimizer.load_state_dict casts state
        # tensors to the parameter's dtype, and the copies are derived data
        # (rewritten by the next update) that a checkpoint need not hold.
        self._bf16 = {}

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        self.begin_step()
        self.step_params()
        return loss

    def begin_step(self) -> None:
        """Advances the step count (bias correction) of a step whose update is
        applied in parts with :meth:`step_params`."""
        self._step += 1
        if self.device_step:
            if self._step_t is None:
                dev = self.param_groups[0]["params"][0].device
                self._step_t = torch.full((1,), self._step, dtype=torch.int64, device=dev)
            else:
                self._step_t.add_(1)

    def set_step(self, n: int) -> None:
        """Sets the number of completed steps (e.g. from a checkpoint)."""
        self._step = int(n)
        if self._step_t is not None:
            self._step_t.fill_(self._step)

    @torch.no_grad()
    def step_params(self, only=None) -> None:
        """Applies the current step to the parameters in ``only`` (all when
        None) that have a gradient. The update is elementwise, so a step split
        into parts (one per gradient bucket, as its all-reduce completes)
        gives the same result as one call."""
        ops = load().ops
        sel = None if only is None else {id(p) for p in only}
        for group in self.param_groups:
            ps, gs, ms, vs, wds, cs = [], [], [], [], [], []
            for p in group["params"]:
                if p.grad is None or (sel is not None and id(p) not in sel):
                    continue
                st = self.state[p]
                if not st:
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
                ps.append(p)
                if self.bf16_copies:
                    if id(p) not in self._bf16:
                        self._bf16[id(p)] = torch.empty(p.shape, dtype=torch.bfloat16,
                                                        device=p.device)
                    cs.append(self._bf16[id(p)])
                gs.append(p.grad if p.grad.is_contiguous() else p.grad.contiguous())
                ms.append(st["exp_avg"])
                vs.append(st["exp_avg_sq"])
                wds.append(float(group["weight_decay"]))
            if ps:
                b1, b2 = group["betas"]
                ops.adamw(ps, gs, ms, vs, wds, float(group["lr"]), float(b1), float(b2),
                          float(group["eps"]), self._step, 1.0,
                          self._step_t if self.device_step else None, cs)
                # The kernel writes through raw pointers, so the parameter's
                # version counter stays put: a copy is current as long as the
                # version is the one recorded here (any other in-place change
                # of the parameter moves it on and retires the copy).
                for p, c in zip(ps, cs):
                    p._tn_bf16 = (c, p._version)


def gpt2_param_groups(model: torch.nn.Module, weight_decay: float = 0.1):
    """2-D weights decay; biases and LayerNorm parameters do not."""
    decay, no_decay = [], []
    for _, p in model.named_parameters():
        if not p.requires_grad:
            continue
        (decay if p.dim() >= 2 else no_decay).append(p)
    return [{"params": decay, "weight_decay": weight_decay},
            {"params": no_decay, "weight_decay": 0.0}]
