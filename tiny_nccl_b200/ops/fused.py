"""Autograd wrappers of the fused sm_100a model kernels (csrc/ops).

Every function calls the native kernel; there is no PyTorch fallback. A
missing extension or an unsupported shape raises.
"""
from __future__ import annotations

import os

import torch

from .._native import load


def _ops():
    return load().ops


class _AddLayerNorm(torch.autograd.Function):
    """x_out = x + delta (optional); y = LayerNorm(x_out) in bf16.

    The residual stream x stays fp32; delta (a bf16 sub-layer output) is added
    in the same pass that normalises, and the backward returns the residual
    gradient (fp32) and the sub-layer gradient (bf16) from one kernel.
    """

    @staticmethod
    def forward(ctx, x, delta, weight, bias, eps):
        C = x.shape[-1]
        x2 = x.reshape(-1, C)
        d2 = delta.reshape(-1, C) if delta is not None else None
        x_out, y, mean, rstd = _ops().ln_fwd(x2, d2, weight, bias, eps)
        ctx.save_for_backward(x_out, weight, mean, rstd)
        ctx.params = (weight, bias)
        ctx.has_delta = delta is not None
        ctx.shape = x.shape
        return x_out.view(x.shape), y.view(x.shape)

    @staticmethod
    def backward(ctx, g_xout, g_y):
        x_out, weight, mean, rstd = ctx.saved_tensors
        C = ctx.shape[-1]
        if g_y is None:
            g_y = torch.zeros(x_out.shape, dtype=torch.bfloat16, device=x_out.device)
        gres = g_xout.reshape(-1, C).contiguous() if g_xout is not None else None
        pw, pb = ctx.params
        dx, dxb, dw, db = _ops().ln_bwd(g_y.reshape(-1, C).contiguous(), gres, x_out, weight,
                                        mean, rstd, ctx.has_delta,
                                        grad_destination(pw), grad_destination(pb))
        ddelta = dxb.view(ctx.shape) if ctx.has_delta else None
        return dx.view(ctx.shape), ddelta, dw, db, None


def add_layer_norm(x: torch.Tensor, delta: torch.Tensor, weight: torch.Tensor,
                   bias: torch.Tensor, eps: float = 1e-5):
    """Returns (x + delta, LayerNorm(x + delta)) with x fp32, delta bf16."""
    x_out, y = _AddLayerNorm.apply(x, delta.contiguous(), weight, bias, eps)
    return x_out, y


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
               eps: float = 1e-5) -> torch.Tensor:
    """bf16 LayerNorm of a fp32 input."""
    return _AddLayerNorm.apply(x.contiguous(), None, weight, bias, eps)[1]


class _CrossEntropy(torch.autograd.Function):
    """Mean softmax cross-entropy of bf16 logits. The forward kernel also
    writes d(loss)/d(logits) into the logits buffer, so the backward only
    rescales when the incoming gradient is not 1 (checked on the device)."""

    @staticmethod
    def forward(ctx, logits, target, classes):
        valid = int(target.numel())
        per_row = _ops().cross_entropy_fwd_bwd(logits, target, valid, classes)
        ctx.save_for_backward(logits)
        return per_row.sum() / valid

    @staticmethod
    def backward(ctx, g):
        (dlogits,) = ctx.saved_tensors
        _ops().scale_bf16_(dlogits, g.reshape(1).float().contiguous())
        return dlogits, None, None


def cross_entropy(logits: torch.Tensor, target: torch.Tensor,
                  reuse_logits: bool = True, classes: int = 0) -> torch.Tensor:
    """Mean cross-entropy of [rows, ld] logits against int64 targets, over the
    first ``classes`` columns (all columns when 0; the rest is vocabulary
    padding, excluded from the softmax and given zero gradient).

    With ``reuse_logits`` (the default, used for the model's temporary logits)
    the gradient is written into the logits storage during the forward pass,
    so the logits values are gone afterwards; pass False to keep them (the
    kernel then works on a copy)."""
    if logits.dtype != torch.bfloat16:
        logits = logits.to(torch.bfloat16)
    elif not reuse_logits:
        logits = logits.clone()
    return _CrossEntropy.apply(logits.contiguous(), target.contiguous(), int(classes))


def bf16_weight(p: torch.Tensor) -> torch.Tensor:
    """The bf16 value of an fp32 parameter for a GEMM operand: the copy the
    fused AdamW wrote in its last update while it is current (the
    parameter's version unchanged since), else a cast."""
    c = getattr(p, "_tn_bf16", None)
    if c is not None and c[1] == p._version:
        return c[0]
    return p.to(torch.bfloat16)


def grad_destination(p: torch.Tensor):
    """Where the gradient of parameter p can be written directly: its slice
    of a flat gradient buffer (FlatGradReducer sets ``p._tn_grad_dest``), as
    long as p has no gradient yet in this backward. The backward functions
    below write their parameter gradients there and return that slice, which
    autograd then adopts as ``p.grad`` as it is (no copy, no accumulation
    kernel). None otherwise: a new tensor is returned and autograd handles it
    as usual."""
    d = getattr(p, "_tn_grad_dest", None)
    # A new tensor object on the same memory: autograd adopts a gradient
    # without copying only when nothing else holds the object.
    return d.detach() if d is not None and p.grad is None else None


def _wgrad(gy: torch.Tensor, x: torch.Tensor, dest: torch.Tensor | None = None) -> torch.Tensor:
    """dW = gy^T x with bf16 operands and the fp32 result written by the GEMM
    itself (no bf16 rounding, no separate cast to the fp32 parameter),
    into ``dest`` when given."""
    if dest is not None:
        return torch.mm(gy.t(), x, out_dtype=torch.float32, out=dest)
    return torch.mm(gy.t(), x, out_dtype=torch.float32)


class _LinearBias(torch.autograd.Function):
    """y = x W^T + b in bf16 (cuBLAS GEMM with bias epilogue) for fp32
    parameters. Backward: dX and dW on cuBLAS (dW written in fp32), db by the
    deterministic column-sum kernel."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        w16 = bf16_weight(weight)
        with torch.autocast("cuda", enabled=False):
            y = torch.addmm(bf16_weight(bias), x, w16.t())
        ctx.save_for_backward(x, w16)
        ctx.params = (weight, bias)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, w16 = ctx.saved_tensors
        pw, pb = ctx.params
        gy = gy.contiguous()
        return (gy @ w16, _wgrad(gy, x, grad_destination(pw)),
                _ops().bias_grad(gy, out=grad_destination(pb)))


# The forward of linear_gelu runs this library's tcgen05 GEMM with its fused
# bias + GELU epilogue: TNCCL_TCGEN05_GEMM=pair (default: persistent CTA
# pairs, cta_group::2), persistent (one CTA per SM) or 1 (one tile per CTA);
# 0 selects cuBLAS and a separate GELU kernel. The persistent variants
# assume they get (nearly) every SM: in training they run in the forward
# pass, when no gradient all-reduce is in flight.
_TCGEN05 = os.environ.get("TNCCL_TCGEN05_GEMM", "pair")
_TCGEN05_VARIANT = {"1": 0, "persistent": 1, "pair": 2}.get(_TCGEN05, 0)


class _LinearGelu(torch.autograd.Function):
    """y = GELU_tanh(x W^T + b): one tcgen05 GEMM with the bias and GELU in
    its epilogue (or cuBLAS + GELU with TNCCL_TCGEN05_GEMM=0). Backward: one
    kernel computes the GELU gradient and the bias gradient (column sums of
    that gradient); dX and dW on cuBLAS."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        w16 = bf16_weight(weight)
        b16 = bf16_weight(bias)
        if _TCGEN05 != "0":
            pre, y = _ops().gemm_bias_act(x, w16, b16, True, _TCGEN05_VARIANT)
        else:
            with torch.autocast("cuda", enabled=False):
                pre = torch.addmm(b16, x, w16.t())
                y = torch.nn.functional.gelu(pre, approximate="tanh")
        ctx.save_for_backward(x, w16, pre)
        ctx.params = (weight, bias)
        return y

    @staticmethod
    def backward(ctx, gy):
        x, w16, pre = ctx.saved_tensors
        pw, pb = ctx.params
        gpre, db = _ops().gelu_bwd_bias(gy.contiguous(), pre, grad_destination(pb))
        return gpre @ w16, _wgrad(gpre, x, grad_destination(pw)), db


class _LinearNoBias(torch.autograd.Function):
    """y = x W^T in bf16 for an fp32 weight (the tied LM head): dX on cuBLAS,
    dW written in fp32 by the GEMM itself."""

    @staticmethod
    def forward(ctx, x, weight):
        w16 = bf16_weight(weight)
        with torch.autocast("cuda", enabled=False):
            y = torch.mm(x, w16.t())
        ctx.save_for_backward(x, w16)
        ctx.weight = weight
        return y

    @staticmethod
    def backward(ctx, gy):
        x, w16 = ctx.saved_tensors
        gy = gy.contiguous()
        return gy @ w16, _wgrad(gy, x, grad_destination(ctx.weight))


def _rows(x: torch.Tensor) -> torch.Tensor:
    x = x.reshape(-1, x.shape[-1])
    return (x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)).contiguous()


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """bf16 x W^T + b over the last dimension of x (fp32 weight and bias)."""
    y = _LinearBias.apply(_rows(x), weight, bias)
    return y.view(*x.shape[:-1], weight.shape[0])


def linear_nobias(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """bf16 x W^T over the last dimension of x (fp32 weight, no bias)."""
    y = _LinearNoBias.apply(_rows(x), weight)
    return y.view(*x.shape[:-1], weight.shape[0])


def linear_gelu(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """GELU(tanh)(x W^T + b) in bf16; the backward fuses the GELU gradient
    with the bias gradient."""
    y = _LinearGelu.apply(_rows(x), weight, bias)
    return y.view(*x.shape[:-1], weight.shape[0])


def launch_count() -> int:
    return _ops().launch_count()
