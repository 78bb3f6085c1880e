"""Host-side logic of the fused ops that needs no GPU: where a parameter's
gradient may be written directly (its flat-buffer slice), and when the bf16
weight copy written by AdamW may stand in for a cast."""
import torch

from tiny_nccl_b200.ops.fused import bf16_weight, grad_destination


def test_grad_destination_follows_the_flat_slice():
    p = torch.nn.Parameter(torch.randn(4, 4))
    assert grad_destination(p) is None  # no flat buffer: a new tensor is returned
    flat = torch.zeros(32)
    p._tn_grad_dest = flat[8:24].view(4, 4)
    d = grad_destination(p)
    # Same memory, a new tensor object (autograd adopts it without a copy
    # only when nothing else holds it).
    assert d is not p._tn_grad_dest
    assert d.data_ptr() == flat[8:].data_ptr() and d.shape == p.shape
    assert not d.requires_grad
    # Once the parameter has a gradient in this backward, accumulation is
    # autograd's job again.
    p.grad = torch.zeros(4, 4)
    assert grad_destination(p) is None


def test_bf16_weight_uses_the_copy_only_while_current():
    p = torch.nn.Parameter(torch.randn(8, 8))
    fresh = bf16_weight(p)  # no copy yet: a cast
    assert fresh.dtype == torch.bfloat16 and torch.equal(fresh, p.detach().to(torch.bfloat16))
    copy = p.detach().to(torch.bfloat16)
    p._tn_bf16 = (copy, p._version)
    assert bf16_weight(p) is copy
    with torch.no_grad():
        p.mul_(2)  # an in-place change bumps the version: the copy is stale
    got = bf16_weight(p)
    assert got is not copy and torch.equal(got, p.detach().to(torch.bfloat16))
