"""Fused sm_100a model kernels vs plain PyTorch fp32 references."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(built):
    import tiny_nccl_b200.ops as o
    assert o.launch_count() >= 0
    return o


@pytest.mark.parametrize("rows,C", [(64, 768), (257, 1024), (8, 128), (33, 640)])
@pytest.mark.parametrize("with_delta", [False, True])
def test_add_layer_norm(ops, rows, C, with_delta):
    torch.manual_seed(0)
    dev = "cuda"
    x = torch.randn(rows, C, device=dev, requires_grad=True)
    d = torch.randn(rows, C, device=dev).to(torch.bfloat16).requires_grad_(with_delta)
    w = (1 + 0.1 * torch.randn(C, device=dev)).requires_grad_()
    b = (0.1 * torch.randn(C, device=dev)).requires_grad_()
    if with_delta:
        xo, y = ops.add_layer_norm(x, d, w, b)
    else:
        y = ops.layer_norm(x, w, b)
        xo = x
    gy = torch.randn(rows, C, device=dev).to(torch.bfloat16)
    gx = torch.randn(rows, C, device=dev)
    (y.float() * gy.float()).sum().backward(retain_graph=True) if not with_delta else \
        ((y.float() * gy.float()).sum() + (xo * gx).sum()).backward()
    # fp32 reference
    xr = x.detach().clone().requires_grad_()
    dr = d.detach().float().clone().requires_grad_(with_delta)
    wr = w.detach().clone().requires_grad_()
    br = b.detach().clone().requires_grad_()
    xor = xr + dr if with_delta else xr
    yr = torch.nn.functional.layer_norm(xor, (C,), wr, br, 1e-5)
    lr = (yr * gy.float()).sum() + ((xor * gx).sum() if with_delta else 0)
    lr.backward()
    torch.testing.assert_close(y.float(), yr, atol=2e-2, rtol=1e-2)
    if with_delta:
        torch.testing.assert_close(xo, xor, atol=1e-6, rtol=1e-6)
        torch.testing.assert_close(d.grad.float(), dr.grad, atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(x.grad, xr.grad, atol=1e-3, rtol=1e-3)
    torch.testing.assert_close(w.grad, wr.grad, atol=1e-2, rtol=1e-3)
    torch.testing.assert_close(b.grad, br.grad, atol=1e-2, rtol=1e-3)


@pytest.mark.parametrize("rows,V", [(16, 50257), (7, 1000), (3, 9)])
def test_cross_entropy(ops, rows, V):
    torch.manual_seed(1)
    logits = (3 * torch.randn(rows, V, device="cuda")).to(torch.bfloat16)
    tgt = torch.randint(0, V, (rows,), device="cuda")
    ref_in = logits.float().clone().requires_grad_()
    ref = torch.nn.functional.cross_entropy(ref_in, tgt)
    ref.backward()
    x = logits.clone().requires_grad_()
    loss = ops.cross_entropy(x, tgt)
    loss.backward()
    torch.testing.assert_close(loss, ref, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(x.grad.float(), ref_in.grad, atol=2e-4, rtol=2e-2)


def test_cross_entropy_grad_scale(ops):
    logits = torch.randn(5, 300, device="cuda").to(torch.bfloat16).requires_grad_()
    tgt = torch.randint(0, 300, (5,), device="cuda")
    ref_in = logits.detach().float().clone().requires_grad_()
    kept = logits.detach().clone()
    (ops.cross_entropy(logits, tgt, reuse_logits=False) * 3.0).backward()
    assert torch.equal(logits.detach(), kept)  # reuse_logits=False keeps the input
    (torch.nn.functional.cross_entropy(ref_in, tgt) * 3.0).backward()
    torch.testing.assert_close(logits.grad.float(), ref_in.grad, atol=1e-3, rtol=3e-2)


def test_adamw_matches_torch(ops):
    torch.manual_seed(2)
    shapes = [(768, 768), (3,), (1000, 7), (50257, 16)]
    a = [torch.randn(s, device="cuda", requires_grad=True) for s in shapes]
    b = [t.detach().clone().requires_grad_() for t in a]
    opt_a = ops.AdamW([{"params": a[:2], "weight_decay": 0.1},
                       {"params": a[2:], "weight_decay": 0.0}], lr=1e-3, betas=(0.9, 0.95))
    opt_b = torch.optim.AdamW([{"params": b[:2], "weight_decay": 0.1},
                               {"params": b[2:], "weight_decay": 0.0}], lr=1e-3, betas=(0.9, 0.95),
                              eps=1e-8)
    for step in range(5):
        g = [torch.randn(s, device="cuda") for s in shapes]
        for t, gg in zip(a, g):
            t.grad = gg.clone()
        for t, gg in zip(b, g):
            t.grad = gg.clone()
        opt_a.step()
        opt_b.step()
    for x, y in zip(a, b):
        torch.testing.assert_close(x, y, atol=1e-6, rtol=1e-5)
