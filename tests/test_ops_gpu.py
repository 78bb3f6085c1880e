"""Fused sm_100a model kernels vs plain PyTorch fp32 references."""
import sys

import pytest
import torch

from conftest import run

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(built):
    import tiny_nccl_b200.ops as o
    assert o.launch_count() >= 0
    return o


# C % 8 == 0 takes the pipelined backward (cp.async row stages), C = 772 and
# 36 the one-row-per-warp kernel; 4096 rows give every warp several rows.
@pytest.mark.parametrize("rows,C", [(64, 768), (257, 1024), (8, 128), (33, 640), (4096, 768),
                                    (100, 772), (3, 36)])
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


@pytest.mark.parametrize("variant", ["group", "warp"])
def test_ln_bwd_kernel_variants(built, variant):
    """Both LayerNorm backward kernels (row groups, the default; one warp
    per row, TNOPS_LN_BWD=warp) against fp32 autograd, in a fresh process
    because the library reads the switch once."""
    r = run([sys.executable, "tests/workers/ln_bwd_variant_worker.py"],
            env={"TNOPS_LN_BWD": variant})
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]


def test_ln_bwd_refuses_misaligned_rows(ops):
    """Rows that do not start on 16 bytes are refused before any launch."""
    import tiny_nccl_b200 as tn
    C, rows = 768, 4
    base = torch.zeros(rows * C + 1, device="cuda")
    xo = base[1:].view(rows, C)  # 4 bytes past a 16-byte boundary
    w = torch.ones(C, device="cuda")
    stats = torch.ones(rows, device="cuda")
    gy = torch.zeros(rows, C, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        tn.load().ops.ln_bwd(gy, None, xo, w, stats, stats, True)


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


@pytest.mark.parametrize("M,N", [(8192, 768), (1000, 3072), (37, 2304), (5, 8)])
def test_bias_grad(ops, M, N):
    """Column sums of a bf16 gradient (the bias gradient) vs fp32 torch."""
    from tiny_nccl_b200._native import load
    torch.manual_seed(M + N)
    g = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    db = load().ops.bias_grad(g)
    ref = g.float().sum(0)
    assert db.dtype == torch.float32
    torch.testing.assert_close(db, ref, rtol=1e-5, atol=1e-4)
    # deterministic: the same bits on a second call
    assert torch.equal(db, load().ops.bias_grad(g))


def _gelu_tanh_grad64(x):
    k0, k1 = (2.0 / torch.pi) ** 0.5, 0.044715
    t = torch.tanh(k0 * (x + k1 * x ** 3))
    return 0.5 * (1 + t) + 0.5 * x * (1 - t * t) * k0 * (1 + 3 * k1 * x * x)


@pytest.mark.parametrize("M,N", [(4096, 3072), (129, 64)])
def test_gelu_bwd_bias(ops, M, N):
    """Fused tanh-GELU backward + bias gradient vs an fp64 reference of the
    same formula: the bf16 gradient within one rounding, the bias gradient
    as the fp32 column sum of the kernel's own bf16 gradient."""
    from tiny_nccl_b200._native import load
    torch.manual_seed(N)
    gy = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    pre = (2 * torch.randn(M, N, device="cuda")).to(torch.bfloat16)
    gpre, db = load().ops.gelu_bwd_bias(gy, pre)
    ref = (gy.double() * _gelu_tanh_grad64(pre.double())).to(torch.bfloat16)
    # One bf16 rounding of the product, plus the fp32 evaluation error of
    # gelu' (absolute, scaled by |gy|) where the derivative nearly cancels.
    diff = (gpre.float() - ref.float()).abs()
    bound = ref.float().abs() * 2.0 ** -7 + gy.float().abs() * 1e-5 + 1e-30
    assert bool((diff <= bound).all()), float((diff / bound).max())
    torch.testing.assert_close(db, gpre.float().sum(0), rtol=1e-5, atol=1e-4)


def test_linear_autograd_matches_torch(ops):
    """ops.linear / ops.linear_gelu (custom backward: fp32 weight gradient
    from the GEMM, fused bias / GELU gradients) vs autocast nn.functional."""
    torch.manual_seed(3)
    x = torch.randn(4, 256, 768, device="cuda")
    lin = torch.nn.Linear(768, 3072).cuda()
    lin2 = torch.nn.Linear(3072, 768).cuda()
    gy = torch.randn(4, 256, 768, device="cuda")

    def run(fused):
        for p in (*lin.parameters(), *lin2.parameters()):
            p.grad = None
        xi = x.clone().requires_grad_()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            if fused:
                h = ops.linear_gelu(xi, lin.weight, lin.bias)
                y = ops.linear(h, lin2.weight, lin2.bias)
            else:
                h = torch.nn.functional.gelu(lin(xi), approximate="tanh")
                y = lin2(h)
        (y.float() * gy).sum().backward()
        return y.float(), xi.grad, [p.grad.clone() for p in (*lin.parameters(), *lin2.parameters())]

    yf, gxf, gpf = run(True)
    yt, gxt, gpt = run(False)
    torch.testing.assert_close(yf, yt, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(gxf, gxt, rtol=5e-2, atol=5e-2)
    for a, b in zip(gpf, gpt):
        assert a.dtype == torch.float32
        rel = (a - b).norm() / b.norm()
        assert rel < 2e-2, float(rel)
