"""LayerNorm backward of the kernel that TNOPS_LN_BWD selects (read once by
the library, hence a separate process) against an fp32 PyTorch autograd
reference. Exits 0 when every shape matches."""
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))


def main():
    import tiny_nccl_b200 as tn
    ops = tn.load().ops
    for rows, C in [(64, 768), (4096, 768), (257, 1024), (100, 772), (3, 36)]:
        g = torch.Generator(device="cuda")
        g.manual_seed(rows + C)
        x = torch.randn(rows, C, device="cuda", generator=g)
        w = 1 + 0.1 * torch.randn(C, device="cuda", generator=g)
        b = torch.zeros(C, device="cuda")
        xo, _, mean, rstd = ops.ln_fwd(x, None, w, b, 1e-5)
        gy = torch.randn(rows, C, device="cuda", generator=g).to(torch.bfloat16)
        gres = torch.randn(rows, C, device="cuda", generator=g)
        dx, dxb, dw, db = ops.ln_bwd(gy, gres, xo, w, mean, rstd, True)
        xr = x.clone().requires_grad_(True)
        wr = w.clone().requires_grad_(True)
        br = b.clone().requires_grad_(True)
        torch.nn.functional.layer_norm(xr, (C,), wr, br, 1e-5).backward(gy.float())
        torch.testing.assert_close(dx, xr.grad + gres, rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(dxb.float(), xr.grad + gres, rtol=8e-3, atol=1e-3)
        torch.testing.assert_close(dw, wr.grad, rtol=1e-4, atol=5e-3)
        torch.testing.assert_close(db, br.grad, rtol=1e-4, atol=5e-3)
    print("ln_bwd", os.environ.get("TNOPS_LN_BWD", "group"), "ok")


if __name__ == "__main__":
    main()
