"""The tcgen05 GEMM with the fused bias + GELU epilogue (csrc/ops/
gemm_tcgen05.cu), one CTA per tile, persistent, and persistent CTA pairs
(cta_group::2, 256 x 256 tiles), against an fp32 PyTorch
reference of the same op, on the GPT-2 MLP shape and on shapes with M, N and
K tails."""
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(128, 256, 64), (256, 264, 72), (1000, 3072, 768), (8192, 3072, 768)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("gelu", [True, False])
@pytest.mark.parametrize("persistent", [0, 1, 2])  # one tile per CTA, persistent, CTA pairs
def test_gemm_bias_act_matches_fp32_reference(built, M, N, K, gelu, persistent):
    import tiny_nccl_b200 as tn

    ops = tn.load().ops
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = (torch.randn(M, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    b = (torch.randn(N, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    out = ops.gemm_bias_act(x, w, b, gelu, persistent)
    torch.cuda.synchronize()
    assert ops.tcgen05_status(True) == 0
    ref = x.float() @ w.float().t() + b.float()
    # One bf16 rounding of an fp32 sum whose order differs from the reference's.
    tol = dict(rtol=1.6e-2, atol=2e-3 * float(ref.abs().max()))
    torch.testing.assert_close(out[0].float(), ref, **tol)
    if gelu:
        # GELU of the kernel's own bf16 pre: one bf16 rounding (half an ulp,
        # 2^-9 relative) of an accurate evaluation.
        act_ref = torch.nn.functional.gelu(out[0].float(), approximate="tanh")
        torch.testing.assert_close(out[1].float(), act_ref, rtol=8e-3, atol=1e-5)


def test_gemm_without_bias_and_argument_checks(built):
    import tiny_nccl_b200 as tn

    ops = tn.load().ops
    x = torch.randn(300, 128, device="cuda").to(torch.bfloat16)
    w = torch.randn(512, 128, device="cuda").to(torch.bfloat16)
    (pre,) = ops.gemm_bias_act(x, w, None, False)
    torch.cuda.synchronize()
    torch.testing.assert_close(pre.float(), x.float() @ w.float().t(), rtol=1.6e-2, atol=0.1)
    with pytest.raises(RuntimeError):
        ops.gemm_bias_act(x[:, :100].contiguous(), w[:, :100].contiguous(), None, False)  # K % 8
    assert ops.tcgen05_status(True) == 0
