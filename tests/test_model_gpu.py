"""GPT-2 with the fused kernels vs the same model on stock PyTorch ops."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _pair(cfg):
    from tiny_nccl_b200.models import GPT2
    torch.manual_seed(0)
    fused = GPT2(cfg, impl="fused").cuda()
    ref = GPT2(cfg, impl="torch").cuda()
    ref.load_state_dict(fused.state_dict())
    return fused, ref


def test_gpt2_fused_matches_torch(built):
    from tiny_nccl_b200.models import GPT2Config
    cfg = GPT2Config(n_layer=2, n_head=4, n_embd=256, vocab_size=1000, block_size=128)
    fused, ref = _pair(cfg)
    idx = torch.randint(0, 1000, (2, 128), device="cuda")
    tgt = torch.randint(0, 1000, (2, 128), device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        lf = fused(idx, tgt)
        lr = ref(idx, tgt)
    lf.backward()
    lr.backward()
    assert abs(lf.item() - lr.item()) < 2e-2, (lf.item(), lr.item())
    for (n, a), (_, b) in zip(fused.named_parameters(), ref.named_parameters()):
        cos = torch.nn.functional.cosine_similarity(a.grad.flatten(), b.grad.flatten(), dim=0)
        assert cos > 0.99, (n, cos.item())


def test_gpt2_small_trains(built):
    from tiny_nccl_b200.models import GPT2, GPT2Config
    from tiny_nccl_b200.ops import AdamW, gpt2_param_groups
    torch.manual_seed(0)
    cfg = GPT2Config(n_layer=2, n_head=4, n_embd=128, vocab_size=512, block_size=64)
    m = GPT2(cfg, impl="fused").cuda()
    opt = AdamW(gpt2_param_groups(m), lr=3e-3)
    data = torch.randint(0, 64, (4, 65), device="cuda")  # small vocabulary subset: learnable
    losses = []
    for _ in range(30):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = m(data[:, :-1], data[:, 1:])
        loss.backward()
        opt.step()
        opt.zero_grad()
        losses.append(loss.item())
    assert losses[-1] < losses[0] - 1.0, losses
