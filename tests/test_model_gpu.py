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


def test_cuda_graph_step_matches_eager(built):
    """The trainer's CUDA-graph step (flat reducer, one rank) follows the
    same loss trajectory as the eager step from the same initialisation:
    three eager warm-up steps, then capture and replays whose optimizer step
    count advances on the device."""
    import datetime
    import os

    import torch.distributed as dist

    import tiny_nccl_b200 as tn
    from conftest import free_port
    from tiny_nccl_b200.models import GPT2, GPT2Config
    from tiny_nccl_b200.parallel import DataParallelTrainer

    own_group = not dist.is_initialized()
    if own_group:
        os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(free_port())})
        dist.init_process_group("nccl", rank=0, world_size=1,
                                device_id=torch.device("cuda", 0),
                                timeout=datetime.timedelta(seconds=60))
    cfg = GPT2Config(n_layer=2, n_head=4, n_embd=128, vocab_size=512, block_size=64)
    data = torch.randint(0, 64, (4, 65), device="cuda", generator=torch.Generator(
        device="cuda").manual_seed(5))
    runs = {}
    try:
        for graph in (False, True):
            comm = tn.init_from_torch_distributed(device=0)
            torch.manual_seed(0)
            model = GPT2(cfg, impl="fused").cuda()
            tr = DataParallelTrainer(model, comm, lr=3e-3, reducer="flat", cuda_graph=graph)
            losses = [tr.step(data[:, :-1], data[:, 1:]).item() for _ in range(8)]
            runs[graph] = (losses, [p.detach().clone() for p in model.parameters()])
            tr.close()  # releases the captured graph before the group goes away
            comm.destroy()
    finally:
        if own_group:
            dist.destroy_process_group()
    (le, pe), (lg, pg) = runs[False], runs[True]
    assert lg[-1] < lg[0] - 0.5, lg
    for a, b in zip(le, lg):
        assert abs(a - b) < 2e-2 * max(1.0, abs(a)), (le, lg)
    for a, b in zip(pe, pg):
        torch.testing.assert_close(a, b, rtol=2e-2, atol=2e-3)
