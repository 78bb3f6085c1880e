"""Collective library on GPUs: single-rank path through the PyTorch layer,
multi-rank correctness (skipped with fewer than 2 GPUs), the C example."""
import os

import pytest
import torch

from conftest import ROOT, gpu_count, run

pytestmark = pytest.mark.gpu


def test_single_rank_paths(built):
    import tiny_nccl_b200 as tn
    comm = tn.Communicator(tn.get_unique_id(), 1, 0, device=0)
    x = torch.randn(1 << 20, device="cuda")
    y = torch.empty_like(x)
    n0 = tn.launch_count()
    comm.all_reduce(x, y)  # identity copy
    torch.testing.assert_close(y, x, atol=0, rtol=0)
    comm.all_reduce(x, y, scale=0.5)  # fused pre-scale kernel
    torch.testing.assert_close(y, x * 0.5, atol=0, rtol=0)
    xb = torch.randn(12345, device="cuda").to(torch.bfloat16)
    comm.all_reduce(xb, op="avg", scale=3.0)
    assert tn.launch_count() >= n0 + 2
    with pytest.raises(RuntimeError):
        comm.all_reduce(torch.randn(4))  # CPU tensor
    comm.destroy()


def test_example_single_gpu(built):
    r = run([os.path.join(ROOT, "build", "bin", "tnccl_allreduce"), "1", "1048576"], timeout=120)
    assert r.returncode == 0 and "all ranks: ok" in r.stdout, r.stdout + r.stderr


def test_example_registered_buffers(built):
    # One rank: tncclMemAlloc / tncclMemFree and a refused registration (no
    # NVLS); two or more: registered buffers on the zero-copy NVLS kernel.
    n = min(gpu_count(), 8)
    r = run([os.path.join(ROOT, "build", "bin", "tnccl_allreduce"), str(n), str(1 << 22)],
            timeout=300, env={"TNCCL_EXAMPLE_REGISTERED": "1", "TNCCL_NVLS_ZERO_COPY": "1",
                              "TNCCL_TIMEOUT_MS": "10000", "TNCCL_DEBUG": "TRACE"})
    assert r.returncode == 0 and "all ranks: ok" in r.stdout, r.stdout + r.stderr[-4000:]


@pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")
def test_two_rank_bit_exact(built):
    r = run([os.path.join(ROOT, "build", "bin", "allreduce_gpu_test"), "2", "quick"], timeout=600,
            env={"TNCCL_TIMEOUT_MS": "10000"})
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")
def test_two_rank_config2_stress(built):
    r = run([os.path.join(ROOT, "build", "bin", "allreduce_gpu_test"), "2", "stress"], timeout=600,
            env={"TNCCL_TIMEOUT_MS": "10000"})
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.skipif(gpu_count() < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("P", [4, 8])
def test_multi_rank_bit_exact(built, P):
    """Every algorithm on P ranks: counts 1 .. 1,048,581 across tile
    boundaries, fp32 / bf16 / fp16, in and out of place, averaging,
    misaligned buffers; ring, one-shot and two-shot bit for bit against the
    order-aware oracle; constant communication memory; guard lines intact."""
    if gpu_count() < P:
        pytest.skip(f"needs {P} GPUs")
    r = run([os.path.join(ROOT, "build", "bin", "allreduce_gpu_test"), str(P), "quick"],
            timeout=900, env={"TNCCL_TIMEOUT_MS": "10000"})
    assert r.returncode == 0, r.stdout + r.stderr[-4000:]


@pytest.mark.skipif(gpu_count() < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("P", [4, 8])
def test_multi_rank_stress(built, P):
    """100 consecutive checked all-reduces of 1,048,576 fp32 on one stream."""
    if gpu_count() < P:
        pytest.skip(f"needs {P} GPUs")
    r = run([os.path.join(ROOT, "build", "bin", "allreduce_gpu_test"), str(P), "stress"],
            timeout=900, env={"TNCCL_TIMEOUT_MS": "10000"})
    assert r.returncode == 0, r.stdout + r.stderr[-4000:]


@pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")
def test_nvls_summation_order_is_stable(built):
    """The switch's fp32 reduction on all visible GPUs (up to 8): five runs
    on the same inputs agree bit for bit; the printed study says which
    candidate summation order reproduces the result."""
    P = min(gpu_count(), 8)
    r = run([os.path.join(ROOT, "build", "bin", "allreduce_gpu_test"), str(P), "nvls_order"],
            timeout=600, env={"TNCCL_TIMEOUT_MS": "10000"})
    assert r.returncode == 0, r.stdout + r.stderr[-4000:]
    print(r.stdout)


def test_bounded_wait_self_test(built):
    """A device wait on a word nothing writes gives up after its bound and
    reports TNCCL_TIMEOUT; the communicator then refuses collectives."""
    import time

    import tiny_nccl_b200 as tn
    comm = tn.Communicator(tn.get_unique_id(), 1, 0, device=0)
    t0 = time.time()
    comm._c.diag_wait_timeout(300)
    torch.cuda.synchronize()
    assert 0.2 < time.time() - t0 < 20
    assert comm.async_error() == 5
    with pytest.raises(RuntimeError):
        comm.all_reduce(torch.ones(16, device="cuda"), scale=2.0)
    comm.destroy()
