"""Multi-process tests. GPU ones need 2 GPUs (skipped otherwise); the store
exchange runs on CPU with gloo ranks."""

import pytest

from conftest import gpu_count, torchrun


@pytest.mark.skipif(gpu_count() > 0, reason="CPU-only behaviour")
def test_flat_reducer_matches_ddp_cpu_ranks():
    r = torchrun(2, ["tests/workers/flat_reducer_worker.py"], timeout=180)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.skipif(gpu_count() > 0, reason="CPU-only behaviour")
def test_store_exchange_cpu_ranks(built):
    r = torchrun(2, ["tests/workers/store_exchange_worker.py"], timeout=180)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.gpu
@pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")
def test_ddp_hook_matches_nccl_ddp(built):
    r = torchrun(2, ["tests/workers/ddp_hook_worker.py"], timeout=600)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.gpu
@pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")
def test_cuda_graph_capture_replay(built):
    r = torchrun(2, ["tests/workers/graph_capture_worker.py"], timeout=600)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.gpu
def test_trainer_checkpoint_resume(built):
    n = 2 if gpu_count() >= 2 else 1
    r = torchrun(n, ["tests/workers/checkpoint_worker.py"], timeout=600)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.gpu
@pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")
def test_mailbox_guard_lines(built):
    r = torchrun(2, ["tests/workers/canary_worker.py"], timeout=600)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.gpu
@pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")
def test_bounded_wait_timeout_two_ranks(built):
    env = {"TNCCL_TIMEOUT_MS": "1500", "TNCCL_NVLS_ENABLE": "0", "NCCL_NVLS_ENABLE": "0"}
    r = torchrun(2, ["tests/workers/timeout_worker.py"], timeout=300, env=env)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.gpu
@pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")
def test_graph_trainer_matches_ddp(built):
    """Flat gradient buffer + whole-step CUDA graph on 2 ranks against the
    eager DDP + tnccl hook trainer (NVLS off: the bucket all-reduces take the
    peer-memory kernels)."""
    r = torchrun(2, ["tests/workers/graph_trainer_worker.py"], timeout=600,
                 env={"TNCCL_TIMEOUT_MS": "10000", "TNCCL_NVLS_ENABLE": "0"})
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.gpu
@pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")
def test_nvls_zero_copy_registered_buffers(built):
    r = torchrun(2, ["tests/workers/nvls_zero_copy_worker.py"], timeout=600,
                 env={"TNCCL_NVLS_ZERO_COPY": "1", "TNCCL_DEBUG": "TRACE",
                      "TNCCL_TIMEOUT_MS": "5000"})
    out = r.stdout + r.stderr
    assert r.returncode == 0 and ("PASS" in r.stdout or "SKIP" in r.stdout), out[-4000:]
    if "PASS" in r.stdout:
        assert "(zero-copy)" in r.stderr, "the zero-copy kernel never ran"


@pytest.mark.gpu
@pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")
def test_flat_reducer_registered_buffer(built):
    r = torchrun(2, ["tests/workers/flat_trainer_worker.py"], timeout=600,
                 # 2 ranks: AUTO never picks the zero-copy kernel by itself
                 # (two-shot is faster there); a 1 MiB minimum makes every
                 # bucket take it, which is what this test is about.
                 env={"TNCCL_NVLS_ZERO_COPY": "1", "TNCCL_NVLS_ZC_MIN_BYTES": "1048576",
                      "TNCCL_TIMEOUT_MS": "10000"})
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
