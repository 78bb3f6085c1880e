"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device (B200); everything else runs on CPU.
Multi-GPU tests additionally skip when fewer GPUs are visible.
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU")


@pytest.fixture(scope="session")
def built():
    """Builds the native library, extension and C++ programs once per session."""
    from tiny_nccl_b200 import _build
    _build.build_all()
    return _build


def gpu_count() -> int:
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:  # noqa: BLE001
        return 0


def run(cmd, timeout=300, env=None):
    e = dict(os.environ)
    if env:
        e.update(env)
    return subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=timeout, env=e)


def free_port() -> int:
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def torchrun(nproc, script_args, timeout=600, env=None):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1",
           f"--master-port={free_port()}", *script_args]
    return run(cmd, timeout=timeout, env=env)
