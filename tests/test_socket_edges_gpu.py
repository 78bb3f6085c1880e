"""Socket ring edges (TNCCL_NET) on 2 GPUs: the ring kernel with host-mapped
FIFOs and the proxy thread, on one host with every edge forced onto sockets,
with every rank posing as its own host over a TCP rendezvous, and the
failure path of a rank that leaves between steps. The host side of the same
path is covered on CPU by tests/cpp/net_proxy_test.cc."""
import pytest

from conftest import gpu_count, torchrun

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs"),
]

_BASE = {"TNCCL_NVLS_ENABLE": "0", "NCCL_NVLS_ENABLE": "0", "TNCCL_TIMEOUT_MS": "20000"}


def test_every_edge_a_socket_edge(built):
    env = dict(_BASE, TNCCL_NET="force")
    r = torchrun(2, ["tests/workers/socket_edge_worker.py", "force"], timeout=600, env=env)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_ranks_as_separate_hosts_over_tcp(built):
    r = torchrun(2, ["tests/workers/socket_edge_worker.py", "hosts"], timeout=600, env=dict(_BASE))
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_rank_leaving_fails_the_socket_edge(built):
    env = dict(_BASE, TNCCL_NET="force", TNCCL_BOOTSTRAP_TIMEOUT_MS="3000")
    r = torchrun(2, ["tests/workers/socket_edge_worker.py", "fail"], timeout=300, env=env)
    assert "PASS" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
