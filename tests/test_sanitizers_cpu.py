"""Host sanitizer runs (compute-sanitizer is closed on the GPU pool): the
threaded CPU rank model under ThreadSanitizer (data races in the flag
protocol model) and the bootstrap tests under AddressSanitizer +
UndefinedBehaviorSanitizer (memory errors in the socket control plane), the
socket proxy under both, the registered-buffer control plane under
AddressSanitizer + UndefinedBehaviorSanitizer, and the LayerNorm plan test
under both."""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

OUT = os.path.join(ROOT, "build", "sanitize")


def _build(name, srcs, flags):
    os.makedirs(OUT, exist_ok=True)
    exe = os.path.join(OUT, name)
    cmd = ["g++", "-std=c++17", "-O1", "-g", *flags, f"-I{ROOT}/include", f"-I{ROOT}/csrc/tnccl",
           f"-I{ROOT}/tests/cpp", "-I/usr/local/cuda/include", *srcs, "-o", exe, "-lpthread"]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    return exe


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_rank_model_under_tsan():
    exe = _build("rank_model_tsan", ["tests/cpp/rank_model_test.cc"], ["-fsanitize=thread"])
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1 second_deadlock_stack=1")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0 and "rank_model_test: PASS" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
    assert "WARNING: ThreadSanitizer" not in r.stderr, r.stderr[-4000:]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_bootstrap_under_asan_ubsan():
    exe = _build("bootstrap_asan", ["tests/cpp/bootstrap_test.cc", "csrc/tnccl/bootstrap.cc",
                                    "csrc/tnccl/common.cc", "csrc/tnccl/sockio.cc"],
                 ["-fsanitize=address,undefined", "-fno-omit-frame-pointer",
                  "-fno-sanitize-recover=undefined"])
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=1")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0 and "bootstrap_test: PASS" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]


_NET_SRCS = ["tests/cpp/net_proxy_test.cc", "csrc/tnccl/net.cc", "csrc/tnccl/sockio.cc",
             "csrc/tnccl/bootstrap.cc", "csrc/tnccl/common.cc"]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_socket_proxy_under_tsan():
    exe = _build("net_proxy_tsan", _NET_SRCS, ["-fsanitize=thread"])
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1 second_deadlock_stack=1")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0 and "net_proxy_test: PASS" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
    assert "WARNING: ThreadSanitizer" not in r.stderr, r.stderr[-4000:]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_socket_proxy_under_asan_ubsan():
    exe = _build("net_proxy_asan", _NET_SRCS,
                 ["-fsanitize=address,undefined", "-fno-omit-frame-pointer",
                  "-fno-sanitize-recover=undefined"])
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=1")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0 and "net_proxy_test: PASS" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_gemm_pipeline_model_under_tsan():
    exe = _build("gemm_pipeline_tsan", ["tests/cpp/gemm_pipeline_model_test.cc"],
                 ["-fsanitize=thread"])
    env = dict(os.environ, TSAN_OPTIONS="halt_on_error=1")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0 and "gemm_pipeline_model_test: PASS" in r.stdout, \
        r.stdout[-2000:] + r.stderr[-4000:]
    assert "WARNING: ThreadSanitizer" not in r.stderr, r.stderr[-4000:]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_registration_under_asan_ubsan():
    exe = _build("register_asan", ["tests/cpp/register_test.cc", "csrc/tnccl/register.cc",
                                   "csrc/tnccl/enqueue.cc", "csrc/tnccl/bootstrap.cc",
                                   "csrc/tnccl/common.cc", "csrc/tnccl/sockio.cc"],
                 ["-fsanitize=address,undefined", "-fno-omit-frame-pointer",
                  "-fno-sanitize-recover=undefined"])
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=1")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0 and "register_test: PASS" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_ln_plan_under_tsan_and_asan():
    """The LayerNorm plan test (its parity-slot check runs real threads)
    under ThreadSanitizer, and its host restatements under ASan / UBSan."""
    for name, flags, opts in (
            ("ln_plan_tsan", ["-fsanitize=thread"], ("TSAN_OPTIONS", "halt_on_error=1")),
            ("ln_plan_asan", ["-fsanitize=address,undefined", "-fno-omit-frame-pointer",
                              "-fno-sanitize-recover=undefined"],
             ("ASAN_OPTIONS", "detect_leaks=1:abort_on_error=1"))):
        exe = _build(name, ["tests/cpp/ln_plan_test.cc"], [*flags, f"-I{ROOT}/csrc/ops"])
        env = dict(os.environ, **{opts[0]: opts[1]})
        r = subprocess.run([exe], capture_output=True, text=True, timeout=600, env=env)
        assert r.returncode == 0 and "PASS" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
        assert "WARNING: ThreadSanitizer" not in r.stderr, r.stderr[-4000:]
