"""CPU tests of the native layer: build, C ABI surface, bootstrap control
plane (fork-based ranks) and the threaded CPU model of the device protocols."""
import ctypes
import os

import pytest

from conftest import ROOT, run


def test_build_and_import(built):
    import tiny_nccl_b200 as tn
    assert tn.load().version() == 10000
    assert len(tn.get_unique_id()) == 128
    assert os.path.exists(tn.library_path())


def test_c_abi_surface(built):
    lib = ctypes.CDLL(os.path.join(ROOT, "tiny_nccl_b200", "lib", "libtnccl.so"))
    names = ["tncclGetUniqueId", "tncclCommInitRank", "tncclAllReduceSumF32", "tncclCommDestroy",
             "tncclGetErrorString", "tncclAllReduce", "tncclAllReduceEx", "tncclCommGetInfo",
             "tncclCommGetAsyncError", "tncclCommAbort", "tncclCommSelectAlgo", "tncclGetVersion",
             "tncclGetLaunchCount"]
    for n in names:
        assert hasattr(lib, n), n
    lib.tncclGetErrorString.restype = ctypes.c_char_p
    # Values of the tiny-nccl result codes are kept; new codes are appended.
    assert lib.tncclGetErrorString(0) == b"success"
    assert lib.tncclGetErrorString(1) == b"invalid argument"
    assert lib.tncclGetErrorString(2) == b"unsupported configuration"
    assert lib.tncclGetErrorString(3) == b"system error"
    assert lib.tncclGetErrorString(4) == b"CUDA error"
    assert lib.tncclGetErrorString(5) == b"timed out waiting for a peer"
    # Argument validation before any device work.
    comm = ctypes.c_void_p()
    class Uid(ctypes.Structure):
        _fields_ = [("bytes", ctypes.c_ubyte * 128)]
    lib.tncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, Uid,
                                      ctypes.c_int]
    uid = Uid()
    assert lib.tncclCommInitRank(ctypes.byref(comm), 0, uid, 0) == 1
    assert lib.tncclCommInitRank(ctypes.byref(comm), 2, uid, 2) == 1
    assert lib.tncclCommInitRank(None, 2, uid, 0) == 1
    assert lib.tncclCommDestroy(None) == 1
    assert lib.tncclAllReduceSumF32(None, None, 0, None, None) == 1
    assert lib.tncclGetUniqueId(None) == 1


def test_bootstrap_forked_ranks(built):
    r = run([os.path.join(ROOT, "build", "bin", "bootstrap_test")], timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "bootstrap_test: PASS" in r.stdout


def test_rank_model(built):
    r = run([os.path.join(ROOT, "build", "bin", "rank_model_test")], timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "rank_model_test: PASS" in r.stdout
    for line in ("config1 P=4 8x64KiB ring fp32", "reference matrix (twoshot",
                 "dropped flag -> bounded timeout (ring)"):
        assert line in r.stdout


def test_config_and_partitions(built):
    r = run([os.path.join(ROOT, "build", "bin", "config_test")], timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "config_test: PASS" in r.stdout


@pytest.mark.skipif(__import__("conftest").gpu_count() > 0, reason="CPU-only behaviour")
def test_init_without_gpu_fails_cleanly(built):
    import tiny_nccl_b200 as tn
    with pytest.raises(RuntimeError, match="CUDA error"):
        tn.Communicator(tn.get_unique_id(), 1, 0)
