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
             "tncclGetLaunchCount", "tncclGetUniqueIdTcp", "tncclCommGetNetStats",
             "tncclMemAlloc", "tncclMemFree", "tncclCommRegister", "tncclCommDeregister"]
    for n in names:
        assert hasattr(lib, n), n
    # Every function the public header declares is exported.
    import re
    with open(os.path.join(ROOT, "include", "tnccl.h")) as f:
        declared = set(re.findall(r"^\s*(?:[A-Za-z_][\w\s\*]*?)\b(tnccl[A-Z]\w*)\s*\(",
                                  f.read(), re.M))
    assert len(declared) >= 25
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing
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
    # Registered-buffer entry points: argument checks before any device work.
    ptr = ctypes.c_void_p()
    lib.tncclMemAlloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t]
    lib.tncclMemFree.argtypes = [ctypes.c_void_p]
    lib.tncclCommRegister.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                      ctypes.POINTER(ctypes.c_void_p)]
    lib.tncclCommDeregister.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    assert lib.tncclMemAlloc(None, 4096) == 1
    assert lib.tncclMemAlloc(ctypes.byref(ptr), 0) == 1
    assert lib.tncclMemFree(None) == 0
    assert lib.tncclMemFree(ctypes.c_void_p(0x1000)) == 1  # not from tncclMemAlloc
    assert lib.tncclCommRegister(None, ctypes.c_void_p(0x1000), 4096, ctypes.byref(ptr)) == 1
    assert lib.tncclCommDeregister(None, None) == 1
    if __import__("conftest").gpu_count() == 0:
        assert lib.tncclMemAlloc(ctypes.byref(ptr), 1 << 20) == 2  # no driver
    # TCP rendezvous ids: address and port are validated.
    lib.tncclGetUniqueIdTcp.argtypes = [ctypes.POINTER(Uid), ctypes.c_char_p, ctypes.c_int]
    tcp = Uid()
    assert lib.tncclGetUniqueIdTcp(ctypes.byref(tcp), b"127.0.0.1", 29500) == 0
    assert bytes(tcp.bytes[:8]) == b"TNCBT003"
    assert lib.tncclGetUniqueIdTcp(ctypes.byref(tcp), b"localhost", 29500) == 1
    assert lib.tncclGetUniqueIdTcp(ctypes.byref(tcp), b"127.0.0.1", 0) == 1


def test_registration_control_plane(built):
    # tncclMemAlloc / tncclCommRegister / tncclCommDeregister over forked
    # ranks, a real bootstrap and a fake driver with failures injected.
    r = run([os.path.join(ROOT, "build", "bin", "register_test")], timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "register_test: PASS" in r.stdout


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


def test_socket_ring_edges(built):
    """Socket data plane (TCP ring edges + proxy thread) on host threads:
    stream integrity under back-pressure, ring all-reduce over mixed NVLink /
    socket edges vs the ring oracle, and the host-made failure paths."""
    r = run([os.path.join(ROOT, "build", "bin", "net_proxy_test")], timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "net_proxy_test: PASS" in r.stdout


def test_socket_edge_loopback_throughput_mode(built):
    """The loopback throughput mode of the socket-edge test (full frames
    through both proxies) completes for every channel count and frame size."""
    r = run([os.path.join(ROOT, "build", "bin", "net_proxy_test"), "--bench", "64"], timeout=120)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    rates = [float(line.split(":")[-1].split()[0]) for line in r.stdout.splitlines()
             if line.startswith("socket edge loopback")]
    assert len(rates) == 9 and min(rates) > 0, r.stdout


def test_gemm_pipeline_model(built):
    """The mbarrier hand-offs of both tcgen05 GEMM kernels (stage ring,
    accumulator buffers, abort path) as threads with asynchronous TMA / MMA
    units, under random timing."""
    r = run([os.path.join(ROOT, "build", "bin", "gemm_pipeline_model_test")], timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "gemm_pipeline_model_test: PASS" in r.stdout


def test_ln_plan(built):
    """Launch geometry of the row-group LayerNorm backward (the header the
    launcher uses) for every C and a spread of row counts, its row walk and
    stage ring, and the parity-buffered warp sums with real threads."""
    r = run([os.path.join(ROOT, "build", "bin", "ln_plan_test")], timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "ln_plan_test:" in r.stdout and "PASS" in r.stdout


def test_config_and_partitions(built):
    r = run([os.path.join(ROOT, "build", "bin", "config_test")], timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "config_test: PASS" in r.stdout


@pytest.mark.skipif(__import__("conftest").gpu_count() > 0, reason="CPU-only behaviour")
def test_init_without_gpu_fails_cleanly(built):
    import tiny_nccl_b200 as tn
    with pytest.raises(RuntimeError, match="CUDA error"):
        tn.Communicator(tn.get_unique_id(), 1, 0)


def test_make_tuning_table(tmp_path):
    """benchmarks/make_tuning_table.py: fastest algorithm per size, merged
    into runs per rank count, last run unbounded."""
    import json
    import subprocess
    import sys
    recs = []
    for n, algo_bw in ((2, {1024: {"oneshot": 1.0, "twoshot": 0.5},
                            1 << 20: {"oneshot": 50.0, "twoshot": 40.0},
                            1 << 24: {"oneshot": 30.0, "twoshot": 300.0, "nccl": 400.0}}),
                       (8, {1024: {"oneshot": 1.0, "ring": 2.0}})):
        for size, d in algo_bw.items():
            for impl, bw in d.items():
                recs.append({"impl": impl, "n_gpus": n, "bytes": size, "busbw_gbs": bw})
    src = tmp_path / "sweep.jsonl"
    src.write_text("\n".join(json.dumps(r) for r in recs))
    out = tmp_path / "tuning.txt"
    r = subprocess.run([sys.executable, os.path.join(ROOT, "benchmarks", "make_tuning_table.py"),
                        str(src), "-o", str(out)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    lines = [l for l in out.read_text().splitlines() if not l.startswith("#")]
    assert lines == [f"2 {1 << 20} oneshot", f"2 {(1 << 64) - 1} twoshot",
                     f"8 {(1 << 64) - 1} ring"], lines


def test_bench_record_contract():
    """The JSON line of bench.py carries every key the benchmark contract
    names, with whole-job tokens/s derived from the device step time."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    e2e = {"value": 1.0, "unit": "tokens/s", "h2d_bytes_per_step": 65600, "d2h_bytes_per_step": 4}
    clocks = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []}
    rec = bench.make_record("tnccl", 8, 8, 1024, 20, 5, 16.0, clocks, 1234, e2e, 10.9)
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "clocks", "e2e", "gpu_launches"):
        assert key in rec, key
    for key in ("model", "global_batch", "seq_len", "parallelism"):
        assert key in rec["config"], key
    assert rec["value"] == 8 * 8 * 1024 / 16.0e-3
    assert rec["config"]["global_batch"] == 64 and rec["config"]["parallelism"] == "dp8"
    assert rec["scaling"] == "weak" and rec["higher_is_better"] is True
    assert rec["dtype"] == "bf16" and rec["gpu_launches"] == 1234


def test_clock_summary_parsing():
    """The clock record bench.py attaches: median SM clock under load, max
    clock, and every throttle reason seen while loaded."""
    from tiny_nccl_b200.utils.clocks import summarize
    na, act = "Not Active", "Active"
    rows = [
        f"0, 1965, 1965, 120.5, 0x0, {na}, {na}, {na}, {na}",   # idle, below the load cut
        f"0, 1965, 1965, 650.0, 0x0, {na}, {na}, {na}, {na}",
        f"0, 1800, 1965, 980.0, 0x4, {na}, {na}, {na}, {act}",
        f"0, 1700, 1965, 990.0, 0x4, {na}, {na}, {na}, {act}",
        "garbage line",
    ]
    s = summarize("\n".join(rows))
    assert s["sm_mhz"] == 1800 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"]
    assert s["samples"] == 4 and s["samples_under_load"] == 3 and s["power_w_max"] == 990.0
    assert summarize("")["available"] is False


def test_store_keys_change_per_communicator(monkeypatch):
    """init_from_store: a default key is new for every communicator, so a
    second communicator never reads the first one's id from the store."""
    from tiny_nccl_b200.parallel import comm as C

    made = []

    class FakeComm:
        def __init__(self, uid, nranks, rank, device=None):
            made.append((uid, nranks, rank))

    class Store(dict):
        def set(self, k, v):
            self[k] = v

        def get(self, k):
            return self[k]

    ids = iter([b"first", b"second"])
    monkeypatch.setattr(C, "Communicator", FakeComm)
    monkeypatch.setattr(C, "get_unique_id", lambda bootstrap_addr=None: next(ids))
    store = Store()
    C.init_from_store(store, 0, 2)
    C.init_from_store(store, 0, 2)
    assert len(store) == 2 and sorted(store.values()) == [b"first", b"second"]
    assert C._store_key("explicit") == "explicit"


def test_tcp_rendezvous_ids_and_default_address(built):
    import tiny_nccl_b200 as tn

    a, b = tn.get_unique_id("127.0.0.1:29500"), tn.get_unique_id("127.0.0.1:29500")
    assert len(a) == 128 and a[:8] == b"TNCBT003" and a != b  # fresh nonce each time
    assert tn.get_unique_id()[:8] == b"TNCBB002"  # AF_UNIX path id
    for bad in ("127.0.0.1", "127.0.0.1:0", ":29500", "127.0.0.1:x"):
        with pytest.raises(ValueError):
            tn.get_unique_id(bad)
    with pytest.raises(RuntimeError):
        tn.get_unique_id("not-an-ip:29500")
    one_host = {"WORLD_SIZE": "8", "LOCAL_WORLD_SIZE": "8", "MASTER_ADDR": "127.0.0.1",
                "MASTER_PORT": "29400"}
    assert tn.default_bootstrap_addr(one_host) is None
    two_hosts = dict(one_host, LOCAL_WORLD_SIZE="4")
    assert tn.default_bootstrap_addr(two_hosts) == "127.0.0.1:29401"
    assert tn.default_bootstrap_addr(dict(two_hosts, TNCCL_BOOTSTRAP_PORT="31000")) == \
        "127.0.0.1:31000"
    assert tn.default_bootstrap_addr({"WORLD_SIZE": "1"}) is None


def test_kernels_compile_with_device_checks(tmp_path):
    """The debug build (TNCCL_DEVICE_CHECKS=1: plan capacities and exact ring
    sequence numbers checked in the kernels) compiles for sm_100a."""
    import shutil

    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    if not os.path.exists(nvcc) and shutil.which("nvcc") is None:
        pytest.skip("needs nvcc")
    cmd = [nvcc if os.path.exists(nvcc) else "nvcc", "-gencode", "arch=compute_100a,code=sm_100a",
           "-O3", "-std=c++17", "--expt-relaxed-constexpr", "-diag-suppress", "177",
           "-DTNCCL_DEVICE_CHECKS=1", f"-I{ROOT}/include", f"-I{ROOT}/csrc/tnccl", "-c",
           os.path.join(ROOT, "csrc", "tnccl", "allreduce.cu"), "-o", str(tmp_path / "ar.o")]
    r = run(cmd, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]


def test_tcgen05_gemm_rejects_bad_arguments_before_device_work(built):
    """The tcgen05 GEMM launcher validates shapes and alignment on the host
    and returns 1 (invalid argument) without touching the device."""
    lib = ctypes.CDLL(os.path.join(ROOT, "tiny_nccl_b200", "lib", "libtnccl_ops.so"))
    f = lib.tnops_gemm_bias_act
    f.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 5 + [ctypes.c_void_p]
    f.restype = ctypes.c_int
    p = 1 << 20  # aligned address; never dereferenced on these paths
    cases = [
        (p, p, 0, p, p, 128, 256, 60, 1),     # K % 8 != 0
        (p, p, 0, p, p, 128, 250, 64, 1),     # N % 8 != 0
        (p + 8, p, 0, p, p, 128, 256, 64, 1),  # x not 16-byte aligned
        (p, p, 0, p, 0, 128, 256, 64, 1),     # GELU without an act output
        (p, p, 0, 0, p, 128, 256, 64, 0),     # no GELU and no pre output
        (p, p, 0, p, p, 0, 256, 64, 1),       # empty M
    ]
    for x, w, b, pre, act, M, N, K, gelu in cases:
        for persistent in (0, 1):
            assert f(x, w, b or None, pre or None, act or None, M, N, K, gelu, persistent,
                     None) == 1


def test_model_kernels_reject_misaligned_rows_before_device_work(built):
    """The LayerNorm and column-sum launchers move 8- and 16-byte pieces of
    each row; a base pointer off those boundaries is refused on the host
    (return 1) before any CUDA call, instead of faulting in the kernel."""
    lib = ctypes.CDLL(os.path.join(ROOT, "tiny_nccl_b200", "lib", "libtnccl_ops.so"))
    P, I = ctypes.c_void_p, ctypes.c_int
    p = 1 << 20  # aligned address; never dereferenced on these paths
    fwd = lib.tnops_ln_fwd
    fwd.argtypes = [P] * 8 + [I, I, ctypes.c_float, P]
    fwd.restype = I
    # x, delta, w, b, x_out, y, mean, rstd
    ok = [p, p, p, p, p, p, p, p]
    for i, off in [(0, 4), (2, 8), (3, 4), (4, 8), (1, 2), (5, 4)]:
        args = list(ok)
        args[i] += off
        assert fwd(*args, 16, 768, 1e-5, None) == 1, (i, off)
    bwd = lib.tnops_ln_bwd
    bwd.argtypes = [P] * 11 + [I, I, P]
    bwd.restype = I
    # gy, g_res, x_out, w, mean, rstd, dx, dx_bf16, dw, db, partial
    ok = [p] * 11
    for i, off in [(0, 4), (1, 8), (2, 4), (3, 8), (6, 4), (7, 2)]:
        args = list(ok)
        args[i] += off
        assert bwd(*args, 16, 768, None) == 1, (i, off)
    for name, nargs in (("tnops_bias_grad", 3), ("tnops_gelu_bwd_bias", 5)):
        f = getattr(lib, name)
        f.argtypes = [P] * nargs + [I, I, P]
        f.restype = I
        bf16_args = [0] if nargs == 3 else [0, 1, 2]
        for i in bf16_args:
            args = [p] * nargs
            args[i] += 8
            assert f(*args, 64, 768, None) == 1, (name, i)
        assert f(*([p] * nargs), 64, 770, None) == 1, name  # N % 8 != 0


def test_example_makes_tcp_ids_for_multi_host_runs(built):
    """examples/allreduce.cc --make-id prints a TCP rendezvous id as hex (no
    GPU needed); malformed multi-host arguments are usage errors."""
    exe = os.path.join(ROOT, "build", "bin", "tnccl_allreduce")
    r = run([exe, "--make-id", "127.0.0.1:29500"], timeout=60)
    assert r.returncode == 0, r.stderr
    hexid = r.stdout.strip()
    assert len(hexid) == 256 and bytes.fromhex(hexid)[:8] == b"TNCBT003"
    assert run([exe, "--make-id", "localhost:29500"], timeout=60).returncode == 2
    assert run([exe, "2", "10", "--ranks", "0:1", "--id", "zz"], timeout=60).returncode == 2
    assert run([exe, "2", "10", "--ranks", "1:2", "--id", hexid], timeout=60).returncode == 2


def test_environment_report(built):
    """python -m tiny_nccl_b200 reports versions, devices, the peer matrix and
    the TNCCL_* settings as JSON (no devices on a CPU-only host)."""
    import json
    import sys

    r = run([sys.executable, "-m", "tiny_nccl_b200"], timeout=120,
            env={"TNCCL_NET": "auto"})
    assert r.returncode == 0, r.stderr[-2000:]
    info = json.loads(r.stdout)
    assert info["tnccl_version"] >= 10000 and info["env"]["TNCCL_NET"] == "auto"
    assert isinstance(info["devices"], list) and isinstance(info["peers"], list)
    t = run([sys.executable, "-m", "tiny_nccl_b200", "--text"], timeout=120)
    assert t.returncode == 0 and "tnccl" in t.stdout


def test_trace_to_chrome_conversion(tmp_path):
    """benchmarks/trace_phases.py turns a phase-trace dump into a Chrome /
    Perfetto trace: team busy intervals as spans, other marks as instants."""
    import json
    import sys

    # Two channels of a two-shot trace: (globaltimer ns, phase, tile).
    raw = {"0": [[1000, 0, 0], [1500, 1, 0], [4000, 2, 0], [4500, 4, 0], [9000, 5, 0]],
           "3": [[1200, 0, 0], [2000, 1, 0], [5000, 2, 0]]}
    dump = tmp_path / "dump.rank0.json"
    dump.write_text(json.dumps(raw))
    out = tmp_path / "trace.json"
    r = run([sys.executable, os.path.join(ROOT, "benchmarks", "trace_phases.py"), "--convert",
             str(dump), "--algo", "twoshot", "--chrome", str(out)], timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    ev = json.loads(out.read_text())["traceEvents"]
    spans = [e for e in ev if e["ph"] == "X"]
    assert {(e["name"], e["tid"]) for e in spans} == {("reduce", 0), ("gather", 0), ("reduce", 3)}
    red0 = next(e for e in spans if e["name"] == "reduce" and e["tid"] == 0)
    assert abs(red0["ts"] - 0.5) < 1e-9 and abs(red0["dur"] - 2.5) < 1e-9
    assert any(e["ph"] == "i" and e["name"] == "pushed+published" for e in ev)


def test_empty_registrable_views(monkeypatch):
    """empty_registrable: the tncclMemAlloc bytes are viewed as the requested
    dtype and shape (stand-in allocator on the CPU, which records sizes)."""
    import torch

    from tiny_nccl_b200.parallel import comm as C

    asked = []

    class FakeNative:
        def mem_empty(self, nbytes, device):
            asked.append((nbytes, device))
            return torch.empty(nbytes, dtype=torch.uint8)

    monkeypatch.setattr(C, "load", lambda: FakeNative())
    t = C.empty_registrable((3, 5), torch.float32, "cpu")
    assert t.shape == (3, 5) and t.dtype == torch.float32 and asked[-1][0] == 60
    b = C.empty_registrable(7, torch.bfloat16, "cpu")
    assert b.shape == (7,) and b.dtype == torch.bfloat16 and asked[-1][0] == 14
    # Every view starts at the allocation's first byte (offset 0 is what
    # tncclCommRegister binds).
    assert b.untyped_storage().data_ptr() == b.data_ptr()
    z = C.empty_registrable(0, torch.float16, "cpu")
    assert z.numel() == 0 and asked[-1][0] == 2


def test_flat_reducer_launches_in_bucket_order():
    """FlatGradReducer launches bucket all-reduces strictly in bucket order
    (what keeps ranks' collectives in step) even when gradients complete out
    of order; offsets and bucket ends are 16-byte aligned; the .grad tensors
    are views of the flat buffer."""
    import torch

    from tiny_nccl_b200.parallel.reducer import FlatGradReducer

    params = [torch.nn.Parameter(torch.zeros(n)) for n in (5, 3, 9, 4, 7)]
    order = []
    red = FlatGradReducer(params, lambda t: order.append(t.data_ptr()), bucket_bytes=32)
    starts = [red.flat[s:e].data_ptr() for s, e in red.buckets]
    assert len(red.buckets) >= 3
    assert all(s % 4 == 0 and e % 4 == 0 for s, e in red.buckets)
    for p in params:
        assert red.flat.data_ptr() <= p.grad.data_ptr() < red.flat.data_ptr() + red.flat.numel() * 4
        assert (p.grad.data_ptr() - red.flat.data_ptr()) % 16 == 0
    # Complete the buckets back to front: nothing may launch before bucket 0.
    for b in reversed(range(1, len(red.buckets))):
        for p in red.bucket_params[b]:
            red._ready(p)
    assert order == []
    for p in red.bucket_params[0]:
        red._ready(p)
    assert order == starts
    red.finish()
    assert red.launched == len(red.buckets)
    # finish() launches what never completed, still in order, and re-arms.
    order.clear()
    red._ready(red.bucket_params[1][0])
    red.finish()
    assert order == starts
    red.remove()
