"""Multi-rank all-reduce kernels on ONE GPU: emulated ranks run as one
cooperative launch (tncclEmu*), so the ring / one-shot / two-shot device code
is exercised with 2, 4 and 8 ranks even when a single GPU is available.
Results are compared bit for bit with an order-aware fp32 oracle: rank order
0..P-1 for one-shot/two-shot, the ring's s+1 ... s rotation (rounded to the
wire type at every hop) for the ring.

The last test runs this module again in a child process on the build with the
kernels' debug protocol checks (lib/checked/libtnccl.so, preloaded): every
launch checks its plan against the mailbox capacities and the ring checks
each sequence number it waits for, so a protocol slip fails a test instead of
passing silently."""
import os
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(autouse=True)
def _expected_build():
    """In the child process of the device-checks test, the debug build must
    really be the one loaded."""
    if os.environ.get("TNCCL_EXPECT_DEVICE_CHECKS") == "1":
        import tiny_nccl_b200 as tn
        assert tn.load().device_checks() == 1

CHANNELS = 8  # small enough that channels x ranks CTAs are co-resident
RING_CHUNK = 256 << 10
RING_MIN_CHUNK = 4096


def _div_up(a, b):
    return (a + b - 1) // b


def _round_up(a, b):
    return _div_up(a, b) * b


def ring_chunk_index(count, P, es, channels=CHANNELS):
    """Chunk (segment) owning each element under the ring's chunk plan
    (protocol.h makeChunkPlan / chunkSpan)."""
    V = 16 // es
    want = _round_up(_div_up(count, P * channels), V)
    want = max(want, RING_MIN_CHUNK // es)
    want = min(want, RING_CHUNK // es)
    tile_elems = want * P
    e = torch.arange(count, device="cuda", dtype=torch.int64)
    tile = e // tile_elems
    off = e - tile * tile_elems
    base = tile * tile_elems
    length = torch.clamp(count - base, max=tile_elems)
    partial = _round_up_t(_div_up_t(length, P), V)
    cl = torch.where(length == tile_elems, torch.full_like(length, want), partial)
    return torch.clamp(off // cl, max=P - 1)


def _div_up_t(a, b):
    return (a + b - 1) // b


def _round_up_t(a, b):
    return _div_up_t(a, b) * b


def oracle(xs, algo, alpha, dtype, channels=CHANNELS):
    P = len(xs)
    f = [x.float() for x in xs]
    a = torch.tensor(alpha, dtype=torch.float32, device="cuda")
    if algo in ("oneshot", "twoshot"):
        acc = f[0] * a
        for k in range(1, P):
            acc = acc + f[k] * a
        return acc.to(dtype)
    es = xs[0].element_size()
    j = ring_chunk_index(xs[0].numel(), P, es, channels)
    stack = torch.stack(f)  # [P, n]
    cols = torch.arange(xs[0].numel(), device="cuda")
    acc = (stack[(j + 1) % P, cols] * a).to(dtype).float()
    for k in range(2, P + 1):
        acc = (acc + stack[(j + k) % P, cols] * a).to(dtype).float()
    return acc.to(dtype)


@pytest.fixture(scope="module")
def emulators(built):
    os.environ["TNCCL_NCHANNELS"] = str(CHANNELS)
    os.environ["TNCCL_ONESHOT_CHANNELS"] = str(CHANNELS)
    import tiny_nccl_b200 as tn
    emus = {P: tn.load().Emulator(P) for P in (2, 4, 8)}
    yield emus
    for e in emus.values():
        e.destroy()


@pytest.mark.parametrize("P", [2, 4, 8])
@pytest.mark.parametrize("algo", ["oneshot", "twoshot", "ring"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_emulated_bit_exact(emulators, P, algo, dtype):
    emu = emulators[P]
    g = torch.Generator(device="cuda")
    for count, op in ((1, "sum"), (4097, "sum"), (300_001, "avg"), (2_500_000, "sum")):
        g.manual_seed(count + P)
        xs = [(torch.rand(count, device="cuda", generator=g) * 2 - 1).to(dtype) for _ in range(P)]
        ys = [torch.full_like(x, float("nan")) for x in xs]
        emu.all_reduce(xs, ys, op=op, algo=algo)
        torch.cuda.synchronize()
        assert emu.async_error() == 0
        want = oracle(xs, algo, (1.0 / P) if op == "avg" else 1.0, dtype)
        for r, y in enumerate(ys):
            bad = (y.float() != want.float()).nonzero()
            assert bad.numel() == 0, (algo, P, count, r, bad[:5].flatten().tolist())


def test_emulated_in_place_and_sequence(emulators):
    """In-place operation and 50 consecutive collectives of varying size on
    the same mailboxes (device-resident sequence numbers)."""
    emu = emulators[4]
    for it in range(50):
        n = 1 + (it * 7919) % 200_000
        algo = ("oneshot", "twoshot", "ring")[it % 3]
        xs = [torch.full((n,), float(r + it), device="cuda") for r in range(4)]
        emu.all_reduce(xs, xs, algo=algo)
        torch.cuda.synchronize()
        want = float(sum(r + it for r in range(4)))
        for x in xs:
            assert bool(torch.all(x == want)), (it, algo)
    assert emu.async_error() == 0


@pytest.mark.parametrize("P", [2, 4, 8])
@pytest.mark.parametrize("stage_min", [0, 1 << 30])
def test_emulated_twoshot_staging_paths(built, P, stage_min):
    """Two-shot with every copy staged through shared memory by TMA
    (TNCCL_STAGE_MIN_BYTES=0, opt-in) and with none staged (the default),
    bit for bit against the oracle."""
    import tiny_nccl_b200 as tn
    old = os.environ.get("TNCCL_STAGE_MIN_BYTES")
    os.environ["TNCCL_STAGE_MIN_BYTES"] = str(stage_min)
    os.environ["TNCCL_NCHANNELS"] = str(CHANNELS)
    try:
        emu = tn.load().Emulator(P)
    finally:
        if old is None:
            del os.environ["TNCCL_STAGE_MIN_BYTES"]
        else:
            os.environ["TNCCL_STAGE_MIN_BYTES"] = old
    try:
        g = torch.Generator(device="cuda")
        for count in (4097, 1_000_003, 3_000_000):
            for dtype in (torch.float32, torch.bfloat16):
                g.manual_seed(count + P)
                xs = [(torch.rand(count, device="cuda", generator=g) * 2 - 1).to(dtype)
                      for _ in range(P)]
                ys = [torch.empty_like(x) for x in xs]
                emu.all_reduce(xs, ys, algo="twoshot")
                torch.cuda.synchronize()
                assert emu.async_error() == 0
                want = oracle(xs, "twoshot", 1.0, dtype)
                for y in ys:
                    assert bool(torch.equal(y, want)), (P, stage_min, count, dtype)
    finally:
        emu.destroy()


@pytest.mark.parametrize("P,hosts", [(2, None), (4, None), (4, "0,0,1,1"), (8, "0,0,0,1,1,2,2,2")])
def test_emulated_socket_ring(built, P, hosts):
    """The ring over socket edges on one GPU: emulated ranks joined by
    host-mapped FIFOs, in-process proxy threads and loopback TCP (every edge
    with TNCCL_NET=force; with TNCCL_EMU_HOSTS only the edges between
    different host ids, the others over mailboxes), 2 channels, bit for bit
    against the ring oracle, then 30 collectives in a row on the same FIFOs."""
    import tiny_nccl_b200 as tn
    env = {"TNCCL_NET_CHANNELS": "2", "TNCCL_NCHANNELS": str(CHANNELS)}
    if hosts is None:
        env["TNCCL_NET"] = "force"
    else:
        env["TNCCL_EMU_HOSTS"] = hosts
    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        emu = tn.load().Emulator(P)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    try:
        g = torch.Generator(device="cuda")
        for count in (1, 4097, 1_000_003):
            for dtype in (torch.float32, torch.bfloat16):
                g.manual_seed(count + P)
                xs = [(torch.rand(count, device="cuda", generator=g) * 2 - 1).to(dtype)
                      for _ in range(P)]
                ys = [torch.full_like(x, float("nan")) for x in xs]
                emu.all_reduce(xs, ys, algo="ring")
                torch.cuda.synchronize()
                assert emu.async_error() == 0
                want = oracle(xs, "ring", 1.0, dtype, channels=2)
                for y in ys:
                    assert bool(torch.equal(y, want)), (P, count, dtype)
        for it in range(30):
            n = 1 + (it * 7919) % 100_000
            xs = [torch.full((n,), float(r + it), device="cuda") for r in range(P)]
            emu.all_reduce(xs, xs, algo="ring")
            torch.cuda.synchronize()
            want = float(sum(r + it for r in range(P)))
            assert all(bool(torch.all(x == want)) for x in xs), it
        assert emu.async_error() == 0
    finally:
        emu.destroy()


@pytest.mark.skipif(os.environ.get("TNCCL_EXPECT_DEVICE_CHECKS") == "1",
                    reason="already inside the device-checks run")
def test_emulated_suite_with_device_checks(built):
    """Every other test of this module, on the debug build of the library."""
    from conftest import run
    lib = os.path.join(ROOT, "tiny_nccl_b200", "lib", "checked", "libtnccl.so")
    assert os.path.exists(lib), "build_all() builds lib/checked/libtnccl.so"
    env = {"LD_PRELOAD": lib, "TNCCL_EXPECT_DEVICE_CHECKS": "1"}
    r = run([sys.executable, "-m", "pytest", "tests/test_emulated_gpu.py", "-q", "-x", "-m", "gpu",
             "-p", "no:cacheprovider"], timeout=1200, env=env)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    assert " passed" in r.stdout and " failed" not in r.stdout, r.stdout[-2000:]
