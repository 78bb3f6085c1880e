"""Communicator creation and the tensor-level all-reduce.

A communicator is created collectively by every rank: rank 0 draws a unique id
(a rendezvous path for the AF_UNIX bootstrap) and shares it through any
key-value store, typically the ``torch.distributed`` TCPStore of the job. The
tensor data never goes through the store or the bootstrap socket; it moves
over NVLink through the library's mailboxes.

Mirrors tiny-nccl's ``tncclGetUniqueId`` / ``tncclCommInitRank`` /
``tncclAllReduceSumF32`` / ``tncclCommDestroy`` (include/tnccl.h:25-51) with
dtype, pre-scale and algorithm choice added. Ranks on several hosts meet
through a TCP rendezvous (``bootstrap_addr``) and are linked by socket ring
edges (``TNCCL_NET``).
"""
from __future__ import annotations

import os
import socket

import torch

from .._native import load

ALGOS = ("auto", "ring", "oneshot", "twoshot", "nvls")


def _split_addr(addr: str) -> tuple[str, int]:
    host, sep, port = addr.rpartition(":")
    if not sep or not host or not port.isdigit() or not 0 < int(port) < 65536:
        raise ValueError(f"bootstrap address must be <ipv4>:<port>, got {addr!r}")
    return host, int(port)


def get_unique_id(bootstrap_addr: str | None = None) -> bytes:
    """128-byte rendezvous id (same role as tncclGetUniqueId).

    With ``bootstrap_addr="<ipv4>:<port>"`` the id names a TCP rendezvous
    where rank 0 listens at that address (ranks on several hosts,
    tncclGetUniqueIdTcp); otherwise an AF_UNIX path on this host.
    """
    if bootstrap_addr is None:
        return load().get_unique_id()
    host, port = _split_addr(bootstrap_addr)
    return load().get_unique_id_tcp(host, port)


def default_bootstrap_addr(env=None) -> str | None:
    """Rank 0's TCP rendezvous address for a job whose ranks span several
    hosts (torchrun's ``LOCAL_WORLD_SIZE < WORLD_SIZE``): ``MASTER_ADDR``
    resolved to IPv4 and ``MASTER_PORT + 1`` (``TNCCL_BOOTSTRAP_PORT``
    overrides the port). None when every rank is on one host, where the
    AF_UNIX rendezvous is used."""
    env = os.environ if env is None else env
    world = int(env.get("WORLD_SIZE", "1"))
    local = int(env.get("LOCAL_WORLD_SIZE", str(world)))
    if local >= world or "MASTER_ADDR" not in env:
        return None
    port = int(env.get("TNCCL_BOOTSTRAP_PORT", int(env.get("MASTER_PORT", "29500")) + 1))
    return f"{socket.gethostbyname(env['MASTER_ADDR'])}:{port}"


def empty_registrable(shape, dtype: torch.dtype, device=None) -> torch.Tensor:
    """An uninitialised tensor in ``tncclMemAlloc`` memory, which, unlike the
    caching allocator's ``cudaMalloc`` memory, :meth:`Communicator.register`
    can bind to an NVSwitch multicast object. The memory is rounded up to the
    multicast granularity (2 MiB or more) and freed with the tensor, which
    must be deregistered first (memory still registered is not freed)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None \
        else torch.device(device)
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    numel = 1
    for d in shape:
        numel *= int(d)
    es = torch.empty((), dtype=dtype).element_size()
    raw = load().mem_empty(max(numel * es, es), dev.index)
    return raw.view(dtype)[:numel].view(shape)


class Communicator:
    """One rank's handle on a tnccl communicator.

    Creation and :meth:`destroy` are blocking collectives. The communicator
    captures the current CUDA device at creation; the first collective binds it
    to the caller's current stream and later collectives must use that stream.
    """

    def __init__(self, unique_id: bytes, nranks: int, rank: int, device: int | None = None):
        if device is not None:
            torch.cuda.set_device(device)
        self._c = load().Communicator(unique_id, nranks, rank)
        self._side = None

    # -- properties -----------------------------------------------------------
    @property
    def rank(self) -> int:
        return self._c.rank

    @property
    def size(self) -> int:
        return self._c.size

    @property
    def device(self) -> torch.device:
        return torch.device("cuda", self._c.device)

    def info(self) -> dict:
        return self._c.info()

    def net_stats(self) -> dict:
        """Traffic of this rank's socket ring edges: frames and bytes each
        way, frames that took several socket calls, received frames that
        waited for the kernel's credit, and the proxy's failure code."""
        return self._c.net_stats()

    # -- collectives ----------------------------------------------------------
    def all_reduce(self, tensor: torch.Tensor, out: torch.Tensor | None = None, op: str = "sum",
                   scale: float = 1.0, algo: str = "auto") -> torch.Tensor:
        """out = sum over ranks of (scale * tensor) with fp32 accumulation.

        In place when ``out`` is None. ``op="avg"`` multiplies the pre-scale by
        1/nranks. Enqueued on the current CUDA stream; returns immediately.
        """
        return self._c.all_reduce(tensor, out, op, float(scale), algo)

    def all_reduce_ptr(self, send: int, recv: int, count: int, dtype: torch.dtype,
                       op: str = "sum", scale: float = 1.0, algo: str = "auto",
                       stream: int | None = None) -> None:
        """Pointer-level all-reduce for preallocated buffers."""
        code = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[dtype]
        if stream is None:
            stream = torch.cuda.current_stream(self.device).cuda_stream
        self._c.all_reduce_ptr(send, recv, count, code, op, float(scale), algo, stream)

    def register(self, tensor: torch.Tensor) -> int:
        """Collective: binds ``tensor`` (from :func:`empty_registrable`, the
        same size on every rank) to an NVSwitch multicast object of its own,
        so that an NVLS all-reduce on it reads and writes it in place instead
        of copying it through the communicator's region (on by default,
        ``TNCCL_NVLS_ZERO_COPY=0`` turns it off). Returns a handle for
        :meth:`deregister`."""
        return self._c.register(tensor)

    def deregister(self, handle: int) -> None:
        """Collective: waits for the bound stream and unbinds on every rank."""
        self._c.deregister(int(handle))

    def validate(self) -> int:
        """Waits for the bound stream and returns how many of this rank's
        mailbox guard lines were overwritten (0 = intact)."""
        return self._c.validate()

    def side_stream(self) -> torch.cuda.Stream:
        """A stream of this communicator's device, created once and shared by
        the components (DDP hooks, trainers) that enqueue on it; the
        communicator binds to the first stream a collective runs on."""
        if self._side is None:
            self._side = torch.cuda.Stream(device=self.device)
        return self._side

    def set_max_channels(self, max_channels: int) -> None:
        """Caps the CTAs of later collectives (0 restores the configured count);
        a collective that overlaps with compute leaves the other SMs to it."""
        self._c.set_max_channels(int(max_channels))

    def select_algo(self, numel: int, dtype: torch.dtype) -> str:
        return self._c.select_algo(numel, dtype)

    # -- failure handling -----------------------------------------------------
    def async_error(self) -> int:
        """0 when no device wait failed, else a tncclResult code (5: timeout)."""
        return self._c.async_error()

    def check(self) -> None:
        err = self._c.async_error()
        if err:
            raise RuntimeError(f"tnccl: {load().error_string(err)}")

    def abort(self) -> None:
        self._c.abort()

    def destroy(self) -> None:
        self._c.destroy()

    @property
    def alive(self) -> bool:
        return self._c.alive


_created = 0  # communicators created through a store by this process


def _store_key(key: str | None) -> str:
    """The store key of the next communicator: the caller's, or a default
    that changes with every communicator this process creates, so a later
    communicator never picks up an earlier id left in the store (every rank
    creates its communicators in the same order, so the keys agree)."""
    global _created
    _created += 1
    return key if key is not None else f"tnccl/uid/{_created}"


def init_from_store(store, rank: int, world_size: int, key: str | None = None,
                    device: int | None = None,
                    bootstrap_addr: str | None = None) -> Communicator:
    """Creates a communicator, sharing the unique id through ``store``
    (anything with ``set(key, bytes)`` and a blocking ``get(key)``).
    ``bootstrap_addr`` (rank 0's ``<ipv4>:<port>``) selects a TCP
    rendezvous, needed when the ranks span several hosts."""
    key = _store_key(key)
    if rank == 0:
        uid = get_unique_id(bootstrap_addr)
        store.set(key, uid)
    else:
        uid = bytes(store.get(key))
    return Communicator(uid, world_size, rank, device=device)


def init_from_torch_distributed(key: str | None = None, device: int | None = None,
                                bootstrap_addr: str | None = None) -> Communicator:
    """Creates a communicator over the ranks of the default process group.
    Across hosts the rendezvous is TCP at ``bootstrap_addr``, by default
    :func:`default_bootstrap_addr` (``MASTER_ADDR``, ``MASTER_PORT + 1``)."""
    import torch.distributed as dist

    if not dist.is_initialized():
        raise RuntimeError("torch.distributed is not initialized")
    store = dist.distributed_c10d._get_default_store()
    if bootstrap_addr is None and dist.get_rank() == 0:
        bootstrap_addr = default_bootstrap_addr()
    return init_from_store(store, dist.get_rank(), dist.get_world_size(), key=key, device=device,
                           bootstrap_addr=bootstrap_addr)
