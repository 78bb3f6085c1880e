"""tiny_nccl_b200: a B200-native collective library (tnccl) and its PyTorch layer.

* ``tiny_nccl_b200.parallel`` - communicators, all-reduce, the DDP comm hook.
* ``tiny_nccl_b200.ops``      - fused sm_100a model kernels.
* ``tiny_nccl_b200.models``   - GPT-2 built on those kernels.
* ``tiny_nccl_b200.utils``    - device timing and clock sampling.
"""
from ._native import library_path, load
from .parallel import (Communicator, TncclHookState, default_bootstrap_addr, get_unique_id,
                       init_from_store, init_from_torch_distributed, register_tnccl_hook,
                       tnccl_allreduce_hook)

__version__ = "1.0.0"


def launch_count() -> int:
    """Kernels launched by the collective library in this process."""
    return load().launch_count()


__all__ = [
    "Communicator", "default_bootstrap_addr", "get_unique_id", "init_from_store",
    "init_from_torch_distributed", "TncclHookState", "register_tnccl_hook", "tnccl_allreduce_hook", "launch_count", "load",
    "library_path", "__version__",
]
