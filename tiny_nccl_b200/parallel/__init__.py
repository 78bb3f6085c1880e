"""Parallelism layer: communicators, the DDP comm hook and the DP trainer."""
from .comm import (Communicator, default_bootstrap_addr, empty_registrable, get_unique_id,
                   init_from_store, init_from_torch_distributed)
from .ddp import TncclHookState, register_tnccl_hook, tnccl_allreduce_hook

__all__ = [
    "Communicator", "default_bootstrap_addr", "empty_registrable", "get_unique_id",
    "init_from_store",
    "init_from_torch_distributed", "TncclHookState", "register_tnccl_hook", "tnccl_allreduce_hook",
]
from .reducer import FlatGradReducer  # noqa: E402
from .trainer import DataParallelTrainer  # noqa: E402

__all__ += ["FlatGradReducer", "DataParallelTrainer"]
