"""Fused sm_100a model kernels (LayerNorm, cross-entropy, AdamW) and the
functional all-reduce."""
from .fused import (add_layer_norm, cross_entropy, launch_count, layer_norm, linear,
                    linear_gelu)
from .optim import AdamW, gpt2_param_groups

__all__ = ["add_layer_norm", "layer_norm", "cross_entropy", "linear", "linear_gelu", "AdamW",
           "gpt2_param_groups", "launch_count"]
