"""Fused sm_100a model kernels: residual-add + LayerNorm, softmax
cross-entropy, multi-tensor AdamW, and the bias / GELU-backward gradients
behind the autograd linears."""
from .fused import (add_layer_norm, bf16_weight, cross_entropy, launch_count, layer_norm,
                    linear, linear_gelu, linear_nobias)
from .optim import AdamW, gpt2_param_groups

__all__ = ["add_layer_norm", "layer_norm", "cross_entropy", "linear", "linear_gelu",
           "linear_nobias", "bf16_weight", "AdamW", "gpt2_param_groups", "launch_count"]
