"""GPT-2 (124M "small" by default) for data-parallel training benchmarks.

Architecture of GPT-2 small: 12 layers, d_model 768, 12 heads, vocabulary
50257, context 1024, pre-LayerNorm blocks, tanh-GELU MLP with 4x expansion,
learned positional embeddings, LM head tied to the token embedding.

Two implementations share one parameter layout:

* ``impl="fused"`` (training on B200): LayerNorm, bias+GELU, residual adds and
  the softmax cross-entropy (forward and backward) run as hand-written sm_100a
  kernels from ``tiny_nccl_b200.ops``; GEMMs use cuBLAS through
  ``torch.nn.functional.linear`` and attention uses
  ``scaled_dot_product_attention`` (flash attention), all in bf16.
* ``impl="torch"``: the same math in stock PyTorch ops; it is the fp32
  numerics reference for the fused kernels and the path the CPU tests use.

The reference (tiny-nccl) has no model; this is the workload of the
"GPT-2 small DP tokens/s" headline metric.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class GPT2Config:
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768
    vocab_size: int = 50257
    block_size: int = 1024
    # Rows of the token-embedding / LM-head matrix are padded to a multiple of
    # this, so the LM-head GEMMs (N = vocabulary) run on aligned tensor-core
    # kernels; padded rows are never looked up and padded logits are excluded
    # from the softmax, so the model computes exactly the same function.
    vocab_multiple: int = 128

    @property
    def vocab_padded(self) -> int:
        m = self.vocab_multiple
        return (self.vocab_size + m - 1) // m * m

    @property
    def n_params(self) -> int:
        """Parameters of the model (padding rows of the embedding excluded)."""
        d, v, L, t = self.n_embd, self.vocab_size, self.n_layer, self.block_size
        per_layer = 12 * d * d + 13 * d
        return v * d + t * d + L * per_layer + 2 * d

    def flops_per_token(self, seq: int) -> float:
        """Training FLOPs per token (forward + backward, dense matmuls and
        attention scores), 6N + 12 L d T."""
        n_matmul = 12 * self.n_layer * self.n_embd ** 2 + self.vocab_size * self.n_embd
        return 6.0 * n_matmul + 12.0 * self.n_layer * self.n_embd * seq


class Block(nn.Module):
    def __init__(self, cfg: GPT2Config):
        super().__init__()
        d = cfg.n_embd
        self.n_head = cfg.n_head
        self.ln_1 = nn.LayerNorm(d)
        self.attn_qkv = nn.Linear(d, 3 * d)
        self.attn_proj = nn.Linear(d, d)
        self.ln_2 = nn.LayerNorm(d)
        self.mlp_fc = nn.Linear(d, 4 * d)
        self.mlp_proj = nn.Linear(4 * d, d)

    def attention(self, h: torch.Tensor, ops=None) -> torch.Tensor:
        B, T, C = h.shape
        qkv = ops.linear(h, self.attn_qkv.weight, self.attn_qkv.bias) if ops else self.attn_qkv(h)
        q, k, v = qkv.split(C, dim=2)
        hd = C // self.n_head
        q = q.view(B, T, self.n_head, hd).transpose(1, 2)
        k = k.view(B, T, self.n_head, hd).transpose(1, 2)
        v = v.view(B, T, self.n_head, hd).transpose(1, 2)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        y = y.transpose(1, 2).contiguous().view(B, T, C)
        if ops:
            return ops.linear(y, self.attn_proj.weight, self.attn_proj.bias)
        return self.attn_proj(y)

    def forward_torch(self, x: torch.Tensor) -> torch.Tensor:
        x = x + self.attention(self.ln_1(x))
        h = F.gelu(self.mlp_fc(self.ln_2(x)), approximate="tanh")
        return x + self.mlp_proj(h)

    def mlp_fused(self, h: torch.Tensor, ops) -> torch.Tensor:
        g = ops.linear_gelu(h, self.mlp_fc.weight, self.mlp_fc.bias)
        return ops.linear(g, self.mlp_proj.weight, self.mlp_proj.bias)


class GPT2(nn.Module):
    def __init__(self, cfg: GPT2Config | None = None, impl: str = "fused"):
        super().__init__()
        self.cfg = cfg or GPT2Config()
        if impl not in ("fused", "torch"):
            raise ValueError(f"unknown impl {impl!r}")
        self.impl = impl
        c = self.cfg
        self.wte = nn.Embedding(c.vocab_padded, c.n_embd)
        self.wpe = nn.Embedding(c.block_size, c.n_embd)
        self.blocks = nn.ModuleList([Block(c) for _ in range(c.n_layer)])
        self.ln_f = nn.LayerNorm(c.n_embd)
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self, seed: int | None = None) -> None:
        """GPT-2 initialisation: N(0, 0.02), residual projections scaled by
        1/sqrt(2 L), zero biases, unit LayerNorm gains."""
        g = None
        if seed is not None:
            g = torch.Generator(device=self.wte.weight.device)
            g.manual_seed(seed)
        std = 0.02
        proj_std = std / math.sqrt(2 * self.cfg.n_layer)
        for name, p in self.named_parameters():
            if name.endswith("bias"):
                p.zero_()
            elif ".ln_" in name or name.startswith("ln_"):
                p.fill_(1.0)
            elif name.endswith("attn_proj.weight") or name.endswith("mlp_proj.weight"):
                p.normal_(0.0, proj_std, generator=g)
            else:
                p.normal_(0.0, std, generator=g)
        self.wte.weight[self.cfg.vocab_size:].zero_()  # padding rows

    def _ops(self):
        from .. import ops
        return ops

    def forward(self, idx: torch.Tensor, targets: torch.Tensor | None = None):
        """Returns the mean cross-entropy loss when targets are given, else the
        logits of the last position."""
        B, T = idx.shape
        pos = torch.arange(T, device=idx.device)
        x = self.wte(idx) + self.wpe(pos)  # fp32 residual stream
        if self.impl == "fused":
            return self._forward_fused(x, targets)
        for blk in self.blocks:
            x = blk.forward_torch(x)
        x = self.ln_f(x)
        if targets is None:
            return F.linear(x[:, -1], self.wte.weight)[..., :self.cfg.vocab_size]
        logits = F.linear(x, self.wte.weight)
        V = self.cfg.vocab_size
        return F.cross_entropy(logits.view(B * T, -1)[:, :V].float(), targets.reshape(-1))

    def _forward_fused(self, x: torch.Tensor, targets: torch.Tensor | None):
        """Residual stream kept in fp32; every residual add is fused with the
        LayerNorm that follows it; sub-layer outputs are bf16 (autocast)."""
        ops = self._ops()
        B, T, C = x.shape
        x = x.reshape(B * T, C)
        first = self.blocks[0].ln_1
        h = ops.layer_norm(x, first.weight, first.bias)
        L = len(self.blocks)
        for i, blk in enumerate(self.blocks):
            a = blk.attention(h.view(B, T, C), ops)
            x, h = ops.add_layer_norm(x, a.reshape(B * T, C), blk.ln_2.weight, blk.ln_2.bias)
            m = blk.mlp_fused(h, ops)
            nxt = self.blocks[i + 1].ln_1 if i + 1 < L else self.ln_f
            x, h = ops.add_layer_norm(x, m, nxt.weight, nxt.bias)
        if targets is None:
            last = h.view(B, T, C)[:, -1]
            return ops.linear_nobias(last, self.wte.weight)[..., :self.cfg.vocab_size]
        logits = ops.linear_nobias(h, self.wte.weight)
        return ops.cross_entropy(logits, targets.reshape(-1), classes=self.cfg.vocab_size)
