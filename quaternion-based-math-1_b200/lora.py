"""LoRA residual over a frozen quaternion base, fused into the kernel.

Same module contract as the reference (``quaternion/lora.py:30-111``):
``LoRAQuaternionLinear(base, rank=8, alpha=None, dropout=0.0)`` with
``scale = alpha / rank`` (``alpha`` defaults to ``2 * rank``), ``lora_A
[rank, in]`` kaiming-uniform, ``lora_B [out, rank]`` zeros, the base frozen,
and ``forward = base(x) + scale * ((dropout(x) A^T) B^T)``.

Without dropout the whole expression (quaternion product, bias, LoRA) is one
device call: the kernel adds ``scale * (x A^T) B^T`` in fp32 before the single
output rounding.  With dropout active (training, ``p > 0``) the residual's
input differs from the base's, so the base runs fused with its bias and the
residual is added from the dropped-out input.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from .linear import QuaternionLinear, fused_quaternion_linear

__all__ = [
    "LoRAQuaternionLinear",
    "inject_lora",
    "lora_parameters",
    "mark_only_lora_trainable",
    "count_trainable",
]


class LoRAQuaternionLinear(nn.Module):
    """A ``QuaternionLinear`` whose weights stay fixed, with a learnable rank-r
    residual ``scale * B (A x)`` added on the same fused device call."""

    def __init__(self, base: QuaternionLinear, rank: int = 8, alpha: float | None = None,
                 dropout: float = 0.0):
        super().__init__()
        if rank <= 0:
            raise ValueError(f"LoRA rank must be at least 1, got {rank}")
        self.base = base
        for p in self.base.parameters():
            p.requires_grad_(False)
        self.in_features = base.in_features
        self.out_features = base.out_features
        self.rank = rank
        self.alpha = alpha if alpha is not None else 2 * rank
        self.scale = self.alpha / rank
        ref = next(base.parameters())
        self.lora_A = nn.Parameter(torch.empty(rank, self.in_features, device=ref.device,
                                               dtype=ref.dtype))
        self.lora_B = nn.Parameter(torch.zeros(self.out_features, rank, device=ref.device,
                                               dtype=ref.dtype))
        nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
        self.lora_dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()

    @property
    def bias(self):
        return self.base.bias

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b = self.base
        if isinstance(self.lora_dropout, nn.Dropout) and self.training:
            out = fused_quaternion_linear(x, b.wr, b.wi, b.wj, b.wk, b.bias)
            lora = (self.lora_dropout(x) @ self.lora_A.t()) @ self.lora_B.t()
            return out + self.scale * lora
        return fused_quaternion_linear(x, b.wr, b.wi, b.wj, b.wk, b.bias, self.lora_A, self.lora_B,
                                       self.scale, static_weights=b.static_weights,
                                       packed=b._packed_for_call(x, self.lora_A, self.lora_B))

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"rank={self.rank}, alpha={self.alpha}, base=frozen")


def inject_lora(model: nn.Module, rank: int = 8, alpha: float | None = None, dropout: float = 0.0):
    """Wrap every ``QuaternionLinear`` of ``model`` in place; return the wrapped names."""
    targets = [(n, m) for n, m in model.named_modules() if isinstance(m, QuaternionLinear)]
    wrapped = []
    for name, mod in targets:
        parent_name, _, leaf = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, leaf, LoRAQuaternionLinear(mod, rank=rank, alpha=alpha, dropout=dropout))
        wrapped.append(name)
    return wrapped


def lora_parameters(model: nn.Module):
    """Yield ``(name, parameter)`` for the LoRA parameters only."""
    for name, p in model.named_parameters():
        if "lora_" in name:
            yield name, p


def mark_only_lora_trainable(model: nn.Module) -> None:
    for name, p in model.named_parameters():
        p.requires_grad_("lora_" in name)


def count_trainable(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters() if p.requires_grad)
