"""Converting a model's dense projections to quaternion layers.

The caller that puts the quaternion kernels under a whole model: the
reference's ``matrix`` conversion (``conversion/convert_model.py:239-299``
with ``_build_layer``, ``:69-80``) replaces each eligible projection with a
:class:`QuaternionLinear` whose components are the closed-form least-squares
projection of the dense weight onto the quaternion block structure
(``conversion/fit_linear.py:35-61``), bias copied.  Eligible projections
follow ``conversion/model_utils.py:37-90`` and ``convert_model.py:58-69``:
``nn.Linear`` or GPT-2 ``Conv1D`` modules named ``q/k/v/o/gate/up/down_proj``,
``c_attn`` (kept whole), ``c_fc`` or ``c_proj``, both dimensions divisible by
4, never the LM head.

The reference's ``activation`` method (activation-aware fitting on a
calibration corpus) is not provided: it is calibration and optimisation
machinery, not part of the layer's forward.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn as nn

from .linear import QuaternionLinear
from .packing import build_block_matrix, check_divisible

__all__ = ["ConversionRecord", "project_onto_quaternion", "module_weight_out_in", "eligible_modules",
           "convert_model"]

_NAMED_PROJECTIONS = {"q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"}


@dataclass
class ConversionRecord:
    name: str
    in_features: int
    out_features: int
    kind: str
    method: str
    metrics: dict = field(default_factory=dict)


def project_onto_quaternion(weight: torch.Tensor):
    """``(wr, wi, wj, wk)`` minimising ``||Block(wr, wi, wj, wk) - weight||_F``.

    Each component is the signed mean of the four entries of every 4x4 block
    that the block structure assigns to it (reference
    ``conversion/fit_linear.py:35-61``); computed in float64.
    """
    if weight.dim() != 2:
        raise ValueError("weight must be 2D [out, in]")
    check_divisible(weight.shape[0], "out_features")
    check_divisible(weight.shape[1], "in_features")
    w = weight.double()
    blk = lambda a, q: w[a::4, q::4]  # entry (a, q) of every 4x4 block
    wr = (blk(0, 0) + blk(1, 1) + blk(2, 2) + blk(3, 3)) / 4
    wi = (blk(1, 0) - blk(0, 1) + blk(3, 2) - blk(2, 3)) / 4
    wj = (blk(2, 0) - blk(0, 2) + blk(1, 3) - blk(3, 1)) / 4
    wk = (blk(3, 0) - blk(0, 3) + blk(2, 1) - blk(1, 2)) / 4
    return wr, wi, wj, wk


def _is_linear_like(mod: nn.Module) -> bool:
    if isinstance(mod, nn.Linear):
        return True
    return type(mod).__name__ == "Conv1D" and hasattr(mod, "weight") and mod.weight.dim() == 2


def module_weight_out_in(mod: nn.Module) -> torch.Tensor:
    """The ``[out, in]`` weight of an ``nn.Linear`` or a GPT-2 ``Conv1D``
    (which stores ``[in, out]``)."""
    w = mod.weight.detach()
    return w if isinstance(mod, nn.Linear) else w.t()


def eligible_modules(model: nn.Module) -> list[tuple[str, nn.Module]]:
    """``(name, module)`` of every projection the conversion replaces, each module once."""
    out, seen = [], set()
    for name, mod in model.named_modules():
        if not _is_linear_like(mod) or name.endswith("lm_head") or ".lm_head" in name:
            continue
        leaf = name.rsplit(".", 1)[-1]
        if leaf not in _NAMED_PROJECTIONS and leaf not in ("c_attn", "c_fc", "c_proj"):
            continue
        w = module_weight_out_in(mod)
        if w.shape[0] % 4 or w.shape[1] % 4 or id(mod) in seen:
            continue
        seen.add(id(mod))
        out.append((name, mod))
    return out


def _kind(name: str) -> str:
    leaf = name.rsplit(".", 1)[-1]
    if leaf in _NAMED_PROJECTIONS:
        return leaf
    if leaf == "c_attn":
        return "qkv_proj"
    if leaf == "c_fc":
        return "up_proj"
    return "o_proj" if ".attn." in f".{name}." else "down_proj"


def _build_layer(module: nn.Module, wr, wi, wj, wk, bias) -> QuaternionLinear:
    w = module_weight_out_in(module)
    out_features, in_features = w.shape
    layer = QuaternionLinear(in_features, out_features, bias=bias is not None, device=w.device, dtype=w.dtype)
    with torch.no_grad():
        for dst, src in zip((layer.wr, layer.wi, layer.wj, layer.wk), (wr, wi, wj, wk)):
            dst.copy_(src.to(dst.dtype))
        if bias is not None:
            layer.bias.copy_(bias.to(layer.bias.dtype))
    return layer


def convert_model(model: nn.Module, method: str = "matrix", verbose: bool = False):
    """Replace the eligible projections of ``model`` in place with
    :class:`QuaternionLinear` layers on the same device and dtype.  Returns
    ``(model, records)`` with one :class:`ConversionRecord` per replaced
    module; each record's metrics hold the relative Frobenius error of the
    projection."""
    if method == "activation":
        raise ValueError("the activation-aware conversion is not provided; use method='matrix'")
    if method != "matrix":
        raise ValueError("method must be 'matrix'")
    records = []
    for name, module in eligible_modules(model):
        w = module_weight_out_in(module)
        comps = project_onto_quaternion(w)
        bias = module.bias.detach() if getattr(module, "bias", None) is not None else None
        layer = _build_layer(module, *comps, bias)
        wd = w.double()
        err = float((build_block_matrix(*comps) - wd).norm() / wd.norm().clamp_min(1e-30))
        parent_name, _, leaf = name.rpartition(".")
        setattr(model.get_submodule(parent_name) if parent_name else model, leaf, layer)
        records.append(ConversionRecord(name, w.shape[1], w.shape[0], _kind(name), method,
                                        {"relative_frobenius_error": err}))
        if verbose:
            print(f"[convert] {name}: {w.shape[1]}->{w.shape[0]} rel err {err:.3f}", flush=True)
    return model, records
