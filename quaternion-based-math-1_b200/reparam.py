"""Re-parameterised quaternion layers: factorized and unit-quaternion weights.

Drop-ins for the reference's ``FactorizedQuaternionLinear`` /
``parameter_count`` (``quaternion/factorized.py:35-137``) and
``UnitQuaternionLinear`` / ``normalize_quaternion``
(``quaternion/unit.py:26-95``): the same constructor arguments, parameter
names and shapes (state dicts load unchanged), initialisation and errors.

Both rebuild the four dense components ``wr, wi, wj, wk`` from their
parameters with ordinary tensor operations -- a small matrix product per
component (factorized) or an element-wise normalisation and scale (unit) --
and then run the Hamilton-product layer, bias fused, on this package's device
kernels (``fused_quaternion_linear``; gradients reach the parameters through
the rebuild).  Like the rest of the package there is no CPU forward: CPU
tensors raise ``RuntimeError``.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from .linear import fused_quaternion_linear
from .packing import check_divisible

__all__ = ["FactorizedQuaternionLinear", "parameter_count", "UnitQuaternionLinear", "normalize_quaternion"]

_FACTOR_MODES = ("independent", "shared_input", "shared_output")
_COMPONENTS = ("r", "i", "j", "k")


def parameter_count(in_features: int, out_features: int, rank: int, mode: str) -> int:
    """Scalar parameters of a factorized quaternion weight
    (reference ``quaternion/factorized.py:35-49``)."""
    if mode not in _FACTOR_MODES:
        raise ValueError(f"mode must be one of {_FACTOR_MODES}, got {mode!r}")
    og, ig = out_features // 4, in_features // 4
    left, right = og * rank, rank * ig
    if mode == "independent":
        return 4 * (left + right)
    return 4 * left + right if mode == "shared_input" else left + 4 * right


def _uniform_param(shape, fan_in, device, dtype) -> nn.Parameter:
    """U(-1/sqrt(fan_in), 1/sqrt(fan_in)), zero bound for fan_in 0 (the
    reference's factor initialisation, ``quaternion/factorized.py:52-55``)."""
    bound = 1.0 / math.sqrt(fan_in) if fan_in > 0 else 0.0
    return nn.Parameter(torch.empty(*shape, device=device, dtype=dtype).uniform_(-bound, bound))


class FactorizedQuaternionLinear(nn.Module):
    """Quaternion linear layer whose four components are low-rank products.

    ``independent``: W_c = A_c B_c; ``shared_input``: W_c = A_c B (one input
    factor); ``shared_output``: W_c = A B_c (one output factor).  A factors are
    ``[out_groups, rank]``, B factors ``[rank, in_groups]``.
    """

    def __init__(self, in_features: int, out_features: int, rank: int, mode: str = "independent",
                 bias: bool = False, device=None, dtype=None) -> None:
        super().__init__()
        if mode not in _FACTOR_MODES:
            raise ValueError(f"mode must be one of {_FACTOR_MODES}, got {mode!r}")
        in_g = check_divisible(in_features, "in_features")
        out_g = check_divisible(out_features, "out_features")
        if rank <= 0:
            raise ValueError("rank must be positive")
        self.in_features, self.out_features = in_features, out_features
        self.in_groups, self.out_groups = in_g, out_g
        self.rank, self.mode = rank, mode
        kw = dict(device=device, dtype=dtype)
        left = lambda: _uniform_param((out_g, rank), rank, **kw)
        right = lambda: _uniform_param((rank, in_g), in_g, **kw)
        # drawn in the reference's order, so one seed gives the same factors
        if mode == "independent":
            for c in _COMPONENTS:
                setattr(self, f"a_{c}", left())
                setattr(self, f"b_{c}", right())
        elif mode == "shared_input":
            for c in _COMPONENTS:
                setattr(self, f"a_{c}", left())
            self.b = right()
        else:
            self.a = left()
            for c in _COMPONENTS:
                setattr(self, f"b_{c}", right())
        if bias:
            self.bias = _uniform_param((out_features,), in_features, **kw)
        else:
            self.register_parameter("bias", None)

    @property
    def compression_ratio(self) -> float:
        return (self.out_features * self.in_features) / parameter_count(
            self.in_features, self.out_features, self.rank, self.mode)

    def reconstruct_weights(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        """The dense components ``(wr, wi, wj, wk)``, each ``[out_groups, in_groups]``."""
        left = [getattr(self, f"a_{c}") for c in _COMPONENTS] if self.mode != "shared_output" else [self.a] * 4
        right = [getattr(self, f"b_{c}") for c in _COMPONENTS] if self.mode != "shared_input" else [self.b] * 4
        return tuple(a @ b for a, b in zip(left, right))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fused_quaternion_linear(x, *self.reconstruct_weights(), self.bias)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"rank={self.rank}, mode={self.mode}, bias={self.bias is not None}")


def normalize_quaternion(wr: torch.Tensor, wi: torch.Tensor, wj: torch.Tensor, wk: torch.Tensor,
                         eps: float = 1e-8):
    """Divide four components element-wise by their quaternion norm (clamped
    below at ``eps``), reference ``quaternion/unit.py:26-34``."""
    norm = (wr * wr + wi * wi + wj * wj + wk * wk).sqrt().clamp_min(eps)
    return wr / norm, wi / norm, wj / norm, wk / norm


class UnitQuaternionLinear(nn.Module):
    """Quaternion linear layer with rotation-constrained weights:
    W = exp(log_magnitude) * unit(v), the magnitude per output group
    (``per_output``, ``[out_groups, 1]``) or per element (``per_element``)."""

    def __init__(self, in_features: int, out_features: int, magnitude: str = "per_output",
                 bias: bool = False, device=None, dtype=None) -> None:
        super().__init__()
        if magnitude not in ("per_output", "per_element"):
            raise ValueError("magnitude must be 'per_output' or 'per_element'")
        in_g = check_divisible(in_features, "in_features")
        out_g = check_divisible(out_features, "out_features")
        self.in_features, self.out_features = in_features, out_features
        self.in_groups, self.out_groups = in_g, out_g
        self.magnitude = magnitude
        bound = 1.0 / math.sqrt(in_features)
        for name in ("vr", "vi", "vj", "vk"):
            setattr(self, name, nn.Parameter(
                torch.empty(out_g, in_g, device=device, dtype=dtype).uniform_(-bound, bound)))
        mag_shape = (out_g, 1) if magnitude == "per_output" else (out_g, in_g)
        self.log_magnitude = nn.Parameter(torch.zeros(*mag_shape, device=device, dtype=dtype))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype))
        else:
            self.register_parameter("bias", None)

    def reconstruct_weights(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        scale = self.log_magnitude.exp()
        return tuple(c * scale for c in normalize_quaternion(self.vr, self.vi, self.vj, self.vk))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fused_quaternion_linear(x, *self.reconstruct_weights(), self.bias)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"magnitude={self.magnitude}, bias={self.bias is not None}")
