"""K1 "naive" and K2 "planar" operator entry points on the B200 kernels.

The reference keeps two deliberately different CPU/ATen formulations of the
same operator (``quaternion/planar.py:39-61`` sixteen separate products,
``quaternion/planar.py:100-129`` one batched contraction with the sparse
coefficient tensor ``C[a, q, p]``).  Here both names keep their signatures and
error behaviour and run the fused device kernel: the kernel's sixteen
sign-tagged tensor-core products *are* the planar contraction, applied tile by
tile without the ``P[n, q, p, o]`` intermediate.

``quaternion_linear_planar(..., coefficient=C)`` accepts the reference's
optional coefficient tensor; the kernel implements the Hamilton coefficients,
so any other ``C`` raises ``ValueError`` rather than being silently ignored.
"""

from __future__ import annotations

import torch

from .linear import fused_quaternion_linear
from .packing import check_divisible

__all__ = ["quaternion_linear_naive", "quaternion_linear_planar", "planar_coefficient_tensor"]


def planar_coefficient_tensor(device=None, dtype=None) -> torch.Tensor:
    """``C[a, q, p]`` with sixteen +-1 entries (reference planar.py:64-97).

    ``Y[n, a, o] = sum_{q,p} C[a, q, p] * sum_i X[n, q, i] W[p, o, i]``.
    """
    c = torch.zeros(4, 4, 4, device=device, dtype=dtype)
    entries = (
        (0, 0, 0, 1), (0, 1, 1, -1), (0, 2, 2, -1), (0, 3, 3, -1),
        (1, 0, 1, 1), (1, 1, 0, 1), (1, 2, 3, -1), (1, 3, 2, 1),
        (2, 0, 2, 1), (2, 1, 3, 1), (2, 2, 0, 1), (2, 3, 1, -1),
        (3, 0, 3, 1), (3, 1, 2, -1), (3, 2, 1, 1), (3, 3, 0, 1),
    )
    for a, q, p, s in entries:
        c[a, q, p] = s
    return c


def _check(x, wr):
    in_groups = check_divisible(x.shape[-1], "in_features")
    if wr.shape[1] != in_groups:
        raise ValueError("weight in_groups must match input in_groups")


def quaternion_linear_naive(x, wr, wi, wj, wk) -> torch.Tensor:
    """K1 entry point (planar.py:39-61): same math, fused device kernel."""
    _check(x, wr)
    return fused_quaternion_linear(x, wr, wi, wj, wk)


def quaternion_linear_planar(x, wr, wi, wj, wk, coefficient=None) -> torch.Tensor:
    """K2 entry point (planar.py:100-129): same math, fused device kernel."""
    _check(x, wr)
    if coefficient is not None:
        c = torch.as_tensor(coefficient).detach().to("cpu", torch.float64)
        if c.shape != (4, 4, 4) or not torch.equal(c, planar_coefficient_tensor(dtype=torch.float64)):
            raise ValueError("the device kernel implements the Hamilton coefficient tensor only")
    return fused_quaternion_linear(x, wr, wi, wj, wk)
