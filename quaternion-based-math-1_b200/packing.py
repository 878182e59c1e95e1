"""Real <-> quaternion channel packing (the layout contract the kernels honour).

Same convention as the reference (``quaternion/packing.py:5-25``): a real
tensor ``[..., D]`` with ``D % 4 == 0`` holds ``D // 4`` quaternions whose
four components are consecutive channels ordered (r, i, j, k).  Weight
components ``Wr, Wi, Wj, Wk`` are ``[out_groups, in_groups]``.  The real block
matrix of a quaternion weight places, for every (o, i) pair, the
left-multiplication block

    [ Wr  -Wi  -Wj  -Wk ]
    [ Wi   Wr  -Wk   Wj ]
    [ Wj   Wk   Wr  -Wi ]
    [ Wk  -Wj   Wi   Wr ]

at rows 4o..4o+3 and columns 4i..4i+3.  These helpers are views / small
tensor ops (no GEMM) and work on any device; ``build_block_matrix`` exists for
verification only -- the device kernels never form it.
"""

from __future__ import annotations

import torch

__all__ = [
    "QUATERNION_GROUPS",
    "check_divisible",
    "pack_real_to_quaternion",
    "unpack_quaternion_to_real",
    "split_components",
    "pack_components",
    "build_block_matrix",
]

QUATERNION_GROUPS = 4


def check_divisible(dim: int, name: str = "dimension") -> int:
    """Return ``dim // 4``; ``ValueError`` unless ``dim % 4 == 0`` (packing.py:45-52)."""
    if dim % QUATERNION_GROUPS:
        raise ValueError(
            f"{name} must be divisible by {QUATERNION_GROUPS} for quaternion packing, got {dim}"
        )
    return dim // QUATERNION_GROUPS


def pack_real_to_quaternion(x: torch.Tensor) -> torch.Tensor:
    """``[..., D] -> [..., D // 4, 4]`` (a view), last axis (r, i, j, k)."""
    groups = check_divisible(x.shape[-1], "last dimension")
    return x.reshape(*x.shape[:-1], groups, QUATERNION_GROUPS)


def unpack_quaternion_to_real(q: torch.Tensor) -> torch.Tensor:
    """``[..., G, 4] -> [..., 4G]``, inverse of :func:`pack_real_to_quaternion`."""
    if q.shape[-1] != QUATERNION_GROUPS:
        raise ValueError(f"last dimension must be {QUATERNION_GROUPS}, got {q.shape[-1]}")
    return q.reshape(*q.shape[:-2], q.shape[-2] * QUATERNION_GROUPS)


def split_components(q: torch.Tensor):
    """``[..., G, 4] -> (qr, qi, qj, qk)``, each ``[..., G]`` (views)."""
    if q.shape[-1] != QUATERNION_GROUPS:
        raise ValueError(f"last dimension must be {QUATERNION_GROUPS}, got {q.shape[-1]}")
    return tuple(q.unbind(-1))


def pack_components(qr, qi, qj, qk) -> torch.Tensor:
    """``(qr, qi, qj, qk)`` each ``[..., G]`` -> ``[..., G, 4]`` ordered (r, i, j, k)."""
    return torch.stack((qr, qi, qj, qk), dim=-1)


# Signed component permutation of the block matrix: row a holds
# sign * W_{_BLOCK_COMP[a][q]} in column q.
_BLOCK_COMP = ((0, 1, 2, 3), (1, 0, 3, 2), (2, 3, 0, 1), (3, 2, 1, 0))
_BLOCK_SIGN = ((1, -1, -1, -1), (1, 1, -1, 1), (1, 1, 1, -1), (1, -1, 1, 1))


def build_block_matrix(wr, wi, wj, wk) -> torch.Tensor:
    """The real ``[4*out_groups, 4*in_groups]`` matrix of the quaternion weight.

    Verification only (packing.py:89-127): it is 4x the parameter memory.
    """
    ws = (wr, wi, wj, wk)
    for w, name in zip(ws, ("wr", "wi", "wj", "wk")):
        if w.dim() != 2:
            raise ValueError(f"{name} must be 2D [out_groups, in_groups]")
    if not (wr.shape == wi.shape == wj.shape == wk.shape):
        raise ValueError("all four weight components must share the same shape")
    og, ig = wr.shape
    block = wr.new_empty(og, 4, ig, 4)
    for a in range(4):
        for q in range(4):
            block[:, a, :, q] = _BLOCK_SIGN[a][q] * ws[_BLOCK_COMP[a][q]]
    return block.reshape(og * 4, ig * 4)
