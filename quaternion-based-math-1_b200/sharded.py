"""Column-partitioned quaternion linear layer over ``torch.distributed``.

For layers too large for one GPU the output quaternion rows are split across
the ranks of a process group: rank ``r`` of ``G`` owns output groups
``[r*n, (r+1)*n)`` (``n = ceil(N_g / G)``) of every weight component, the
matching 4n slice of the bias and of LoRA ``B``; ``x`` and LoRA ``A`` are
replicated.  Each rank runs the single-GPU kernel on its shard (no
communication inside the kernel), then one all-gather of the ``[M, 4n]``
outputs over NCCL (NVLink/NVSwitch on one box) and one column-gather kernel
produce the full ``[M, 4*N_g]`` output on every rank.  The reference has no
distributed path; this is the partitioning of the layer it describes for
large layers.

Works with any backend whose all-gather accepts the tensors' device (NCCL for
CUDA tensors).  The shard arithmetic itself is device-free and is tested on
CPU with gloo ranks.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from . import _lib
from .linear import QuaternionLinear, fused_quaternion_linear
from .packing import check_divisible

__all__ = ["shard_bounds", "ColumnParallelQuaternionLinear", "gather_columns"]


def shard_bounds(out_groups: int, world: int, rank: int) -> tuple[int, int, int]:
    """Return ``(begin, end, n)``: this rank's output groups and the padded shard size."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    n = -(-out_groups // world)
    begin = min(rank * n, out_groups)
    end = min(begin + n, out_groups)
    return begin, end, n


def gather_columns(shards: torch.Tensor, M: int, n_cols: int, out: torch.Tensor | None = None):
    """``[G, M, n_cols] -> [M, G*n_cols]`` on the device (C ABI qlin_gather_columns)."""
    G = shards.shape[0]
    if out is None:
        out = torch.empty((M, G * n_cols), dtype=shards.dtype, device=shards.device)
    if M == 0:
        return out
    with torch.cuda.device(shards.device):
        _lib.check(
            _lib.load().qlin_gather_columns(
                _lib.dtype_code(shards.dtype), shards.data_ptr(), out.data_ptr(), G, M, n_cols,
                out.stride(0), _lib.stream_handle(shards.device)),
            "qlin_gather_columns",
        )
    return out


class ColumnParallelQuaternionLinear(nn.Module):
    """One rank's shard of a ``QuaternionLinear`` partitioned along out/4."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 process_group=None, device=None, dtype=None, world_size: int | None = None,
                 rank: int | None = None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.in_groups = check_divisible(in_features, "in_features")
        self.out_groups = check_divisible(out_features, "out_features")
        self.process_group = process_group
        if world_size is None:
            world_size = dist.get_world_size(process_group) if dist.is_initialized() else 1
        if rank is None:
            rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.world_size, self.rank = world_size, rank
        self.begin, self.end, self.shard = shard_bounds(self.out_groups, world_size, rank)
        fk = {"device": device, "dtype": dtype}
        # Every rank holds `shard` rows; rows past out_groups are zero padding.
        self.wr = nn.Parameter(torch.zeros(self.shard, self.in_groups, **fk))
        self.wi = nn.Parameter(torch.zeros(self.shard, self.in_groups, **fk))
        self.wj = nn.Parameter(torch.zeros(self.shard, self.in_groups, **fk))
        self.wk = nn.Parameter(torch.zeros(self.shard, self.in_groups, **fk))
        self.bias = nn.Parameter(torch.zeros(4 * self.shard, **fk)) if bias else None
        self.lora_A = None
        self.lora_B = None
        self.lora_scale = 0.0

    @classmethod
    def from_full(cls, layer: QuaternionLinear, process_group=None, world_size=None, rank=None,
                  lora_A=None, lora_B=None, lora_scale: float = 0.0, device=None):
        """Cut this rank's shard out of a full layer (and optional LoRA A/B)."""
        dev = device if device is not None else layer.wr.device
        m = cls(layer.in_features, layer.out_features, bias=layer.bias is not None,
                process_group=process_group, device=dev, dtype=layer.wr.dtype,
                world_size=world_size, rank=rank)
        rows = m.end - m.begin
        with torch.no_grad():
            for name in ("wr", "wi", "wj", "wk"):
                getattr(m, name)[:rows].copy_(getattr(layer, name)[m.begin:m.end])
            if layer.bias is not None:
                m.bias[:4 * rows].copy_(layer.bias[4 * m.begin:4 * m.end])
        if lora_A is not None:
            r = lora_A.shape[0]
            m.lora_A = lora_A.detach().to(dev)
            b = torch.zeros(4 * m.shard, r, dtype=lora_B.dtype, device=dev)
            b[:4 * rows] = lora_B.detach()[4 * m.begin:4 * m.end]
            m.lora_B = b
            m.lora_scale = float(lora_scale)
        return m

    def local_forward(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's ``[..., 4*shard]`` columns (no communication)."""
        return fused_quaternion_linear(x, self.wr, self.wi, self.wj, self.wk, self.bias,
                                       self.lora_A, self.lora_B, self.lora_scale)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        y_local = self.local_forward(x).reshape(-1, 4 * self.shard)
        M = y_local.shape[0]
        G = self.world_size
        if G == 1:
            y = y_local
        else:
            flat = torch.empty((G * M, 4 * self.shard), dtype=y_local.dtype, device=y_local.device)
            dist.all_gather_into_tensor(flat, y_local.contiguous(), group=self.process_group)
            buf = flat.view(G, M, 4 * self.shard)
            y = buf.view(M, G * 4 * self.shard) if M == 1 else gather_columns(buf, M, 4 * self.shard)
        if G * self.shard != self.out_groups:
            y = y[:, :self.out_features]
        return y.reshape(*lead, self.out_features)
