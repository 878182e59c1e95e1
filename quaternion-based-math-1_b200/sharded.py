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

With ``fused_allgather=True`` (bf16/f16, one process per GPU of one box) the
all-gather is fused into the kernel instead (``"auto"``, the default, does so
for calls of at least 64 tokens, where it measured faster: 2 GPUs, 5120→27648,
M=512 98 vs 175 us, M=8192 1054 vs 2103 us; at M=1 and 16 the NCCL path was
slightly faster): every rank's full output is
mapped into every other rank (CUDA IPC, exchanged once per output shape),
each rank's epilogue stores its columns into all of them over NVLink, and
bounded cross-rank flag barriers open the call (no rank writes into an
output that a peer may still be copying from) and end it
(``qlin_forward_allgather``).  Where the box offers NVLink multicast
(NVSwitch; torch's symmetric memory reports it), the full outputs are one
symmetric-memory buffer per rank bound to a multicast object and each output
piece is stored once through the multicast address (``multimem.st``): every
rank sends its columns over NVLink once instead of once per peer
(``qlin_forward_allgather_mc``).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
import torch.nn as nn

from . import _lib
from .linear import QuaternionLinear, fused_quaternion_linear
from .packing import check_divisible

__all__ = ["shard_bounds", "ColumnParallelQuaternionLinear", "gather_columns", "PeerOutputs", "MulticastOutputs"]


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


class PeerOutputs:
    """Every rank's full ``[M, cols]`` output, mapped into this process.

    Built collectively (every rank of ``group`` constructs it with the same
    shape): each rank allocates its output and its barrier flags
    ``[2 * world]`` (entry and exit barrier) plus two call counters with
    ``qlin_ipc_alloc`` (plain cudaMalloc, zero-filled),
    the CUDA IPC handles are exchanged with ``all_gather_object``, and the
    peers' buffers are mapped with this rank's GPU current (``qlin_ipc_open``:
    plain peer mappings, no multicast objects).  The buffers must outlive
    every use by the peers: instances live for the process's life unless
    ``close`` is called on every rank after a final barrier.
    """

    def __init__(self, M: int, cols: int, dtype, device, group=None):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        lib = _lib.load()
        elem = torch.empty((), dtype=dtype).element_size()
        self._owned = []   # this rank's allocations (qlin_ipc_alloc)
        self._mapped = []  # peers' mapped bases (qlin_ipc_open)
        with torch.cuda.device(self.device):
            out_ptr, out_h = self._alloc(lib, M * cols * elem)
            # flags[2 * world] (exit, entry) + the two barriers' call counters
            flag_ptr, flag_h = self._alloc(lib, 4 * (2 * self.world + 2))
        self.out = _device_view(out_ptr, (M, cols), dtype, self.device, self)
        self.flags = _device_view(flag_ptr, (2 * self.world,), torch.int32, self.device, self)
        self.epoch = _device_view(flag_ptr + 8 * self.world, (2,), torch.int32, self.device, self)
        everyone = [None] * self.world
        dist.all_gather_object(everyone, (out_h, flag_h), group=group)
        outs, flags = [], []
        with torch.cuda.device(self.device):
            for q, (oh, fh) in enumerate(everyone):
                if q == self.rank:
                    outs.append(out_ptr)
                    flags.append(flag_ptr)
                    continue
                outs.append(self._open(lib, oh))
                flags.append(self._open(lib, fh))
        P = ctypes.c_void_p
        self._outs = (P * self.world)(*outs)
        self._flags = (P * self.world)(*flags)

    def _alloc(self, lib, nbytes):
        p = ctypes.c_void_p()
        h = ctypes.create_string_buffer(64)
        _lib.check(lib.qlin_ipc_alloc(nbytes, ctypes.byref(p), h), "qlin_ipc_alloc")
        self._owned.append(p.value)
        return p.value, h.raw

    def _open(self, lib, handle):
        p = ctypes.c_void_p()
        _lib.check(lib.qlin_ipc_open(handle, 0, ctypes.byref(p)), "qlin_ipc_open")
        self._mapped.append(p.value)
        return p.value

    def close(self):
        """Unmap the peers' buffers and free this rank's (after every rank is done with them)."""
        lib = _lib.load()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for b in self._mapped:
                lib.qlin_ipc_close(b)
            for p in self._owned:
                lib.qlin_ipc_free(p)
        self._mapped, self._owned = [], []


class MulticastOutputs:
    """Every rank's full ``[M, cols]`` output in one NVLink multicast group.

    Built collectively (every rank of ``group`` constructs it with the same
    shape) from torch's symmetric memory: ``out`` is this rank's buffer,
    ``mc`` the multicast address of the same offset (a store through it lands
    in every rank's ``out``), the barrier flags ``[2 * world]`` and two call
    counters live in a second symmetric buffer, zero-filled before any rank
    uses them (``_flags``: every rank's flag array as mapped here).  Raises
    RuntimeError where multicast is not available (see ``available``).
    """

    @staticmethod
    def available(device) -> bool:
        """Whether this process's GPU offers NVLink multicast (torch's check)."""
        try:
            from torch._C._distributed_c10d import _SymmetricMemory
            dev = torch.device(device)
            return bool(_SymmetricMemory.has_multicast_support(torch._C._autograd.DeviceType.CUDA, dev.index))
        except Exception:  # an older torch or no CUDA: the peer-store path
            return False

    def __init__(self, M: int, cols: int, dtype, device, group=None):
        import torch.distributed._symmetric_memory as symm_mem
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        gname = (group if group is not None else dist.group.WORLD).group_name
        self.out = symm_mem.empty((M, cols), dtype=dtype, device=self.device)
        self._h_out = symm_mem.rendezvous(self.out, gname)
        base = self._h_out.buffer_ptrs[self.rank]
        if not self._h_out.multicast_ptr:
            raise RuntimeError("NVLink multicast is not available for this group")
        self.mc = self._h_out.multicast_ptr + (self.out.data_ptr() - base)
        flags = symm_mem.empty((2 * self.world + 2,), dtype=torch.int32, device=self.device)
        flags.zero_()
        self._h_flags = symm_mem.rendezvous(flags, gname)
        torch.cuda.synchronize(self.device)
        dist.barrier(group)  # every rank's flags are zero before any rank signals
        off = flags.data_ptr() - self._h_flags.buffer_ptrs[self.rank]
        self._flag_buf = flags
        self.flags = flags[:2 * self.world]
        self.epoch = flags[2 * self.world:]
        P = ctypes.c_void_p
        self._flags = (P * self.world)(*(p + off for p in self._h_flags.buffer_ptrs))


class _CudaArray:
    """__cuda_array_interface__ of a raw device buffer (zero-copy torch view)."""

    def __init__(self, ptr, shape, typestr, owner):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}
        self.owner = owner


_TYPESTR = {torch.bfloat16: "<V2", torch.float16: "<f2", torch.int32: "<i4"}


def _device_view(ptr, shape, dtype, device, owner):
    if dtype == torch.bfloat16:  # no bf16 typestr: view int16 storage as bf16
        t = torch.as_tensor(_CudaArray(ptr, shape, "<i2", owner), device=device)
        return t.view(torch.bfloat16)
    return torch.as_tensor(_CudaArray(ptr, shape, _TYPESTR[dtype], owner), device=device)


class ColumnParallelQuaternionLinear(nn.Module):
    """One rank's shard of a ``QuaternionLinear`` partitioned along out/4."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 process_group=None, device=None, dtype=None, world_size: int | None = None,
                 rank: int | None = None, fused_allgather: bool | str = "auto"):
        super().__init__()
        if fused_allgather not in (True, False, "auto"):
            raise ValueError("fused_allgather must be True, False or 'auto'")
        self.fused_allgather = fused_allgather
        self._peer_outputs: dict[int, PeerOutputs | MulticastOutputs] = {}
        self._multicast: bool | None = None  # decided on the first fused call
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

    def _fused_forward(self, x: torch.Tensor) -> torch.Tensor:
        """Shard GEMM with the all-gather fused into its epilogue (see module doc)."""
        x2 = x.reshape(-1, self.in_features).contiguous()
        M = x2.shape[0]
        G = self.world_size
        cols = 4 * self.shard * G
        if self._multicast is None:
            # the same answer on every rank: all must take the same (collective) path
            ok = torch.tensor([int(MulticastOutputs.available(x2.device))], device=x2.device)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.process_group)
            self._multicast = bool(ok.item())
        po = self._peer_outputs.get(M)
        if po is None:
            make = MulticastOutputs if self._multicast else PeerOutputs
            po = self._peer_outputs[M] = make(M, cols, x2.dtype, x2.device, self.process_group)
        la, lb = self.lora_A, self.lora_B
        rank_l = 0 if la is None else la.shape[0]
        if rank_l % 8:
            # the tensor-core path takes ranks in multiples of 8: zero-pad
            pad = 8 - rank_l % 8
            la = torch.cat((la, la.new_zeros(pad, la.shape[1])), 0)
            lb = torch.cat((lb, lb.new_zeros(lb.shape[0], pad)), 1).contiguous()
            rank_l += pad
        K_g, n = self.in_groups, self.shard
        ws_bytes = _lib.workspace_size(x2.dtype, M, K_g, n, rank_l)
        ws = _lib.zeroed_workspace(x2.device, ws_bytes) if ws_bytes else None
        flags = _lib.FLAG_ZEROED_WORKSPACE if ws is not None else 0
        ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        common = (_lib.dtype_code(x2.dtype), x2.data_ptr(), self.in_features,
                  self.wr.data_ptr(), self.wi.data_ptr(), self.wj.data_ptr(), self.wk.data_ptr(), K_g,
                  ptr(self.bias), ptr(la), ptr(lb), rank_l, float(self.lora_scale),
                  M, K_g, n, ptr(ws), ws_bytes, flags, G, self.rank)
        with torch.cuda.device(x2.device):
            if isinstance(po, MulticastOutputs):
                code = _lib.load().qlin_forward_allgather_mc(
                    *common, po.out.data_ptr(), po.mc, cols, 4 * n * self.rank, po._flags, po.epoch.data_ptr(),
                    _lib.stream_handle(x2.device))
            else:
                code = _lib.load().qlin_forward_allgather(
                    *common, po._outs, cols, 4 * n * self.rank, po._flags, po.epoch.data_ptr(),
                    _lib.stream_handle(x2.device))
        _lib.check(code, "qlin_forward_allgather")
        return po.out[:, :self.out_features].clone()

    def _use_fused(self, x: torch.Tensor) -> bool:
        if self.world_size <= 1 or self.fused_allgather is False:
            return False
        if self.fused_allgather is True:
            return True
        rows = x.numel() // max(self.in_features, 1)
        return x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and rows >= 64

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        if self._use_fused(x):
            return self._fused_forward(x).reshape(*lead, self.out_features)
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
