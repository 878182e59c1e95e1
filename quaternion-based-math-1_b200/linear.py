"""Quaternion linear layer on the B200 kernels (drop-in for the reference's
``quaternion/linear.py``).

``quaternion_linear(x, wr, wi, wj, wk)`` keeps the reference signature and
error behaviour (``quaternion/linear.py:41-72``): ``ValueError`` when
``in_features % 4 != 0``, when ``wr.shape[1]`` differs from ``in_features // 4``
or when the four weight components differ in shape.  The computation itself
is one call into the C ABI (``qlin_forward``); CPU tensors raise
``RuntimeError`` -- there is no CPU path.

``QuaternionLinear`` keeps the module signature, parameter names
(``wr, wi, wj, wk, bias``), initialisation and helpers of
``quaternion/linear.py:75-163``, so reference state dicts load unchanged; its
bias is fused into the kernel epilogue.

Gradients.  ``y = x B^T`` with ``B`` the block matrix, so
``dX = dY B``, i.e. the quaternion layer with weights
``conj(W)^T = (Wr^T, -Wi^T, -Wj^T, -Wk^T)`` (run on the same kernel), and
``dW[o, i] = sum_m dY[m, o] (x) conj(X[m, i])``, whose conjugate
``sum_m X[m, i] (x) conj(dY[m, o])`` is again the quaternion layer, with the
tokens as the reduction axis.  Both directions therefore use the device
kernel; only transposes and sign flips are plain tensor ops.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import _lib
from .packing import build_block_matrix, check_divisible

__all__ = ["quaternion_linear", "QuaternionLinear", "fused_quaternion_linear"]


def _validate(x: torch.Tensor, wr, wi, wj, wk) -> tuple[int, int]:
    in_groups = check_divisible(x.shape[-1], "in_features")
    for w in (wr, wi, wj, wk):
        if w.dim() != 2:
            raise ValueError("weight components must be 2D [out_groups, in_groups]")
    if wr.shape[1] != in_groups:
        raise ValueError(
            f"weight in_groups ({wr.shape[1]}) must match input in_groups ({in_groups})"
        )
    if not (wr.shape == wi.shape == wj.shape == wk.shape):
        raise ValueError("all four weight components must share the same shape")
    return in_groups, wr.shape[0]


def _check_device(tensors) -> torch.device:
    x = tensors[0]
    if x.is_cuda:
        # common case: every tensor on x's device with x's dtype
        dev, dtype = x.device, x.dtype
        ok = True
        for t in tensors:
            if t is not None and (t.device != dev or t.dtype != dtype):
                ok = False
                break
        if ok:
            if dtype not in _lib._DTYPE_CODE:
                _lib.dtype_code(dtype)
            return dev
    dev = None
    dtype = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "the B200 quaternion linear kernels require CUDA tensors (there is no CPU path); "
                f"got a tensor on {t.device}"
            )
        if dev is None:
            dev, dtype = t.device, t.dtype
        elif t.device != dev:
            raise RuntimeError(f"all tensors must be on one device, got {dev} and {t.device}")
        elif t.dtype != dtype:
            raise RuntimeError(f"all tensors must share one dtype, got {dtype} and {t.dtype}")
    _lib.dtype_code(dtype)
    return dev


def _rows(x: torch.Tensor, K: int) -> tuple[torch.Tensor, int]:
    if x.is_contiguous():
        return x.view(-1, K), K
    x2 = x.reshape(-1, K)
    if x2.stride(-1) != 1 or (x2.shape[0] > 1 and x2.stride(0) < K):
        x2 = x2.contiguous()
    ld = x2.stride(0) if x2.shape[0] > 1 else K
    return x2, ld


def _weights(ws):
    w0, w1, w2, w3 = ws
    if w0.is_contiguous() and w1.is_contiguous() and w2.is_contiguous() and w3.is_contiguous():
        return ws, w0.shape[1]
    ld = ws[0].stride(0)
    if any(w.stride(1) != 1 or w.stride(0) != ld for w in ws) or ld < ws[0].shape[1]:
        ws = tuple(w.contiguous() for w in ws)
        ld = ws[0].shape[1]
    return ws, ld


def _forward_impl(x, wr, wi, wj, wk, bias=None, lora_a=None, lora_b=None, lora_scale=0.0,
                  algo=_lib.ALGO_AUTO, static_weights=False, packed=None):
    if algo == _lib.ALGO_AUTO:
        ext = _lib._torch_ext if _lib._lib is not None else (_lib.load() and _lib._torch_ext)
        if ext is not None:
            # the same checks, allocation and call in C++ (csrc/qlin_torch_ext.cpp)
            return ext.forward(x, wr, wi, wj, wk, bias, lora_a, lora_b, float(lora_scale),
                               bool(static_weights), packed)
    in_groups, out_groups = _validate(x, wr, wi, wj, wk)
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != 4 * out_groups):
        raise ValueError(f"bias must be [{4 * out_groups}], got {tuple(bias.shape)}")
    rank = 0
    if lora_a is not None or lora_b is not None:
        if lora_a is None or lora_b is None:
            raise ValueError("LoRA needs both A and B")
        rank = lora_a.shape[0]
        if lora_a.shape != (rank, 4 * in_groups) or lora_b.shape != (4 * out_groups, rank):
            raise ValueError(
                f"LoRA shapes must be A [r, {4 * in_groups}] and B [{4 * out_groups}, r], got "
                f"{tuple(lora_a.shape)} and {tuple(lora_b.shape)}"
            )
    dev = _check_device((x, wr, wi, wj, wk, bias, lora_a, lora_b))
    K = 4 * in_groups
    lead = x.shape[:-1]
    x2, ld_x = _rows(x, K)
    M = x2.shape[0]
    ws, ld_w = _weights((wr, wi, wj, wk))
    b = bias if bias is None or bias.is_contiguous() else bias.contiguous()
    la = (lora_a if lora_a.is_contiguous() else lora_a.contiguous()) if rank else None
    lb = (lora_b if lora_b.is_contiguous() else lora_b.contiguous()) if rank else None
    if rank % 8 and x.dtype != torch.float32:
        # The tensor-core path reads B through TMA with rows of rank elements;
        # zero-padding the rank to a multiple of 8 keeps it on that path and
        # adds exact zeros.
        pad = 8 - rank % 8
        la = torch.cat((la, la.new_zeros(pad, la.shape[1])), 0)
        lb = torch.cat((lb, lb.new_zeros(lb.shape[0], pad)), 1)
        rank += pad
    y = torch.empty((M, 4 * out_groups), dtype=x.dtype, device=dev)
    if M:
        flags = _lib.FLAG_STATIC_WEIGHTS if static_weights else 0
        # the library launches on the current device: switch only when needed
        if torch._C._cuda_getDevice() == dev.index:
            _lib.forward_raw(x2, ld_x, ws, ld_w, b, la, lb, rank, float(lora_scale), y, 4 * out_groups,
                             M, in_groups, out_groups, int(algo), flags, packed=packed)
        else:
            with torch.cuda.device(dev):
                _lib.forward_raw(x2, ld_x, ws, ld_w, b, la, lb, rank, float(lora_scale), y,
                                 4 * out_groups, M, in_groups, out_groups, int(algo), flags, packed=packed)
    return y.reshape(*lead, 4 * out_groups)


def _conj_t(wr, wi, wj, wk):
    """Weights of the adjoint layer: conj(W)^T."""
    return (wr.t().contiguous(), (-wi).t().contiguous(), (-wj).t().contiguous(),
            (-wk).t().contiguous())


def _weight_grad(x2: torch.Tensor, g2: torch.Tensor):
    """dW[o, i] = sum_m g[m, o] (x) conj(x[m, i]) via the kernel on transposed operands.

    conj(dW[o, i]) = sum_m x[m, i] (x) conj(g[m, o]): a quaternion layer whose
    "tokens" are the output groups o, whose input groups are the tokens m,
    with weight X^T (quaternion [K_g, M]) and input conj(G)^T ([N_g, 4M]).
    """
    M = x2.shape[0]
    K_g, N_g = x2.shape[1] // 4, g2.shape[1] // 4
    xq = x2.reshape(M, K_g, 4)
    wt = tuple(xq[:, :, c].t().contiguous() for c in range(4))  # [K_g, M] each
    gq = g2.reshape(M, N_g, 4)
    sign = g2.new_tensor([1.0, -1.0, -1.0, -1.0])
    gin = (gq * sign).permute(1, 0, 2).reshape(N_g, 4 * M).contiguous()  # conj(G)^T
    cw = _forward_impl(gin, *wt)  # [N_g, 4*K_g] = conj(dW) in (o, i, comp) order
    cw = cw.reshape(N_g, K_g, 4)
    return cw[..., 0], -cw[..., 1], -cw[..., 2], -cw[..., 3]


class _QLinFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, wr, wi, wj, wk, bias, lora_a, lora_b, lora_scale):
        ctx.save_for_backward(x, wr, wi, wj, wk, bias, lora_a, lora_b)
        ctx.lora_scale = lora_scale
        return _forward_impl(x, wr, wi, wj, wk, bias, lora_a, lora_b, lora_scale)

    @staticmethod
    def backward(ctx, gy):
        x, wr, wi, wj, wk, bias, lora_a, lora_b = ctx.saved_tensors
        K = x.shape[-1]
        N = gy.shape[-1]
        g2 = gy.reshape(-1, N).contiguous()
        x2 = x.reshape(-1, K).contiguous()
        need = ctx.needs_input_grad
        dx = dwr = dwi = dwj = dwk = db = da = dbl = None
        t = None
        if lora_a is not None and (need[0] or need[6] or need[7]):
            t = x2 @ lora_a.t()  # [M, r]
        if need[0]:
            dx = _forward_impl(g2, *_conj_t(wr, wi, wj, wk))
            if lora_a is not None:
                dx = dx + ctx.lora_scale * ((g2 @ lora_b) @ lora_a)
            dx = dx.reshape(x.shape)
        if any(need[1:5]):
            dwr, dwi, dwj, dwk = _weight_grad(x2, g2)
        if bias is not None and need[5]:
            db = g2.sum(0)
        if lora_a is not None:
            if need[6]:
                da = ctx.lora_scale * ((g2 @ lora_b).t() @ x2)
            if need[7]:
                dbl = ctx.lora_scale * (g2.t() @ t)
        return dx, dwr, dwi, dwj, dwk, db, da, dbl, None


def fused_quaternion_linear(x, wr, wi, wj, wk, bias=None, lora_a=None, lora_b=None,
                            lora_scale: float = 0.0, static_weights: bool = False, packed=None):
    """``quaternion_linear(x) + bias + lora_scale * (x A^T) B^T`` in one device call.

    ``static_weights=True`` declares that nothing queued earlier on the current
    stream writes the weights, bias or LoRA A/B (inference with fixed weights):
    the kernel may then stream them while the previous kernel finishes.
    ``packed``: the same weights as one ``[out_groups, in_groups, 4]`` tensor
    (:func:`pack_quaternion_weights`), read by the kernels that take it (the
    decode GEMV and the CTA-pair prefill kernel); ignored under autograd.
    """
    if torch.is_grad_enabled():
        for t in (x, wr, wi, wj, wk, bias, lora_a, lora_b):
            if t is not None and t.requires_grad:
                return _QLinFn.apply(x, wr, wi, wj, wk, bias, lora_a, lora_b, float(lora_scale))
    return _forward_impl(x, wr, wi, wj, wk, bias, lora_a, lora_b, lora_scale,
                         static_weights=static_weights, packed=packed)


def pack_quaternion_weights(wr, wi, wj, wk) -> torch.Tensor:
    """The packed weight layout ``[out_groups, in_groups, 4]``: component p of
    weight quaternion (o, i) at ``[o, i, p]`` -- the layout of ``x`` rows, so
    one 16-byte load holds two whole weight quaternions."""
    with torch.no_grad():
        return torch.stack((wr, wi, wj, wk), dim=-1).contiguous()


def quaternion_linear(x, wr, wi, wj, wk) -> torch.Tensor:
    """Quaternion linear transform without bias (reference quaternion/linear.py:41-72).

    ``x``: ``[..., in_features]``; weights ``[out_groups, in_groups]``; returns
    ``[..., out_features]``.
    """
    return fused_quaternion_linear(x, wr, wi, wj, wk)


class QuaternionLinear(nn.Module):
    """Drop-in for the reference ``QuaternionLinear`` (quaternion/linear.py:75-163)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, device=None,
                 dtype=None) -> None:
        super().__init__()
        in_groups = check_divisible(in_features, "in_features")
        out_groups = check_divisible(out_features, "out_features")
        self.in_features = in_features
        self.out_features = out_features
        self.in_groups = in_groups
        self.out_groups = out_groups
        fk = {"device": device, "dtype": dtype}
        self.wr = nn.Parameter(torch.empty(out_groups, in_groups, **fk))
        self.wi = nn.Parameter(torch.empty(out_groups, in_groups, **fk))
        self.wj = nn.Parameter(torch.empty(out_groups, in_groups, **fk))
        self.wk = nn.Parameter(torch.empty(out_groups, in_groups, **fk))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, **fk))
        else:
            self.register_parameter("bias", None)
        # Inference hint (not part of the state dict): when True, forward
        # declares the weights static for the duration of the call, letting
        # the kernel stream them while the previous kernel of the stream ends.
        self.static_weights = False
        # Inference option (not part of the state dict; the parameters stay
        # wr, wi, wj, wk): when True, forward without autograd also keeps the
        # packed weight cache (packed_weights) and hands it to the kernels
        # that read it.
        self.packed = False
        self._packed_cache = None
        self.reset_parameters()

    def reset_parameters(self) -> None:
        # U(-1/sqrt(in), 1/sqrt(in)) for all four components and the bias,
        # the variance of the equivalent real layer (linear.py:111-118).
        bound = 1.0 / math.sqrt(self.in_features)
        for w in (self.wr, self.wi, self.wj, self.wk):
            nn.init.uniform_(w, -bound, bound)
        if self.bias is not None:
            nn.init.uniform_(self.bias, -bound, bound)

    def packed_weights(self) -> torch.Tensor:
        """The packed weight cache ``[out_groups, in_groups, 4]``
        (:func:`pack_quaternion_weights`), rebuilt whenever a component is
        replaced, moved or updated in place (its version counter advances)."""
        key = tuple((w.data_ptr(), w._version, w.dtype, w.device, tuple(w.shape))
                    for w in (self.wr, self.wi, self.wj, self.wk))
        cache = self._packed_cache
        if cache is None or cache[0] != key:
            cache = self._packed_cache = (key, pack_quaternion_weights(self.wr, self.wi, self.wj, self.wk))
        return cache[1]

    def _packed_for_call(self, *tensors):
        """The packed cache when this call may use it (``packed`` set, no autograd)."""
        if not getattr(self, "packed", False):
            return None
        if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors):
            return None
        return self.packed_weights()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fused_quaternion_linear(x, self.wr, self.wi, self.wj, self.wk, self.bias,
                                       static_weights=self.static_weights,
                                       packed=self._packed_for_call(x, self.wr, self.wi, self.wj, self.wk,
                                                                    self.bias))

    def real_block_matrix(self) -> torch.Tensor:
        """The equivalent real ``[out_features, in_features]`` matrix (verification only)."""
        return build_block_matrix(self.wr, self.wi, self.wj, self.wk)

    @classmethod
    def from_real_block_matrix(cls, weight: torch.Tensor, bias: torch.Tensor | None = None):
        """Exact inverse of :meth:`real_block_matrix` (linear.py:126-157)."""
        if weight.dim() != 2:
            raise ValueError("weight must be 2D [out_features, in_features]")
        out_features, in_features = weight.shape
        check_divisible(out_features, "out_features")
        check_divisible(in_features, "in_features")
        layer = cls(in_features, out_features, bias=bias is not None, device=weight.device,
                    dtype=weight.dtype)
        with torch.no_grad():
            layer.wr.copy_(weight[0::4, 0::4])
            layer.wi.copy_(weight[1::4, 0::4])
            layer.wj.copy_(weight[2::4, 0::4])
            layer.wk.copy_(weight[3::4, 0::4])
            if bias is not None:
                layer.bias.copy_(bias)
        return layer

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}")
