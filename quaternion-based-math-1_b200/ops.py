"""Kernel operator interface ``fn(x, wr, wi, wj, wk) -> y`` and timing harness.

Mirrors the reference's operator layer: ``kernels/pytorch/ops.py:20-72``
(``dense_gemm``, ``naive``, ``planar``, ``benchmark_operator``) and
``kernels/cuda/loader.py:13-49`` (``cuda_kernel_available``,
``quaternion_linear_cuda``).  Every quaternion operator here is the fused
sm_100a kernel; ``dense_gemm`` stays the cuBLAS comparator of the same
logical shape.  Unlike the reference loader, weights are consumed in their
native ``[out_groups, in_groups]`` layout (no per-call transpose) and the
kernel runs on the caller's current stream.
"""

from __future__ import annotations

import os
import time

import torch

from . import _lib
from .linear import fused_quaternion_linear
from .planar import quaternion_linear_naive, quaternion_linear_planar

__all__ = [
    "dense_gemm",
    "naive",
    "planar",
    "fused",
    "quaternion_linear_cuda",
    "cuda_kernel_available",
    "benchmark_operator",
]


def dense_gemm(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """cuBLAS comparator ``x @ weight.T`` (reference ops.py:20-22)."""
    return x @ weight.t()


def naive(x, wr, wi, wj, wk):
    return quaternion_linear_naive(x, wr, wi, wj, wk)


def planar(x, wr, wi, wj, wk):
    return quaternion_linear_planar(x, wr, wi, wj, wk)


def fused(x, wr, wi, wj, wk, bias=None, lora_a=None, lora_b=None, lora_scale=0.0):
    return fused_quaternion_linear(x, wr, wi, wj, wk, bias, lora_a, lora_b, lora_scale)


def cuda_kernel_available() -> bool:
    """True when a CUDA device is present and the in-tree library loads."""
    if not torch.cuda.is_available():
        return False
    try:
        _lib.load()
    except (RuntimeError, OSError):
        return False
    return True


def quaternion_linear_cuda(x, wr, wi, wj, wk):
    """Fused quaternion linear on the device (reference kernels/cuda/loader.py:39-49)."""
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is not available")
    return fused_quaternion_linear(x, wr, wi, wj, wk)


def benchmark_operator(fn, args, warmup: int = 10, iters: int = 50, device=None) -> dict:
    """Time ``fn(*args)``; same result keys as reference ops.py:38-72.

    On CUDA each iteration is bracketed by CUDA events on the current stream
    (device time, not host time); on CPU by ``perf_counter``.
    """
    if device is not None and not isinstance(device, torch.device):
        device = torch.device(device)
    cuda = device is not None and device.type == "cuda"
    for _ in range(warmup):
        fn(*args)
    if cuda:
        torch.cuda.synchronize(device)
    times = []
    out = None
    for _ in range(iters):
        if cuda:
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            out = fn(*args)
            e.record()
            e.synchronize()
            times.append(s.elapsed_time(e))
        else:
            t0 = time.perf_counter()
            out = fn(*args)
            times.append((time.perf_counter() - t0) * 1e3)
    t = torch.tensor(times, dtype=torch.float64)
    mean_ms = t.mean().item()
    n_out = out.numel() if hasattr(out, "numel") else 0
    return {
        "latency_ms_mean": mean_ms,
        "latency_ms_min": t.min().item(),
        "latency_ms_p50": t.median().item(),
        "output_elements": n_out,
        "gelem_per_s": n_out / (mean_ms * 1e6) if mean_ms > 0 else float("inf"),
        "iters": iters,
        "warmup": warmup,
        "threads": torch.get_num_threads() if not cuda else None,
        "cpu_count": os.cpu_count(),
    }
