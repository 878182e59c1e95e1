"""Helpers for the GPU parity tests: move a workload to the device, run it
through the C ABI (qlin_forward_ex via the package's ctypes binding) and
compare with the double-precision oracle."""

from __future__ import annotations

import numpy as np
import torch

TORCH_DTYPE = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}

# Tolerances (relative Frobenius error against the float64 oracle on the same
# rounded inputs): fp32 <= 1e-5, bf16/f16 <= 1e-2 with fp32 accumulation.
REL_TOL = {"f32": 1e-5, "bf16": 1e-2, "f16": 1e-2}


def to_device(lay, device):
    dt = TORCH_DTYPE[lay.dtype]

    def t(a):
        return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(device).to(dt)

    return dict(x=t(lay.x), w=[t(a) for a in lay.weights], bias=t(lay.bias), lora_a=t(lora_a_of(lay)),
                lora_b=t(lay.lora_b), scale=lay.lora_scale)


def lora_a_of(lay):
    return lay.lora_a


def run(qb, d, algo=0):
    lin = qb.linear
    return lin._forward_impl(d["x"], *d["w"], d["bias"], d["lora_a"], d["lora_b"], d["scale"],
                             algo=algo)


def oracle_rows(oracle, lay, rows=None):
    return oracle.forward_rows(lay.x, *lay.weights, bias=lay.bias, lora_a=lay.lora_a,
                               lora_b=lay.lora_b, lora_scale=lay.lora_scale, rows=rows)


def rel_err(oracle, got, want) -> float:
    return oracle.relative_frobenius_error(np.asarray(got, np.float64), want)


def sample_rows(M: int, n: int = 12) -> np.ndarray:
    base = {0, 1, M // 2, M - 1}
    rng = np.random.default_rng(M)
    base.update(int(v) for v in rng.integers(0, M, size=max(0, n - len(base))))
    return np.array(sorted(r for r in base if 0 <= r < M), dtype=np.int64)
