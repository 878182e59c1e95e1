"""Seeded synthetic workloads with the shapes and value distributions of the
reference's benchmark configurations.

No dataset is involved anywhere on this path; every input is drawn from a
seeded ``numpy.random.default_rng`` and rounded to the element type the device
computes in, so the oracle and the device see bit-identical values.

Distribution convention: ``N(0, 1/fan)`` is a *variance* (std = 1/sqrt(fan)),
matching the reference's ``randn / sqrt(fan)`` style
(``tests/test_matrix_equivalence.py:19-24``, ``scripts/benchmark_kernel.py:26-35``);
``N(0, 0.02)`` and ``N(0, 0.01)`` are standard deviations.

Layers (``QuaternionLinear(in, out)``, reference ``quaternion/linear.py:75-124``):

* ``fp32_1024``     -- in=out=1024 fp32, x [128, 1024], bias zeros.
* ``decode_4096``   -- in=out=4096 bf16, x [M, 4096] with M in {1, 16}, bias
  N(0, 0.02), LoRA rank 32 (A [32, 4096], B [4096, 32], N(0, 0.01)),
  scale = alpha/rank = 2 (``quaternion/lora.py:43-44``).
* ``prefill_11008`` -- in=4096, out=11008 bf16, x [2048, 4096], no bias.
* ``gpt2_stack``    -- 12 blocks of {768->2304, 768->768, 768->3072, 3072->768}
  bf16, M = 8 * 1024 tokens.
* ``sharded_27648`` -- in=5120, out=27648 bf16, M in {1, 16, 512, 8192}.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


def _bf16_round(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).copy()


def round_to(dtype: str, a: np.ndarray) -> np.ndarray:
    if dtype == "bf16":
        return _bf16_round(a)
    if dtype == "f16":
        return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)
    if dtype == "f32":
        return np.ascontiguousarray(a, dtype=np.float32)
    raise ValueError(f"unknown dtype {dtype!r}")


@dataclass
class LayerInputs:
    """Host copies (float32 arrays holding values on the dtype's grid)."""

    dtype: str
    x: np.ndarray
    wr: np.ndarray
    wi: np.ndarray
    wj: np.ndarray
    wk: np.ndarray
    bias: np.ndarray | None = None
    lora_a: np.ndarray | None = None
    lora_b: np.ndarray | None = None
    lora_scale: float = 0.0
    meta: dict = field(default_factory=dict)

    @property
    def weights(self):
        return (self.wr, self.wi, self.wj, self.wk)

    @property
    def M(self) -> int:
        return self.x.shape[0]

    @property
    def K_g(self) -> int:
        return self.wr.shape[1]

    @property
    def N_g(self) -> int:
        return self.wr.shape[0]


def make_layer(dtype: str, M: int, in_features: int, out_features: int, seed: int,
               w_std: float | None = None, bias: str | None = None, bias_std: float = 0.02,
               lora_rank: int = 0, lora_std: float = 0.01, lora_alpha: float | None = None,
               x_std: float = 1.0) -> LayerInputs:
    """Draw one layer's inputs.  ``bias`` is None, "zeros" or "normal"."""
    if in_features % 4 or out_features % 4:
        raise ValueError("in_features and out_features must be divisible by 4")
    rng = np.random.default_rng(seed)
    kg, ng = in_features // 4, out_features // 4
    if w_std is None:
        w_std = 1.0 / np.sqrt(in_features)
    w = [round_to(dtype, rng.standard_normal((ng, kg), dtype=np.float32) * np.float32(w_std))
         for _ in range(4)]
    x = round_to(dtype, rng.standard_normal((M, in_features), dtype=np.float32) * np.float32(x_std))
    b = None
    if bias == "zeros":
        b = np.zeros(out_features, dtype=np.float32)
    elif bias == "normal":
        b = round_to(dtype, rng.standard_normal(out_features, dtype=np.float32) * np.float32(bias_std))
    la = lb = None
    scale = 0.0
    if lora_rank > 0:
        la = round_to(dtype, rng.standard_normal((lora_rank, in_features), dtype=np.float32)
                      * np.float32(lora_std))
        lb = round_to(dtype, rng.standard_normal((out_features, lora_rank), dtype=np.float32)
                      * np.float32(lora_std))
        alpha = lora_alpha if lora_alpha is not None else 2 * lora_rank
        scale = float(alpha) / lora_rank
    return LayerInputs(dtype, x, *w, bias=b, lora_a=la, lora_b=lb, lora_scale=scale,
                       meta=dict(M=M, in_features=in_features, out_features=out_features,
                                 seed=seed, w_std=float(w_std), lora_rank=lora_rank))


def fp32_1024(seed: int = 1) -> LayerInputs:
    return make_layer("f32", 128, 1024, 1024, seed, w_std=1.0 / 32.0, bias="zeros")


def decode_4096(M: int = 1, seed: int = 2) -> LayerInputs:
    return make_layer("bf16", M, 4096, 4096, seed, w_std=1.0 / 64.0, bias="normal",
                      bias_std=0.02, lora_rank=32, lora_std=0.01)


def prefill_11008(M: int = 2048, seed: int = 3) -> LayerInputs:
    return make_layer("bf16", M, 4096, 11008, seed, w_std=1.0 / 64.0)


GPT2_LINEARS = (("qkv", 768, 2304), ("proj", 768, 768), ("fc", 768, 3072), ("fc2", 3072, 768))


def gpt2_stack(M: int = 8 * 1024, blocks: int = 12, seed: int = 4):
    """Inputs for every quaternion linear of the GPT-2-small-shaped stack."""
    out = []
    for b in range(blocks):
        for li, (name, fin, fout) in enumerate(GPT2_LINEARS):
            lay = make_layer("bf16", M, fin, fout, seed * 1000 + b * 8 + li)
            lay.meta["name"] = f"h{b}.{name}"
            out.append(lay)
    return out


def sharded_27648(M: int = 16, seed: int = 5) -> LayerInputs:
    return make_layer("bf16", M, 5120, 27648, seed, w_std=1.0 / np.sqrt(5120.0))


def input_digest(lay: LayerInputs) -> str:
    """Short content hash of a layer's inputs (pins the generator across hosts)."""
    import hashlib

    h = hashlib.sha256()
    for a in (lay.x, *lay.weights, lay.bias, lay.lora_a, lay.lora_b):
        if a is not None:
            h.update(np.ascontiguousarray(a, dtype=np.float32).tobytes())
    return h.hexdigest()[:16]
