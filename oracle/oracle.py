"""CPU oracle for the quaternion linear forward -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and ``--impl reference`` arm) may import this module, and
only to check device results or as the timed CPU baseline.  The product package never
imports it and has no CPU path of its own.

Each function restates the reference's algorithm in numpy (or calls the C
restatement in ``qlin_oracle.c`` through ctypes) and cites the reference line
it follows.  The restatement is pinned against golden vectors produced by the
reference itself (``tests/golden/make_golden.py``; checked by
``tests/test_oracle_golden.py``).

Packing convention (reference ``quaternion/packing.py:5-25``): a real vector
``[..., 4G]`` is ``G`` quaternions with components ordered (r, i, j, k) on the
last axis; weight components ``W_c`` are ``[out_groups, in_groups]``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libqlin_oracle.so")
_lib = None
_lib_lock = threading.Lock()


# ---------------------------------------------------------------------------
# rounding helpers (inputs are rounded exactly as the device sees them)
# ---------------------------------------------------------------------------


def bf16_round(a) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); float32 out."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    nan = np.isnan(a)
    out = r.astype(np.uint32).view(np.float32).copy()
    out[nan] = np.nan
    return out


def bf16_bits(a) -> np.ndarray:
    """bfloat16 bit patterns (uint16) of float32 values already on the bf16 grid."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    return (a.view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f16_round(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(dtype: str, a) -> np.ndarray:
    if dtype in ("bf16", "bfloat16"):
        return bf16_round(a)
    if dtype in ("f16", "float16"):
        return f16_round(a)
    return np.asarray(a, dtype=np.float32)


# ---------------------------------------------------------------------------
# numpy restatements
# ---------------------------------------------------------------------------


def check_divisible(dim: int, name: str = "dimension") -> int:
    """quaternion/packing.py:45-52."""
    if dim % 4 != 0:
        raise ValueError(f"{name} must be divisible by 4, got {dim}")
    return dim // 4


def hamilton_product(a, b) -> np.ndarray:
    """quaternion/reference.py:31-45; last axis (r, i, j, k), broadcasting."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    if a.shape[-1] != 4 or b.shape[-1] != 4:
        raise ValueError("last dimension of both inputs must be 4")
    ar, ai, aj, ak = np.moveaxis(a, -1, 0)
    br, bi, bj, bk = np.moveaxis(b, -1, 0)
    r = ar * br - ai * bi - aj * bj - ak * bk
    i = ar * bi + ai * br + aj * bk - ak * bj
    j = ar * bj - ai * bk + aj * br + ak * bi
    k = ar * bk + ai * bj - aj * bi + ak * br
    return np.stack((r, i, j, k), axis=-1)


def quaternion_linear_reference(x, wr, wi, wj, wk) -> np.ndarray:
    """quaternion/reference.py:48-86: explicit product per (out, in) pair, summed.

    Materialises ``[..., out_groups, in_groups, 4]``; small shapes only.
    """
    x = np.asarray(x, dtype=np.float64)
    in_groups = check_divisible(x.shape[-1], "in_features")
    wr, wi, wj, wk = (np.asarray(w, dtype=np.float64) for w in (wr, wi, wj, wk))
    if not (wr.shape == wi.shape == wj.shape == wk.shape):
        raise ValueError("all four weight components must share the same shape")
    if wr.shape[1] != in_groups:
        raise ValueError("weight in_groups must match input in_groups")
    xq = x.reshape(*x.shape[:-1], in_groups, 4)[..., None, :, :]
    wq = np.stack((wr, wi, wj, wk), axis=-1)
    yq = hamilton_product(wq, xq).sum(axis=-2)
    return yq.reshape(*yq.shape[:-2], wr.shape[0] * 4)


def quaternion_linear_naive(x, wr, wi, wj, wk, dtype=np.float64) -> np.ndarray:
    """quaternion/planar.py:39-61 (K1): sixteen real products with signs.

    ``dtype`` selects the arithmetic (float64 for checking, float32 for the
    timed CPU baseline, where the sixteen products run as BLAS sgemm calls).
    """
    x = np.asarray(x, dtype=dtype)
    in_groups = check_divisible(x.shape[-1], "in_features")
    wr, wi, wj, wk = (np.asarray(w, dtype=dtype) for w in (wr, wi, wj, wk))
    if wr.shape[1] != in_groups:
        raise ValueError("weight in_groups must match input in_groups")
    lead = x.shape[:-1]
    xq = x.reshape(-1, in_groups, 4)
    xr, xi, xj, xk = (np.ascontiguousarray(xq[..., c]) for c in range(4))
    tr, ti, tj, tk = wr.T, wi.T, wj.T, wk.T
    yr = xr @ tr - xi @ ti - xj @ tj - xk @ tk
    yi = xr @ ti + xi @ tr - xj @ tk + xk @ tj
    yj = xr @ tj + xi @ tk + xj @ tr - xk @ ti
    yk = xr @ tk - xi @ tj + xj @ ti + xk @ tr
    y = np.stack((yr, yi, yj, yk), axis=-1)
    return y.reshape(*lead, wr.shape[0] * 4)


def planar_coefficient_tensor() -> np.ndarray:
    """quaternion/planar.py:64-97: C[a, q, p] with sixteen +-1 entries."""
    c = np.zeros((4, 4, 4))
    c[0, 0, 0], c[0, 1, 1], c[0, 2, 2], c[0, 3, 3] = 1, -1, -1, -1
    c[1, 0, 1], c[1, 1, 0], c[1, 2, 3], c[1, 3, 2] = 1, 1, -1, 1
    c[2, 0, 2], c[2, 1, 3], c[2, 2, 0], c[2, 3, 1] = 1, 1, 1, -1
    c[3, 0, 3], c[3, 1, 2], c[3, 2, 1], c[3, 3, 0] = 1, -1, 1, 1
    return c


def quaternion_linear_planar(x, wr, wi, wj, wk, coefficient=None) -> np.ndarray:
    """quaternion/planar.py:100-129 (K2): one batched contraction then C."""
    x = np.asarray(x, dtype=np.float64)
    in_groups = check_divisible(x.shape[-1], "in_features")
    wr, wi, wj, wk = (np.asarray(w, dtype=np.float64) for w in (wr, wi, wj, wk))
    if wr.shape[1] != in_groups:
        raise ValueError("weight in_groups must match input in_groups")
    lead = x.shape[:-1]
    xf = x.reshape(-1, in_groups, 4).transpose(0, 2, 1)
    wf = np.stack((wr, wi, wj, wk), axis=0)
    p = np.einsum("nqi,poi->nqpo", xf, wf)
    c = planar_coefficient_tensor() if coefficient is None else np.asarray(coefficient, np.float64)
    y = np.einsum("aqp,nqpo->nao", c, p).transpose(0, 2, 1)
    return y.reshape(*lead, wr.shape[0] * 4)


def build_block_matrix(wr, wi, wj, wk) -> np.ndarray:
    """quaternion/packing.py:89-127: the real [4*out_g, 4*in_g] block matrix."""
    wr, wi, wj, wk = (np.asarray(w, dtype=np.float64) for w in (wr, wi, wj, wk))
    rows = [
        np.stack((wr, -wi, -wj, -wk), axis=-1),
        np.stack((wi, wr, -wk, wj), axis=-1),
        np.stack((wj, wk, wr, -wi), axis=-1),
        np.stack((wk, -wj, wi, wr), axis=-1),
    ]
    block = np.stack(rows, axis=-2)  # [og, ig, 4 (row), 4 (col)]
    og, ig = wr.shape
    return block.transpose(0, 2, 1, 3).reshape(og * 4, ig * 4)


def lora_forward(base_y, x, lora_a, lora_b, scale) -> np.ndarray:
    """quaternion/lora.py:60-63: base(x) + scale * ((x A^T) B^T) in float64."""
    x = np.asarray(x, dtype=np.float64)
    t = x @ np.asarray(lora_a, np.float64).T
    return np.asarray(base_y, np.float64) + scale * (t @ np.asarray(lora_b, np.float64).T)


FACTORIZED_MODES = ("independent", "shared_input", "shared_output")


def factorized_parameter_count(in_features: int, out_features: int, rank: int, mode: str) -> int:
    """quaternion/factorized.py:35-49: scalar parameters of a factorized weight."""
    if mode not in FACTORIZED_MODES:
        raise ValueError(f"mode must be one of {FACTORIZED_MODES}, got {mode!r}")
    og, ig = out_features // 4, in_features // 4
    if mode == "independent":
        return 4 * (og * rank + rank * ig)
    if mode == "shared_input":
        return 4 * og * rank + rank * ig
    return og * rank + 4 * rank * ig


def factorized_weights(mode: str, a, b):
    """quaternion/factorized.py:113-124: the dense components from the factors.

    ``a`` and ``b`` are the four left / right factors ([og, rank] / [rank, ig])
    where the mode keeps them per component, or a single shared array."""
    if mode not in FACTORIZED_MODES:
        raise ValueError(f"mode must be one of {FACTORIZED_MODES}, got {mode!r}")
    f64 = lambda t: np.asarray(t, dtype=np.float64)
    if mode == "independent":
        return tuple(f64(ac) @ f64(bc) for ac, bc in zip(a, b))
    if mode == "shared_input":
        return tuple(f64(ac) @ f64(b) for ac in a)
    return tuple(f64(a) @ f64(bc) for bc in b)


def normalize_quaternion(wr, wi, wj, wk, eps: float = 1e-8):
    """quaternion/unit.py:26-34: element-wise projection onto the unit sphere."""
    c = [np.asarray(t, dtype=np.float64) for t in (wr, wi, wj, wk)]
    norm = np.maximum(np.sqrt(c[0] * c[0] + c[1] * c[1] + c[2] * c[2] + c[3] * c[3]), eps)
    return tuple(t / norm for t in c)


def unit_weights(vr, vi, vj, vk, log_magnitude):
    """quaternion/unit.py:77-81: exp(log_magnitude) * the unit quaternion of v
    (log_magnitude [og, 1] per output group or [og, ig] per element)."""
    scale = np.exp(np.asarray(log_magnitude, dtype=np.float64))
    return tuple(t * scale for t in normalize_quaternion(vr, vi, vj, vk))


def project_onto_quaternion(weight):
    """conversion/fit_linear.py:35-61: the least-squares quaternion components
    of a real [4*og, 4*ig] matrix -- for each component, the signed mean of
    the four block entries the block structure (build_block_matrix) gives it."""
    w = np.asarray(weight, dtype=np.float64)
    if w.ndim != 2 or w.shape[0] % 4 or w.shape[1] % 4:
        raise ValueError("weight must be 2D with both dimensions divisible by 4")
    og, ig = w.shape[0] // 4, w.shape[1] // 4
    blocks = w.reshape(og, 4, ig, 4).transpose(0, 2, 1, 3)  # [og, ig, row, col]
    # sign of component c at block entry (row, col): read off the block structure
    basis = [build_block_matrix(*(np.eye(4)[c][k] * np.ones((1, 1)) for k in range(4))) for c in range(4)]
    return tuple((blocks * basis[c][None, None]).sum(axis=(2, 3)) / 4.0 for c in range(4))


def relative_frobenius_error(a, b) -> float:
    """quaternion/metrics.py:38-43: ||a - b|| / ||b|| in float64."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    if a.shape != b.shape:
        raise ValueError(f"shape mismatch: {a.shape} vs {b.shape}")
    d = np.linalg.norm(b)
    if d == 0:
        return float(np.linalg.norm(a))
    return float(np.linalg.norm(a - b) / d)


# ---------------------------------------------------------------------------
# C restatement (double precision, OpenMP), for checking large layers by rows
# ---------------------------------------------------------------------------


def build_c_oracle(force: bool = False) -> str:
    """Compile qlin_oracle.c into oracle/_build/ with the committed Makefile."""
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    with _lib_lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                build_c_oracle()
            lib = ctypes.CDLL(_LIB_PATH)
            P = ctypes.c_void_p
            I64 = ctypes.c_int64
            lib.qlin_oracle_forward.argtypes = [
                P, I64, P, P, P, P, I64, P, P, P, ctypes.c_int, ctypes.c_double,
                P, I64, I64, I64, I64, P, I64, ctypes.c_int,
            ]
            lib.qlin_oracle_forward.restype = ctypes.c_int
            lib.qlin_oracle_threads.restype = ctypes.c_int
            _lib = lib
    return _lib


def c_oracle_threads() -> int:
    return int(_load().qlin_oracle_threads())


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return None if a is None else a.ctypes.data


def forward_rows(x, wr, wi, wj, wk, bias=None, lora_a=None, lora_b=None,
                 lora_scale: float = 0.0, rows=None, threads: int = 0) -> np.ndarray:
    """Double-precision y for the tokens in ``rows`` (all tokens when None).

    ``x`` is ``[M, 4*K_g]``; weights ``[N_g, K_g]``; bias ``[4*N_g]``;
    ``lora_a`` ``[r, 4*K_g]``; ``lora_b`` ``[4*N_g, r]``.  Values should already
    be rounded to the device dtype (``round_to``).  Follows
    reference.py:48-86 + linear.py:120-124 + lora.py:60-63.
    """
    lib = _load()
    x = _f32(x)
    M, K = x.shape
    K_g = check_divisible(K, "in_features")
    w = [_f32(t) for t in (wr, wi, wj, wk)]
    N_g = w[0].shape[0]
    for t in w:
        if t.shape != (N_g, K_g):
            raise ValueError("weight shapes must all be [N_g, K_g]")
    bias = _f32(bias)
    rank = 0
    la = lb = None
    if lora_a is not None:
        la, lb = _f32(lora_a), _f32(lora_b)
        rank = la.shape[0]
    idx = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    n_rows = M if idx is None else idx.shape[0]
    y = np.empty((n_rows, 4 * N_g), dtype=np.float64)
    rc = lib.qlin_oracle_forward(
        _ptr(x), K, _ptr(w[0]), _ptr(w[1]), _ptr(w[2]), _ptr(w[3]), K_g,
        _ptr(bias), _ptr(la), _ptr(lb), rank, float(lora_scale),
        _ptr(y), 4 * N_g, M, K_g, N_g, _ptr(idx), n_rows, int(threads),
    )
    if rc != 0:
        raise ValueError("oracle rejected its arguments")
    return y
