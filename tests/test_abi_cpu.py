"""The C ABI library loads without a GPU, exports every function that
include/qlin_b200.h declares, and validates arguments before touching the
device (so shape errors surface with the reference's error class)."""

import ctypes
import os
import re

import pytest

from conftest import REPO


def _declared_functions():
    src = open(os.path.join(REPO, "include", "qlin_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qlin_\w+)\s*\(", src)))


def test_header_declares_the_entry_points():
    names = _declared_functions()
    for n in ("qlin_forward", "qlin_forward_ex", "qlin_workspace_size", "qlin_gather_columns",
              "qlin_get_device_error", "qlin_status_string"):
        assert n in names


def test_library_exports_every_declared_symbol(qb):
    lib = qb._lib.load()
    raw = ctypes.CDLL(qb._lib.LIB_PATH)
    for name in _declared_functions():
        assert hasattr(raw, name), f"{name} not exported"
    assert set(qb._lib.EXPORTED) <= set(_declared_functions())
    assert lib.qlin_abi_version() >= 100


def test_status_strings(qb):
    for code in range(0, 10):
        assert qb._lib.status_string(code)
    assert qb._lib.status_string(1).startswith("invalid shape")


def test_workspace_size(qb):
    import torch
    # fp32, the 1024 layer at 128 tokens: counters + the fp32 partials of an
    # 8-way K split (16 tiles of 64 tokens x 32 output quaternions)
    assert qb._lib.workspace_size(torch.float32, 128, 256, 256, 0) == 4096 + 8 * 128 * 1024 * 4
    # decode-sized: LoRA t (bf16 and fp32 copies) + split-K partials, no planar x
    ws = qb._lib.workspace_size(torch.bfloat16, 16, 1024, 1024, 32)
    assert ws >= 16 * 32 * 2 + 16 * 32 * 4 + 2 * 8 * 16 * 128 * 16
    # prefill-sized: planar copy of x
    assert qb._lib.workspace_size(torch.bfloat16, 2048, 1024, 2752, 0) >= 4 * 2048 * 1024 * 2
    with pytest.raises(ValueError):
        qb._lib.workspace_size(torch.bfloat16, -1, 1024, 1024, 0)
    # an empty batch needs no split-K partials (and must not divide by zero tiles)
    assert qb._lib.workspace_size(torch.bfloat16, 0, 1024, 1024, 0) == 0
    # every non-empty workspace starts with the 4096 counter bytes of the
    # fused split-K reduction, which nothing else uses
    assert qb._lib.workspace_size(torch.bfloat16, 1, 1024, 1024, 0) >= 4096 + 16 * 16 * 8 * 128 * 16
    # fp32, one token: counters + LoRA t (fp32, 256-byte rounded) + a 5-way K split's partials
    assert qb._lib.workspace_size(torch.float32, 1, 1024, 1024, 8) == 4096 + 256 + 5 * 4096 * 4


def test_shape_errors_are_reported_before_device_use(qb):
    lib = qb._lib.load()
    P = None
    # ld_x < 4*K_g -> QLIN_ERR_SHAPE, no CUDA call needed
    code = lib.qlin_forward(1, 1, 10, 1, 1, 1, 1, 4, P, P, P, 0, 0.0, 1, 16, 2, 4, 4, P, 0, P)
    assert code == 1
    # unknown flag bits are refused (after the shape checks, before any device use)
    code = lib.qlin_forward_ex(1, 1, 16, 1, 1, 1, 1, 4, P, P, P, 0, 0.0, 1, 16, 2, 4, 4, P, 0, 0, 16, P)
    assert code == 8
    # kernel choices: AUTO, SIMT, TC, GEMV (0-3); anything else is refused before device use
    for algo in (-1, 4):
        code = lib.qlin_forward_ex(1, 1, 16, 1, 1, 1, 1, 4, P, P, P, 0, 0.0, 1, 16, 2, 4, 4, P, 0, algo, 0, P)
        assert code == 8, algo
    assert qb._lib.ALGO_GEMV == 3
    # M == 0 is a no-op that succeeds without a device
    code = lib.qlin_forward(1, P, 16, P, P, P, P, 4, P, P, P, 0, 0.0, P, 16, 0, 4, 4, P, 0, P)
    assert code == 0
    # unknown dtype
    code = lib.qlin_forward(7, 1, 16, 1, 1, 1, 1, 4, P, P, P, 0, 0.0, 1, 16, 2, 4, 4, P, 0, P)
    assert code == 2
    # rank > 0 without LoRA pointers
    code = lib.qlin_forward(1, 1, 16, 1, 1, 1, 1, 4, P, P, P, 8, 1.0, 1, 16, 2, 4, 4, P, 0, P)
    assert code == 8
    assert lib.qlin_gather_columns(1, P, P, 0, 1, 1, 1, P) == 1


def test_shape_status_maps_to_valueerror(qb):
    with pytest.raises(ValueError):
        qb._lib.check(1, "x")
    with pytest.raises(RuntimeError):
        qb._lib.check(5, "x")


def test_cpython_binding_matches_ctypes_on_refusals(qb):
    # the per-call path's CPython binding of qlin_forward_ex (built next to
    # the library) gives the same status codes as the ctypes binding
    lib = qb._lib.load()
    fast = qb._lib._fast
    assert fast is not None, "lib/_qlin_call*.so not built"
    P = None
    cases = [
        (1, 1, 10, 1, 1, 1, 1, 4, P, P, P, 0, 0.0, 1, 16, 2, 4, 4, P, 0, 0, 0, P),  # ld_x < 4*K_g
        (1, 1, 16, 1, 1, 1, 1, 4, P, P, P, 0, 0.0, 1, 16, 2, 4, 4, P, 0, 0, 16, P),  # unknown flag
        (7, 1, 16, 1, 1, 1, 1, 4, P, P, P, 0, 0.0, 1, 16, 2, 4, 4, P, 0, 0, 0, P),  # dtype
        (1, P, 16, P, P, P, P, 4, P, P, P, 0, 0.0, P, 16, 0, 4, 4, P, 0, 0, 0, P),  # M == 0
    ]
    for c in cases:
        assert fast.forward_ex(*c) == lib.qlin_forward_ex(*c)
    with pytest.raises(TypeError):
        fast.forward_ex(1, 2, 3)


def test_sharded_nccl_entry_refusals_and_workspace(qb):
    # qlin_sharded_fwd checks its arguments before any device or NCCL use
    lib = qb._lib.load()
    P = None
    comm = ctypes.c_void_p(1)  # never dereferenced: every call below is refused first
    args = (1, 1, 16, 1, 1, 1, 1, 4, P, P, P, 0, 0.0, 1, 32, 2, 4, 4, P, 0, 0)
    assert lib.qlin_sharded_fwd(*args, P, 2, 0, P) == 8          # no communicator
    assert lib.qlin_sharded_fwd(*args, comm, 0, 0, P) == 8       # empty world
    assert lib.qlin_sharded_fwd(*args, comm, 2, 2, P) == 8       # rank outside the world
    bad_ld = (1, 1, 16, 1, 1, 1, 1, 4, P, P, P, 0, 0.0, 1, 31, 2, 4, 4, P, 0, 0)
    assert lib.qlin_sharded_fwd(*bad_ld, comm, 2, 1, P) == 1     # ld_y < world * 4 * N_g
    assert lib.qlin_sharded_fwd(*args, comm, 2, 1, P) == 4       # M > 1 needs the gather buffer
    assert lib.qlin_nccl_comm_init(None, 1, b"\0" * 128, 0) == 8
    assert lib.qlin_nccl_comm_destroy(None) == 8
    assert qb._lib.status_string(9).startswith("NCCL")
    n = ctypes.c_size_t(0)
    assert lib.qlin_sharded_workspace_size(1, 16, 1024, 128, 0, 4, ctypes.byref(n)) == 0
    one = ctypes.c_size_t(0)
    assert lib.qlin_workspace_size(1, 16, 1024, 128, 0, ctypes.byref(one)) == 0
    # the gathered [world, M, 4 N_g] blocks (bf16, 256-byte rounded) ahead of the forward's workspace
    assert n.value == 4 * 16 * 512 * 2 + one.value
    assert lib.qlin_sharded_workspace_size(1, 1, 1024, 128, 0, 4, ctypes.byref(n)) == 0
    assert n.value == qb._lib.workspace_size(__import__("torch").bfloat16, 1, 1024, 128, 0)


def test_nccl_is_found_without_a_gpu(qb):
    # the library resolves NCCL at run time (here: the copy torch loaded) and
    # its bootstrap helper returns a 128-byte unique id, no device needed
    import torch  # noqa: F401  (loads torch's NCCL into the process)
    lib = qb._lib.load()
    uid = ctypes.create_string_buffer(128)
    assert lib.qlin_nccl_unique_id(uid) == 0
    assert any(uid.raw)


def test_host_entry_refusals_and_workspace(qb):
    # qlin_forward_host checks shapes, host pointers and the staging size before any device use
    lib = qb._lib.load()
    P = None
    base = (1, 1, 16, 1, 1, 1, 1, 4, P, P, P, 0, 0.0, 1, 16, 2, 4, 4)
    assert lib.qlin_forward_host(1, 1, 10, 1, 1, 1, 1, 4, P, P, P, 0, 0.0, 1, 16, 2, 4, 4, P, 0, 0, 0, P) == 1
    assert lib.qlin_forward_host(1, P, 16, 1, 1, 1, 1, 4, P, P, P, 0, 0.0, 1, 16, 2, 4, 4, P, 0, 0, 0, P) == 8
    assert lib.qlin_forward_host(*base, P, 0, 0, 0, P) == 4
    assert lib.qlin_forward_host(1, P, 16, P, P, P, P, 4, P, P, P, 0, 0.0, P, 16, 0, 4, 4, P, 0, 0, 0, P) == 0
    n = ctypes.c_size_t(0)
    one = ctypes.c_size_t(0)
    assert lib.qlin_host_workspace_size(1, 3, 256, 128, 0, ctypes.byref(n)) == 0
    assert lib.qlin_workspace_size(1, 3, 256, 128, 0, ctypes.byref(one)) == 0
    # staged x [3, 1024] and y [3, 512] bf16, each rounded to 256 bytes, then the forward's workspace
    assert n.value == 6144 + 3072 + one.value
