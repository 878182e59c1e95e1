"""Single-GPU checks of the column-partitioned path's plumbing.

* qlin_forward_allgather with a world of one (no peers, no barrier) writes
  the same output, at its column offset of a wider buffer, as qlin_forward.
* qlin_ipc_alloc / qlin_ipc_open: a buffer allocated and filled in a child
  process is mapped and read in this one (processes on the same GPU only
  exchange memory here; nothing waits on another process's kernels)."""

import ctypes

import pytest
import torch

from gpu_helpers import to_device

pytestmark = pytest.mark.gpu


def _ptr(t):
    return None if t is None else t.data_ptr()


def test_allgather_world_one_matches_forward(qb, workloads, cuda):
    lib = qb._lib.load()
    code = qb._lib.dtype_code(torch.bfloat16)
    stream = qb._lib.stream_handle(cuda)
    for M, rank in ((1, 32), (16, 0), (200, 8)):
        lay = workloads.make_layer("bf16", M, 1024, 512, 40 + M, bias="normal", lora_rank=rank, lora_std=0.05)
        d = to_device(lay, cuda)
        K_g, N_g = 256, 128
        n = qb._lib.workspace_size(torch.bfloat16, M, K_g, N_g, rank)
        ws = torch.zeros(max(n, 256), dtype=torch.uint8, device=cuda)
        want = torch.empty(M, 512, dtype=torch.bfloat16, device=cuda)
        args = (code, _ptr(d["x"]), 1024, *(_ptr(w) for w in d["w"]), K_g, _ptr(d["bias"]), _ptr(d["lora_a"]),
                _ptr(d["lora_b"]), rank, float(d["scale"]))
        # the fused all-gather runs the tensor-core kernel: compare with the same kernel
        assert lib.qlin_forward_ex(*args, _ptr(want), 512, M, K_g, N_g, _ptr(ws), n, 2, 0, stream) == 0
        wide = torch.zeros(M, 512 * 3, dtype=torch.bfloat16, device=cuda)
        outs = (ctypes.c_void_p * 1)(wide.data_ptr())
        flags = (ctypes.c_void_p * 1)(None)
        ws2 = torch.zeros(max(n, 256), dtype=torch.uint8, device=cuda)
        assert lib.qlin_forward_allgather(*args, M, K_g, N_g, _ptr(ws2), n, 0, 1, 0, outs, 1536, 512, flags,
                                          None, stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(wide[:, 512:1024], want)
        assert int(wide[:, :512].count_nonzero()) == 0 and int(wide[:, 1024:].count_nonzero()) == 0
    # argument checks happen before any device work
    assert lib.qlin_forward_allgather(code, 1, 16, 1, 1, 1, 1, 4, None, None, None, 0, 0.0, 2, 4, 4, None, 0, 0,
                                      9, 0, outs, 16, 0, flags, None, stream) == 8
    assert qb.device_error(cuda) == 0


def _child(q_out, q_in):
    import importlib
    import os
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if repo not in sys.path:
        sys.path.insert(0, repo)
    qb = importlib.import_module("quaternion-based-math-1_b200")
    torch.cuda.set_device(0)
    lib = qb._lib.load()
    p = ctypes.c_void_p()
    h = ctypes.create_string_buffer(64)
    assert lib.qlin_ipc_alloc(4096, ctypes.byref(p), h) == 0
    view = qb.sharded._device_view(p.value, (1024,), torch.int32, torch.device("cuda", 0), None)
    assert int(view.count_nonzero()) == 0  # zero-filled
    view.copy_(torch.arange(1024, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    q_out.put(h.raw)
    q_in.get(timeout=120)  # the parent has read it
    assert lib.qlin_ipc_free(p) == 0


def test_ipc_buffer_between_processes(qb, cuda):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q_out, q_in = ctx.Queue(), ctx.Queue()
    child = ctx.Process(target=_child, args=(q_out, q_in))
    child.start()
    try:
        handle = q_out.get(timeout=120)
        lib = qb._lib.load()
        p = ctypes.c_void_p()
        assert lib.qlin_ipc_open(handle, 0, ctypes.byref(p)) == 0
        view = qb.sharded._device_view(p.value, (1024,), torch.int32, cuda, None)
        got = view.clone()
        torch.cuda.synchronize()
        assert torch.equal(got, torch.arange(1024, dtype=torch.int32, device=cuda))
        assert lib.qlin_ipc_close(p) == 0
        q_in.put(True)
        child.join(timeout=60)
        assert child.exitcode == 0
    finally:
        if child.is_alive():
            child.kill()
