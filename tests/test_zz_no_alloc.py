"""The allocation-free entry point, qlin_forward_noalloc.

It exists for callers that cannot allocate device memory where they run the
layer -- code that must not call cudaMalloc mid-stream because that can
synchronise the device, framework plugins handed only their input and output
buffers, runtimes that forbid allocation after start-up.  It must give the
same result as qlin_forward with a caller-provided workspace, on consecutive
calls that reuse its one fixed scratch buffer, and must refuse problems whose
scratch does not fit that buffer.

This file is collected last so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process."""

import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import rel_err, to_device


def _ptr(t):
    return None if t is None else t.data_ptr()


def _noalloc(lib, code, d, y, M, K_g, N_g, rank, stream):
    return lib.qlin_forward_noalloc(code, _ptr(d["x"]), 4 * K_g, *(_ptr(w) for w in d["w"]), K_g,
                                    _ptr(d["bias"]), _ptr(d["lora_a"]), _ptr(d["lora_b"]), rank,
                                    float(d["scale"]), _ptr(y), 4 * N_g, M, K_g, N_g, stream)


def _with_workspace(qb, lib, code, d, y, M, K_g, N_g, rank, stream):
    n = qb._lib.workspace_size(d["x"].dtype, M, K_g, N_g, rank)
    ws = torch.empty(max(n, 256), dtype=torch.uint8, device=d["x"].device)
    return lib.qlin_forward(code, _ptr(d["x"]), 4 * K_g, *(_ptr(w) for w in d["w"]), K_g,
                            _ptr(d["bias"]), _ptr(d["lora_a"]), _ptr(d["lora_b"]), rank,
                            float(d["scale"]), _ptr(y), 4 * N_g, M, K_g, N_g, _ptr(ws), n, stream)


@pytest.mark.gpu
# M = 3 and 4 run the tensor-core kernel's K split summed inside the kernel
# (arrival counters in the scratch): the second call of each pair relies on
# the first leaving those counters at zero.
@pytest.mark.parametrize("M", [1, 3, 4, 16, 100])
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(qb, oracle, workloads, cuda, M):
    lib = qb._lib.load()
    stream = qb._lib.stream_handle(cuda)
    code = qb._lib.dtype_code(torch.bfloat16)
    # decode-shaped layer with bias and LoRA: its scratch holds the LoRA down
    # projection and the split-K partials (M = 100 also the planar copy of x)
    first = workloads.make_layer("bf16", M, 1024, 1024, 31, bias="normal", lora_rank=32, lora_std=0.02)
    second = workloads.make_layer("bf16", M, 1024, 1024, 32, bias="normal", lora_rank=32, lora_std=0.02)
    K_g = N_g = 256
    assert qb._lib.workspace_size(torch.bfloat16, M, K_g, N_g, 32) <= lib_max()
    for lay in (first, second):  # two calls in a row share the fixed scratch
        d = to_device(lay, cuda)
        y_na = torch.empty(M, 4 * N_g, dtype=torch.bfloat16, device=cuda)
        y_ws = torch.empty_like(y_na)
        assert _noalloc(lib, code, d, y_na, M, K_g, N_g, 32, stream) == 0
        assert _with_workspace(qb, lib, code, d, y_ws, M, K_g, N_g, 32, stream) == 0
        torch.cuda.synchronize()
        got = y_na.float().cpu().numpy()
        want = y_ws.float().cpu().numpy()
        assert rel_err(oracle, got, want.astype(np.float64)) <= 1e-2
        assert rel_err(oracle, got, oracle.forward_rows(lay.x, *lay.weights, bias=lay.bias,
                                                         lora_a=lay.lora_a, lora_b=lay.lora_b,
                                                         lora_scale=lay.lora_scale)) <= 1e-2
    assert qb.device_error(cuda) == 0


def lib_max():
    return 8 * 1024 * 1024


def test_noalloc_refuses_problems_beyond_its_scratch(qb):
    lib = qb._lib.load()
    # prefill-sized: the planar copy of x alone is 16 MiB > 8 MiB; refused
    # with QLIN_ERR_WORKSPACE before any device work (no device needed)
    code = lib.qlin_forward_noalloc(1, 1, 4096, 1, 1, 1, 1, 1024, None, None, None, 0, 0.0,
                                    1, 11008, 2048, 1024, 2752, None)
    assert code == 4
    assert "workspace" in qb._lib.status_string(code)
