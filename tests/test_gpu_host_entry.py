"""qlin_forward_host: the layer with x and y in host memory, the copies
enqueued on the stream around the forward (decode-sized, page-locked,
16-byte-word rows: the stage-in / stage-out kernels; otherwise copy-engine
transfers).  Its output must equal
qlin_forward_ex on the same device inputs (the same kernels run on the
staged copies), for one token (GEMV, LoRA), a strided host x and y (row
copies) and a prefill-sized problem (the CTA-pair kernel), with page-locked
and with pageable host buffers; a workspace smaller than the staging is
refused before any device work."""

import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import oracle_rows, rel_err, to_device

pytestmark = pytest.mark.gpu

FLAG_ZEROED = 2
ERR_WORKSPACE = 4


def _ptr(t):
    return None if t is None else t.data_ptr()


@pytest.mark.parametrize("M,fin,fout,rank,pad_x,pad_y,pinned", [
    (1, 4096, 4096, 32, 0, 0, True),
    (3, 1024, 512, 8, 12, 20, True),
    (300, 1024, 1040, 0, 0, 0, True),
    (2, 512, 256, 0, 4, 0, False),
    (2, 512, 256, 16, 8, 8, True),   # strided rows in whole 16-byte words: the stage kernels
])
def test_host_entry_matches_the_device_entry(qb, oracle, workloads, cuda, M, fin, fout, rank, pad_x, pad_y, pinned):
    lib = qb._lib.load()
    lay = workloads.make_layer("bf16", M, fin, fout, 500 + M + rank, bias="normal", lora_rank=rank, lora_std=0.02)
    d = to_device(lay, cuda)
    K_g, N_g = fin // 4, fout // 4
    code = qb._lib.dtype_code(torch.bfloat16)
    stream = qb._lib.stream_handle(cuda)
    ld_x, ld_y = fin + pad_x, fout + pad_y
    x_host = torch.zeros(M, ld_x, dtype=torch.bfloat16)
    x_host[:, :fin] = d["x"].cpu()
    y_host = torch.full((M, ld_y), 3.0, dtype=torch.bfloat16)
    if pinned:
        x_host, y_host = x_host.pin_memory(), y_host.pin_memory()
    n = ctypes.c_size_t(0)
    assert lib.qlin_host_workspace_size(code, M, K_g, N_g, rank, ctypes.byref(n)) == 0
    ws = torch.zeros(n.value, dtype=torch.uint8, device=cuda)
    args = (code, x_host.data_ptr(), ld_x, *(_ptr(w) for w in d["w"]), K_g, _ptr(d["bias"]), _ptr(d["lora_a"]),
            _ptr(d["lora_b"]), rank, float(d["scale"]), y_host.data_ptr(), ld_y, M, K_g, N_g)
    for _ in range(2):  # the second call runs on the counters the first left at zero
        assert lib.qlin_forward_host(*args, _ptr(ws), n.value, 0, FLAG_ZEROED, stream) == 0
        torch.cuda.synchronize()
    # the device entry on the same inputs
    nd = qb._lib.workspace_size(torch.bfloat16, M, K_g, N_g, rank)
    wsd = torch.zeros(max(nd, 256), dtype=torch.uint8, device=cuda)
    want = torch.empty(M, fout, dtype=torch.bfloat16, device=cuda)
    assert lib.qlin_forward_ex(code, _ptr(d["x"]), fin, *(_ptr(w) for w in d["w"]), K_g, _ptr(d["bias"]),
                               _ptr(d["lora_a"]), _ptr(d["lora_b"]), rank, float(d["scale"]), _ptr(want), fout,
                               M, K_g, N_g, _ptr(wsd), nd, 0, FLAG_ZEROED, stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(y_host[:, :fout], want.cpu())
    assert bool((y_host[:, fout:] == 3.0).all())  # the padding of the host rows is not written
    rows = np.arange(min(M, 8))
    assert rel_err(oracle, y_host[:len(rows), :fout].float().numpy(), oracle_rows(oracle, lay, rows)) <= 1e-2
    # too small a workspace: refused before any copy
    assert lib.qlin_forward_host(*args, _ptr(ws), 256, 0, FLAG_ZEROED, stream) == ERR_WORKSPACE
    assert qb.device_error(cuda) == 0



def test_host_entry_reads_fresh_inputs_and_captures_in_a_graph(qb, workloads, cuda):
    # repeated calls read each call's host x and write that call's y; the
    # call's launches (the stage kernels reading and writing host memory
    # through its device mapping) can be captured in the caller's CUDA graph
    lib = qb._lib.load()
    M, fin, fout, rank = 1, 1024, 1024, 16
    lay = workloads.make_layer("bf16", M, fin, fout, 77, bias="normal", lora_rank=rank, lora_std=0.02)
    d = to_device(lay, cuda)
    K_g, N_g = fin // 4, fout // 4
    code = qb._lib.dtype_code(torch.bfloat16)
    x_host = torch.empty(M, fin, dtype=torch.bfloat16).pin_memory()
    y_host = torch.empty(M, fout, dtype=torch.bfloat16).pin_memory()
    n = ctypes.c_size_t(0)
    assert lib.qlin_host_workspace_size(code, M, K_g, N_g, rank, ctypes.byref(n)) == 0
    ws = torch.zeros(n.value, dtype=torch.uint8, device=cuda)

    def call(stream):
        return lib.qlin_forward_host(code, x_host.data_ptr(), fin, *(_ptr(t) for t in d["w"]), K_g, _ptr(d["bias"]),
                                     _ptr(d["lora_a"]), _ptr(d["lora_b"]), rank, float(d["scale"]), y_host.data_ptr(),
                                     fout, M, K_g, N_g, _ptr(ws), n.value, 0, FLAG_ZEROED, stream)

    def device_result():
        want = torch.empty(M, fout, dtype=torch.bfloat16, device=cuda)
        nd = qb._lib.workspace_size(torch.bfloat16, M, K_g, N_g, rank)
        wsd = torch.zeros(max(nd, 256), dtype=torch.uint8, device=cuda)
        assert lib.qlin_forward_ex(code, _ptr(x_host.to(cuda)), fin, *(_ptr(t) for t in d["w"]), K_g,
                                   _ptr(d["bias"]), _ptr(d["lora_a"]), _ptr(d["lora_b"]), rank, float(d["scale"]),
                                   _ptr(want), fout, M, K_g, N_g, _ptr(wsd), nd, 0, FLAG_ZEROED,
                                   qb._lib.stream_handle(cuda)) == 0
        torch.cuda.synchronize()
        return want.cpu()

    g = torch.Generator().manual_seed(5)
    for _ in range(4):
        x_host.copy_(torch.randn(M, fin, generator=g).to(torch.bfloat16))
        assert call(qb._lib.stream_handle(cuda)) == 0
        torch.cuda.synchronize()
        assert torch.equal(y_host, device_result())
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        assert call(s.cuda_stream) == 0
    for _ in range(2):
        x_host.copy_(torch.randn(M, fin, generator=g).to(torch.bfloat16))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(y_host, device_result())
    del graph
    assert qb.device_error(cuda) == 0
