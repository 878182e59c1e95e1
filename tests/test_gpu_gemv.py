"""Parity of the CUDA-core decode kernel (QLIN_ALGO_GEMV) with the oracle.

The decode GEMV gives each output quaternion to one warp, which walks the
whole input width with 16-byte weight loads (8 input quaternions per lane,
256 per chunk, four chunks in flight), and leaves a rank <= 32 LoRA down
projection to this call's prologue kernel, whose programmatic dependent it
is.  The cases cover ragged input widths
(a partial last chunk, more chunks than are in flight), output counts that
leave whole warps and CTAs idle, 1-4 tokens, both 16-bit types, bias and
LoRA ranks 4-32 on their own and together, strided x, static weights, and
agreement with the tensor-core kernel on the same inputs.  Tolerance: 1e-2
relative Frobenius error against the float64 oracle on the same rounded
inputs (fp32 accumulation)."""

import numpy as np
import pytest
import torch

from gpu_helpers import oracle_rows, rel_err, run, to_device

pytestmark = pytest.mark.gpu

ALGO_AUTO, ALGO_SIMT, ALGO_TC, ALGO_GEMV = 0, 1, 2, 3

SHAPES = [
    # (in_features, out_features)
    (32, 4),        # one input chunk, 8 lanes live; one output quaternion
    (96, 20),       # 24 input quaternions; 5 outputs (3 idle warps)
    (128, 512),
    (1024, 1032),   # 258 outputs: a last CTA with 2 live warps
    (4000, 64),     # 1000 input quaternions: a partial fourth chunk
    (5120, 256),    # 1280 input quaternions: five chunks, one refill
    (8192, 64),     # eight chunks: every in-flight slot refilled
    (4096, 4096),   # the decode layer
]


@pytest.mark.parametrize("fin,fout", SHAPES)
@pytest.mark.parametrize("M", [1, 2, 3, 4])
def test_gemv_shapes_bf16(qb, oracle, workloads, cuda, fin, fout, M):
    lay = workloads.make_layer("bf16", M, fin, fout, 31 * M + fin + fout, bias="normal")
    got = run(qb, to_device(lay, cuda), ALGO_GEMV).float().cpu().numpy()
    assert rel_err(oracle, got, oracle_rows(oracle, lay)) <= 1e-2


@pytest.mark.parametrize("fin,fout", [(96, 20), (1024, 1032), (5120, 256)])
@pytest.mark.parametrize("M", [1, 4])
def test_gemv_shapes_f16_no_bias(qb, oracle, workloads, cuda, fin, fout, M):
    lay = workloads.make_layer("f16", M, fin, fout, 7 * M + fin, bias=None)
    got = run(qb, to_device(lay, cuda), ALGO_GEMV).float().cpu().numpy()
    assert rel_err(oracle, got, oracle_rows(oracle, lay)) <= 1e-2


@pytest.mark.parametrize("M,rank,fin,fout", [(1, 32, 4096, 4096), (2, 32, 4096, 512), (3, 8, 2048, 256),
                                             (4, 16, 1024, 64), (1, 24, 160, 36), (2, 4, 96, 8),
                                             (1, 32, 8192, 64), (4, 32, 128, 4)])
def test_gemv_bias_and_lora(qb, oracle, workloads, cuda, M, rank, fin, fout):
    lay = workloads.make_layer("bf16", M, fin, fout, 300 + M + rank, bias="normal", lora_rank=rank,
                               lora_std=0.05)
    d = to_device(lay, cuda)
    want = oracle_rows(oracle, lay)
    got = run(qb, d, ALGO_GEMV).float().cpu().numpy()
    assert rel_err(oracle, got, want) <= 1e-2
    tc = run(qb, d, ALGO_TC).float().cpu().numpy()
    assert rel_err(oracle, tc, want) <= 1e-2


@pytest.mark.parametrize("M,rank,fin", [(1, 32, 4096), (2, 16, 160), (4, 32, 1024), (1, 8, 32)])
def test_gemv_lora_term_alone(qb, oracle, workloads, cuda, M, rank, fin):
    # zero quaternion weights: the output is bias + LoRA only, so the split
    # down projection is checked on its own (160 features over 8 slices of 24
    # elements: the last slices partly or wholly past the input width)
    lay = workloads.make_layer("bf16", M, fin, 256, 950 + M, bias="normal", lora_rank=rank, lora_std=0.05)
    lay.wr, lay.wi, lay.wj, lay.wk = (np.zeros_like(w) for w in lay.weights)
    want = oracle_rows(oracle, lay)
    got = run(qb, to_device(lay, cuda), ALGO_GEMV).float().cpu().numpy()
    assert np.abs(want).max() > 0.05
    assert rel_err(oracle, got, want) <= 1e-2


@pytest.mark.parametrize("rank,offset,width", [(0, 4, 524), (16, 8, 528)])
def test_gemv_strided_input_and_3d_batch(qb, oracle, workloads, cuda, rank, offset, width):
    # rows of x 524 / 528 elements apart, starting 8 / 16 bytes into the buffer
    # (with LoRA the prologue reads x in 16-byte vectors)
    lay = workloads.make_layer("bf16", 2, 512, 128, 41, bias="normal", lora_rank=rank, lora_std=0.05)
    d = to_device(lay, cuda)
    wide = torch.zeros(2, width, dtype=torch.bfloat16, device=cuda)
    wide[:, offset:offset + 512] = d["x"]
    x = wide[:, offset:offset + 512]
    got = qb.linear._forward_impl(x, *d["w"], d["bias"], d["lora_a"], d["lora_b"], d["scale"],
                                  algo=ALGO_GEMV)
    want = oracle_rows(oracle, lay)
    assert rel_err(oracle, got.float().cpu().numpy(), want) <= 1e-2
    y3 = qb.linear._forward_impl(d["x"].reshape(1, 2, 512), *d["w"], d["bias"], d["lora_a"], d["lora_b"],
                                 d["scale"], algo=ALGO_GEMV)
    assert y3.shape == (1, 2, 128)
    assert torch.equal(y3.reshape(2, 128), got)


def test_gemv_static_weights_same_result(qb, workloads, cuda):
    lay = workloads.make_layer("bf16", 1, 4096, 4096, 12, bias="normal", lora_rank=32, lora_std=0.01)
    d = to_device(lay, cuda)
    args = (d["x"], *d["w"], d["bias"], d["lora_a"], d["lora_b"], d["scale"])
    a = qb.linear._forward_impl(*args, algo=ALGO_GEMV)
    b = qb.linear._forward_impl(*args, algo=ALGO_GEMV, static_weights=True)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_gemv_agrees_with_tensor_core_kernel(qb, workloads, cuda):
    # two independent device kernels on the full decode layer: the output
    # difference is fp32 summation order only, well below bf16 resolution
    lay = workloads.make_layer("bf16", 2, 4096, 4096, 13, bias="normal", lora_rank=32, lora_std=0.01)
    d = to_device(lay, cuda)
    g = run(qb, d, ALGO_GEMV).float()
    t = run(qb, d, ALGO_TC).float()
    assert ((g - t).norm() / t.norm()).item() <= 4e-3


def test_auto_picks_gemv_for_decode(qb, cuda):
    for M in (1, 2):
        for rank in (0, 32):
            p = qb._lib.plan(torch.bfloat16, M, 1024, 1024, rank)
            assert p["algo"] == "gemv" and p["split_k"] == 1, (M, rank, p)
            assert p["launches"] == (2 if rank else 1), (M, rank, p)  # LoRA: the prologue first
    # a layer too wide for one wave of the decode kernel keeps the tensor-core kernel
    assert qb._lib.plan(torch.bfloat16, 1, 1280, 6912, 0)["algo"] == "tcgen05"
    # more tokens, a rank above 32 or fp32 keep the other kernels
    assert qb._lib.plan(torch.bfloat16, 3, 1024, 1024, 0)["algo"] == "tcgen05"
    assert qb._lib.plan(torch.bfloat16, 1, 1024, 1024, 64)["algo"] == "tcgen05"
    assert qb._lib.plan(torch.float32, 1, 1024, 1024, 0)["algo"] == "simt"


def test_gemv_rejects_what_it_cannot_run(qb, workloads, cuda):
    lay = workloads.make_layer("bf16", 1, 24, 16, 3)  # K_g = 6: not a multiple of 8
    with pytest.raises(RuntimeError, match="alignment"):
        run(qb, to_device(lay, cuda), ALGO_GEMV)
    lay = workloads.make_layer("bf16", 5, 64, 16, 3)  # more than 4 tokens
    with pytest.raises(RuntimeError, match="alignment"):
        run(qb, to_device(lay, cuda), ALGO_GEMV)
    assert qb.device_error(cuda) == 0


def test_gemv_in_a_graph_back_to_back(qb, workloads, cuda):
    lay = workloads.make_layer("bf16", 1, 4096, 4096, 14, bias="normal", lora_rank=32, lora_std=0.01)
    d = to_device(lay, cuda)
    args = (d["x"], *d["w"], d["bias"], d["lora_a"], d["lora_b"], d["scale"])
    want = qb.linear._forward_impl(*args, algo=ALGO_GEMV)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up: the side stream's zeroed workspace exists before capture
        qb.linear._forward_impl(*args, algo=ALGO_GEMV)
    outs = []
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for _ in range(8):
            outs.append(qb.linear._forward_impl(*args, algo=ALGO_GEMV, static_weights=True))
    for _ in range(4):
        graph.replay()
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, want)
    del graph
    assert qb.device_error(cuda) == 0


# ---- LoRA: the down projection from this call's prologue ----

FLAG_ZEROED = 2
COUNTER_BYTES = 4096


def _ptr(t):
    return None if t is None else t.data_ptr()


def _call_gemv(qb, d, y, M, K_g, N_g, rank, ws, flags):
    lib = qb._lib.load()
    n = qb._lib.workspace_size(d["x"].dtype, M, K_g, N_g, rank)
    return lib.qlin_forward_ex(qb._lib.dtype_code(d["x"].dtype), _ptr(d["x"]), 4 * K_g,
                               *(_ptr(w) for w in d["w"]), K_g, _ptr(d["bias"]), _ptr(d["lora_a"]),
                               _ptr(d["lora_b"]), rank, float(d["scale"]), _ptr(y), 4 * N_g, M, K_g, N_g,
                               _ptr(ws), n if ws is not None else 0, ALGO_GEMV, flags,
                               qb._lib.stream_handle(d["x"].device))


@pytest.mark.parametrize("M,fin,fout,rank", [(1, 4096, 4096, 32), (2, 1024, 512, 16), (1, 160, 36, 8),
                                             (4, 2048, 256, 32), (3, 8192, 1024, 24), (1, 256, 16384, 8)])
def test_gemv_lora_repeatable_on_any_workspace(qb, oracle, workloads, cuda, M, fin, fout, rank):
    # LoRA: this call's prologue computes t into the workspace and the decode
    # kernel follows it; a zero-filled and a plain workspace give the same
    # output, call after call, agreeing with the oracle and the tensor-core kernel
    lay = workloads.make_layer("bf16", M, fin, fout, 700 + M + rank, bias="normal", lora_rank=rank,
                               lora_std=0.05)
    d = to_device(lay, cuda)
    K_g, N_g = fin // 4, fout // 4
    ws = torch.zeros(8 << 20, dtype=torch.uint8, device=cuda)
    plain = torch.empty(max(qb._lib.workspace_size(torch.bfloat16, M, K_g, N_g, rank), 1), dtype=torch.uint8,
                        device=cuda)
    y = torch.empty(M, fout, dtype=torch.bfloat16, device=cuda)
    outs = []
    for i in range(4):
        assert _call_gemv(qb, d, y, M, K_g, N_g, rank, ws if i % 2 else plain, FLAG_ZEROED if i % 2 else 0) == 0
        outs.append(y.clone())
    torch.cuda.synchronize()
    assert all(torch.equal(o, outs[0]) for o in outs)
    want = oracle_rows(oracle, lay)
    assert rel_err(oracle, y.float().cpu().numpy(), want) <= 1e-2
    tc = run(qb, d, ALGO_TC).float().cpu().numpy()
    assert rel_err(oracle, tc, want) <= 1e-2
    assert int(ws[:COUNTER_BYTES].count_nonzero()) == 0
    assert qb.device_error(cuda) == 0


def test_gemv_lora_needs_a_workspace(qb, workloads, cuda):
    # t, the prologue's output, lives in the workspace
    lay = workloads.make_layer("bf16", 1, 1024, 1024, 5, bias="normal", lora_rank=16, lora_std=0.05)
    d = to_device(lay, cuda)
    y = torch.empty(1, 1024, dtype=torch.bfloat16, device=cuda)
    assert _call_gemv(qb, d, y, 1, 256, 256, 16, None, 0) == 4  # QLIN_ERR_WORKSPACE
    assert qb.device_error(cuda) == 0


def test_gemv_grid_exchange_in_a_graph(qb, workloads, cuda):
    lay = workloads.make_layer("bf16", 1, 4096, 4096, 15, bias="normal", lora_rank=32, lora_std=0.01)
    d = to_device(lay, cuda)
    K_g = N_g = 1024
    ws = torch.zeros(qb._lib.workspace_size(torch.bfloat16, 1, K_g, N_g, 32), dtype=torch.uint8, device=cuda)
    want = torch.empty(1, 4096, dtype=torch.bfloat16, device=cuda)
    assert _call_gemv(qb, d, want, 1, K_g, N_g, 32, ws, FLAG_ZEROED) == 0
    torch.cuda.synchronize()
    outs = [torch.empty_like(want) for _ in range(8)]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for i, o in enumerate(outs):  # eight calls back to back on one workspace
            assert _call_gemv(qb, d, o, 1, K_g, N_g, 32, ws, FLAG_ZEROED | (i & 1)) == 0
    for _ in range(5):
        graph.replay()
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, want)
    assert int(ws[:COUNTER_BYTES].count_nonzero()) == 0
    del graph
    assert qb.device_error(cuda) == 0
