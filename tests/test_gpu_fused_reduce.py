"""The K-split reduction fused into the main kernel (QLIN_FLAG_ZEROED_WORKSPACE).

Decode-sized problems split K over several CTAs per output tile.  On a
zero-filled workspace the last CTA of each tile to finish sums the fp32
partials (an arrival counter in the workspace's first 4096 bytes, reset by
that CTA) instead of a separate reduction kernel.  The sum runs over the same
slots in the same order as the reduction kernel, so results must be
bit-identical with and without the flag; the counters must be back at zero
after every call, whatever sequence of problems shares the workspace."""

import pytest
import torch

from gpu_helpers import rel_err, to_device

pytestmark = pytest.mark.gpu

FLAG_ZEROED = 2
FLAG_NO_CLUSTER = 8  # the workspace reductions, not the cluster reduce-scatter
COUNTER_BYTES = 4096
ALGO_AUTO, ALGO_TC = 0, 2  # the fused reduction is a property of the tensor-core kernel

def _ptr(t):
    return None if t is None else t.data_ptr()

def _call(qb, d, y, M, K_g, N_g, rank, ws, flags, algo=ALGO_TC):
    lib = qb._lib.load()
    n = qb._lib.workspace_size(d["x"].dtype, M, K_g, N_g, rank)
    assert ws is None or ws.numel() >= n
    return lib.qlin_forward_ex(qb._lib.dtype_code(d["x"].dtype), _ptr(d["x"]), 4 * K_g,
                               *(_ptr(w) for w in d["w"]), K_g, _ptr(d["bias"]), _ptr(d["lora_a"]),
                               _ptr(d["lora_b"]), rank, float(d["scale"]), _ptr(y), 4 * N_g, M, K_g,
                               N_g, _ptr(ws), n, algo, flags, qb._lib.stream_handle(d["x"].device))

def _both(qb, workloads, cuda, dtype, M, K, N, seed, rank, bias, zeroed_ws):
    lay = workloads.make_layer(dtype, M, K, N, seed, bias=bias, lora_rank=rank, lora_std=0.02)
    d = to_device(lay, cuda)
    K_g, N_g = K // 4, N // 4
    y_f = torch.empty(M, N, dtype=d["x"].dtype, device=cuda)
    y_r = torch.empty_like(y_f)
    ws_plain = torch.empty(max(qb._lib.workspace_size(d["x"].dtype, M, K_g, N_g, rank), 1),
                           dtype=torch.uint8, device=cuda)
    assert _call(qb, d, y_f, M, K_g, N_g, rank, zeroed_ws, FLAG_ZEROED | FLAG_NO_CLUSTER) == 0
    assert _call(qb, d, y_r, M, K_g, N_g, rank, ws_plain, FLAG_NO_CLUSTER) == 0
    torch.cuda.synchronize()
    return lay, y_f, y_r

@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("M", [1, 2, 3, 4, 5])
@pytest.mark.parametrize("rank,bias", [(0, None), (32, "normal")])
def test_fused_reduction_is_bit_identical(qb, oracle, workloads, cuda, dtype, M, rank, bias):
    K, N = 2048, 1024
    ws = torch.zeros(8 << 20, dtype=torch.uint8, device=cuda)
    lay, y_f, y_r = _both(qb, workloads, cuda, dtype, M, K, N, 100 + M, rank, bias, ws)
    assert torch.equal(y_f, y_r)
    want = oracle.forward_rows(lay.x, *lay.weights, bias=lay.bias, lora_a=lay.lora_a,
                               lora_b=lay.lora_b, lora_scale=lay.lora_scale)
    assert rel_err(oracle, y_f.float().cpu().numpy(), want) <= 1e-2
    assert int(ws[:COUNTER_BYTES].count_nonzero()) == 0
    assert qb.device_error(cuda) == 0

def test_one_zeroed_workspace_serves_a_sequence_of_problems(qb, workloads, cuda):
    # decode, prefill-like and LoRA problems interleaved on one workspace: the
    # larger problems write their scratch past the counter bytes, the small
    # ones keep finding zero counters
    ws = torch.zeros(8 << 20, dtype=torch.uint8, device=cuda)
    seq = [(1, 1024, 1024, 0), (100, 512, 512, 16), (2, 4096, 512, 0), (4, 1024, 4096, 32),
           (1, 1024, 1024, 32), (70, 1024, 256, 0), (3, 2048, 2048, 8), (2, 4096, 4096, 16),
           (1, 1024, 1024, 0)]
    for i, (M, K, N, rank) in enumerate(seq):
        lay, y_f, y_r = _both(qb, workloads, cuda, "bf16", M, K, N, 200 + i, rank, "normal", ws)
        assert torch.equal(y_f, y_r), (M, K, N, rank)
        assert int(ws[:COUNTER_BYTES].count_nonzero()) == 0
        # the automatic choice on the same workspace (the decode kernel, whose
        # LoRA partials meet through the workspace, for 1-2 tokens)
        y_a = torch.empty_like(y_f)
        assert _call(qb, to_device(lay, cuda), y_a, M, K // 4, N // 4, rank, ws, FLAG_ZEROED, ALGO_AUTO) == 0
        torch.cuda.synchronize()
        assert ((y_a.float() - y_r.float()).norm() / y_r.float().norm()).item() <= 4e-3
        assert int(ws[:COUNTER_BYTES].count_nonzero()) == 0
    assert qb.device_error(cuda) == 0

def test_fused_reduction_in_a_graph_and_back_to_back(qb, workloads, cuda):
    lay = workloads.make_layer("bf16", 1, 4096, 4096, 5, bias="normal", lora_rank=0)
    d = to_device(lay, cuda)
    K_g = N_g = 1024
    ws = torch.zeros(qb._lib.workspace_size(torch.bfloat16, 1, K_g, N_g, 0), dtype=torch.uint8,
                     device=cuda)
    want = torch.empty(1, 4096, dtype=torch.bfloat16, device=cuda)
    assert _call(qb, d, want, 1, K_g, N_g, 0, torch.empty_like(ws), 0) == 0
    outs = [torch.empty_like(want) for _ in range(8)]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for o in outs:  # eight calls back to back on one workspace
            assert _call(qb, d, o, 1, K_g, N_g, 0, ws, FLAG_ZEROED) == 0
    for _ in range(5):
        graph.replay()
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o, want)
    assert int(ws[:COUNTER_BYTES].count_nonzero()) == 0
    del graph
    assert qb.device_error(cuda) == 0

def test_plan_counts_the_fused_reduction(qb, cuda):
    # three or four tokens: the K split is summed by the last CTA of each tile
    # on a zero-filled workspace, else by the reduction kernel
    p0 = qb._lib.plan(torch.bfloat16, 3, 1024, 1024, 0, flags=FLAG_NO_CLUSTER)
    p1 = qb._lib.plan(torch.bfloat16, 3, 1024, 1024, 0, flags=FLAG_ZEROED | FLAG_NO_CLUSTER)
    assert p0["split_k"] > 1
    assert p1["launches"] == p0["launches"] - 1 == 1
    # above four tokens the separate reduction kernel stays
    p5 = qb._lib.plan(torch.bfloat16, 5, 1024, 1024, 0, flags=FLAG_ZEROED | FLAG_NO_CLUSTER)
    assert p5["launches"] == 2
    # by default 3..8 tokens sum the split through a cluster: one launch, no workspace use
    for M in (3, 5, 8):
        for rank in (0, 32):
            p = qb._lib.plan(torch.bfloat16, M, 1024, 1024, rank, flags=0)
            assert p["launches"] == 1 and p["split_k"] in (8, 16), (M, rank, p)
    # one or two tokens: the CUDA-core decode kernel, no K split, whatever
    # the flags; one launch, two with LoRA (the down-projection prologue)
    for M in (1, 2):
        for flags in (0, 1, FLAG_ZEROED, 1 | FLAG_ZEROED):
            for rank in (0, 32):
                p = qb._lib.plan(torch.bfloat16, M, 1024, 1024, rank, flags=flags)
                assert p["algo"] == "gemv" and p["split_k"] == 1, (M, flags, rank, p)
                assert p["launches"] == (2 if rank else 1), (M, flags, rank, p)


def test_module_path_keeps_its_workspace_counters_zero(qb, cuda):
    g = torch.Generator().manual_seed(11)
    w = [(torch.randn(256, 256, generator=g) / 32).to(cuda, torch.bfloat16) for _ in range(4)]
    for M in (1, 3, 4, 1):
        x = torch.randn(M, 1024, generator=g).to(cuda, torch.bfloat16)
        y = qb.quaternion_linear(x, *w)
        ref = qb.linear._forward_impl(x, *w, None, None, None, 0.0, algo=qb._lib.ALGO_SIMT)
        torch.cuda.synchronize()
        assert (y.float() - ref.float()).abs().max().item() <= 2e-2 * ref.float().abs().max().item()
    bufs = list(qb._lib._zeroed_ws.values())
    if qb._lib._torch_ext is not None:  # the C++ inference forward keeps its own
        bufs += qb._lib._torch_ext.workspaces()
    assert bufs
    for buf in bufs:
        assert int(buf[:COUNTER_BYTES].count_nonzero()) == 0
    assert qb.device_error(cuda) == 0


@pytest.mark.parametrize("M", [3, 4, 5, 8, 13, 16])
@pytest.mark.parametrize("rank,bias", [(0, None), (32, "normal")])
def test_cluster_reduce_scatter_matches_reduction_kernel(qb, oracle, workloads, cuda, M, rank, bias):
    """Decode tiles of 3..16 tokens: the K split summed through distributed
    shared memory (each CTA of the cluster owns some tokens, receives the
    other splits' partials of them and adds all splits in order) against the
    reduction kernel over the workspace.  Same split count: bit-identical."""
    K, N = 4096, 4096
    lay = workloads.make_layer("bf16", M, K, N, 300 + M, bias=bias, lora_rank=rank, lora_std=0.02)
    d = to_device(lay, cuda)
    K_g, N_g = K // 4, N // 4
    p_c = qb._lib.plan(torch.bfloat16, M, K_g, N_g, rank, flags=0)
    p_r = qb._lib.plan(torch.bfloat16, M, K_g, N_g, rank, flags=FLAG_NO_CLUSTER)
    assert p_c["launches"] == 1 or M > 8  # more tokens: clusters of 16 CTAs when they fit
    y_c = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    y_r = torch.empty_like(y_c)
    ws = torch.empty(max(qb._lib.workspace_size(torch.bfloat16, M, K_g, N_g, rank), 1), dtype=torch.uint8,
                     device=cuda)
    for _ in range(2):  # twice: nothing of the first call may leak into the second
        assert _call(qb, d, y_c, M, K_g, N_g, rank, ws, 0) == 0
        assert _call(qb, d, y_r, M, K_g, N_g, rank, ws, FLAG_NO_CLUSTER) == 0
        torch.cuda.synchronize()
        if p_c["split_k"] == p_r["split_k"]:
            assert torch.equal(y_c, y_r)
        want = oracle.forward_rows(lay.x, *lay.weights, bias=lay.bias, lora_a=lay.lora_a,
                                   lora_b=lay.lora_b, lora_scale=lay.lora_scale)
        assert rel_err(oracle, y_c.float().cpu().numpy(), want) <= 1e-2
    assert qb.device_error(cuda) == 0
