"""Module-level behaviour on the device: module == functional, fused bias,
LoRA (the reference's exact-equality start, golden outputs), gradients,
CUDA-graph capture, operator interface, and the sharded layer emulated on one
GPU (every shard's kernel + the column-gather kernel)."""

import numpy as np
import pytest
import torch

from gpu_helpers import oracle_rows, rel_err, to_device

pytestmark = pytest.mark.gpu


def test_module_matches_functional_and_bias(qb, cuda):
    torch.manual_seed(0)
    layer = qb.QuaternionLinear(256, 128, bias=True, device=cuda, dtype=torch.bfloat16)
    x = torch.randn(4, 3, 256, device=cuda, dtype=torch.bfloat16)
    y = layer(x)
    want = qb.quaternion_linear(x, layer.wr, layer.wi, layer.wj, layer.wk).float() + layer.bias.float()
    assert y.shape == (4, 3, 128)
    assert torch.allclose(y.float(), want, atol=2e-2, rtol=2e-2)


def test_naive_planar_entry_points_agree(qb, cuda):
    g = torch.Generator().manual_seed(3)
    w = [(torch.randn(32, 64, generator=g) / 16).to(cuda, torch.bfloat16) for _ in range(4)]
    x = torch.randn(20, 256, generator=g).to(cuda, torch.bfloat16)
    a = qb.quaternion_linear(x, *w)
    assert torch.equal(a, qb.quaternion_linear_naive(x, *w))
    assert torch.equal(a, qb.quaternion_linear_planar(x, *w))
    assert torch.equal(a, qb.ops.quaternion_linear_cuda(x, *w))
    assert qb.ops.cuda_kernel_available()


def test_block_matrix_equivalence_on_device(qb, cuda):
    g = torch.Generator().manual_seed(5)
    w = [(torch.randn(16, 24, generator=g) / 5).to(cuda) for _ in range(4)]
    x = torch.randn(9, 96, generator=g).to(cuda)
    block = qb.build_block_matrix(*w)
    got = qb.quaternion_linear(x, *w)
    assert torch.allclose(got, x @ block.t(), atol=1e-5, rtol=1e-5)
    layer = qb.QuaternionLinear.from_real_block_matrix(block)
    assert torch.allclose(layer(x), got, atol=1e-6, rtol=1e-6)


def test_lora_initial_output_equals_base_exactly(qb, cuda):
    torch.manual_seed(0)
    base = qb.QuaternionLinear(256, 128, bias=True, device=cuda, dtype=torch.bfloat16)
    layer = qb.LoRAQuaternionLinear(base, rank=8)
    x = torch.randn(5, 256, device=cuda, dtype=torch.bfloat16)
    assert torch.equal(layer(x), base(x))


def test_lora_matches_reference_golden(qb, oracle, golden, cuda):
    # float64 golden data -> fp32 device path; compare at fp32 input precision
    w = [torch.from_numpy(a).float().to(cuda) for a in golden["lora_w"]]
    base = qb.QuaternionLinear(24, 16, bias=True, device=cuda)
    with torch.no_grad():
        for n, a in zip(("wr", "wi", "wj", "wk"), w):
            getattr(base, n).copy_(a)
        base.bias.copy_(torch.from_numpy(golden["lora_bias"]).float())
    layer = qb.LoRAQuaternionLinear(base, rank=4, alpha=12.0)
    with torch.no_grad():
        layer.lora_A.copy_(torch.from_numpy(golden["lora_a"]).float())
        layer.lora_B.copy_(torch.from_numpy(golden["lora_b"]).float())
    x = torch.from_numpy(golden["lora_x"]).float().to(cuda)
    got = layer(x).detach().cpu().numpy()
    assert np.abs(got - golden["lora_y"]).max() < 1e-5


def test_lora_forward_shape_and_gradients(qb, cuda):
    base = qb.QuaternionLinear(24, 16, bias=True, device=cuda)
    layer = qb.LoRAQuaternionLinear(base, rank=4)
    x = torch.randn(3, 7, 24, device=cuda, requires_grad=True)
    out = layer(x)
    assert out.shape == (3, 7, 16)
    out.sum().backward()
    assert layer.lora_A.grad is not None and layer.lora_B.grad is not None
    assert layer.base.wr.grad is None


def test_gradients_match_reference_golden(qb, golden, cuda):
    x = torch.from_numpy(golden["grad_x"]).float().to(cuda).requires_grad_(True)
    w = [torch.from_numpy(a).float().to(cuda).requires_grad_(True) for a in golden["grad_w"]]
    qb.quaternion_linear(x, *w).pow(2).sum().backward()
    assert np.abs(x.grad.cpu().numpy() - golden["grad_dx"]).max() < 1e-4
    for a, want in zip(w, golden["grad_dw"]):
        assert np.abs(a.grad.cpu().numpy() - want).max() < 1e-4


def test_gradients_tensor_core_path(qb, oracle, cuda):
    g = torch.Generator().manual_seed(11)
    M, K_g, N_g = 64, 64, 32
    x = (torch.randn(M, 4 * K_g, generator=g)).to(cuda, torch.bfloat16).requires_grad_(True)
    w = [(torch.randn(N_g, K_g, generator=g) / 16).to(cuda, torch.bfloat16).requires_grad_(True)
         for _ in range(4)]
    y = qb.quaternion_linear(x, *w)
    gy = torch.randn_like(y)
    y.backward(gy)
    # float64 reference gradients of <gy, y> through the block matrix
    x64 = x.detach().double().cpu()
    w64 = [a.detach().double().cpu() for a in w]
    block = qb.build_block_matrix(*w64)
    g64 = gy.double().cpu()
    dx = (g64 @ block).numpy()
    assert rel_err(oracle, x.grad.float().cpu().numpy(), dx) <= 2e-2
    dblock = g64.t() @ x64
    for c, a in enumerate(w):
        # dW_c collects the signed entries of the block gradient
        want = sum(qb.packing._BLOCK_SIGN[r][q] * dblock[r::4, q::4]
                   for r in range(4) for q in range(4) if qb.packing._BLOCK_COMP[r][q] == c)
        assert rel_err(oracle, a.grad.float().cpu().numpy(), want.numpy()) <= 2e-2


def test_cuda_graph_capture_and_replay(qb, cuda):
    g = torch.Generator().manual_seed(2)
    w = [(torch.randn(256, 256, generator=g) / 32).to(cuda, torch.bfloat16) for _ in range(4)]
    b = torch.randn(1024, generator=g).to(cuda, torch.bfloat16)
    x = torch.randn(16, 1024, generator=g).to(cuda, torch.bfloat16)
    eager = qb.fused_quaternion_linear(x, *w, b)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        qb.fused_quaternion_linear(x, *w, b)  # warm-up on the side stream
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = qb.fused_quaternion_linear(x, *w, b)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_dtype_mismatch_raises(qb, cuda):
    w = [torch.randn(8, 8, device=cuda) for _ in range(4)]
    with pytest.raises(RuntimeError):
        qb.quaternion_linear(torch.randn(2, 32, device=cuda, dtype=torch.bfloat16), *w)
    with pytest.raises(RuntimeError):
        qb.quaternion_linear(torch.randn(2, 32, device=cuda, dtype=torch.float64),
                             *[a.double() for a in w])


def test_benchmark_operator_keys(qb, cuda):
    w = [torch.randn(64, 64, device=cuda, dtype=torch.bfloat16) for _ in range(4)]
    x = torch.randn(16, 256, device=cuda, dtype=torch.bfloat16)
    r = qb.ops.benchmark_operator(qb.ops.naive, (x, *w), warmup=2, iters=3, device=cuda)
    for k in ("latency_ms_mean", "latency_ms_min", "latency_ms_p50", "output_elements", "gelem_per_s"):
        assert k in r
    assert r["output_elements"] == 16 * 256


@pytest.mark.parametrize("G,M", [(2, 1), (4, 16), (8, 37), (3, 5)])
def test_sharded_layer_emulated_on_one_gpu(qb, oracle, workloads, cuda, G, M):
    lay = workloads.make_layer("bf16", M, 512, 1040, 77 + G, bias="normal", lora_rank=16,
                               lora_std=0.05)
    d = to_device(lay, cuda)
    full = qb.QuaternionLinear(512, 1040, bias=True, device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        for n, a in zip(("wr", "wi", "wj", "wk"), d["w"]):
            getattr(full, n).copy_(a)
        full.bias.copy_(d["bias"])
    shards = [qb.ColumnParallelQuaternionLinear.from_full(full, world_size=G, rank=r,
                                                          lora_A=d["lora_a"], lora_B=d["lora_b"],
                                                          lora_scale=d["scale"])
              for r in range(G)]
    n = shards[0].shard
    buf = torch.stack([s.local_forward(d["x"]) for s in shards])  # what all-gather yields
    y = qb.gather_columns(buf, M, 4 * n)[:, :1040]
    assert rel_err(oracle, y.float().cpu().numpy(), oracle_rows(oracle, lay)) <= 1e-2
