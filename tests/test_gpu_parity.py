"""Parity of the device path with the oracle, through the C ABI.

Every case runs seeded inputs (rounded to the device dtype) through
qlin_forward_ex and compares with the double-precision oracle on the same
inputs: relative Frobenius error <= 1e-5 for fp32 and <= 1e-2 for bf16/f16
(fp32 accumulation), plus the reference tests' own max-abs bounds where they
apply.  Full-size layers are checked on sampled rows (all columns) and against
the second, independent device kernel on the whole output."""

import numpy as np
import pytest
import torch

from gpu_helpers import REL_TOL, oracle_rows, rel_err, run, sample_rows, to_device

pytestmark = pytest.mark.gpu

ALGO_AUTO, ALGO_SIMT, ALGO_TC = 0, 1, 2


def _layer(workloads, dtype, M, fin, fout, seed, bias=None, rank=0):
    return workloads.make_layer(dtype, M, fin, fout, seed, bias=bias, lora_rank=rank)


# ---- the reference kernel tests' case: M=37, og=8, ig=6 (test_kernels.py:30-47) ----

@pytest.mark.parametrize("dt,tol", [("f32", 1e-4), ("bf16", 5e-2), ("f16", 2e-2)])
def test_reference_kernel_case(qb, oracle, golden, cuda, dt, tol):
    x = torch.from_numpy(golden[f"dtype_{dt}_x"]).to(cuda)
    w = [torch.from_numpy(a).to(cuda) for a in golden[f"dtype_{dt}_w"]]
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[dt]
    got = qb.quaternion_linear(x.to(tdt), *[a.to(tdt) for a in w]).float().cpu().numpy()
    assert got.shape == (37, 32)
    assert np.abs(got - golden[f"dtype_{dt}_y32"]).max() < tol
    assert rel_err(oracle, got, golden[f"dtype_{dt}_y64"]) <= REL_TOL[dt]


def test_decode_shaped_golden_from_reference(qb, oracle, golden, workloads, cuda):
    lay = workloads.make_layer("bf16", 16, 256, 256, 11, w_std=1.0 / 16.0, bias="normal",
                               lora_rank=32, lora_std=0.01)
    d = to_device(lay, cuda)
    for algo in (ALGO_TC, ALGO_SIMT):
        got = run(qb, d, algo).float().cpu().numpy()
        assert rel_err(oracle, got, golden["decode_small_y"]) <= 1e-2


# ---- tensor-core path over ragged shapes, both dtypes, bias / LoRA ----

TC_SHAPES = [
    # (M, in_features, out_features)
    (1, 32, 4),
    (1, 128, 512),
    (3, 96, 20),
    (16, 256, 512),
    (17, 128, 1032),
    (37, 160, 260),
    (64, 1024, 512),
    (100, 256, 516),
    (128, 512, 512),
    (129, 128, 1028),
    (300, 384, 768),
]


@pytest.mark.parametrize("M,fin,fout", TC_SHAPES)
@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_tc_path_ragged_shapes(qb, oracle, workloads, cuda, M, fin, fout, dt):
    lay = _layer(workloads, dt, M, fin, fout, seed=M * 7 + fin + fout)
    d = to_device(lay, cuda)
    tc = run(qb, d, ALGO_TC).float().cpu().numpy()
    want = oracle_rows(oracle, lay)
    assert rel_err(oracle, tc, want) <= REL_TOL[dt]
    simt = run(qb, d, ALGO_SIMT).float().cpu().numpy()
    assert rel_err(oracle, simt, want) <= REL_TOL[dt]


@pytest.mark.parametrize("M,rank", [(1, 8), (5, 16), (16, 32), (20, 24), (32, 32), (1, 64), (33, 8),
                                    (40, 40), (130, 64), (7, 4)])
def test_tc_path_bias_and_lora(qb, oracle, workloads, cuda, M, rank):
    lay = workloads.make_layer("bf16", M, 256, 384, 100 + M, bias="normal", lora_rank=rank,
                               lora_std=0.05)
    d = to_device(lay, cuda)
    want = oracle_rows(oracle, lay)
    for algo in (ALGO_AUTO, ALGO_TC, ALGO_SIMT):
        got = run(qb, d, algo).float().cpu().numpy()
        assert rel_err(oracle, got, want) <= 1e-2, algo


@pytest.mark.parametrize("M,rank,fin", [(1, 32, 4096), (3, 8, 2048), (4, 32, 1024), (2, 16, 160),
                                        (4, 32, 128), (16, 24, 1024), (20, 32, 512), (32, 16, 4096),
                                        (1, 64, 1024)])
def test_lora_term_alone(qb, oracle, workloads, cuda, M, rank, fin):
    # zero quaternion weights: the output is bias + LoRA only, so the down
    # projection is checked on its own against the oracle: on the builder
    # warps' CUDA cores (<= 4 tokens, <= 4 K chunks per split: 160 features
    # also has a ragged last chunk), on the tensor cores (<= 32 tokens), both
    # per K split with every split applying its own partial, or in the
    # prologue kernel (rank 64)
    lay = workloads.make_layer("bf16", M, fin, 512, 900 + M, bias="normal", lora_rank=rank,
                               lora_std=0.05)
    lay.wr, lay.wi, lay.wj, lay.wk = (np.zeros_like(w) for w in lay.weights)
    d = to_device(lay, cuda)
    want = oracle_rows(oracle, lay)
    got = run(qb, d, ALGO_TC).float().cpu().numpy()
    assert np.abs(want).max() > 0.05
    assert rel_err(oracle, got, want) <= 1e-2


@pytest.mark.parametrize("M", [1, 7, 33, 128])
def test_fp32_path(qb, oracle, workloads, cuda, M):
    lay = workloads.make_layer("f32", M, 256, 260, 500 + M, bias="normal", lora_rank=8, lora_std=0.1)
    got = run(qb, to_device(lay, cuda)).cpu().numpy()
    assert rel_err(oracle, got, oracle_rows(oracle, lay)) <= 1e-5


def test_tc_path_rejects_unaligned(qb, workloads, cuda):
    lay = _layer(workloads, "bf16", 4, 24, 16, seed=1)  # K_g = 6: no TMA path
    with pytest.raises(RuntimeError, match="alignment"):
        run(qb, to_device(lay, cuda), ALGO_TC)
    got = run(qb, to_device(lay, cuda), ALGO_AUTO)  # auto picks the CUDA-core kernel
    assert got.shape == (4, 16)


def test_strided_input_rows(qb, oracle, workloads, cuda):
    lay = _layer(workloads, "bf16", 40, 256, 256, seed=9)
    d = to_device(lay, cuda)
    wide = torch.zeros(40, 512, dtype=torch.bfloat16, device=cuda)
    wide[:, 128:384] = d["x"]
    d["x"] = wide[:, 128:384]  # ld_x = 512, 16-byte aligned offset
    got = run(qb, d).float().cpu().numpy()
    assert rel_err(oracle, got, oracle_rows(oracle, lay)) <= 1e-2


def test_batched_leading_dims(qb, oracle, workloads, cuda):
    lay = _layer(workloads, "bf16", 2 * 5 * 3, 128, 64, seed=4)
    d = to_device(lay, cuda)
    x3 = d["x"].reshape(2, 5, 3, 128)
    y = qb.quaternion_linear(x3, *d["w"])
    assert y.shape == (2, 5, 3, 64)
    assert rel_err(oracle, y.reshape(30, 64).float().cpu().numpy(), oracle_rows(oracle, lay)) <= 1e-2


def test_zero_rows_is_noop(qb, cuda):
    w = [torch.randn(8, 8, device=cuda, dtype=torch.bfloat16) for _ in range(4)]
    y = qb.quaternion_linear(torch.empty(0, 32, device=cuda, dtype=torch.bfloat16), *w)
    assert y.shape == (0, 32)


# ---- the benchmark configurations at full size ----

def test_config_fp32_1024_full(qb, oracle, golden, workloads, cuda):
    lay = workloads.fp32_1024()
    got = run(qb, to_device(lay, cuda)).cpu().numpy()
    want = oracle_rows(oracle, lay)
    assert rel_err(oracle, got, want) <= 1e-5
    rows = golden["fp32_1024_rows"]
    assert rel_err(oracle, got[rows], golden["fp32_1024_y_rows"]) <= 1e-5
    np.testing.assert_allclose(got.astype(np.float64).sum(0), golden["fp32_1024_colsum"], atol=2e-3)


@pytest.mark.parametrize("M", [1, 16])
def test_config_decode_4096_full(qb, oracle, workloads, cuda, M):
    lay = workloads.decode_4096(M)
    d = to_device(lay, cuda)
    want = oracle_rows(oracle, lay)
    got = run(qb, d).float().cpu().numpy()
    assert rel_err(oracle, got, want) <= 1e-2
    simt = run(qb, d, ALGO_SIMT).float().cpu().numpy()
    assert rel_err(oracle, simt, want) <= 1e-2


def test_config_prefill_11008_sampled(qb, oracle, workloads, cuda):
    lay = workloads.prefill_11008()
    d = to_device(lay, cuda)
    got = run(qb, d).float()
    rows = sample_rows(lay.M, 12)
    want = oracle_rows(oracle, lay, rows)
    assert rel_err(oracle, got[torch.from_numpy(rows).to(cuda)].cpu().numpy(), want) <= 1e-2
    # whole-output agreement with the independent CUDA-core kernel
    simt = run(qb, d, ALGO_SIMT).float()
    assert float(torch.linalg.norm(got - simt) / torch.linalg.norm(simt)) <= 1e-2


@pytest.mark.parametrize("li", [0, 1, 2, 3])
def test_config_gpt2_layers_sampled(qb, oracle, workloads, cuda, li):
    lay = workloads.gpt2_stack(blocks=1)[li]
    got = run(qb, to_device(lay, cuda)).float()
    rows = sample_rows(lay.M, 8)
    want = oracle_rows(oracle, lay, rows)
    assert rel_err(oracle, got[torch.from_numpy(rows).to(cuda)].cpu().numpy(), want) <= 1e-2


@pytest.mark.parametrize("M", [1, 16, 512, 8192])
def test_config_sharded_layer_sampled(qb, oracle, workloads, cuda, M):
    lay = workloads.sharded_27648(M)
    d = to_device(lay, cuda)
    got = run(qb, d).float()
    rows = sample_rows(lay.M, 6)
    want = oracle_rows(oracle, lay, rows)
    assert rel_err(oracle, got[torch.from_numpy(rows).to(cuda)].cpu().numpy(), want) <= 1e-2
    if M == 8192:
        # every row: agreement with the independent CUDA-core kernel
        simt = run(qb, d, ALGO_SIMT).float()
        assert float(torch.linalg.norm(got - simt) / torch.linalg.norm(simt)) <= 1e-2


@pytest.mark.parametrize("M", [16, 512])
@pytest.mark.parametrize("G", [2, 4, 8])
def test_config_sharded_layer_every_shard(qb, oracle, workloads, cuda, G, M):
    """The 5120->27648 layer cut into G column shards (6912 / G = 3456, 1728 or
    864 output quaternions per rank; 864 is not a multiple of the 128-row
    tile), each shard run on this GPU as its rank would run it
    (local_forward); the shards side by side equal the oracle."""
    lay = workloads.sharded_27648(M)
    d = to_device(lay, cuda)
    full = qb.QuaternionLinear(5120, 27648, device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        for name, w in zip(("wr", "wi", "wj", "wk"), d["w"]):
            getattr(full, name).copy_(w)
    parts = []
    with torch.no_grad():
        for r in range(G):
            shard = qb.ColumnParallelQuaternionLinear.from_full(full, world_size=G, rank=r)
            assert shard.shard == 6912 // G
            parts.append(shard.local_forward(d["x"])[:, :4 * (shard.end - shard.begin)])
    got = torch.cat(parts, 1).float()
    assert got.shape == (M, 27648)
    rows = sample_rows(lay.M, 4)
    want = oracle_rows(oracle, lay, rows)
    assert rel_err(oracle, got[torch.from_numpy(rows).to(cuda)].cpu().numpy(), want) <= 1e-2
    whole = run(qb, d).float()
    assert float(torch.linalg.norm(got - whole) / torch.linalg.norm(whole)) <= 1e-2


def test_no_device_error_recorded(qb, cuda):
    assert qb.device_error(cuda) == 0
