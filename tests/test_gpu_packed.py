"""The packed weight cache: one [out_groups, in_groups, 4] tensor holding the
four components of every weight quaternion side by side (the layout of x),
read by the decode GEMV and the CTA-pair prefill kernel.

* qlin_forward_packed with the packed buffer only (planar pointers NULL)
  against the float64 oracle and against qlin_forward on the planar weights:
  the CTA-pair kernel builds the same expanded operand either way (bit-equal
  results); the GEMV assigns input quaternions to lanes differently (same
  tolerance as every bf16 path);
* a problem only planar kernels serve (16 tokens) is refused without them;
* QuaternionLinear(packed=True): same outputs as the planar module, the
  cache rebuilt after an in-place weight update, state-dict keys unchanged;
  LoRAQuaternionLinear on a packed base."""

import numpy as np
import pytest
import torch

from gpu_helpers import oracle_rows, rel_err, sample_rows, to_device

pytestmark = pytest.mark.gpu

ERR_ALIGN = 3


def _ptr(t):
    return None if t is None else t.data_ptr()


def _packed_call(qb, d, wq, M, K_g, N_g, rank, planar=False):
    lib = qb._lib.load()
    dt = d["x"].dtype
    y = torch.empty(M, 4 * N_g, dtype=dt, device=d["x"].device)
    n = qb._lib.workspace_size(dt, M, K_g, N_g, rank)
    ws = torch.zeros(max(n, 256), dtype=torch.uint8, device=d["x"].device)
    w = d["w"] if planar else (None, None, None, None)
    st = lib.qlin_forward_packed(qb._lib.dtype_code(dt), d["x"].data_ptr(), 4 * K_g, wq.data_ptr(), K_g,
                                 *(_ptr(t) for t in w), K_g, _ptr(d["bias"]), _ptr(d["lora_a"]), _ptr(d["lora_b"]),
                                 rank, float(d["scale"]), y.data_ptr(), 4 * N_g, M, K_g, N_g, ws.data_ptr(), n, 0,
                                 qb._lib.stream_handle(d["x"].device))
    return st, y


def _planar_call(qb, d, M, K_g, N_g, rank):
    lib = qb._lib.load()
    dt = d["x"].dtype
    y = torch.empty(M, 4 * N_g, dtype=dt, device=d["x"].device)
    n = qb._lib.workspace_size(dt, M, K_g, N_g, rank)
    ws = torch.zeros(max(n, 256), dtype=torch.uint8, device=d["x"].device)
    st = lib.qlin_forward(qb._lib.dtype_code(dt), d["x"].data_ptr(), 4 * K_g, *(w.data_ptr() for w in d["w"]), K_g,
                          _ptr(d["bias"]), _ptr(d["lora_a"]), _ptr(d["lora_b"]), rank, float(d["scale"]),
                          y.data_ptr(), 4 * N_g, M, K_g, N_g, ws.data_ptr(), n, qb._lib.stream_handle(d["x"].device))
    assert st == 0
    return y


@pytest.mark.parametrize("dtype,M,fin,fout,rank", [
    ("bf16", 1, 4096, 4096, 32),   # decode GEMV with its LoRA prologue
    ("bf16", 2, 1024, 2048, 0),
    ("f16", 1, 544, 264, 8),       # 136 input quaternions: a partial 256-quaternion chunk
    ("bf16", 300, 1024, 1040, 0),  # CTA-pair kernel, partial tiles
    ("bf16", 2048, 4096, 11008, 0),
])
def test_packed_only_matches_oracle_and_planar(qb, oracle, workloads, cuda, dtype, M, fin, fout, rank):
    lay = workloads.make_layer(dtype, M, fin, fout, 700 + M, bias="normal", lora_rank=rank, lora_std=0.02)
    d = to_device(lay, cuda)
    K_g, N_g = fin // 4, fout // 4
    wq = qb.pack_quaternion_weights(*d["w"])
    assert wq.shape == (N_g, K_g, 4)
    for planar in (False, True):
        st, got = _packed_call(qb, d, wq, M, K_g, N_g, rank, planar=planar)
        assert st == 0
        want_plan = _planar_call(qb, d, M, K_g, N_g, rank)
        torch.cuda.synchronize()
        rows = np.arange(M) if M <= 64 else sample_rows(M, 8)
        want = oracle_rows(oracle, lay, rows)
        assert rel_err(oracle, got.float()[torch.from_numpy(rows).to(cuda)].cpu().numpy(), want) <= 1e-2
        if M > 64:  # the same expanded operand and UMMA sequence
            assert torch.equal(got, want_plan)
        else:
            diff = (got.float() - want_plan.float()).norm() / want_plan.float().norm()
            assert float(diff) <= 4e-3
    assert qb.device_error(cuda) == 0


def test_packed_only_refuses_paths_that_need_planar_weights(qb, workloads, cuda):
    lay = workloads.make_layer("bf16", 16, 1024, 1024, 5, bias="normal")
    d = to_device(lay, cuda)
    wq = qb.pack_quaternion_weights(*d["w"])
    st, _ = _packed_call(qb, d, wq, 16, 256, 256, 0, planar=False)
    assert st == ERR_ALIGN
    st, y = _packed_call(qb, d, wq, 16, 256, 256, 0, planar=True)  # with the planar weights it runs
    assert st == 0
    torch.cuda.synchronize()
    assert qb.device_error(cuda) == 0


@pytest.mark.parametrize("M", [1, 16, 200])
def test_module_packed_cache(qb, oracle, cuda, M):
    torch.manual_seed(3)
    layer = qb.QuaternionLinear(1024, 2048, bias=True, device=cuda, dtype=torch.bfloat16)
    ref = qb.QuaternionLinear(1024, 2048, bias=True, device=cuda, dtype=torch.bfloat16)
    ref.load_state_dict(layer.state_dict())
    layer.packed = True
    assert list(layer.state_dict()) == ["wr", "wi", "wj", "wk", "bias"]
    x = torch.randn(M, 1024, device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        y, y_ref = layer(x), ref(x)
        torch.cuda.synchronize()
        assert float((y.float() - y_ref.float()).norm() / y_ref.float().norm()) <= 4e-3
        first = layer.packed_weights()
        # an in-place update (an optimiser step) invalidates the cache
        layer.wj.mul_(-0.5)
        ref.wj.mul_(-0.5)
        y2, y2_ref = layer(x), ref(x)
        torch.cuda.synchronize()
        assert layer.packed_weights() is not first
        assert torch.equal(layer.packed_weights()[..., 2], layer.wj)
        assert float((y2.float() - y2_ref.float()).norm() / y2_ref.float().norm()) <= 4e-3
        assert not torch.equal(y2, y)
    # with autograd the planar path runs (the cache is an inference cache)
    xg = x.float().to(torch.bfloat16).requires_grad_(True)
    yg = layer(xg)
    yg.float().sum().backward()
    assert xg.grad is not None
    assert qb.device_error(cuda) == 0


def test_lora_on_packed_base(qb, cuda):
    torch.manual_seed(4)
    base = qb.QuaternionLinear(4096, 4096, bias=True, device=cuda, dtype=torch.bfloat16)
    lora = qb.LoRAQuaternionLinear(base, rank=32)
    with torch.no_grad():
        lora.lora_B.normal_(0, 0.02)
    lora.eval()
    x = torch.randn(1, 4096, device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        want = lora(x)
        base.packed = True
        got = lora(x)
    torch.cuda.synchronize()
    assert float((got.float() - want.float()).norm() / want.float().norm()) <= 4e-3
    assert qb.device_error(cuda) == 0
