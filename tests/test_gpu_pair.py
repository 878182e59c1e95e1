"""The CTA-pair prefill kernel (2-SM tcgen05 UMMA, expanded weight rows in
tensor memory, x straight from TMA) against the float64 oracle and against
the one-CTA tensor-core kernel (QLIN_FLAG_NO_PAIR) on the same inputs.

Shapes cover: token counts just above the stacked-tile limit and not a
multiple of the 128-token tile, output widths that leave a partial
256-output tile, input widths whose last 32-quaternion stage is partial,
tiles per CTA pair above one (the persistent loop and both accumulator
buffers), bias and no bias, bf16 and f16 (tolerances of the reference:
1e-2 relative Frobenius error with fp32 accumulation)."""

import numpy as np
import pytest
import torch

from gpu_helpers import oracle_rows, rel_err, sample_rows, to_device

pytestmark = pytest.mark.gpu

ALGO_AUTO, ALGO_TC = 0, 2


def _call(qb, d, M, K_g, N_g, flags, algo=ALGO_AUTO):
    lib = qb._lib.load()
    dt = d["x"].dtype
    y = torch.empty(M, 4 * N_g, dtype=dt, device=d["x"].device)
    n = qb._lib.workspace_size(dt, M, K_g, N_g, 0)
    ws = torch.zeros(max(n, 256), dtype=torch.uint8, device=d["x"].device)
    st = lib.qlin_forward_ex(qb._lib.dtype_code(dt), d["x"].data_ptr(), 4 * K_g, *(w.data_ptr() for w in d["w"]),
                             K_g, None if d["bias"] is None else d["bias"].data_ptr(), None, None, 0, 0.0,
                             y.data_ptr(), 4 * N_g, M, K_g, N_g, ws.data_ptr(), n, algo, flags,
                             qb._lib.stream_handle(d["x"].device))
    qb._lib.check(st, "qlin_forward_ex")
    return y


CASES = [
    # dtype, M, in_features, out_features, bias
    ("bf16", 65, 128, 512, "normal"),
    ("bf16", 128, 32, 256, None),         # one stage, one tile
    ("bf16", 200, 96, 520, "normal"),     # K tail (24 quaternions), partial output tile
    ("bf16", 300, 1056, 1048, "normal"),  # 264 quaternions: partial last stage
    ("bf16", 1000, 768, 2304, None),      # many tiles per pair
    ("f16", 257, 512, 1024, "normal"),
    ("bf16", 2048, 4096, 11008, None),    # the prefill configuration
]


@pytest.mark.parametrize("dtype,M,fin,fout,bias", CASES)
def test_pair_kernel_matches_oracle_and_one_cta_kernel(qb, oracle, workloads, cuda, dtype, M, fin, fout, bias):
    K_g, N_g = fin // 4, fout // 4
    plan = qb._lib.plan({"bf16": torch.bfloat16, "f16": torch.float16}[dtype], M, K_g, N_g, 0)
    assert plan["algo"] == "tcgen05-pair" and plan["launches"] == 1
    lay = workloads.make_layer(dtype, M, fin, fout, 900 + M, bias=bias)
    d = to_device(lay, cuda)
    got = _call(qb, d, M, K_g, N_g, 0).float()
    ref = _call(qb, d, M, K_g, N_g, qb._lib.FLAG_NO_PAIR, ALGO_TC).float()
    torch.cuda.synchronize()
    rows = np.arange(M) if M * fout <= 2_000_000 else sample_rows(M, 8)
    want = oracle_rows(oracle, lay, rows)
    idx = torch.from_numpy(rows).to(cuda)
    assert rel_err(oracle, got[idx].cpu().numpy(), want) <= 1e-2
    assert float(torch.linalg.norm(got - ref) / torch.linalg.norm(ref)) <= 4e-3
    assert qb.device_error(cuda) == 0


def test_pair_kernel_repeated_calls_and_module(qb, oracle, workloads, cuda):
    """Back-to-back calls (the next call's CTAs start while the previous
    call's tail runs) through the module API give identical results."""
    lay = workloads.make_layer("bf16", 384, 512, 1024, 77, bias="normal")
    d = to_device(lay, cuda)
    layer = qb.QuaternionLinear(512, 1024, bias=True, device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        for name, w in zip(("wr", "wi", "wj", "wk"), d["w"]):
            getattr(layer, name).copy_(w)
        layer.bias.copy_(d["bias"])
        outs = [layer(d["x"]) for _ in range(5)]
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    want = oracle_rows(oracle, lay)
    assert rel_err(oracle, outs[0].float().cpu().numpy(), want) <= 1e-2
    assert qb.device_error(cuda) == 0
