"""A converted model on the device: a transformers GPT-2 (random init from a
config; no checkpoints offline) in bf16 whose c_attn / c_proj / c_fc
projections are replaced by QuaternionLinear (matrix method).  Every
converted layer, at 1 token (decode GEMV) and 16 tokens (tensor-core
kernel), against float64 F.linear with its real block matrix (relative
Frobenius error <= 1e-2); the whole model's logits finite."""


import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def test_converted_gpt2_runs_on_the_device_kernels(qb, cuda):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.GPT2Config(n_layer=2, n_embd=256, n_head=4, n_positions=64, vocab_size=512)
    torch.manual_seed(0)
    model = transformers.GPT2LMHeadModel(cfg).to(cuda, torch.bfloat16).eval()
    _, records = qb.convert_model(model)
    assert len(records) == 8
    for r in records:
        layer = model.get_submodule(r.name)
        block = qb.build_block_matrix(*(getattr(layer, n).double() for n in ("wr", "wi", "wj", "wk")))
        for M in (1, 16):
            x = torch.randn(M, layer.in_features, device=cuda, dtype=torch.bfloat16)
            with torch.no_grad():
                y = layer(x).double()
            want = F.linear(x.double(), block) + layer.bias.detach().double()
            assert ((y - want).norm() / want.norm()).item() <= 1e-2, (r.name, M)
    ids = torch.randint(0, 512, (2, 16), device=cuda)
    with torch.no_grad():
        assert torch.isfinite(model(ids).logits).all()
        assert torch.isfinite(model(ids[:, :1]).logits).all()
    assert qb.device_error(cuda) == 0
