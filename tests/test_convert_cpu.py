"""Model conversion (reference conversion/convert_model.py, matrix method):
the closed-form projection onto the quaternion structure against golden
vectors from the reference, and the replacement of a model's projections by
QuaternionLinear layers -- which modules, which weights -- on the CPU (the
replaced layers' forward is the device kernels', tested elsewhere)."""

import numpy as np
import pytest
import torch
import torch.nn as nn


def test_oracle_projection_matches_reference(oracle, golden):
    got = np.stack(oracle.project_onto_quaternion(golden["proj_w"]))
    np.testing.assert_allclose(got, golden["proj_out"], rtol=0, atol=1e-15)


def test_projection_matches_reference_and_inverts_the_block_matrix(qb, golden):
    got = torch.stack(qb.project_onto_quaternion(torch.from_numpy(golden["proj_w"]))).numpy()
    np.testing.assert_allclose(got, golden["proj_out"], rtol=0, atol=1e-15)
    g = torch.Generator().manual_seed(3)
    w = [torch.randn(5, 7, generator=g, dtype=torch.float64) for _ in range(4)]
    back = qb.project_onto_quaternion(qb.build_block_matrix(*w))
    assert all(torch.allclose(a, b, atol=1e-15) for a, b in zip(back, w))
    with pytest.raises(ValueError):
        qb.project_onto_quaternion(torch.randn(6, 8))
    with pytest.raises(ValueError):
        qb.project_onto_quaternion(torch.randn(8))


class _Attn(nn.Module):
    def __init__(self):
        super().__init__()
        self.q_proj = nn.Linear(16, 16)
        self.v_proj = nn.Linear(16, 8, bias=False)
        self.o_proj = nn.Linear(16, 10)      # 10 outputs: not divisible by 4, kept
        self.scores = nn.Linear(16, 16)      # not a projection name, kept


class _Toy(nn.Module):
    def __init__(self):
        super().__init__()
        self.attn = _Attn()
        self.lm_head = nn.Linear(16, 32)     # never converted


def test_convert_model_replaces_named_projections(qb):
    torch.manual_seed(0)
    model = _Toy().double()
    q_w, q_b, v_w = (p.detach().clone() for p in (model.attn.q_proj.weight, model.attn.q_proj.bias,
                                                   model.attn.v_proj.weight))
    _, records = qb.convert_model(model)
    assert [r.name for r in records] == ["attn.q_proj", "attn.v_proj"]
    assert [r.kind for r in records] == ["q_proj", "v_proj"]
    assert isinstance(model.attn.q_proj, qb.QuaternionLinear) and isinstance(model.attn.v_proj, qb.QuaternionLinear)
    for keep in (model.attn.o_proj, model.attn.scores, model.lm_head):
        assert type(keep) is nn.Linear
    q = model.attn.q_proj
    want = qb.project_onto_quaternion(q_w)
    assert all(torch.equal(getattr(q, n), w) for n, w in zip(("wr", "wi", "wj", "wk"), want))
    assert torch.equal(q.bias, q_b) and q.wr.dtype == torch.float64
    assert model.attn.v_proj.bias is None and model.attn.v_proj.out_features == 8
    err = float((qb.build_block_matrix(*qb.project_onto_quaternion(v_w)) - v_w).norm() / v_w.norm())
    assert abs(records[1].metrics["relative_frobenius_error"] - err) < 1e-12
    with pytest.raises(ValueError):
        qb.convert_model(_Toy(), method="activation")
    with pytest.raises(ValueError):
        qb.convert_model(_Toy(), method="bogus")


def test_convert_gpt2_conv1d_projections(qb):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.GPT2Config(n_layer=2, n_embd=64, n_head=4, n_positions=32, vocab_size=128)
    torch.manual_seed(1)
    model = transformers.GPT2LMHeadModel(cfg).eval()
    originals = {n: m.weight.detach().t().clone() for n, m in model.named_modules()
                 if type(m).__name__ == "Conv1D"}  # Conv1D stores [in, out]
    assert {n.rsplit(".", 1)[-1] for n in originals} == {"c_attn", "c_proj", "c_fc"}
    _, records = qb.convert_model(model)
    assert sorted(r.name for r in records) == sorted(originals)
    kinds = {r.name: r.kind for r in records}
    assert kinds["transformer.h.0.attn.c_attn"] == "qkv_proj"
    assert kinds["transformer.h.0.attn.c_proj"] == "o_proj"
    assert kinds["transformer.h.0.mlp.c_fc"] == "up_proj" and kinds["transformer.h.1.mlp.c_proj"] == "down_proj"
    for name, w in originals.items():
        layer = model.get_submodule(name)
        assert isinstance(layer, qb.QuaternionLinear)
        assert (layer.out_features, layer.in_features) == tuple(w.shape)
        want = qb.project_onto_quaternion(w)
        assert all(torch.allclose(getattr(layer, n).double(), c, atol=1e-7) for n, c in zip(("wr", "wi", "wj", "wk"), want))
    assert isinstance(model.lm_head, nn.Linear)
