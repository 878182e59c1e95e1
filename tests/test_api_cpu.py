"""Host-side behaviour of the package on CPU: the reference's packing
contract, its error classes, module construction, LoRA bookkeeping, and the
refusal to compute on CPU tensors (there is no CPU path)."""

import pytest
import torch
import torch.nn as nn


# ---- packing (reference tests/test_matrix_equivalence.py:32-68) ----

@pytest.mark.parametrize("shape", [(4,), (8,), (2, 12), (2, 3, 16), (1, 1, 4)])
def test_pack_roundtrip(qb, shape):
    x = torch.randn(*shape)
    q = qb.pack_real_to_quaternion(x)
    assert q.shape == (*shape[:-1], shape[-1] // 4, 4)
    assert torch.equal(qb.unpack_quaternion_to_real(q), x)


def test_pack_channel_order_is_r_i_j_k(qb, golden):
    q = qb.pack_real_to_quaternion(torch.arange(8, dtype=torch.float64))
    assert torch.equal(q, torch.from_numpy(golden["pack_order"]))
    r, i, j, k = qb.split_components(q)
    assert torch.equal(r, torch.tensor([0.0, 4], dtype=torch.float64))
    assert torch.equal(k, torch.tensor([3.0, 7], dtype=torch.float64))


def test_split_pack_components_roundtrip(qb):
    q = torch.randn(5, 3, 4)
    assert torch.equal(qb.pack_components(*qb.split_components(q)), q)


@pytest.mark.parametrize("bad", [1, 2, 3, 5, 6, 7, 9])
def test_invalid_hidden_dim_raises(qb, bad):
    with pytest.raises(ValueError):
        qb.pack_real_to_quaternion(torch.randn(bad))


def test_block_matrix_matches_reference(qb, golden):
    w = [torch.from_numpy(a) for a in golden["block_16x24_w"]]
    assert torch.equal(qb.build_block_matrix(*w), torch.from_numpy(golden["block_16x24"]))


def test_block_matrix_rejects_bad_weights(qb):
    with pytest.raises(ValueError):
        qb.build_block_matrix(torch.zeros(2, 3), torch.zeros(2, 3), torch.zeros(2, 3), torch.zeros(3))
    with pytest.raises(ValueError):
        qb.build_block_matrix(torch.zeros(2, 3), torch.zeros(2, 3), torch.zeros(2, 3), torch.zeros(3, 2))


# ---- module construction (reference linear.py:75-163) ----

def test_invalid_linear_features_raise(qb):
    with pytest.raises(ValueError):
        qb.QuaternionLinear(in_features=10, out_features=8)
    with pytest.raises(ValueError):
        qb.QuaternionLinear(in_features=8, out_features=10)


def test_parameter_count_is_quarter_and_names(qb):
    layer = qb.QuaternionLinear(64, 32, bias=True)
    assert sum(p.numel() for p in (layer.wr, layer.wi, layer.wj, layer.wk)) == 64 * 32 // 4
    assert set(layer.state_dict()) == {"wr", "wi", "wj", "wk", "bias"}
    assert (layer.in_groups, layer.out_groups) == (16, 8)
    assert "bias=True" in layer.extra_repr()
    bound = 1.0 / 64 ** 0.5
    assert float(layer.wr.abs().max()) <= bound


def test_from_real_block_matrix_roundtrip(qb):
    g = torch.Generator().manual_seed(0)
    w = [torch.randn(4, 6, generator=g) for _ in range(4)]
    block = qb.build_block_matrix(*w)
    layer = qb.QuaternionLinear.from_real_block_matrix(block, bias=torch.ones(16))
    for got, want in zip((layer.wr, layer.wi, layer.wj, layer.wk), w):
        assert torch.equal(got, want)
    assert torch.equal(layer.real_block_matrix(), block)


# ---- error classes of the functional entry points ----

def _w(og, ig, dtype=torch.float32):
    return [torch.randn(og, ig, dtype=dtype) for _ in range(4)]


@pytest.mark.parametrize("fn_name", ["quaternion_linear", "quaternion_linear_naive",
                                     "quaternion_linear_planar"])
def test_feature_dim_mismatch_raises_valueerror(qb, fn_name):
    fn = getattr(qb, fn_name)
    with pytest.raises(ValueError):
        fn(torch.randn(4, 8), *_w(2, 3))        # in_groups 2 vs 3
    with pytest.raises(ValueError):
        fn(torch.randn(5, 10), *_w(4, 3))       # 10 not divisible by 4


def test_unequal_weight_shapes_raise(qb):
    w = _w(2, 3)
    w[2] = torch.randn(3, 3)
    with pytest.raises(ValueError):
        qb.quaternion_linear(torch.randn(4, 12), *w)


def test_cpu_tensors_are_refused(qb):
    with pytest.raises(RuntimeError, match="CUDA"):
        qb.quaternion_linear(torch.randn(4, 12), *_w(2, 3))
    layer = qb.QuaternionLinear(12, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        layer(torch.randn(4, 12))


def test_planar_coefficient_tensor(qb, oracle):
    c = qb.planar_coefficient_tensor(dtype=torch.float64)
    assert c.shape == (4, 4, 4) and int((c != 0).sum()) == 16
    assert torch.equal(c, torch.from_numpy(oracle.planar_coefficient_tensor()))


def test_planar_rejects_foreign_coefficients(qb):
    c = qb.planar_coefficient_tensor()
    c[0, 0, 0] = 2.0
    with pytest.raises(ValueError):
        qb.quaternion_linear_planar(torch.randn(3, 12), *_w(2, 3), coefficient=c)


# ---- LoRA bookkeeping (reference tests/test_lora.py) ----

def test_lora_scale_frozen_and_shapes(qb):
    base = qb.QuaternionLinear(24, 16, bias=True)
    layer = qb.LoRAQuaternionLinear(base, rank=8, alpha=32)
    assert layer.scale == 4.0
    assert qb.LoRAQuaternionLinear(qb.QuaternionLinear(24, 16), rank=16).scale == 2.0
    for name, p in layer.named_parameters():
        assert p.requires_grad == ("lora_" in name)
    assert layer.lora_A.shape == (8, 24) and layer.lora_B.shape == (16, 8)
    assert torch.count_nonzero(layer.lora_B) == 0
    assert layer.bias is base.bias
    with pytest.raises(ValueError):
        qb.LoRAQuaternionLinear(base, rank=0)


def test_inject_and_count(qb):
    model = nn.Sequential(qb.QuaternionLinear(24, 16), nn.ReLU(), qb.QuaternionLinear(16, 8))
    wrapped = qb.inject_lora(model, rank=4)
    assert wrapped == ["0", "2"]
    assert isinstance(model[0], qb.LoRAQuaternionLinear)
    qb.mark_only_lora_trainable(model)
    assert qb.count_trainable(model) == (4 * 24 + 16 * 4) + (4 * 16 + 8 * 4)
    assert len(list(qb.lora_parameters(model))) == 4


# ---- sharding arithmetic ----

@pytest.mark.parametrize("og,G", [(6912, 8), (6912, 1), (10, 4), (3, 8), (256, 2)])
def test_shard_bounds_cover_rows(qb, og, G):
    seen = []
    for r in range(G):
        b, e, n = qb.shard_bounds(og, G, r)
        assert n == -(-og // G) and 0 <= e - b <= n
        seen.extend(range(b, e))
    assert seen == list(range(og))


def test_shard_bounds_rejects_bad_rank(qb):
    with pytest.raises(ValueError):
        qb.shard_bounds(8, 2, 2)
