"""Factorized and unit-quaternion layers (reference quaternion/factorized.py,
quaternion/unit.py): the oracle's restatement of their weight rebuilds against
golden vectors from the reference, and the package's modules -- parameter
names and counts, rebuilt components, errors -- on the CPU.  The forward runs
on the device kernels only (tests/test_gpu_reparam.py)."""

import numpy as np
import pytest
import torch

MODES = ("independent", "shared_input", "shared_output")
MAGNITUDES = ("per_output", "per_element")


def _factors(golden, mode):
    a, b = golden[f"fact_{mode}_a"], golden[f"fact_{mode}_b"]
    return (list(a) if a.ndim == 3 else a), (list(b) if b.ndim == 3 else b)


@pytest.mark.parametrize("mode", MODES)
def test_oracle_factorized_matches_reference(oracle, golden, mode):
    a, b = _factors(golden, mode)
    w = oracle.factorized_weights(mode, a, b)
    np.testing.assert_allclose(np.stack(w), golden[f"fact_{mode}_w"], rtol=1e-12, atol=1e-14)
    y = oracle.quaternion_linear_reference(golden[f"fact_{mode}_x"], *w) + golden[f"fact_{mode}_bias"]
    np.testing.assert_allclose(y, golden[f"fact_{mode}_y"], rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("magnitude", MAGNITUDES)
def test_oracle_unit_matches_reference(oracle, golden, magnitude):
    k = f"unit_{magnitude}"
    w = oracle.unit_weights(*golden[k + "_v"], golden[k + "_logmag"])
    np.testing.assert_allclose(np.stack(w), golden[k + "_w"], rtol=1e-12, atol=1e-14)
    norm = np.sqrt(sum(c * c for c in w))
    np.testing.assert_allclose(norm, np.broadcast_to(np.exp(golden[k + "_logmag"]), norm.shape), rtol=1e-12)
    y = oracle.quaternion_linear_reference(golden[k + "_x"], *w) + golden[k + "_bias"]
    np.testing.assert_allclose(y, golden[k + "_y"], rtol=1e-10, atol=1e-12)


def _load_factorized(qb, golden, mode):
    layer = qb.FactorizedQuaternionLinear(32, 48, rank=3, mode=mode, bias=True, dtype=torch.float64)
    a, b = _factors(golden, mode)
    with torch.no_grad():
        if mode == "shared_output":
            layer.a.copy_(torch.from_numpy(a))
        else:
            for c, t in zip("rijk", a):
                getattr(layer, f"a_{c}").copy_(torch.from_numpy(t))
        if mode == "shared_input":
            layer.b.copy_(torch.from_numpy(b))
        else:
            for c, t in zip("rijk", b):
                getattr(layer, f"b_{c}").copy_(torch.from_numpy(t))
        layer.bias.copy_(torch.from_numpy(golden[f"fact_{mode}_bias"]))
    return layer


@pytest.mark.parametrize("mode", MODES)
def test_factorized_module_rebuilds_reference_components(qb, golden, mode):
    layer = _load_factorized(qb, golden, mode)
    w = torch.stack(layer.reconstruct_weights()).detach().numpy()
    np.testing.assert_allclose(w, golden[f"fact_{mode}_w"], rtol=1e-12, atol=1e-14)
    for t in layer.reconstruct_weights():
        assert t.shape == (12, 8)


@pytest.mark.parametrize("mode", MODES)
def test_factorized_parameter_names_and_count(qb, oracle, mode):
    layer = qb.FactorizedQuaternionLinear(64, 32, rank=8, mode=mode)
    n = sum(p.numel() for p in layer.parameters())
    assert n == qb.parameter_count(64, 32, 8, mode) == oracle.factorized_parameter_count(64, 32, 8, mode)
    names = set(dict(layer.named_parameters()))
    left = {"a"} if mode == "shared_output" else {f"a_{c}" for c in "rijk"}
    right = {"b"} if mode == "shared_input" else {f"b_{c}" for c in "rijk"}
    assert names == left | right
    assert layer.compression_ratio > 1.0
    assert "mode=" + mode in layer.extra_repr()


def test_factorized_shared_modes_are_smaller_and_errors(qb):
    indep = qb.parameter_count(256, 256, 16, "independent")
    assert qb.parameter_count(256, 256, 16, "shared_input") < indep
    assert qb.parameter_count(256, 256, 16, "shared_output") < indep
    with pytest.raises(ValueError):
        qb.FactorizedQuaternionLinear(8, 8, rank=2, mode="bogus")
    with pytest.raises(ValueError):
        qb.FactorizedQuaternionLinear(8, 8, rank=0)
    with pytest.raises(ValueError):
        qb.FactorizedQuaternionLinear(10, 8, rank=2)
    with pytest.raises(ValueError):
        qb.parameter_count(8, 8, 2, "bogus")


@pytest.mark.parametrize("magnitude", MAGNITUDES)
def test_unit_module_rebuilds_reference_components(qb, golden, magnitude):
    k = f"unit_{magnitude}"
    layer = qb.UnitQuaternionLinear(32, 48, magnitude=magnitude, bias=True, dtype=torch.float64)
    with torch.no_grad():
        for n, t in zip(("vr", "vi", "vj", "vk"), golden[k + "_v"]):
            getattr(layer, n).copy_(torch.from_numpy(t))
        layer.log_magnitude.copy_(torch.from_numpy(golden[k + "_logmag"]))
    w = torch.stack(layer.reconstruct_weights()).detach().numpy()
    np.testing.assert_allclose(w, golden[k + "_w"], rtol=1e-12, atol=1e-14)
    assert layer.log_magnitude.shape == ((12, 1) if magnitude == "per_output" else (12, 8))
    assert set(dict(layer.named_parameters())) == {"vr", "vi", "vj", "vk", "log_magnitude", "bias"}


def test_unit_normalize_and_errors(qb):
    g = torch.Generator().manual_seed(0)
    comps = [torch.randn(4, 6, generator=g, dtype=torch.float64) for _ in range(4)]
    unit = qb.normalize_quaternion(*comps)
    assert torch.allclose(torch.sqrt(sum(c * c for c in unit)), torch.ones(4, 6, dtype=torch.float64), atol=1e-12)
    zero = [torch.zeros(2, 2) for _ in range(4)]
    assert all(torch.equal(c, torch.zeros(2, 2)) for c in qb.normalize_quaternion(*zero))  # eps clamp
    with pytest.raises(ValueError):
        qb.UnitQuaternionLinear(8, 8, magnitude="bogus")
    with pytest.raises(ValueError):
        qb.UnitQuaternionLinear(8, 6)


def test_reparam_forward_has_no_cpu_path(qb):
    with pytest.raises(RuntimeError):
        qb.FactorizedQuaternionLinear(8, 8, rank=2)(torch.randn(2, 8))
    with pytest.raises(RuntimeError):
        qb.UnitQuaternionLinear(8, 8)(torch.randn(2, 8))
