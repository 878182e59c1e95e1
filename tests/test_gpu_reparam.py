"""Factorized and unit-quaternion layers on the device: the rebuilt
components go through the package's kernels (bias fused).  fp32 against the
reference's own float64 outputs (relative Frobenius error <= 1e-5), bf16
against the float64 oracle on the module's bf16 components (<= 1e-2), and
gradients of every parameter against float64 autograd of the real block
matrix."""

import pytest
import torch
import torch.nn.functional as F

from gpu_helpers import rel_err
from test_reparam_cpu import MAGNITUDES, MODES, _load_factorized

pytestmark = pytest.mark.gpu


def _load_unit(qb, golden, magnitude, dtype=torch.float64):
    k = f"unit_{magnitude}"
    layer = qb.UnitQuaternionLinear(32, 48, magnitude=magnitude, bias=True, dtype=dtype)
    with torch.no_grad():
        for n, t in zip(("vr", "vi", "vj", "vk"), golden[k + "_v"]):
            getattr(layer, n).copy_(torch.from_numpy(t))
        layer.log_magnitude.copy_(torch.from_numpy(golden[k + "_logmag"]))
        layer.bias.copy_(torch.from_numpy(golden[k + "_bias"]))
    return layer


def _layers(qb, golden):
    for mode in MODES:
        yield f"fact_{mode}", _load_factorized(qb, golden, mode)
    for magnitude in MAGNITUDES:
        yield f"unit_{magnitude}", _load_unit(qb, golden, magnitude)


def test_fp32_forward_matches_reference(qb, oracle, golden, cuda):
    for key, layer in _layers(qb, golden):
        layer = layer.to(cuda, torch.float32)
        x = torch.from_numpy(golden[key + "_x"]).to(cuda, torch.float32)
        with torch.no_grad():
            y = layer(x).double().cpu().numpy()
        assert rel_err(oracle, y, golden[key + "_y"]) <= 1e-5, key


def test_bf16_forward_matches_oracle(qb, oracle, golden, cuda):
    for key, layer in _layers(qb, golden):
        layer = layer.to(cuda, torch.bfloat16)
        x = torch.from_numpy(golden[key + "_x"]).to(cuda, torch.bfloat16)
        with torch.no_grad():
            y = layer(x).double().cpu().numpy()
            w = [t.double().cpu().numpy() for t in layer.reconstruct_weights()]
        want = oracle.quaternion_linear_reference(x.double().cpu().numpy(), *w) + \
            layer.bias.detach().double().cpu().numpy()
        assert rel_err(oracle, y, want) <= 1e-2, key


def test_gradients_match_block_matrix_autograd(qb, oracle, golden, cuda):
    for key, layer in _layers(qb, golden):
        ref = layer  # float64 on the CPU
        dev = type(layer)(32, 48, **({"rank": 3, "mode": layer.mode} if hasattr(layer, "rank")
                                      else {"magnitude": layer.magnitude}), bias=True).to(cuda)
        dev.load_state_dict({k: v.float() for k, v in ref.state_dict().items()})
        x64 = torch.from_numpy(golden[key + "_x"]).requires_grad_(True)
        g = torch.Generator().manual_seed(3)
        dy = torch.randn(5, 48, generator=g, dtype=torch.float64)
        y_ref = F.linear(x64, qb.build_block_matrix(*ref.reconstruct_weights())) + ref.bias
        (y_ref * dy).sum().backward()
        x32 = x64.detach().float().to(cuda).requires_grad_(True)
        (dev(x32) * dy.float().to(cuda)).sum().backward()
        assert rel_err(oracle, x32.grad.double().cpu().numpy(), x64.grad.numpy()) <= 1e-5, key
        for name, p in ref.named_parameters():
            got = dict(dev.named_parameters())[name].grad
            assert got is not None and torch.isfinite(got).all(), (key, name)
            assert rel_err(oracle, got.double().cpu().numpy(), p.grad.numpy()) <= 1e-4, (key, name)
