"""Pin the CPU oracle to the reference: every golden vector in
tests/golden/golden.npz was produced by the reference's own code
(tests/golden/make_golden.py); the oracle must reproduce them.  CPU only."""

import numpy as np
import pytest


def test_hamilton_basis_table(oracle, golden):
    # 1, i, j, k products: i^2 = j^2 = k^2 = -1, ij = k, ji = -k ... (test_hamilton.py:19-40)
    e = np.eye(4)
    table = np.stack([np.stack([oracle.hamilton_product(e[a], e[b]) for b in range(4)])
                      for a in range(4)])
    np.testing.assert_array_equal(table, golden["hamilton_basis"])
    one, i, j, k = e
    np.testing.assert_array_equal(oracle.hamilton_product(i, j), k)
    np.testing.assert_array_equal(oracle.hamilton_product(j, i), -k)
    for b in (i, j, k):
        np.testing.assert_array_equal(oracle.hamilton_product(b, b), -one)


def test_hamilton_random_pairs(oracle, golden):
    got = oracle.hamilton_product(golden["hamilton_a"], golden["hamilton_b"])
    np.testing.assert_allclose(got, golden["hamilton_ab"], rtol=0, atol=1e-15)


def test_hamilton_norm_multiplicative_and_associative(oracle):
    rng = np.random.default_rng(0)
    a, b, c = (rng.standard_normal((32, 4)) for _ in range(3))
    nab = np.linalg.norm(oracle.hamilton_product(a, b), axis=-1)
    np.testing.assert_allclose(nab, np.linalg.norm(a, axis=-1) * np.linalg.norm(b, axis=-1),
                               rtol=1e-12)
    left = oracle.hamilton_product(oracle.hamilton_product(a, b), c)
    right = oracle.hamilton_product(a, oracle.hamilton_product(b, c))
    np.testing.assert_allclose(left, right, rtol=1e-10, atol=1e-10)


def test_hamilton_rejects_bad_last_dim(oracle):
    with pytest.raises(ValueError):
        oracle.hamilton_product(np.zeros(3), np.zeros(3))


@pytest.mark.parametrize("shape", [(4, 4), (8, 12), (12, 8), (16, 16), (16, 24)])
def test_equivalence_against_reference(oracle, golden, shape):
    key = f"eq_{shape[0]}x{shape[1]}"
    x, w, ref = golden[key + "_x"], golden[key + "_w"], golden[key + "_ref"]
    # the reference's three implementations agree with its oracle
    for other in ("_lin", "_naive", "_planar"):
        np.testing.assert_allclose(golden[key + other], ref, rtol=1e-12, atol=1e-12)
    for fn in (oracle.quaternion_linear_reference, oracle.quaternion_linear_naive,
               oracle.quaternion_linear_planar):
        np.testing.assert_allclose(fn(x, *w), ref, rtol=1e-12, atol=1e-12)
    c = oracle.forward_rows(x, *w)  # C oracle on float32 copies of float64 data
    np.testing.assert_allclose(c, ref, rtol=1e-5, atol=1e-5)


def test_block_matrix(oracle, golden):
    w = golden["block_16x24_w"]
    np.testing.assert_array_equal(oracle.build_block_matrix(*w), golden["block_16x24"])
    x = golden["block_16x24_x"]
    np.testing.assert_allclose(oracle.quaternion_linear_reference(x, *w), golden["block_16x24_y"],
                               rtol=1e-12, atol=1e-12)


def test_batched_shapes(oracle, golden):
    x, w = golden["batched_x"], golden["batched_w"]
    got = oracle.quaternion_linear_reference(x, *w)
    assert got.shape == (3, 4, 7, 12)
    np.testing.assert_allclose(got, golden["batched_ref"], rtol=1e-12, atol=1e-12)


def test_coefficient_tensor(oracle):
    c = oracle.planar_coefficient_tensor()
    assert c.shape == (4, 4, 4) and int((c != 0).sum()) == 16


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
def test_dtype_cases(oracle, golden, dt):
    x, w = golden[f"dtype_{dt}_x"], golden[f"dtype_{dt}_w"]
    np.testing.assert_allclose(oracle.forward_rows(x, *w), golden[f"dtype_{dt}_y64"],
                               rtol=1e-12, atol=1e-12)
    # the reference's float32 result is within float32 rounding of the oracle
    np.testing.assert_allclose(golden[f"dtype_{dt}_y32"], golden[f"dtype_{dt}_y64"], atol=1e-5)


def test_lora_golden(oracle, golden):
    x, w = golden["lora_x"], golden["lora_w"]
    base = oracle.quaternion_linear_reference(x, *w) + golden["lora_bias"]
    got = oracle.lora_forward(base, x, golden["lora_a"], golden["lora_b"], float(golden["lora_scale"]))
    np.testing.assert_allclose(got, golden["lora_y"], rtol=1e-12, atol=1e-12)
    # C oracle with bias + LoRA (inputs exactly representable after float32 rounding? no:
    # float64 golden data, so compare at float32 input precision)
    c = oracle.forward_rows(x, *w, bias=golden["lora_bias"], lora_a=golden["lora_a"],
                            lora_b=golden["lora_b"], lora_scale=float(golden["lora_scale"]))
    np.testing.assert_allclose(c, golden["lora_y"], rtol=1e-5, atol=1e-5)


def test_fp32_layer_rows_and_column_sums(oracle, golden, workloads):
    lay = workloads.fp32_1024()
    assert workloads.input_digest(lay) == str(golden["fp32_1024_digest"])
    rows = golden["fp32_1024_rows"]
    got = oracle.forward_rows(lay.x, *lay.weights, bias=lay.bias, rows=rows)
    np.testing.assert_allclose(got, golden["fp32_1024_y_rows"], rtol=1e-10, atol=1e-10)
    full = oracle.forward_rows(lay.x, *lay.weights, bias=lay.bias)
    np.testing.assert_allclose(full.sum(axis=0), golden["fp32_1024_colsum"], rtol=1e-9, atol=1e-9)


def test_decode_shaped_layer_with_bias_and_lora(oracle, golden, workloads):
    lay = workloads.make_layer("bf16", 16, 256, 256, 11, w_std=1.0 / 16.0, bias="normal",
                               lora_rank=32, lora_std=0.01)
    assert workloads.input_digest(lay) == str(golden["decode_small_digest"])
    assert lay.lora_scale == float(golden["decode_small_scale"]) == 2.0
    got = oracle.forward_rows(lay.x, *lay.weights, bias=lay.bias, lora_a=lay.lora_a,
                              lora_b=lay.lora_b, lora_scale=lay.lora_scale)
    np.testing.assert_allclose(got, golden["decode_small_y"], rtol=1e-10, atol=1e-10)


def test_gradient_golden_consistent(oracle, golden):
    # d/dW sum(y^2) = sum_m (2y) (x) conj(x); d/dx = conj(W)^T (2y): restated in numpy
    x, w = golden["grad_x"], golden["grad_w"]
    y = oracle.quaternion_linear_reference(x, *w)
    g = 2.0 * y
    wt = [w[0].T, -w[1].T, -w[2].T, -w[3].T]
    np.testing.assert_allclose(oracle.quaternion_linear_reference(g, *wt), golden["grad_dx"],
                               rtol=1e-10, atol=1e-10)
    M, K_g, N_g = x.shape[0], w.shape[2], w.shape[1]
    gq = g.reshape(M, N_g, 4)
    xq = x.reshape(M, K_g, 4)
    xc = xq * np.array([1, -1, -1, -1])
    dw = np.zeros((N_g, K_g, 4))
    for m in range(M):
        dw += oracle.hamilton_product(gq[m][:, None, :], xc[m][None, :, :])
    np.testing.assert_allclose(np.moveaxis(dw, -1, 0), golden["grad_dw"], rtol=1e-10, atol=1e-10)


def test_bf16_rounding_helper(oracle):
    v = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.0e-3], dtype=np.float32)
    r = oracle.bf16_round(v)
    np.testing.assert_array_equal(oracle.bf16_from_bits(oracle.bf16_bits(r)), r)
    assert r[1] == 1.0  # tie rounds to even
    assert r[2] == np.float32(1.0078125)
