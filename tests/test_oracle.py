"""The CPU oracle against the golden fixtures (tests/golden/make_golden.py) -- CPU only."""
import numpy as np
import pytest

from oracle import oracle as O
from open_rknpu2_lm_infer_b200 import workloads as W


def test_golden_was_generated_without_rounding_disagreements(golden):
    assert int(golden["floor_round_disagreements"]) == 0


@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_kat_codes_and_scales(golden, coracle, impl):
    x = W.kat_input(256, 256)
    if impl == "numpy":
        codes, scales = O.act_quant(x)
    else:
        codes, scales, _ = coracle.act_quant(x)
    np.testing.assert_array_equal(codes, golden["kat_codes"])
    np.testing.assert_array_equal(scales, golden["kat_scales"])


@pytest.mark.parametrize("bits", [4, 8])
def test_kat_linear_bit_exact(golden, coracle, bits):
    codes, scales = W.kat_matrix(bits)
    x = W.kat_input(256, 256)
    y_np, _, _, acc_np = O.linear(codes, scales, x, return_parts=True)
    y_c, acc_c = coracle.linear(codes, scales, x, want_acc=True)
    np.testing.assert_array_equal(acc_np, golden[f"kat_w{bits}_acc"])
    np.testing.assert_array_equal(acc_c, golden[f"kat_w{bits}_acc"])
    np.testing.assert_array_equal(y_np, golden[f"kat_w{bits}_y"])
    np.testing.assert_array_equal(y_c, golden[f"kat_w{bits}_y"])


@pytest.mark.parametrize("n", [32, 64])
def test_narrow_w8_kat(golden, coracle, n):
    w, sw, x = W.narrow_kat(n)
    y = coracle.linear(w, sw, x)
    np.testing.assert_array_equal(y, golden[f"narrow_n{n}_y"])
    c, s, _ = coracle.act_quant(x)
    np.testing.assert_array_equal(c, golden[f"narrow_n{n}_codes"])
    np.testing.assert_array_equal(s, golden[f"narrow_n{n}_scales"])


@pytest.mark.parametrize("name", ["seed_k2560", "seed_k9728", "seed_k8192", "seed_k100"])
def test_seeded_fp16_codes(golden, coracle, name):
    xh = golden[f"{name}_x"]
    c1, s1 = O.act_quant(xh.astype(np.float32))
    c2, s2, _ = coracle.act_quant(xh)            # fp16 widened inside the C oracle
    for c, s in ((c1, s1), (c2, s2)):
        np.testing.assert_array_equal(c, golden[f"{name}_codes"])
        np.testing.assert_array_equal(s, golden[f"{name}_scales"])


def test_odd_shape_linear(golden, coracle):
    y, acc = coracle.linear(golden["odd_w"], golden["odd_sw"], golden["odd_x"], want_acc=True)
    np.testing.assert_array_equal(acc, golden["odd_acc"])
    np.testing.assert_array_equal(y, golden["odd_y"])


@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_edge_cases(golden, coracle, impl):
    x = golden["edge_x"]
    if impl == "numpy":
        c, s = O.act_quant(x)
    else:
        c, s, _ = coracle.act_quant(x)
    np.testing.assert_array_equal(c, golden["edge_codes"])
    np.testing.assert_array_equal(s, golden["edge_scales"])


def test_round_away_is_not_floor_plus_half():
    v = np.float32(0.5) - np.float32(2.0 ** -25)
    assert O.round_away(np.array([v, -v, 0.5, -0.5, 1.5, 2.5], np.float32)).tolist() == \
        [0.0, 0.0, 1.0, -1.0, 2.0, 3.0]


def test_half_even_mode_differs_only_on_ties(coracle):
    x = np.array([[127, 2.5, -2.5, 0.5, 1.5, 3.3]], np.float32)
    ca, _, _ = coracle.act_quant(x, O.ROUND_AWAY)
    ce, _, _ = coracle.act_quant(x, O.ROUND_EVEN)
    assert ca.tolist() == [[127, 3, -3, 1, 2, 3]]
    assert ce.tolist() == [[127, 2, -2, 0, 2, 3]]
    assert O.count_ties(x) == 4


def test_swiglu_matches_reference_expectation(coracle):
    y = np.random.default_rng(0).standard_normal((3, 64)).astype(np.float32) * 4
    mid = coracle.swiglu(y)
    g, u = y[:, :32].astype(np.float64), y[:, 32:].astype(np.float64)
    want = g / (1 + np.exp(-g)) * u
    np.testing.assert_allclose(mid, want, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(O.swiglu(y), mid, rtol=1e-6, atol=1e-6)
