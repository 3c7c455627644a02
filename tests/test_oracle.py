"""Pins the CPU oracle (oracle/oracle.c) before any device result is compared against it.

1. Known-answer tests: the golden vectors the reference's own tests hold for these ops (tests/ops/ops_test.cpp,
   tests/nn/rope_test.cpp, tests/nn/qwen_mlp_test.cpp, tests/tensors/tensor_test.cpp), same inputs, same tolerances.
2. The reference's own source code, compiled in place (oracle/_ref): bit-exact agreement on seeded inputs for every
   op whose reference implementation runs without oneDNN.
3. The torch 2.11 fixtures (tests/golden/torch_*.npz), within the op's tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle.oracle import as_float, bf16_to_f32, f32_to_bf16, ulp_distance


def bf16(values):
    return f32_to_bf16(np.asarray(values, dtype=np.float32))


# ---------------------------------------------------------------------------------------------------------------
# 1. Reference known-answer tests
# ---------------------------------------------------------------------------------------------------------------


def test_given_matching_f32_tensors_when_adding_then_elementwise_sum(oracle):
    # tests/ops/ops_test.cpp:47-53
    out = oracle.add(np.array([1, 2, 3, 4], np.float32), np.array([10, 20, 30, 40], np.float32))
    assert out.tolist() == [11.0, 22.0, 33.0, 44.0]


def test_given_matching_bf16_tensors_when_adding_then_elementwise_sum(oracle):
    # tests/ops/ops_test.cpp:229-235
    out = oracle.add(bf16([1, 2, 3, 4]), bf16([10, 20, 30, 40]))
    assert (out == bf16([11, 22, 33, 44])).all()


def test_given_matching_f32_tensors_when_multiplying_then_elementwise_product(oracle):
    # tests/ops/ops_test.cpp:55-61
    out = oracle.mul(np.array([1, 2, 3, 4], np.float32), np.array([10, 20, 30, 40], np.float32))
    assert out.tolist() == [10.0, 40.0, 90.0, 160.0]


def test_given_f32_tensor_when_casting_to_bf16_then_expected_bits(oracle):
    # tests/ops/ops_test.cpp:112-117
    out = oracle.cast(np.array([1.5, -2.25, 0.5, -0.75], np.float32), to_bf16=True)
    assert out.tolist() == [0x3FC0, 0xC010, 0x3F00, 0xBF40]


def test_given_bf16_tensor_when_casting_to_f32_then_expected_values(oracle):
    # tests/ops/ops_test.cpp:119-124
    out = oracle.cast(np.array([0x3FC0, 0xC010, 0x3F00, 0xBF40], np.uint16), to_bf16=False)
    assert out.tolist() == [1.5, -2.25, 0.5, -0.75]


def test_given_float_when_converting_through_bf16_then_round_trips(oracle):
    # tests/tensors/tensor_test.cpp:61-65
    assert bf16_to_f32(f32_to_bf16(np.array([1.5], np.float32)))[0] == 1.5


def test_given_torch_oracle_bf16_tensor_when_applying_silu_then_expected_values(oracle):
    # tests/ops/ops_test.cpp:260-278 (tolerance 1e-6)
    x = bf16([-1.5, -0.25, 0.5, 2.0, 3.0, -4.5, 1.25, 0.75])
    expected = [-0.2734375, -0.109375, 0.310546875, 1.7578125, 2.859375, -0.0495605469, 0.97265625, 0.5078125]
    np.testing.assert_allclose(bf16_to_f32(oracle.silu(x)), expected, atol=1e-6, rtol=0)


def test_given_torch_oracle_bf16_tensor_when_applying_softmax_then_expected_values(oracle):
    # tests/ops/ops_test.cpp:280-298
    x = bf16([1.0, -2.5, 3.25, 0.75, 4.5, 0.5, -1.75, 2.25]).reshape(2, 4)
    expected = [0.0883789062, 0.0026702881, 0.83984375, 0.0688476562, 0.88671875, 0.0162353516, 0.0017166138,
                0.09375]
    np.testing.assert_allclose(bf16_to_f32(oracle.softmax_last_dim(x)).ravel(), expected, atol=1e-6, rtol=0)


def test_given_attention_scores_when_applying_scaled_causal_softmax_then_future_masked(oracle):
    # tests/ops/ops_test.cpp:300-310
    x = np.array([1.0, 1000.0, 3.0, 4.0], np.float32).reshape(1, 2, 2)
    out = oracle.scaled_causal_softmax(x, 1.0)
    np.testing.assert_allclose(out.ravel(), [1.0, 0.0, 0.2689414322, 0.7310585976], atol=1e-6, rtol=0)


def test_given_torch_oracle_bf16_tensor_when_applying_rms_norm_then_expected_values(oracle):
    # tests/ops/ops_test.cpp:312-332 (eps 1e-5, negative weight)
    x = bf16([-1.5, -0.25, 0.5, 2.0, 3.0, -4.5, 1.25, 0.75]).reshape(2, 4)
    w = bf16([1.0, 0.5, -1.5, 2.0])
    expected = [-1.171875, -0.09765625, -0.5859375, 3.125, 1.0703125, -0.8046875, -0.66796875, 0.53515625]
    for chunk in (1, 0):  # the device order for width 4 (scalar path) and the order-free double sum
        np.testing.assert_allclose(bf16_to_f32(oracle.rms_norm(x, w, 1e-5, chunk=chunk)).ravel(), expected,
                                   atol=1e-6, rtol=0)


def test_given_zero_position_offset_when_applying_rope_then_values_stay_the_same(oracle):
    # tests/nn/rope_test.cpp:25-30
    x = np.array([1.0, -0.5, 0.25, 1.5], np.float32).reshape(1, 1, 4)
    assert (oracle.rope(x) == x).all()


ROPE_INPUT = [1.0, -0.5, 0.25, 1.5, -1.25, 0.75, 1.0, -0.25, 0.5, 1.25, -0.75, 0.5,
              -0.5, 1.0, 1.5, -1.25, 0.75, -1.5, 0.5, 1.0, 1.25, 0.25, -1.0, 0.75]
ROPE_EXPECTED = [-0.64453125, -0.50390625, 0.8046875, 1.5, 1.09375, 0.75, -1.1640625, -0.248046875, -0.89453125,
                 1.25, 0.11181640625, 0.50390625, -1.15625, 1.0, -1.078125, -1.25, -0.8125, -1.5, -0.388671875,
                 0.99609375, -1.5703125, 0.2470703125, -0.29296875, 0.75]


def test_given_torch_oracle_bf16_inputs_when_applying_rope_then_expected_values(oracle):
    # tests/nn/rope_test.cpp:32-50 (offset 2, tolerance 1e-6)
    x = bf16(ROPE_INPUT).reshape(2, 3, 4)
    np.testing.assert_allclose(bf16_to_f32(oracle.rope(x, offset=2)).ravel(), ROPE_EXPECTED, atol=1e-6, rtol=0)


MLP_HIDDEN = [-1.00, 0.71, -0.91, -1.26, 1.27, -1.03, 1.06, -0.99, 1.05, 0.56, 0.79, 0.46, -0.22, 0.83, -1.14,
              -0.28, 1.28, 1.29]
MLP_GATE = [-1.03, 1.29, -0.58, 0.84, -0.61, 0.98, -0.79, 0.07, 0.61, 0.99, -0.75, -0.30, 0.83, 0.70, -0.55, 1.03,
            1.28, 1.26, -0.51, -1.23, 0.66, 0.61, 0.63, -0.31, 0.84, -0.54, 1.24, -0.70, -0.16, 0.52, 1.20, -0.28,
            0.98, 0.22, -0.48, 1.17, 0.67, 1.26, 1.05, 0.01, -0.49, -0.86, -1.03, -0.68, 1.06, -0.92, -0.61, 0.22,
            -1.16, 0.61, -1.25, 0.75, -0.64, 1.13, -1.20, 0.54, 1.01, 1.15, -0.37, -0.22]
MLP_UP = [-1.00, -0.51, -0.97, -1.00, -0.20, 0.77, -0.43, 0.31, 0.56, 1.24, 0.86, 0.68, -1.26, -0.12, 0.93, 1.18,
          0.20, 0.09, -0.07, 0.42, -0.90, 0.27, 1.17, -0.32, -1.16, 0.95, 0.76, -1.04, 0.58, 0.16, 0.27, 0.71, 0.67,
          0.91, -0.99, -0.69, 0.57, -0.26, 0.36, 0.39, -0.51, -0.05, 0.29, 1.04, 1.13, -1.01, 0.91, -0.86, -0.10,
          -0.72, 0.32, 0.38, -0.21, 1.10, -0.55, -0.34, -0.36, -0.69, 0.27, 1.06]
MLP_DOWN = [0.80, -0.40, -0.50, -0.20, -0.60, -0.59, -0.93, -0.75, 0.30, 0.77, 0.98, 1.16, 0.61, 0.73, 0.71, -0.26,
            -1.04, -0.50, 0.39, 0.21, -0.54, -0.17, 1.22, -1.13, 0.13, 1.27, -1.18, 0.80, 0.45, -0.17, -0.73, 0.30,
            -0.05, -0.34, -0.69, -0.14, 0.83, 0.12, -0.43, 0.28, -0.96, 0.78, 1.25, 0.16, 1.00, 0.35, -0.33, -0.99,
            -1.13, -0.69, -0.94, 1.25, -0.46, -0.68, 0.77, 0.22, -1.06, 1.22, -0.28, 1.13]
MLP_EXPECTED = [-0.22265625, -0.91015625, 0.515625, 1.03125, 0.11767578125, -0.7109375, 2.609375, -2.109375,
                0.5390625, 2.296875, -2.734375, -2.921875, 4.03125, -0.003997802734375, -4.65625, -2.265625,
                -8.3125, -3.234375]


def test_given_torch_oracle_bf16_mlp_when_gating_then_double_rounding_matches(oracle):
    # tests/nn/qwen_mlp_test.cpp:75-118: gate = x Wg^T, up = x Wu^T, out = (bf16(silu(gate)) * up) Wd^T, bf16 after
    # every op. Pins the silu -> mul double rounding of the fused silu*up op.
    x = bf16(MLP_HIDDEN).reshape(3, 6)
    gate = oracle.linear(x, bf16(MLP_GATE).reshape(10, 6))
    up = oracle.linear(x, bf16(MLP_UP).reshape(10, 6))
    gated = oracle.silu_mul(gate, up)
    assert (gated == oracle.mul(oracle.silu(gate), up)).all()
    out = oracle.linear(gated, bf16(MLP_DOWN).reshape(6, 10))
    np.testing.assert_allclose(bf16_to_f32(out).ravel(), MLP_EXPECTED, atol=1e-6, rtol=0)


# ---------------------------------------------------------------------------------------------------------------
# 2. The reference's own code (oracle/_ref), bit for bit
# ---------------------------------------------------------------------------------------------------------------


def test_oracle_bf16_rounding_matches_reference_helper(reference):
    rng = np.random.default_rng(1)
    x = np.concatenate([
        rng.standard_normal(100000).astype(np.float32) * np.float32(10.0),
        np.array([0.0, -0.0, np.inf, -np.inf, 3.4e38, -3.4e38, 1e-40, -1e-40], np.float32),
    ])
    assert (f32_to_bf16(x) == reference.f32_to_bf16(x)).all()


def test_oracle_scaled_causal_softmax_matches_reference_code(oracle, reference):
    rng = np.random.default_rng(2)
    x = (rng.standard_normal((4, 96, 96)) * 2.0).astype(np.float32)
    scale = float(np.float32(1.0 / np.sqrt(128.0)))
    assert np.array_equal(oracle.scaled_causal_softmax(x, scale), reference.scaled_causal_softmax(x, scale))


def test_oracle_position_causal_softmax_matches_reference_code(oracle, reference):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((4, 3, 12, 50)) * 2.0).astype(np.float32)
    args = (0.125, [0, 10, 38, 5], [12, 7, 0, 12], [12, 17, 50, 3])
    assert np.array_equal(oracle.position_causal_softmax(x, *args), reference.position_causal_softmax(x, *args))


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("seq_dim", [0, 1])
def test_oracle_rope_matches_reference_code(oracle, reference, dtype, seq_dim):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((7, 5, 128)).astype(np.float32)
    if dtype == "bf16":
        x = f32_to_bf16(x)
    assert np.array_equal(oracle.rope(x, offset=2041, seq_dim=seq_dim),
                          reference.apply_rope(x, offset=2041, seq_dim=seq_dim))


def test_oracle_rope_table_matches_reference_angles(oracle, reference):
    # Rotating unit vectors through the reference's apply_rope exposes its cos/sin values exactly.
    d, positions = 128, 64
    x = np.zeros((positions, 1, d), np.float32)
    x[:, 0, 0:d // 2] = 1.0
    rotated = reference.apply_rope(x, offset=0, seq_dim=0)[:, 0, :]
    table = oracle.rope_table(1e6, d, positions)
    assert np.array_equal(rotated[:, :d // 2], table[:, :d // 2])  # first*cos - 0*sin
    assert np.array_equal(rotated[:, d // 2:], table[:, d // 2:])  # 0*cos + first*sin


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_oracle_elementwise_matches_reference_code(oracle, reference, dtype):
    rng = np.random.default_rng(5)
    a = (rng.standard_normal(50001) * 4).astype(np.float32)
    b = (rng.standard_normal(50001) * 4).astype(np.float32)
    if dtype == "bf16":
        a, b = f32_to_bf16(a), f32_to_bf16(b)
    assert np.array_equal(oracle.add(a, b), reference.add(a, b))
    assert np.array_equal(oracle.mul(a, b), reference.mul(a, b))
    assert np.array_equal(oracle.silu(a), reference.silu(a))
    assert np.array_equal(oracle.silu_mul(a, b), reference.silu_mul(a, b))
    assert np.array_equal(oracle.cast(a, to_bf16=dtype == "f32"), reference.cast(a, to_bf16=dtype == "f32"))


def test_reference_rms_norm_needs_onednn_and_validation_matches(reference):
    from oracle.oracle import ReferenceUnavailable

    with pytest.raises(ReferenceUnavailable):
        reference.rms_norm(bf16([1, 2, 3, 4]).reshape(1, 4), bf16([1, 1, 1, 1]), 1e-6)
    with pytest.raises(ValueError, match="non-negative epsilon"):
        reference.rms_norm_validate(0, [2, 4], 0, [4], -1.0)
    with pytest.raises(ValueError, match="matching tensor dtypes"):
        reference.rms_norm_validate(0, [2, 4], 1, [4], 1e-6)
    with pytest.raises(ValueError, match="rank-1 weight"):
        reference.rms_norm_validate(0, [2, 4], 0, [1, 4], 1e-6)
    with pytest.raises(ValueError, match="weight size must match"):
        reference.rms_norm_validate(0, [2, 4], 0, [3], 1e-6)
    with pytest.raises(ValueError, match="non-empty last dimension"):
        reference.rms_norm_validate(0, [2, 0], 0, [0], 1e-6)


def test_committed_reference_fixtures_still_match_reference_code(reference, golden):
    g = golden("ref_causal_softmax")
    assert np.array_equal(reference.scaled_causal_softmax(g["x"], float(g["scale"])), g["y"])
    g = golden("ref_elementwise")
    assert np.array_equal(reference.silu_mul(g["gate"], g["up"]), g["silu_mul_bf16"])


# ---------------------------------------------------------------------------------------------------------------
# 3. Oracle against the committed fixtures
# ---------------------------------------------------------------------------------------------------------------


def test_oracle_matches_reference_fixtures_bit_exact(oracle, golden):
    g = golden("ref_causal_softmax")
    assert np.array_equal(oracle.scaled_causal_softmax(g["x"], float(g["scale"])), g["y"])
    g = golden("ref_position_softmax")
    assert np.array_equal(oracle.position_causal_softmax(g["x"], float(g["scale"]), g["offsets"], g["qlens"],
                                                         g["klens"]), g["y"])
    g = golden("ref_rope")
    assert np.array_equal(oracle.rope(g["bf16_seq1_x"], offset=3, seq_dim=1), g["bf16_seq1_y"])
    assert np.array_equal(oracle.rope(g["bf16_seq0_x"], offset=1000, seq_dim=0), g["bf16_seq0_y"])
    assert np.array_equal(oracle.rope(g["f32_seq1_x"], offset=7, base=10000.0, seq_dim=1), g["f32_seq1_y"])
    g = golden("ref_elementwise")
    for dt in ("bf16", "f32"):
        assert np.array_equal(oracle.add(g[f"a_{dt}"], g[f"b_{dt}"]), g[f"add_{dt}"])
        assert np.array_equal(oracle.mul(g[f"a_{dt}"], g[f"b_{dt}"]), g[f"mul_{dt}"])
    assert np.array_equal(oracle.cast(g["a_f32"], True), g["cast_f32_bf16"])
    assert np.array_equal(oracle.cast(g["a_bf16"], False), g["cast_bf16_f32"])
    assert np.array_equal(oracle.silu(g["gate"]), g["silu_bf16"])
    assert np.array_equal(oracle.silu_mul(g["gate"], g["up"]), g["silu_mul_bf16"])
    assert np.array_equal(oracle.silu_mul(g["a_f32"], g["b_f32"]), g["silu_mul_f32"])


def test_oracle_rms_norm_matches_torch_fixture_within_one_ulp(oracle, golden):
    g = golden("torch_rms_norm")
    for chunk in (8, 0):
        y = oracle.rms_norm(g["x"], g["w"], float(g["eps"]), chunk=chunk)
        assert ulp_distance(y, g["y"]).max() <= 1
    g = golden("torch_add_rms_norm")
    s, y = oracle.add_rms_norm(g["a"], g["b"], g["w"], float(g["eps"]))
    assert np.array_equal(s, g["sum"])
    assert ulp_distance(y, g["y"]).max() <= 1


def test_oracle_rms_norm_device_order_is_within_one_ulp_of_exact_order(oracle):
    rng = np.random.default_rng(6)
    x = f32_to_bf16(rng.standard_normal((512, 1024)).astype(np.float32))
    w = f32_to_bf16((1 + 0.1 * rng.standard_normal(1024)).astype(np.float32))
    device_order = oracle.rms_norm(x, w, 1e-6)
    exact = oracle.rms_norm(x, w, 1e-6, chunk=0)
    d = ulp_distance(device_order, exact)
    assert d.max() <= 1
    assert (d == 0).mean() > 0.999


def test_oracle_silu_mul_matches_torch_fixture(oracle, golden):
    g = golden("torch_silu_mul")
    out, alt = oracle.silu_mul(g["gate"], g["up"], with_alternative=True)
    ok = (out == g["out"]) | (alt == g["out"])
    assert ok.all()


def test_oracle_qk_norm_rope_matches_torch_fixture(oracle, golden):
    g = golden("torch_qk_norm_rope")
    q_out, k_out = oracle.qk_norm_rope(g["q"], g["k"], g["qw"], g["kw"], float(g["eps"]), int(g["offset"]),
                                       float(g["base"]))
    # torch computes inv_freq as 1 / base^(2i/D) and rsqrt, the reference powf(base, -i/(D/2)) and 1/sqrt:
    # angles and norms agree to a few f32 ulps, which moves a small fraction of bf16 roundings by one ulp.
    for got, want in ((q_out, g["q_out"]), (k_out, g["k_out"])):
        err = np.abs(as_float(got) - as_float(want))
        tol = np.maximum(np.abs(as_float(want)) * 2.0 ** -7, 2.0 ** -14)
        assert (err <= tol).all()


def test_oracle_causal_softmax_matches_torch_fixture(oracle, golden):
    g = golden("torch_causal_softmax")
    np.testing.assert_allclose(oracle.scaled_causal_softmax(g["x"], float(g["scale"])), g["y"], rtol=1e-5,
                               atol=1e-7)


def test_oracle_softmax_matches_torch_fixture(oracle, golden):
    g = golden("torch_softmax")
    assert ulp_distance(oracle.softmax_last_dim(g["x"]), g["y"]).max() <= 1


def test_oracle_row_argmax_matches_fixture(oracle, golden):
    g = golden("torch_row_argmax")
    assert np.array_equal(oracle.row_argmax(g["x"]), g["index"])
