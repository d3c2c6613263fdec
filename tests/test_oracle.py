"""Pins the CPU oracle (CPU only).

The oracle is checked against the reference's own known-answer tests for
this path (rebuilt in tests/golden/reference_kats.npz from their pattern
formulas, with the reference's tolerances), against the independent numpy
mirror, and against the committed golden vectors.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import DEFAULT_FLOOR, golden, parity_stats


def test_rounding_matches_numpy_f16(oracle_mod):
    rng = np.random.default_rng(0)
    v = np.concatenate([
        rng.standard_normal(50000).astype(np.float32) * 1000,
        rng.standard_normal(50000).astype(np.float32) * 1e-6,
        np.array([6e-8, 3e-8, 2.98e-8, 65504, 65519, 65520, 1e5, -0.0, 0.0], np.float32),
    ])
    with np.errstate(over="ignore"):
        assert np.array_equal(oracle_mod.to_t(v, "f16"), oracle_mod.np_to_t(v, "f16"))
    assert np.array_equal(oracle_mod.to_t(v, "bf16"), oracle_mod.np_to_t(v, "bf16"))
    bits = np.arange(0, 65536, dtype=np.uint16)
    for dt in ("f16", "bf16"):
        a = oracle_mod.from_t(bits, dt)
        b = oracle_mod.np_from_t(bits, dt)
        assert np.array_equal(np.isnan(a), np.isnan(b))
        assert np.array_equal(a[~np.isnan(a)], b[~np.isnan(b)])


def test_reference_kat_quantized_matmul(oracle_mod):
    """crates/nemotron-mlx/tests/quantized_matmul.rs:24-47 (f32 backend path, abs 0.06)."""
    k = golden("reference_kats.npz")
    rows, ind, outd, g = (int(v) for v in k["qmm_meta"])
    w = k["qmm_weight"].reshape(outd, ind)
    q, s, b = oracle_mod.quantize(w, g, "f32", round_input=False)
    y = oracle_mod.qmatmul(k["qmm_input"].reshape(rows, ind), q, s, b, g, "f32")
    err = np.abs(y.ravel() - k["qmm_expected"]).max()
    assert err <= k["tolerances"][0], err


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_reference_kat_linear_with_bias(oracle_mod, dtype):
    """model_layers.rs:35-55: QuantizedLinear::from_f32 + forward_f32 with bias, abs 0.08."""
    k = golden("reference_kats.npz")
    w = k["lin_weight"].reshape(3, 128)
    q, s, b = oracle_mod.quantize(w, 128, dtype)
    y = oracle_mod.qmatmul(oracle_mod.to_t(k["lin_input"].reshape(2, 128), dtype), q, s, b, 128,
                           dtype, oracle_mod.to_t(k["lin_bias"], dtype))
    err = np.abs(oracle_mod.from_t(y, dtype).ravel() - k["lin_expected"]).max()
    assert err <= k["tolerances"][1], err


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_reference_kat_pointwise(oracle_mod, dtype):
    """model_layers.rs:57-78: PointwiseConv1d over [1, 3, 128] -> [1, 3, 2], abs 0.08."""
    k = golden("reference_kats.npz")
    w = k["pw_weight"].reshape(2, 128)
    q, s, b = oracle_mod.quantize(w, 128, dtype)
    y = oracle_mod.qmatmul(oracle_mod.to_t(k["pw_input"].reshape(3, 128), dtype), q, s, b, 128,
                           dtype, oracle_mod.to_t(k["pw_bias"], dtype))
    err = np.abs(oracle_mod.from_t(y, dtype).ravel() - k["pw_expected"]).max()
    assert err <= k["tolerances"][2], err


def test_reference_kat_artifact_roundtrip(oracle_mod):
    """weight_roundtrip.rs:50-90: f16 artifact, dequantised within 0.008."""
    k = golden("reference_kats.npz")
    m = k["rt_matrix"].reshape(2, 128)
    q, s, b = oracle_mod.quantize(m, 128, "f16")
    assert q.dtype == np.uint32 and q.shape == (2, 32)
    assert s.dtype == np.uint16 and b.dtype == np.uint16 and s.shape == (2, 1)
    w = oracle_mod.dequantize(q, s, b, 128, "f16")
    assert np.abs(w - m).max() <= k["tolerances"][3]


def test_reference_kat_packed_artifact_linear(oracle_mod):
    """weight_roundtrip.rs:93-115: layer bound to packed f16 arrays, no bias, abs 0.04."""
    k = golden("reference_kats.npz")
    q, s, b = oracle_mod.quantize(k["art_matrix"].reshape(2, 128), 128, "f16")
    y = oracle_mod.qmatmul(oracle_mod.to_t(k["art_input"].reshape(1, 128), "f16"), q, s, b, 128,
                           "f16")
    err = np.abs(oracle_mod.from_t(y, "f16").ravel() - k["art_expected"]).max()
    assert err <= k["tolerances"][4], err


def test_quantize_c_matches_numpy(oracle_mod):
    rng = np.random.default_rng(3)
    for dtype in ("f16", "bf16", "f32"):
        for g in (32, 64, 128):
            w = (rng.standard_normal((37, 256)) * 0.05).astype(np.float32)
            w[3, :g] = 0.25  # constant group: bias 0.25, codes 0
            w[4, :g] = 0.0  # zero group: bias 0, codes 0
            w[5, :g] = np.abs(w[5, :g]) + 0.01  # one-signed groups
            w[6, :g] = -np.abs(w[6, :g]) - 0.01
            a = oracle_mod.quantize(w, g, dtype, round_input=dtype != "f32")
            b = oracle_mod.np_quantize(w, g, dtype, round_input=dtype != "f32")
            for x, y in zip(a, b):
                assert np.array_equal(x, y), (dtype, g)
            deq = oracle_mod.dequantize(*a, g, dtype)
            assert np.allclose(deq[3, :g], 0.25)


def test_packing_is_lsb_first(oracle_mod):
    """4 codes per u32, first element in the least significant byte (MLX layout)."""
    # min edge -255 with step 1: codes 0, 85, 170, 255
    w = np.tile(np.array([-3.0, -2.0, -1.0, 0.0], np.float32), (1, 16)) * (255.0 / 3.0)
    q, s, b = oracle_mod.quantize(w, 64, "f32", round_input=False)
    word = int(q[0, 0])
    assert [(word >> (8 * i)) & 0xFF for i in range(4)] == [0, 85, 170, 255]


F = np.float32
# (group values, codes, scale, bias), derived by hand from the edge/sign rule:
# edge = the extreme of larger magnitude (the max on a tie), step =
# (max - min) / 255 with the edge's sign, q0 = round(edge / step),
# scale = edge / q0, bias = edge, codes round((w - bias) / scale).
EDGE_SIGN_CASES = [
    # max edge: q0 = round(1 / (-1.5/255)) = -170, the scale is negative
    ([1.0, -0.5, 0.0], [0, 255, 170], F(1.0) / F(-170.0), 1.0),
    # min edge: the mirror image, positive scale
    ([-1.0, 0.5, 0.0], [0, 255, 170], F(-1.0) / F(-170.0), -1.0),
    # all positive: q0 = round(1 / (-0.5/255)) = -510
    ([0.5, 1.0, 0.7], [255, 0, 153], F(1.0) / F(-510.0), 1.0),
    # all negative: q0 = round(-1 / (0.5/255)) = -510
    ([-1.0, -0.5, -0.7], [0, 255, 153], F(-1.0) / F(-510.0), -1.0),
    # |min| == |max| takes the max; 1 / (-2/255) rounds to -127.49999 -> -127,
    # so -1 lands on code 254
    ([-1.0, 1.0, 0.3], [254, 0, 89], F(1.0) / F(-127.0), 1.0),
    # all zero: step is the 1e-7 floor, q0 = 0, bias 0
    ([0.0], [0], -F(1e-7), 0.0),
]


@pytest.mark.parametrize("vals,codes,scale,bias", EDGE_SIGN_CASES)
def test_quantize_edge_sign_rule(oracle_mod, vals, codes, scale, bias):
    """MLX's affine_quantize rule (fp32 form), checked on hand-derived groups."""
    vals = np.array(vals, np.float32)
    w = np.full((1, 32), vals[-1], np.float32)
    w[0, :len(vals)] = vals
    for impl in (oracle_mod.quantize, oracle_mod.np_quantize):
        q, s, b = impl(w, 32, "f32", round_input=False)
        assert list(q.view(np.uint8)[0, :len(vals)]) == codes
        assert s.view(np.float32)[0, 0] == F(scale)
        assert b.view(np.float32)[0, 0] == F(bias)
    # stored in T, the scale and bias are the fp32 values rounded once; the
    # codes still come from the fp32 values
    for dtype in ("f16", "bf16"):
        q, s, b = oracle_mod.quantize(w, 32, dtype)
        assert list(q.view(np.uint8)[0, :len(vals)]) == codes
        assert np.array_equal(s, oracle_mod.to_t(np.array([[scale]], np.float32), dtype))
        assert np.array_equal(b, oracle_mod.to_t(np.array([[bias]], np.float32), dtype))


def test_quantize_constant_group_is_exact(oracle_mod):
    """A constant group keeps its value as the bias with all codes 0."""
    w = np.full((2, 64), 0.25, np.float32)
    w[1] = -3.5
    q, s, b = oracle_mod.quantize(w, 64, "f16")
    assert not q.any()
    assert np.array_equal(oracle_mod.from_t(b, "f16").ravel(), [0.25, -3.5])
    assert np.array_equal(oracle_mod.dequantize(q, s, b, 64, "f16"), w)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_c_oracle_matches_golden(oracle_mod, dtype, group):
    z = golden(f"oracle_{dtype}_g{group}.npz")
    names = sorted({k.rsplit("_", 1)[0] for k in z if k.endswith("_meta")})
    for name in names:
        m, n, kdim, with_bias, act = (int(v) for v in z[f"{name}_meta"])
        bias = z.get(f"{name}_bias")
        y = oracle_mod.qmatmul(z[f"{name}_x"], z[f"{name}_q"], z[f"{name}_s"], z[f"{name}_b"],
                               group, dtype, bias, ["none", "silu", "relu"][act])
        st = parity_stats(y, z[f"{name}_y"], dtype, bias, DEFAULT_FLOOR)
        # fp32 (C) vs fp64 (numpy) contraction: equal up to one rounding flip
        # per T rounding, counted as the GPU parity tests count (at |y| + |bias|
        # + 2^-6 rms(y): fp32 sums of outputs that cancel to near zero carry an
        # absolute error)
        assert st["exact"] >= 0.98 and st["max_ulp"] <= 2, (name, st)


def test_fp32_and_fp64_oracles_agree(oracle_mod):
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((512, 1024)) * 0.02).astype(np.float32)
    q, s, b = oracle_mod.quantize(w, 64, "bf16")
    x = oracle_mod.to_t(rng.standard_normal((14, 1024)).astype(np.float32), "bf16")
    y32 = oracle_mod.from_t(oracle_mod.qmatmul(x, q, s, b, 64, "bf16"), "bf16")
    y64 = oracle_mod.qmatmul_f64(x, q, s, b, 64, "bf16")
    # bf16 output rounding dominates: half an ulp (2^-9 relative) plus fp32 noise
    assert np.all(np.abs(y32 - y64) <= np.abs(y64) * 2.0 ** -8 + 1e-6)
