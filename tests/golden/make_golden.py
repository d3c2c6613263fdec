"""Generates the committed golden fixtures under tests/golden/.

Two kinds of vectors:

* ``reference_kats.npz`` -- the known-answer tests of the reference's own test
  suite for this path, rebuilt from their integer-pattern formulas, with the
  unquantised f32 expected outputs those tests compare against and their
  tolerances:
    - crates/nemotron-mlx/tests/quantized_matmul.rs:24-47   (2x128 . 64x128, g128, abs 0.06)
    - crates/nemotron-mlx/tests/model_layers.rs:35-55       (bias, 2x128 . 3x128, abs 0.08)
    - crates/nemotron-mlx/tests/model_layers.rs:57-78       (pointwise, 1x3x128 -> 2, abs 0.08)
    - crates/nemotron-mlx/tests/weight_roundtrip.rs:50-90   (dequant of 2x128, abs 0.008)
    - crates/nemotron-mlx/tests/weight_roundtrip.rs:93-115  (packed-artifact linear, abs 0.04)
* ``oracle_<dtype>_g<group>.npz`` -- packed weights, activations and outputs
  of the numpy mirror of the oracle (oracle/oracle.py ``np_*``), seeded, for
  the shapes the kernels special-case (ragged N, M < 16 and M > 16, group
  32/64/128, output bias, fused activations).

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle as O  # noqa: E402


def reference_kats() -> dict[str, np.ndarray]:
    out = {}
    # quantized_matmul.rs:24-47
    rows, ind, outd = 2, 128, 64
    x = np.array([((i % 17) - 8) / 16.0 for i in range(rows * ind)], np.float32)
    w = np.array([((i * 7 % 23) - 11) / 32.0 for i in range(outd * ind)], np.float32)
    out["qmm_input"], out["qmm_weight"] = x, w
    out["qmm_expected"] = (x.reshape(rows, ind).astype(np.float64)
                           @ w.reshape(outd, ind).astype(np.float64).T).astype(np.float32).ravel()
    out["qmm_meta"] = np.array([rows, ind, outd, 128], np.int64)
    # model_layers.rs:35-55 (QuantizedLinear with bias)
    ind, outd = 128, 3
    x = np.array([((i % 19) - 9.0) / 11.0 for i in range(256)], np.float32)
    w = np.array([((i * 5 % 31) - 15.0) / 23.0 for i in range(outd * ind)], np.float32)
    bias = np.array([0.25, -0.5, 0.125], np.float32)
    out["lin_input"], out["lin_weight"], out["lin_bias"] = x, w, bias
    out["lin_expected"] = (x.reshape(2, ind).astype(np.float64) @ w.reshape(outd, ind).astype(
        np.float64).T + bias).astype(np.float32).ravel()
    # model_layers.rs:57-78 (PointwiseConv1d)
    ind, outd = 128, 2
    x = np.array([((i % 13) - 6.0) / 8.0 for i in range(3 * ind)], np.float32)
    w = np.array([((i * 3 % 17) - 8.0) / 13.0 for i in range(outd * ind)], np.float32)
    bias = np.array([0.1, -0.2], np.float32)
    out["pw_input"], out["pw_weight"], out["pw_bias"] = x, w, bias
    out["pw_expected"] = (x.reshape(3, ind).astype(np.float64) @ w.reshape(outd, ind).astype(
        np.float64).T + bias).astype(np.float32).ravel()
    # weight_roundtrip.rs:50-90 (dequantised artifact matrix)
    out["rt_matrix"] = np.array([((i % 29) - 14) / 17.0 for i in range(256)], np.float32)
    # weight_roundtrip.rs:93-115 (packed-artifact layer, no bias)
    m = np.array([((i % 17) - 8.0) / 19.0 for i in range(256)], np.float32)
    xin = np.array([i / 127.0 for i in range(128)], np.float32)
    out["art_matrix"], out["art_input"] = m, xin
    out["art_expected"] = (m.reshape(2, 128).astype(np.float64) @ xin.astype(np.float64)).astype(
        np.float32)
    out["tolerances"] = np.array([0.06, 0.08, 0.08, 0.008, 0.04], np.float64)
    return out


CASES = [
    # (name, M, N, K, bias, act)
    ("m14", 14, 96, 224, False, "none"),  # K % 64 == 32 at g32
    ("m1_bias", 1, 80, 192, True, "none"),
    ("m16_silu", 16, 64, 128, True, "silu"),
    ("m21_relu", 21, 48, 320, False, "relu"),
]


def oracle_vectors(dtype: str, group: int, seed: int) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    out = {}
    for name, m, n, k, with_bias, act in CASES:
        if k % group:
            k = (k // group + 1) * group
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        q, s, b = O.np_quantize(w, group, dtype)
        x = O.np_to_t(rng.standard_normal((m, k)).astype(np.float32), dtype)
        bias = O.np_to_t((rng.standard_normal(n) * 0.1).astype(np.float32), dtype) if with_bias else None
        y = O.np_qmatmul(x, q, s, b, group, dtype, bias, act)
        out[f"{name}_q"], out[f"{name}_s"], out[f"{name}_b"] = q, s, b
        out[f"{name}_x"], out[f"{name}_y"] = x, y
        if bias is not None:
            out[f"{name}_bias"] = bias
        out[f"{name}_meta"] = np.array([m, n, k, int(with_bias), O.ACTS[act]], np.int64)
    return out


def main() -> None:
    np.savez_compressed(os.path.join(HERE, "reference_kats.npz"), **reference_kats())
    seed = 100
    for dtype in ("f16", "bf16"):
        for group in (32, 64, 128):
            np.savez_compressed(os.path.join(HERE, f"oracle_{dtype}_g{group}.npz"),
                                **oracle_vectors(dtype, group, seed))
            seed += 1
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
