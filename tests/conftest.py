"""Shared pytest setup: markers, import paths and helpers.

`-m "not gpu"` runs the oracle, host-logic and ABI tests on CPU; `-m gpu`
runs the parity tests through the C ABI on a B200.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "catcher-tippi_b200", ""):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the CUDA library")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cq():
    """The CUDA library's bindings; GPU tests fail (not skip) if it cannot load."""
    import nemotron_cuda
    nemotron_cuda.lib()
    return nemotron_cuda


def golden(name: str) -> dict[str, np.ndarray]:
    with np.load(os.path.join(GOLDEN, name)) as z:
        return {k: z[k] for k in z.files}


def widen(bits: np.ndarray, dtype: str) -> np.ndarray:
    import oracle
    return oracle.np_from_t(bits, dtype).astype(np.float64)


MANT_BITS = {"bf16": 8, "f16": 11}
MIN_ULP = {"bf16": 2.0 ** -133, "f16": 2.0 ** -24}


def ulp(v: np.ndarray, dtype: str) -> np.ndarray:
    """Spacing of T around |v| (T = bf16 or f16)."""
    _, e = np.frexp(np.abs(v))
    return np.maximum(np.ldexp(1.0, e - MANT_BITS[dtype]), MIN_ULP[dtype])


def parity_stats(got_bits: np.ndarray, want_bits: np.ndarray, dtype: str,
                 bias_bits: np.ndarray | None = None, floor_frac: float = 0.0) -> dict[str, float]:
    """max-abs, max distance in T ulps, relative L2 and exact-match fraction.

    Ulps are counted at |y| + |bias|: with an output bias the first rounding
    happens at the magnitude of y - bias, which may be far larger than y.
    floor_frac > 0 adds floor_frac * rms(y) to that magnitude, for paths whose
    accumulation error is absolute (see assert_parity)."""
    g, w = widen(got_bits, dtype), widen(want_bits, dtype)
    diff = np.abs(g - w)
    scale = max(float(np.abs(w).max()), 1e-30)
    if not diff.size:
        return {"max_abs": 0.0, "max_rel_to_max": 0.0, "max_ulp": 0.0, "rel_l2": 0.0, "exact": 1.0}
    base = np.maximum(np.abs(g), np.abs(w))
    if bias_bits is not None:
        base = base + np.abs(widen(bias_bits, dtype))[None, :]
    if floor_frac > 0:
        base = base + floor_frac * float(np.sqrt(np.mean(w * w)))
    return {
        "max_abs": float(diff.max()),
        "max_rel_to_max": float(diff.max() / scale),
        "max_ulp": float((diff / ulp(base, dtype)).max()),
        "rel_l2": float(np.linalg.norm(g - w) / max(np.linalg.norm(w), 1e-30)),
        "exact": float(np.mean(np.asarray(got_bits) == np.asarray(want_bits))),
    }


# Output tolerances of the CUDA path against the oracle on identical packed
# inputs.  Both accumulate in fp32 and differ only in summation order (and,
# on the batched tensor-core path, in the f16 rounding of dequantised
# weights).  The result is rounded to T twice, as QuantizedLinear::forward_array
# does: t = T(acc), y = T(t + bias).  Next to a rounding tie each rounding can
# fall either way, so two correct implementations may differ by
# ulp(t) + ulp(y) <= 2 ulps counted at |y| + |bias| >= |t|; a fused SiLU adds
# a third rounding of a function with slope <= 1.1 (1.5 ulps more).
# The batched tensor-core path also rounds each dequantised weight to f16
# (relative 2^-12); over K terms that perturbs an output by about 2^-13 of the
# output RMS in absolute terms, which is many ulps of an output that cancels
# to near zero.  Its tests count ulps at |y| + |bias| + GEMM_FLOOR[T] * rms(y)
# (rms/4 for bf16, 2 rms for f16 whose ulp is 8x finer), where that
# perturbation stays below half an ulp at five sigma.
#   bf16: rel-L2 <= 4e-3,  every element within that ulp bound
#   f16 : rel-L2 <= 1e-3,  every element within that ulp bound
# The GEMV folds the 1024 offset of its integer weights into the group bias
# term, so each group contributes the difference of two fp32 terms about 2^10
# times larger than its share of the result; near-zero outputs therefore carry
# an absolute error of a few 1e-6 (for these data, ~1e-5 of rms(y)).  Every
# check counts ulps at |y| + |bias| + 2^-6 rms(y) at least (DEFAULT_FLOOR),
# where that error is below one ulp of T.
TOL = {"bf16": 4e-3, "f16": 1e-3}
MAX_ULP = 2.0
DEFAULT_FLOOR = 2.0 ** -6
GEMM_FLOOR = {"bf16": 0.25, "f16": 2.0}


def assert_parity(got_bits, want_bits, dtype: str, min_exact: float = 0.9,
                  bias_bits=None, act: str = "none", floor_frac=DEFAULT_FLOOR):
    if isinstance(floor_frac, dict):
        floor_frac = floor_frac[dtype]
    if act == "silu":
        # SiLU maps the pre-activation wobble onto outputs that may be much
        # smaller (negative inputs) or in a lower binade: count at + rms(y)
        floor_frac = max(floor_frac, 1.0)
    st = parity_stats(got_bits, want_bits, dtype, bias_bits, floor_frac)
    assert st["rel_l2"] <= TOL[dtype], st
    assert st["max_ulp"] <= MAX_ULP + (1.5 if act == "silu" else 0.0), st
    assert st["exact"] >= min_exact, st
    return st
