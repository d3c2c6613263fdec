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


def parity_stats(got_bits: np.ndarray, want_bits: np.ndarray, dtype: str) -> dict[str, float]:
    """max-abs, relative L2 and exact-match fraction of two T bit-pattern arrays."""
    g, w = widen(got_bits, dtype), widen(want_bits, dtype)
    diff = np.abs(g - w)
    scale = max(float(np.abs(w).max()), 1e-30)
    return {
        "max_abs": float(diff.max()) if diff.size else 0.0,
        "max_rel_to_max": float(diff.max() / scale) if diff.size else 0.0,
        "rel_l2": float(np.linalg.norm(g - w) / max(np.linalg.norm(w), 1e-30)),
        "exact": float(np.mean(np.asarray(got_bits) == np.asarray(want_bits))) if diff.size else 1.0,
    }


# Output tolerances of the CUDA path against the oracle on identical packed
# inputs (both accumulate in fp32; they differ only by summation order, so
# results are within one T ulp):
#   bf16: rel-L2 <= 4e-3 and max-abs <= 1e-2 * max|y|
#   f16 : rel-L2 <= 1e-3 and max-abs <= 2e-3 * max|y|
TOL = {"bf16": (4e-3, 1e-2), "f16": (1e-3, 2e-3)}


def assert_parity(got_bits, want_bits, dtype: str, min_exact: float = 0.9):
    st = parity_stats(got_bits, want_bits, dtype)
    rel_l2, rel_max = TOL[dtype]
    assert st["rel_l2"] <= rel_l2, st
    assert st["max_rel_to_max"] <= rel_max, st
    assert st["exact"] >= min_exact, st
    return st
