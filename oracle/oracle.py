"""CPU oracle for the affine INT8 quantized linear (TEST INFRASTRUCTURE).

Only the test suite, ``__graft_entry__.smoke()`` and the benchmark's CPU-baseline
leg import this module.  It is the checker, never the product path: the CUDA
library does not link it, and the product fails loudly when its extension is
missing rather than falling back here.

Two independent restatements of the same algorithm live here:

* ``liboracle.so`` (``qlinear_oracle.c``): OpenMP C, fp32 / fp64 accumulation;
  also the timed CPU baseline.
* ``np_*`` functions: a numpy mirror used to cross-check the C code and to
  generate the golden fixtures under ``tests/golden``.

Both follow crates/nemotron-mlx/src/model/layers.rs:298-310
(``QuantizedLinear::forward_array``: cast x to T, ``quantized_matmul(transpose=true,
bits=8)`` in T, add the T output bias) and MLX's published affine quantisation
in its fp32 (CPU-stream) form: the group's extreme of larger magnitude is the
edge and the bias, step = max((max-min)/255, 1e-7) with the edge's sign,
q0 = round(edge/step), scale = edge/q0 when q0 != 0, codes
clamp(round((w-bias)/scale), 0, 255) from the fp32 scale and bias, which are
then stored in T; round half to even; 4 codes per u32, least significant byte
first.  Bit-level agreement with MLX itself is unpinned (MLX cannot run here);
the oracle is pinned to the reference's own tolerance tests
(crates/nemotron-mlx/tests/quantized_matmul.rs:24-47, model_layers.rs:35-78,
weight_roundtrip.rs:50-115) and to hand-derived cases of the edge/sign rule.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

DTYPES = {"f16": 0, "bf16": 1, "f32": 2}
ACTS = {"none": 0, "silu": 1, "relu": 2}

_lib = None


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        src = os.path.join(HERE, "qlinear_oracle.c")
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
            build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        L.oracle_quantize.argtypes = [vp, i, i, i, i, i, vp, vp, vp]
        L.oracle_dequantize.argtypes = [vp, vp, vp, i, i, i, i, vp]
        L.oracle_qmatmul.argtypes = [vp, i, i, vp, vp, vp, vp, i, i, i, i, vp]
        L.oracle_qmatmul_f64.argtypes = [vp, i, i, vp, vp, vp, vp, i, i, i, vp]
        L.oracle_f32_linear.argtypes = [vp, i, i, vp, i, vp, vp]
        L.oracle_round_array.argtypes = [vp, ctypes.c_size_t, i, vp]
        L.oracle_widen_array.argtypes = [vp, ctypes.c_size_t, i, vp]
        L.oracle_set_threads.argtypes = [i]
        L.oracle_max_threads.restype = i
        L.oracle_f32_to_f16.argtypes = [f]
        L.oracle_f32_to_f16.restype = ctypes.c_uint16
        L.oracle_f32_to_bf16.argtypes = [f]
        L.oracle_f32_to_bf16.restype = ctypes.c_uint16
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _tbits(dtype: str):
    return np.float32 if dtype == "f32" else np.uint16


# ---------------------------------------------------------------- C oracle API


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def to_t(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 values to T; returns uint16 bit patterns (or float32 for f32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=_tbits(dtype))
    lib().oracle_round_array(_p(x), x.size, DTYPES[dtype], _p(out))
    return out


def from_t(x: np.ndarray, dtype: str) -> np.ndarray:
    """Widen T bit patterns (uint16) or float32 to float32."""
    x = np.ascontiguousarray(x)
    out = np.empty(x.shape, dtype=np.float32)
    lib().oracle_widen_array(_p(x), x.size, DTYPES[dtype], _p(out))
    return out


def quantize(w: np.ndarray, group: int, dtype: str, round_input: bool = True):
    """Affine 8-bit quantisation -> (q u32 [N, K/4], scales T [N, K/g], biases T [N, K/g])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    if group <= 0 or k % group:
        raise ValueError(f"input dimension {k} is not divisible by group size {group}")
    if group > 128:
        raise ValueError(f"group size {group} is above MLX's largest (128)")
    q = np.empty((n, k), dtype=np.uint8)
    s = np.empty((n, k // group), dtype=_tbits(dtype))
    b = np.empty_like(s)
    lib().oracle_quantize(_p(w), n, k, group, DTYPES[dtype], int(round_input), _p(q), _p(s), _p(b))
    return q.view(np.uint32), s, b


def dequantize(q: np.ndarray, s: np.ndarray, b: np.ndarray, group: int, dtype: str) -> np.ndarray:
    q8 = np.ascontiguousarray(q).view(np.uint8)
    n, k = q8.shape
    w = np.empty((n, k), dtype=np.float32)
    lib().oracle_dequantize(_p(q8), _p(np.ascontiguousarray(s)), _p(np.ascontiguousarray(b)),
                            n, k, group, DTYPES[dtype], _p(w))
    return w


def qmatmul(x_t: np.ndarray, q: np.ndarray, s: np.ndarray, b: np.ndarray, group: int,
            dtype: str, bias_t: np.ndarray | None = None, act: str = "none") -> np.ndarray:
    """y T [M, N] from x T [M, K] (bit patterns), fp32 accumulation."""
    x_t = np.ascontiguousarray(x_t)
    q8 = np.ascontiguousarray(q).view(np.uint8)
    n, k = q8.shape
    m = x_t.shape[0]
    y = np.empty((m, n), dtype=_tbits(dtype))
    bias_t = None if bias_t is None else np.ascontiguousarray(bias_t)
    lib().oracle_qmatmul(_p(x_t), m, k, _p(q8), _p(np.ascontiguousarray(s)),
                         _p(np.ascontiguousarray(b)), _p(bias_t), n, group, DTYPES[dtype],
                         ACTS[act], _p(y))
    return y


def qmatmul_f64(x_t, q, s, b, group, dtype, bias_t=None) -> np.ndarray:
    x_t = np.ascontiguousarray(x_t)
    q8 = np.ascontiguousarray(q).view(np.uint8)
    n, k = q8.shape
    m = x_t.shape[0]
    y = np.empty((m, n), dtype=np.float64)
    bias_t = None if bias_t is None else np.ascontiguousarray(bias_t)
    lib().oracle_qmatmul_f64(_p(x_t), m, k, _p(q8), _p(np.ascontiguousarray(s)),
                             _p(np.ascontiguousarray(b)), _p(bias_t), n, group, DTYPES[dtype], _p(y))
    return y


def f32_linear(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    m, k = x.shape
    n = w.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().oracle_f32_linear(_p(x), m, k, _p(w), n, _p(bias), _p(y))
    return y


# ---------------------------------------------------------------- numpy mirror


def np_round_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) & 0x8000).astype(np.uint16) | 0x7FC0
    return r


def np_to_t(x: np.ndarray, dtype: str) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f16":
        return x.astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        return np_round_bf16(x)
    return x.copy()


def np_from_t(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "f16":
        return np.asarray(x, dtype=np.uint16).view(np.float16).astype(np.float32)
    if dtype == "bf16":
        return (np.asarray(x, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
    return np.asarray(x, dtype=np.float32)


def np_quantize(w: np.ndarray, group: int, dtype: str, round_input: bool = True):
    """numpy mirror of MLX's edge/sign affine quantisation (oracle_quantize_group)."""
    w = np.asarray(w, dtype=np.float32)
    if round_input:
        w = np_from_t(np_to_t(w, dtype), dtype)
    n, k = w.shape
    f = np.float32
    wg = w.reshape(n, k // group, group)
    lo = wg.min(axis=2)
    hi = wg.max(axis=2)
    low_edge = np.abs(lo) > np.abs(hi)
    step = np.maximum((hi - lo) / f(255.0), f(1e-7)).astype(f)
    scale = np.where(low_edge, step, -step).astype(f)
    edge = np.where(low_edge, lo, hi).astype(f)
    q0 = np.rint(edge / scale).astype(f)
    nz = q0 != 0
    scale = np.where(nz, edge / np.where(nz, q0, f(1.0)), scale).astype(f)
    bias = np.where(nz, edge, f(0.0)).astype(f)
    c = np.rint((wg - bias[..., None]) / scale[..., None])
    q = np.clip(c, 0, 255).astype(np.uint8).reshape(n, k)
    return q.view(np.uint32), np_to_t(scale, dtype), np_to_t(bias, dtype)


def np_dequantize(q, s, b, group, dtype) -> np.ndarray:
    q8 = np.ascontiguousarray(q).view(np.uint8).astype(np.float32)
    n, k = q8.shape
    sf = np.repeat(np_from_t(s, dtype), group, axis=1)
    bf = np.repeat(np_from_t(b, dtype), group, axis=1)
    return (sf * q8 + bf).astype(np.float32)


def np_qmatmul(x_t, q, s, b, group, dtype, bias_t=None, act="none") -> np.ndarray:
    """Small-case mirror: float64 contraction, then the same two T roundings."""
    xf = np_from_t(x_t, dtype).astype(np.float64)
    w = np_dequantize(q, s, b, group, dtype).astype(np.float64)
    y = np_from_t(np_to_t((xf @ w.T).astype(np.float32), dtype), dtype)
    if bias_t is not None:
        y = np_from_t(np_to_t(y + np_from_t(bias_t, dtype)[None, :], dtype), dtype)
    if act == "silu":
        y = np_from_t(np_to_t(y / (1.0 + np.exp(-y)), dtype), dtype)
    elif act == "relu":
        y = np_from_t(np_to_t(np.maximum(y, 0), dtype), dtype)
    return np_to_t(y, dtype)
