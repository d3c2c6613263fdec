"""Persistent linear chain (include/cqchain.h) on the GPU.

Each step of a chain computes QuantizedLinear::forward_array
(crates/nemotron-mlx/src/model/layers.rs:298-310) on the output of earlier
steps.  Checks, per step: the chain's output against the oracle's quantized
matmul applied to the chain's own input for that step (read back), at the
quantized-linear parity bar of conftest.assert_parity; bit equality with the
per-layer K1 launches where both cut K the same way; the dependencies derived
from the buffers; repeated runs (the in-kernel counters reset themselves);
ragged shapes, token tiles past 16 rows, K split over work items, group sizes
32/64/128, fused activations and output biases.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_parity

pytestmark = pytest.mark.gpu

TDT = {"f16": "float16", "bf16": "bfloat16"}


def _bits(t) -> np.ndarray:
    import torch
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _layer(cq, oracle_mod, n, k, group, dtype, seed, with_bias):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    q, s, b = oracle_mod.quantize(w, group, dtype)
    bias = oracle_mod.to_t((rng.standard_normal(n) * 0.1).astype(np.float32), dtype) \
        if with_bias else None
    return cq.QuantizedLinear.from_packed(q, s, b, bias, group, dtype), (q, s, b, bias)


BLOCK = [  # name, N, K, rows, act, input
    ("ffn1_up", 4096, 1024, 14, "silu", "x0"),
    ("ffn1_down", 1024, 4096, 14, "none", "ffn1_up"),
    ("qkv", 3072, 1024, 14, "none", "ffn1_down"),
    ("pos", 1024, 1024, 83, "none", "pe"),
    ("out", 1024, 1024, 14, "none", "qkv"),
    ("pw1", 2048, 1024, 14, "none", "out"),
    ("pw2", 1024, 1024, 14, "none", "pw1"),
    ("ffn2_up", 4096, 1024, 14, "silu", "pw2"),
    ("ffn2_down", 1024, 4096, 14, "none", "ffn2_up"),
]


def _block_chain(cq, oracle_mod, torch, dtype, blocks, group=64):
    tdt = getattr(torch, TDT[dtype])
    rng = np.random.default_rng(1)
    x0 = torch.from_numpy(oracle_mod.to_t(rng.standard_normal((14, 1024)).astype(np.float32),
                                          dtype).view(np.int16)).cuda().view(tdt)
    pe = torch.from_numpy(oracle_mod.to_t(rng.standard_normal((83, 1024)).astype(np.float32),
                                          dtype).view(np.int16)).cuda().view(tdt)
    steps, meta = [], []
    for blk in range(blocks):
        outs = {}
        for i, (name, n, k, rows, act, src) in enumerate(BLOCK):
            layer, arrays = _layer(cq, oracle_mod, n, k, group, dtype, 100 * blk + i,
                                   with_bias=(name == "pos"))
            if src == "x0":
                x = x0 if blk == 0 else prev
            elif src == "pe":
                x = pe
            else:
                x = outs[src]
            y = torch.zeros((rows, n), dtype=tdt, device="cuda")
            outs[name] = y
            steps.append((layer, x, y, act, rows))
            meta.append((name, arrays, act))
        prev = outs["ffn2_down"]
    return steps, meta


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_block_chain_matches_oracle_step_by_step(cq, oracle_mod, dtype):
    import torch
    steps, meta = _block_chain(cq, oracle_mod, torch, dtype, blocks=2)
    chain = cq.LinearChain(steps)
    assert chain.grid > 0 and chain.items > 0
    chain.run()
    torch.cuda.synchronize()
    assert cq.device_status(0) == 0
    for (layer, x, y, act, rows), (name, (q, s, b, bias), _) in zip(steps, meta):
        xin = np.ascontiguousarray(_bits(x)[:rows, :layer.input_dims])  # qkv: the q columns
        want = oracle_mod.qmatmul(xin, q, s, b, 64, dtype, bias, act)
        # f16 inputs enter the MMA unscaled, so the folded 1024 offset leaves
        # an absolute error that grows with |x|; deeper steps see larger
        # activations than N(0, 1): count ulps at + 2^-3 rms(y) in f16
        # (f16 also rounds more often one ulp away: 3 more mantissa bits)
        floor = 2.0 ** -6 if dtype == "bf16" else 2.0 ** -3
        assert_parity(_bits(y), want, dtype, min_exact=0.9 if dtype == "bf16" else 0.8,
                      bias_bits=bias, act=act, floor_frac=floor)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_chain_equals_per_layer_launches_and_replays(cq, oracle_mod, dtype):
    """The per-layer K1 path on the same inputs, step by step; then two more
    runs (captured in a CUDA graph for the last) give identical bits."""
    import torch
    steps, meta = _block_chain(cq, oracle_mod, torch, dtype, blocks=1)
    chain = cq.LinearChain(steps)
    chain.run()
    torch.cuda.synchronize()
    first = [_bits(y) for (_, _, y, _, _) in steps]
    exact = []
    for (layer, x, y, act, rows), got in zip(steps, first):
        ref = torch.empty_like(y)
        layer.forward(x, ref, act=act, rows=rows)
        torch.cuda.synchronize()
        exact.append(float(np.mean(_bits(ref) == got)))
    # same per-sub-block arithmetic; only where K is split differently the
    # reduction order differs
    assert np.mean(exact) > 0.97, exact
    chain.run()
    torch.cuda.synchronize()
    assert all(np.array_equal(_bits(y), f) for (_, _, y, _, _), f in zip(steps, first))
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            chain.run(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert all(np.array_equal(_bits(y), f) for (_, _, y, _, _), f in zip(steps, first))
    assert cq.device_status(0) == 0


def test_dependencies_follow_the_buffers(cq, oracle_mod):
    """Row-aligned single-producer inputs are read through tagged copies (no
    completion wait); reusing a buffer adds completion waits (write after read
    / write after write)."""
    import torch
    steps, _ = _block_chain(cq, oracle_mod, torch, "bf16", blocks=2)
    chain = cq.LinearChain(steps)
    names = [b[0] for b in BLOCK]
    info = [chain.step_info(i) for i in range(len(steps))]
    idx = {n: i for i, n in enumerate(names)}
    nb = len(names)
    assert info[idx["ffn1_up"]]["reads_tagged"] == -1          # chunk input
    assert info[idx["ffn1_down"]]["reads_tagged"] == idx["ffn1_up"]
    assert info[idx["pos"]]["reads_tagged"] == -1              # position table
    assert info[idx["out"]]["reads_tagged"] == idx["qkv"]      # the q columns of q|k|v
    assert info[nb + idx["ffn1_up"]]["reads_tagged"] == idx["ffn2_down"]
    assert all(i["waits_for"] == [] for i in info)             # distinct buffers
    assert info[idx["ffn1_down"]]["kslices"] > 1
    assert info[idx["ffn1_up"]]["kslices"] == 1
    # reuse: a second pass over the first block's buffers
    again = steps + [(l, x, y, a, r) for (l, x, y, a, r) in steps[:2]]
    chain2 = cq.LinearChain(again)
    i0 = len(steps)
    # rewriting ffn1_up's output waits for its readers and writers
    assert chain2.step_info(i0)["waits_for"] != []
    chain2.run()
    torch.cuda.synchronize()
    assert cq.device_status(0) == 0


@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_ragged_shapes_token_tiles_and_groups(cq, oracle_mod, dtype, group):
    """N not a multiple of the band, 1 and 17..40 rows, K = 2048 (split),
    biases and both activations, an input that is a column slice."""
    import torch
    tdt = getattr(torch, TDT[dtype])
    rng = np.random.default_rng(group)
    cases = [(1025, 640, 1, "none", True), (200, 2048, 17, "relu", False),
             (96, 1025 // 1 - 1, 40, "silu", True)]
    steps, meta = [], []
    prev = None
    for i, (n, k, rows, act, with_bias) in enumerate(cases):
        k = k - k % group
        layer, arrays = _layer(cq, oracle_mod, n, k, group, dtype, 7 + i, with_bias)
        if prev is None or prev.shape[1] < k or prev.shape[0] < rows:
            x = torch.from_numpy(oracle_mod.to_t(rng.standard_normal((rows, k + 8))
                                                 .astype(np.float32), dtype).view(np.int16)).cuda().view(tdt)
        else:
            x = prev
        y = torch.zeros((rows, n + 8), dtype=tdt, device="cuda")
        steps.append((layer, x, y, act, rows))
        meta.append((arrays, act, k, n))
        prev = y
    chain = cq.LinearChain(steps)
    for _ in range(2):
        chain.run()
    torch.cuda.synchronize()
    for (layer, x, y, act, rows), ((q, s, b, bias), _, k, n) in zip(steps, meta):
        xin = _bits(x)[:rows, :k]
        want = oracle_mod.qmatmul(np.ascontiguousarray(xin), q, s, b, group, dtype, bias, act)
        assert_parity(_bits(y)[:rows, :n], want, dtype, min_exact=0.9, bias_bits=bias, act=act)
        assert np.all(_bits(y)[:rows, n:] == 0)  # columns past N untouched
    assert cq.device_status(0) == 0


def test_invalid_chains_are_rejected(cq, oracle_mod):
    import torch
    layer, _ = _layer(cq, oracle_mod, 256, 256, 64, "bf16", 1, False)
    other, _ = _layer(cq, oracle_mod, 256, 256, 64, "f16", 2, False)
    x = torch.zeros((14, 256), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((14, 256), dtype=torch.bfloat16, device="cuda")
    big = torch.zeros((300, 256), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(cq.CQError, match="overlap"):
        cq.LinearChain([(layer, x, x, "none")])
    with pytest.raises(cq.CQError, match="rows must be"):
        cq.LinearChain([(layer, big, big.clone(), "none")])
    with pytest.raises(cq.CQError, match="same device, dtype"):
        cq.LinearChain([(layer, x, y, "none"), (other, y, x, "none")])
    with pytest.raises(cq.CQError, match="at least one step"):
        cq.LinearChain([])
