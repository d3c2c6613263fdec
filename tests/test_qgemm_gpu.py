"""GPU parity of the batched (M >= 256) tensor-core path against the oracle.

Many concurrent streams stack their chunk rows (64 streams x 14 frames =
896 rows per linear).  At these row counts the layer runs the tcgen05 GEMM,
which dequantises the weights to f16 in shared memory (the oracle keeps them
in fp32), so a few outputs may round to the neighbouring T value; the
conftest.TOL bounds hold.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GEMM_FLOOR, assert_parity
from test_qlinear_gpu import from_dev, make_case, run_gpu, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_dev(cq):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


BATCHED = [(4096, 1024), (1024, 4096), (3072, 1024), (2048, 1024), (1025, 640), (2560, 640),
           (640, 1024),
           # an odd number of k-tiles (the last pair holds one), and a K split
           # into slices of 18 and 17 k-tiles (M = 896)
           (640, 576), (1024, 2240)]


@pytest.mark.parametrize("n,k", BATCHED)
@pytest.mark.parametrize("m", [256, 896])
def test_batched_bf16_g64(cq, torch_dev, oracle_mod, n, k, m):
    q, s, b, x, bias = make_case(oracle_mod, n, k, m, 64, "bf16", seed=3 * n + k + m, with_bias=True)
    y = run_gpu(cq, torch_dev, q, s, b, bias, x, 64, "bf16")
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, 64, "bf16", bias), "bf16", min_exact=0.6, floor_frac=GEMM_FLOOR,
                  bias_bits=bias)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_batched_dtypes_groups_ragged(cq, torch_dev, oracle_mod, dtype, group):
    """Ragged M (not a multiple of 128), ragged N, and K % 64 == 32 for group 32."""
    k = 1056 if group == 32 else 1152
    q, s, b, x, bias = make_case(oracle_mod, 1000, k, 300, group, dtype, seed=group, with_bias=True)
    y = run_gpu(cq, torch_dev, q, s, b, bias, x, group, dtype, act="silu")
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, group, dtype, bias, "silu"), dtype,
                  min_exact=0.6, floor_frac=GEMM_FLOOR, bias_bits=bias, act="silu")


@pytest.mark.parametrize("m", [139, 255, 256, 257, 383])
def test_row_threshold(cq, torch_dev, oracle_mod, m):
    q, s, b, x, _ = make_case(oracle_mod, 1024, 1024, m, 64, "bf16", seed=m)
    y = run_gpu(cq, torch_dev, q, s, b, None, x, 64, "bf16")
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, 64, "bf16"), "bf16", min_exact=0.6, floor_frac=GEMM_FLOOR)


def test_batched_strided_rows(cq, torch_dev, oracle_mod):
    q, s, b, x, _ = make_case(oracle_mod, 640, 1024, 300, 64, "bf16", seed=5)
    y = run_gpu(cq, torch_dev, q, s, b, None, x, 64, "bf16", ldx_pad=64, ldy_pad=8)
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, 64, "bf16"), "bf16", min_exact=0.6, floor_frac=GEMM_FLOOR)


@pytest.mark.parametrize("xscale", [1e-30, 1e30])
def test_batched_bf16_activation_range(cq, torch_dev, oracle_mod, xscale):
    q, s, b, x, _ = make_case(oracle_mod, 1024, 1024, 256, 64, "bf16", seed=9, xscale=xscale)
    y = run_gpu(cq, torch_dev, q, s, b, None, x, 64, "bf16")
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, 64, "bf16"), "bf16", min_exact=0.6, floor_frac=GEMM_FLOOR)


def test_small_scales_stay_exact(cq, torch_dev, oracle_mod):
    """bf16 scales below the f16 normal range are not dequantised to f16."""
    rng = np.random.default_rng(4)
    w = (rng.standard_normal((512, 1024)) * 1e-6).astype(np.float32)
    q, s, b = oracle_mod.quantize(w, 64, "bf16")
    x = oracle_mod.to_t(rng.standard_normal((256, 1024)).astype(np.float32), "bf16")
    layer = cq.QuantizedLinear.from_packed(q, s, b, None, 64, "bf16")
    torch = torch_dev
    y = layer.forward(to_dev(torch, x, "bf16"))
    torch.cuda.synchronize()
    assert_parity(from_dev(y), oracle_mod.qmatmul(x, q, s, b, 64, "bf16"), "bf16", min_exact=0.9,
                  floor_frac=GEMM_FLOOR)


def test_reserve_then_graph_capture(cq, torch_dev, oracle_mod):
    torch = torch_dev
    q, s, b, x, _ = make_case(oracle_mod, 2048, 1024, 896, 64, "bf16", seed=21)
    layer = cq.QuantizedLinear.from_packed(q, s, b, None, 64, "bf16")
    layer.reserve(896)
    xd = to_dev(torch, x, "bf16")
    y = torch.zeros((896, 2048), dtype=torch.bfloat16, device="cuda")
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        layer.forward(xd, y, stream=st)  # warm: kernel attributes, tensor maps
    torch.cuda.synchronize()
    y.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        layer.forward(xd, y, stream=st)
    g.replay()
    torch.cuda.synchronize()
    assert_parity(from_dev(y), oracle_mod.qmatmul(x, q, s, b, 64, "bf16"), "bf16", min_exact=0.6, floor_frac=GEMM_FLOOR)
    del g


def test_device_status_clean_after_gemm(cq, torch_dev):
    assert cq.device_status(0) == 0


@pytest.mark.parametrize("act", ["none", "silu"])
def test_prescaled_path_is_bit_identical(cq, torch_dev, oracle_mod, act):
    """cq_linear_prescale_activations + cq_linear_forward_prescaled (the
    format the encoder's LayerNorm emits) give exactly cq_linear_forward_ex's
    output, which matches the oracle."""
    torch = torch_dev
    q, s, b, x, bias = make_case(oracle_mod, 4096, 1024, 896, 64, "bf16", seed=77, with_bias=True)
    layer = cq.QuantizedLinear.from_packed(q, s, b, bias, 64, "bf16")
    xd = to_dev(torch, x, "bf16")
    y_ref = layer.forward(xd, act=act)
    x16, rs = layer.prescale_activations(xd)
    y = layer.forward_prescaled(x16, rs, act=act)
    torch.cuda.synchronize()
    # row scales are powers of two that put each row's maximum in [2^14, 2^15)
    amax = x16.float().abs().amax(dim=1)
    assert bool(((amax >= 2.0 ** 14) & (amax < 2.0 ** 15)).all())
    assert torch.equal(torch.log2(rs), torch.round(torch.log2(rs)))
    assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
    assert_parity(from_dev(y), oracle_mod.qmatmul(x, q, s, b, 64, "bf16", bias, act), "bf16",
                  min_exact=0.6, floor_frac=GEMM_FLOOR, bias_bits=bias, act=act)


def test_prescaled_path_rejects_gemv_calls(cq, torch_dev, oracle_mod):
    torch = torch_dev
    q, s, b, x, _ = make_case(oracle_mod, 1024, 1024, 100, 64, "bf16", seed=78)
    layer = cq.QuantizedLinear.from_packed(q, s, b, None, 64, "bf16")
    xd = to_dev(torch, x, "bf16")
    with pytest.raises(cq.CQError) as ei:
        layer.prescale_activations(xd)
    assert "tensor-core activation format" in str(ei.value)
    x16 = torch.zeros((100, 1024), dtype=torch.float16, device="cuda")
    rs = torch.ones((100,), dtype=torch.float32, device="cuda")
    with pytest.raises(cq.CQError):
        layer.forward_prescaled(x16, rs)
