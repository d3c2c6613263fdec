"""GPU parity of the quantized linear against the CPU oracle, through the C ABI.

The CUDA path and the oracle consume identical packed inputs; both accumulate
in fp32 and round to T at the same two points (quantized_matmul result, then
the output-bias add), so outputs agree to within one T ulp (tolerances in
conftest.TOL).  Shapes cover every encoder / RNNT / prompt call site
(crates/nemotron-mlx/src/model/encoder.rs, rnnt.rs, prompt.rs), ragged N and K,
token tiles beyond 16 rows, strided rows, fused activations, and the
reference's own known-answer tests.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_parity, golden, parity_stats

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_dev(cq):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    assert cq.is_device_available(), "no sm_100 device visible to the library"
    return torch


TDT = {"f16": "float16", "bf16": "bfloat16"}


def to_dev(torch, bits: np.ndarray, dtype: str, pad_cols: int = 0):
    a = np.ascontiguousarray(bits).view(np.int16)
    if pad_cols:
        a = np.pad(a, ((0, 0), (0, pad_cols)))
    return torch.from_numpy(a).cuda().view(getattr(torch, TDT[dtype]))


def from_dev(t) -> np.ndarray:
    import torch
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def make_case(oracle_mod, n, k, m, group, dtype, seed, with_bias=False, xscale=1.0):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    q, s, b = oracle_mod.quantize(w, group, dtype)
    x = oracle_mod.to_t((rng.standard_normal((m, k)) * xscale).astype(np.float32), dtype)
    bias = oracle_mod.to_t((rng.standard_normal(n) * 0.1).astype(np.float32), dtype) if with_bias else None
    return q, s, b, x, bias


def run_gpu(cq, torch, q, s, b, bias, x, group, dtype, act="none", ldx_pad=0, ldy_pad=0):
    layer = cq.QuantizedLinear.from_packed(q, s, b, bias, group, dtype)
    xd = to_dev(torch, x, dtype, ldx_pad)
    m = x.shape[0]
    yfull = torch.zeros((m, layer.output_dims + ldy_pad), dtype=xd.dtype, device="cuda")
    layer.forward(xd, yfull, act=act)
    torch.cuda.synchronize()
    return from_dev(yfull[:, : layer.output_dims])


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_golden_vectors(cq, torch_dev, dtype, group):
    z = golden(f"oracle_{dtype}_g{group}.npz")
    names = sorted({k.rsplit("_", 1)[0] for k in z if k.endswith("_meta")})
    for name in names:
        m, n, k, with_bias, act = (int(v) for v in z[f"{name}_meta"])
        y = run_gpu(cq, torch_dev, z[f"{name}_q"], z[f"{name}_s"], z[f"{name}_b"],
                    z.get(f"{name}_bias"), z[f"{name}_x"], group, dtype,
                    ["none", "silu", "relu"][act])
        try:
            assert_parity(y, z[f"{name}_y"], dtype, min_exact=0.97,
                          bias_bits=z.get(f"{name}_bias"), act=["none", "silu", "relu"][act])
        except AssertionError as e:
            raise AssertionError(f"golden case {name}: {e}") from None


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_single_linear_m14_4096x1024_g64(cq, torch_dev, oracle_mod, dtype):
    """The single-linear workload: x [14,1024] . W[4096,1024]^T, group 64."""
    q, s, b, x, _ = make_case(oracle_mod, 4096, 1024, 14, 64, dtype, seed=0)
    y = run_gpu(cq, torch_dev, q, s, b, None, x, 64, dtype)
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, 64, dtype), dtype, min_exact=0.97)


# (N, K) of every quantized-linear call site at batch 1.
CALL_SITES = [
    (4096, 1024),  # FFN linear1 (encoder.rs:300-337)
    (1024, 4096),  # FFN linear2
    (1024, 1024),  # q/k/v/out/pos (encoder.rs:45-267), conv pw2
    (3072, 1024),  # fused q|k|v
    (2048, 1024),  # conv pw1 (encoder.rs:381)
    (1024, 4352),  # subsampling output linear (encoder.rs:797)
    (2048, 1152),  # prompt projector 1 (prompt.rs:105-140)
    (1024, 2048),  # prompt projector 2
    (640, 1024),   # RNNT encoder projector (rnnt.rs:377)
    (2560, 640),   # LSTM ih / hh (rnnt.rs:113-148)
    (640, 640),    # decoder projector (rnnt.rs:296)
    (1025, 640),   # joint head, vocab 1025
]


@pytest.mark.parametrize("n,k", CALL_SITES)
@pytest.mark.parametrize("m", [1, 4, 14])
def test_call_site_shapes_bf16_g64(cq, torch_dev, oracle_mod, n, k, m):
    q, s, b, x, bias = make_case(oracle_mod, n, k, m, 64, "bf16", seed=n + k + m, with_bias=True)
    y = run_gpu(cq, torch_dev, q, s, b, bias, x, 64, "bf16")
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, 64, "bf16", bias), "bf16", min_exact=0.97,
                  bias_bits=bias)


@pytest.mark.parametrize("n,k", [(4096, 1024), (1024, 4096), (1025, 640), (13088, 640)])
@pytest.mark.parametrize("group", [32, 128])
def test_call_site_shapes_f16_other_groups(cq, torch_dev, oracle_mod, n, k, group):
    """The reference's release artifact: f16 scales, group 128 (manifest.rs:344-357)."""
    q, s, b, x, bias = make_case(oracle_mod, n, k, 14, group, "f16", seed=7 * n + k, with_bias=True)
    y = run_gpu(cq, torch_dev, q, s, b, bias, x, group, "f16")
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, group, "f16", bias), "f16", min_exact=0.97,
                  bias_bits=bias)


@pytest.mark.parametrize("m", [15, 16, 17, 31, 33, 100, 139, 255])
def test_token_tiles_beyond_16_rows(cq, torch_dev, oracle_mod, m):
    """16 < M < 256 spreads 16-row token tiles over CTAs (256 rows and more run the GEMM)."""
    q, s, b, x, bias = make_case(oracle_mod, 1024, 1024, m, 64, "bf16", seed=m, with_bias=True)
    y = run_gpu(cq, torch_dev, q, s, b, bias, x, 64, "bf16")
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, 64, "bf16", bias), "bf16", min_exact=0.97,
                  bias_bits=bias)


@pytest.mark.parametrize("m", [14, 17, 33, 100, 139])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_k_split_token_tiles(cq, torch_dev, oracle_mod, m, dtype):
    """K = 4096 splits over a 4-CTA cluster whose partials meet in the leader's shared
    memory: one token tile per CTA (M <= 33 here) or several per CTA (100, 139), where
    the leader's slots are reused from tile to tile."""
    q, s, b, x, bias = make_case(oracle_mod, 1024, 4096, m, 64, dtype, seed=40 + m, with_bias=True)
    y = run_gpu(cq, torch_dev, q, s, b, bias, x, 64, dtype)
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, 64, dtype, bias), dtype, min_exact=0.97,
                  bias_bits=bias)


@pytest.mark.parametrize("act", ["silu", "relu"])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_fused_activation(cq, torch_dev, oracle_mod, act, dtype):
    q, s, b, x, bias = make_case(oracle_mod, 4096, 1024, 14, 64, dtype, seed=11, with_bias=True)
    y = run_gpu(cq, torch_dev, q, s, b, bias, x, 64, dtype, act=act)
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, 64, dtype, bias, act), dtype, min_exact=0.97,
                  bias_bits=bias, act=act)


@pytest.mark.parametrize("ldx_pad", [64, 8])
def test_strided_rows(cq, torch_dev, oracle_mod, ldx_pad):
    """Row strides of 1088 and 1032 elements: 32-byte aligned rows take the 256-bit
    activation loads, 16-byte aligned ones the pairs of 128-bit loads."""
    q, s, b, x, _ = make_case(oracle_mod, 640, 1024, 9, 64, "bf16", seed=21)
    y = run_gpu(cq, torch_dev, q, s, b, None, x, 64, "bf16", ldx_pad=ldx_pad, ldy_pad=5)
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, 64, "bf16"), "bf16", min_exact=0.97)


@pytest.mark.parametrize("xscale", [1e-30, 1e-3, 1e3, 1e30])
def test_bf16_activation_range(cq, torch_dev, oracle_mod, xscale):
    """bf16 activations far outside the f16 range stay exact (the bf16 MMA takes them as
    they are)."""
    q, s, b, x, _ = make_case(oracle_mod, 1024, 1024, 14, 64, "bf16", seed=3, xscale=xscale)
    y = run_gpu(cq, torch_dev, q, s, b, None, x, 64, "bf16")
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, 64, "bf16"), "bf16", min_exact=0.97)


def test_constant_groups_and_zero_input(cq, torch_dev, oracle_mod):
    rng = np.random.default_rng(8)
    w = (rng.standard_normal((256, 512)) * 0.02).astype(np.float32)
    w[:, :64] = 0.125    # constant group: scale 0
    w[7, :] = -0.5       # constant row
    q, s, b = oracle_mod.quantize(w, 64, "bf16")
    x = oracle_mod.to_t(rng.standard_normal((14, 512)).astype(np.float32), "bf16")
    x[3, :] = 0          # an all-zero token
    y = run_gpu(cq, torch_dev, q, s, b, None, x, 64, "bf16")
    want = oracle_mod.qmatmul(x, q, s, b, 64, "bf16")
    assert_parity(y, want, "bf16", min_exact=0.97)
    assert np.all(oracle_mod.from_t(y[3], "bf16") == 0)


def test_bit_identical_reruns(cq, torch_dev, oracle_mod):
    q, s, b, x, _ = make_case(oracle_mod, 1024, 4096, 14, 64, "bf16", seed=12)
    y1 = run_gpu(cq, torch_dev, q, s, b, None, x, 64, "bf16")
    y2 = run_gpu(cq, torch_dev, q, s, b, None, x, 64, "bf16")
    assert np.array_equal(y1, y2)


def test_concat_matches_separate_layers(cq, torch_dev, oracle_mod):
    torch = torch_dev
    parts, outs, biases = [], [], []
    x = None
    for i, n in enumerate((1024, 1024, 512)):
        q, s, b, xx, bias = make_case(oracle_mod, n, 1024, 14, 64, "bf16", seed=40 + i,
                                      with_bias=(i == 1))
        x = xx if x is None else x
        parts.append(cq.QuantizedLinear.from_packed(q, s, b, bias, 64, "bf16"))
        outs.append(oracle_mod.qmatmul(x, q, s, b, 64, "bf16", bias))
        biases.append(bias if bias is not None else np.zeros(n, np.uint16))
    fused = cq.QuantizedLinear.concat(parts)
    assert fused.output_dims == 2560
    y = fused.forward(to_dev(torch, x, "bf16"))
    torch.cuda.synchronize()
    assert_parity(from_dev(y), np.concatenate(outs, axis=1), "bf16", min_exact=0.97,
                  bias_bits=np.concatenate(biases))


# ---------------------------------------------------------------- reference KATs


def test_reference_kat_quantized_matmul(cq, torch_dev):
    """crates/nemotron-mlx/tests/quantized_matmul.rs:24-47, abs 0.06, via cq_quantized_matmul."""
    k = golden("reference_kats.npz")
    rows, ind, outd, g = (int(v) for v in k["qmm_meta"])
    y = cq.quantized_matmul(k["qmm_input"], rows, ind, k["qmm_weight"], outd, g)
    assert y.shape == k["qmm_expected"].shape
    assert np.abs(y - k["qmm_expected"]).max() <= k["tolerances"][0]


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_reference_kat_linear_with_bias(cq, torch_dev, dtype):
    """model_layers.rs:35-55, abs 0.08, via from_f32 + forward_f32."""
    k = golden("reference_kats.npz")
    layer = cq.QuantizedLinear.from_f32(k["lin_weight"], 3, 128, k["lin_bias"], 128, dtype)
    y = layer.forward_f32(k["lin_input"], 2)
    assert np.abs(y - k["lin_expected"]).max() <= k["tolerances"][1]


def test_reference_kat_pointwise(cq, torch_dev):
    """model_layers.rs:57-78: shape [1, 3, 2] preserved, abs 0.08."""
    k = golden("reference_kats.npz")
    conv = cq.PointwiseConv1d.from_f32(k["pw_weight"], 2, 128, k["pw_bias"], 128)
    y = conv.forward_f32(k["pw_input"], 1, 3)
    assert y.shape == (1, 3, 2)
    assert np.abs(y.ravel() - k["pw_expected"]).max() <= k["tolerances"][2]


def test_reference_kat_packed_artifact_layer(cq, torch_dev, oracle_mod):
    """weight_roundtrip.rs:50-115: f16 artifact arrays bound without requantising."""
    k = golden("reference_kats.npz")
    q, s, b = oracle_mod.quantize(k["art_matrix"].reshape(2, 128), 128, "f16")
    layer = cq.QuantizedLinear.from_packed(q, s, b, None, 128, "f16")
    y = layer.forward_f32(k["art_input"], 1)
    assert np.abs(y - k["art_expected"]).max() <= k["tolerances"][4]
    # the same packed arrays dequantise within 0.008 of the source matrix
    torch = torch_dev
    qd = torch.from_numpy(q.view(np.int32)).cuda()
    sd = to_dev(torch, s, "f16")
    bd = to_dev(torch, b, "f16")
    q2, s2, b2 = oracle_mod.quantize(k["rt_matrix"].reshape(2, 128), 128, "f16")
    w = cq.dequantize(torch.from_numpy(q2.view(np.int32)).cuda(), to_dev(torch, s2, "f16"),
                      to_dev(torch, b2, "f16"), 128, "f16")
    torch.cuda.synchronize()
    assert np.abs(w.cpu().numpy().ravel() - k["rt_matrix"]).max() <= k["tolerances"][3]
    del qd, sd, bd


def test_forward_f32_rejects_wrong_input_length(cq, torch_dev):
    layer = cq.QuantizedLinear.from_f32(np.zeros(128), 1, 128, np.zeros(1), 128)
    with pytest.raises(cq.CQError) as ei:
        layer.forward_f32(np.zeros(127), 1)
    assert "linear input has 127 values, expected 1x128" in str(ei.value)
    assert ei.value.status == cq.CQ_INVALID_ARGUMENT


@pytest.mark.parametrize("dtype", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_device_quantize_is_bit_exact(cq, torch_dev, oracle_mod, dtype, group):
    torch = torch_dev
    rng = np.random.default_rng(group)
    w = (rng.standard_normal((300, 512)) * 0.03).astype(np.float32)
    # groups that separate MLX's edge/sign rule from a plain min/max rule:
    # constant, all zero, one-signed either way, max edge, min edge, |min| == |max|
    w[5, :group] = 0.75
    w[6, :group] = 0.0
    w[7] = np.abs(w[7]) + 0.01
    w[8] = -np.abs(w[8]) - 0.01
    w[9, :3] = [1.0, -0.5, 0.0]
    w[10, :3] = [-1.0, 0.5, 0.0]
    w[11, :2] = [-1.0, 1.0]
    w[12] *= 1e4  # large values
    w[13] *= 1e-4  # small values
    q, s, b = cq.quantize(torch.from_numpy(w).cuda(), group, dtype, round_input=dtype != "f32")
    torch.cuda.synchronize()
    q0, s0, b0 = oracle_mod.quantize(w, group, dtype, round_input=dtype != "f32")
    assert np.array_equal(q.cpu().numpy().view(np.uint32), q0)
    if dtype == "f32":
        assert np.array_equal(s.cpu().numpy(), s0) and np.array_equal(b.cpu().numpy(), b0)
    else:
        assert np.array_equal(from_dev(s), s0) and np.array_equal(from_dev(b), b0)
    wd = cq.dequantize(q, s, b, group, dtype)
    torch.cuda.synchronize()
    assert np.array_equal(wd.cpu().numpy(), oracle_mod.dequantize(q0, s0, b0, group, dtype))


def test_from_f32_matches_oracle_quantiser(cq, torch_dev, oracle_mod):
    """QuantizedLinear::from_f32 (layers.rs:259-280) == oracle quantise + forward."""
    rng = np.random.default_rng(77)
    w = (rng.standard_normal((1024, 1024)) * 0.02).astype(np.float32)
    bias = (rng.standard_normal(1024) * 0.1).astype(np.float32)
    x = rng.standard_normal((14, 1024)).astype(np.float32)
    layer = cq.QuantizedLinear.from_f32(w, 1024, 1024, bias, 64, "bf16")
    y = layer.forward_f32(x, 14).reshape(14, 1024)
    q, s, b = oracle_mod.quantize(w, 64, "bf16")
    want = oracle_mod.qmatmul(oracle_mod.to_t(x, "bf16"), q, s, b, 64, "bf16",
                              oracle_mod.to_t(bias, "bf16"))
    assert_parity(oracle_mod.to_t(y, "bf16"), want, "bf16", min_exact=0.97,
                  bias_bits=oracle_mod.to_t(bias, "bf16"))


def test_device_status_clean(cq, torch_dev):
    assert cq.device_status(0) == 0


# The diarizer's Fast-Conformer (crates/sortformer-mlx/src/model/encoder.rs)
# binds the same QuantizedLinear, with output biases everywhere: d_model 512,
# ff 2048, 8 heads, 256 subsampling channels over 16 frequency bins
# (tests/fixtures/sortformer_config.json); a 188-frame chunk with context
# runs about 190 rows per call.
SORTFORMER_SITES = [
    (2048, 512),  # FFN linear1 (encoder.rs:413-431)
    (512, 2048),  # FFN linear2
    (512, 512),   # q/k/v/out/pos (encoder.rs:446-480), conv pointwise2
    (1024, 512),  # conv pointwise1 (encoder.rs:570-612)
    (256, 256),   # subsampling pointwise convs (encoder.rs:283-335)
    (512, 4096),  # subsampling output linear
]


@pytest.mark.parametrize("n,k", SORTFORMER_SITES)
@pytest.mark.parametrize("m", [1, 190])
def test_sortformer_call_sites_f16(cq, torch_dev, oracle_mod, n, k, m):
    q, s, b, x, bias = make_case(oracle_mod, n, k, m, 64, "f16", seed=5 * n + k + m, with_bias=True)
    y = run_gpu(cq, torch_dev, q, s, b, bias, x, 64, "f16")
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, 64, "f16", bias), "f16", min_exact=0.97,
                  bias_bits=bias)


@pytest.mark.parametrize("n,k", [(2048, 512), (512, 2048), (512, 4096)])
def test_sortformer_call_sites_batched(cq, torch_dev, oracle_mod, n, k):
    """Two streams' chunks stacked (400 rows): the tensor-core GEMM."""
    from conftest import GEMM_FLOOR
    q, s, b, x, bias = make_case(oracle_mod, n, k, 400, 128, "f16", seed=n + 3 * k, with_bias=True)
    y = run_gpu(cq, torch_dev, q, s, b, bias, x, 128, "f16")
    assert_parity(y, oracle_mod.qmatmul(x, q, s, b, 128, "f16", bias), "f16", min_exact=0.6,
                  floor_frac=GEMM_FLOOR, bias_bits=bias)
