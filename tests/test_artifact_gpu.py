"""Models bound from a release artifact on the GPU (include/cqartifact.h)
against the oracles bound from the same files through the numpy reader in
oracle/artifact_oracle.py.

* the reference's converted-artifact fixture (crates/nemotron-mlx/tests/
  encoder_artifact.rs:14-242): the one-block encoder it builds, a 9-frame
  chunk of 0.25 -> [1, 2, 128], then more chunks of seeded mel frames;
* a seeded two-block encoder artifact, two streams, several chunks;
* QuantizedLinear::from_artifact with and without output bias, both dtypes,
  on the GEMV and GEMM paths;
* an RNNT decoder artifact, greedy paths checked by teacher forcing.
The artifact holds F16 scales and biases; a bf16 model rounds them to bf16 on
load, and the oracle is handed the same rounding.  Tolerances are those of
test_encoder_gpu.py and test_rnnt_gpu.py.
"""
from __future__ import annotations

import numpy as np
import pytest

import artifact_oracle as ao
from conftest import GEMM_FLOOR, assert_parity
import encoder_oracle as eo
import rnnt_oracle as ro

pytestmark = pytest.mark.gpu

TOL = {"bf16": (2e-2, 8e-2), "f16": (4e-3, 1.6e-2)}

SMALL_ENCODER = dict(hidden=256, ff=512, layers=2, heads=2, conv_kernel=9, sliding_window=21,
                     mel_bins=32, sub_channels=64, num_prompts=64, prompt_hidden=256,
                     group_size=64)
SMALL_RNNT = dict(enc_hidden=256, pred_hidden=128, joint_hidden=128, vocab=65, max_symbols=3,
                  group_size=64)


def _ecfg(d):
    return eo.EncoderConfig(hidden=d["hidden"], ff=d["ff"], layers=d["layers"], heads=d["heads"],
                            conv_kernel=d["conv_kernel"], sliding_window=d["sliding_window"],
                            mel_bins=d["mel_bins"], sub_channels=d["sub_channels"],
                            num_prompts=d["num_prompts"], prompt_hidden=d["prompt_hidden"],
                            group=d["group_size"])


def _compare(got_t, want, dtype, what):
    got = got_t.float().cpu().numpy().astype(np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    assert np.all(np.isfinite(got)), what
    diff = np.abs(got - want)
    rel_l2 = float(np.sqrt((diff ** 2).sum() / max((want ** 2).sum(), 1e-30)))
    rel_max = float(diff.max() / max(np.abs(want).max(), 1e-30))
    l2_tol, max_tol = TOL[dtype]
    assert rel_l2 <= l2_tol and rel_max <= max_tol, (what, rel_l2, rel_max)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_encoder_binds_the_reference_fixture(cq, oracle_mod, tmp_path, dtype):
    import torch
    from nemotron_cuda.artifact import Artifact
    from nemotron_cuda.encoder import Encoder, EncoderConfig
    path = str(tmp_path / "artifact")
    ao.convert_tensors(path, "fixture/subsampling", ao.reference_fixture_specs())
    d = ao.REFERENCE_FIXTURE_CONFIG
    cfg = _ecfg(d)
    with Artifact(path) as art:
        enc = Encoder.from_artifact(art, EncoderConfig.default(**d), dtype)
    ref_art = ao.Artifact(path)
    ref = eo.Encoder(cfg, ao.model_params(ref_art, eo.linear_names(cfg), eo.dense_names(cfg),
                                          dtype), dtype)
    cache = ref.new_cache()
    state = enc.state(1, 9)
    mel = np.full((1, 9, 8), 0.25, np.float32)
    out = state.encode_chunk(torch.from_numpy(mel).cuda())
    torch.cuda.synchronize()
    assert tuple(out.shape) == (2, 128)  # [1, 2, channels] in the reference test
    _compare(out, ref.encode_chunk(mel[0], 101, cache), dtype, "fixture chunk 0")
    rng = np.random.default_rng(2)
    for chunk in range(1, 4):
        mel = rng.standard_normal((1, 9, 8)).astype(np.float32)
        out = state.encode_chunk(torch.from_numpy(mel).cuda())
        torch.cuda.synchronize()
        _compare(out, ref.encode_chunk(mel[0], 101, cache), dtype, f"fixture chunk {chunk}")
    assert cq.device_status(0) == 0


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_seeded_encoder_artifact_matches_oracle(cq, oracle_mod, tmp_path, dtype):
    import torch
    from nemotron_cuda.artifact import Artifact
    from nemotron_cuda.encoder import Encoder, EncoderConfig
    cfg = _ecfg(SMALL_ENCODER)
    path = str(tmp_path / "artifact")
    ao.convert_tensors(path, "fixture/encoder", ao.random_specs(
        eo.linear_names(cfg), eo.dense_names(cfg), cfg.group, seed=17))
    enc = Encoder(EncoderConfig.default(**SMALL_ENCODER), dtype)
    with Artifact(path) as art:
        enc.bind_artifact(art)
    ref = eo.Encoder(cfg, ao.model_params(ao.Artifact(path), eo.linear_names(cfg),
                                          eo.dense_names(cfg), dtype), dtype)
    streams = 2
    state = enc.state(streams, 112)
    state.set_prompts([5, 9])
    caches = [ref.new_cache() for _ in range(streams)]
    rng = np.random.default_rng(4)
    for chunk in range(3):
        mel = rng.standard_normal((streams, 112, cfg.mel_bins)).astype(np.float32)
        out = state.encode_chunk(torch.from_numpy(mel).cuda())
        torch.cuda.synchronize()
        frames = out.shape[0] // streams
        for s, pid in enumerate((5, 9)):
            _compare(out[s * frames:(s + 1) * frames], ref.encode_chunk(mel[s], pid, caches[s]),
                     dtype, f"chunk {chunk} stream {s}")
    assert cq.device_status(0) == 0


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("rows", [1, 300])
def test_linear_from_artifact_matches_oracle(cq, oracle_mod, tmp_path, dtype, rows):
    import torch
    from nemotron_cuda import QuantizedLinear
    from nemotron_cuda.artifact import Artifact
    path = str(tmp_path / "artifact")
    names = {"joint.head.weight": (1025, 640, True), "decoder.lstm.weight_ih_l0": (2560, 640, False)}
    ao.convert_tensors(path, "fixture/linears", ao.random_specs(names, {}, 64, seed=3))
    ref = ao.model_params(ao.Artifact(path), names, {}, dtype)
    rng = np.random.default_rng(rows)
    with Artifact(path) as art:
        for name, (n, k, has_bias) in names.items():
            bias_name = "joint.head.bias" if has_bias else None
            L = QuantizedLinear.from_artifact(art, name, bias_name, dtype)
            assert (L.output_dims, L.input_dims, L.group_size) == (n, k, 64)
            x = oracle_mod.to_t(rng.standard_normal((rows, k)).astype(np.float32), dtype)
            tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
            xd = torch.from_numpy(x.view(np.int16)).cuda().view(tdt)
            y = L.forward(xd)
            torch.cuda.synchronize()
            q, s, b, bias = ref[name]
            want = oracle_mod.qmatmul(x, q, s, b, 64, dtype, bias)
            got = y.cpu().view(torch.int16).numpy().view(np.uint16)
            # the quantized-linear parity bar (conftest.assert_parity): within
            # two T ulps; the GEMV keeps the oracle's summation order closely
            # (>= 95% bit-exact), the tensor-core GEMM sums in tiles, so in f16
            # (3 more mantissa bits than bf16) about 40% of outputs sit one ulp
            # away
            if rows == 1:
                assert_parity(got, want, dtype, min_exact=0.95, bias_bits=bias)
            else:
                assert_parity(got, want, dtype, min_exact=0.5, bias_bits=bias,
                              floor_frac=GEMM_FLOOR)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_rnnt_artifact_greedy_paths_match_oracle(cq, oracle_mod, tmp_path, dtype):
    import torch
    from nemotron_cuda.artifact import Artifact
    from nemotron_cuda.rnnt import Rnnt, RnntConfig
    cfg = ro.RnntConfig(enc_hidden=256, pred_hidden=128, joint_hidden=128, vocab=65,
                        max_symbols=3, group=64)
    path = str(tmp_path / "artifact")
    ao.convert_tensors(path, "fixture/rnnt", ao.random_specs(
        ro.linear_names(cfg), ro.dense_names(cfg), 64, seed=23,
        std={"decoder.embedding.weight": 1.0}))
    with Artifact(path) as art:
        dec = Rnnt.from_artifact(art, RnntConfig.default(**SMALL_RNNT), dtype)
    ref = ro.RnntDecoder(cfg, ao.model_params(ao.Artifact(path), ro.linear_names(cfg),
                                              ro.dense_names(cfg), dtype), dtype)
    streams, frames = 2, 5
    state = dec.state(streams, frames)
    caches = [ref.new_state() for _ in range(streams)]
    rng = np.random.default_rng(6)
    decisions = differ = 0
    for _ in range(2):
        enc = rng.standard_normal((streams, frames, cfg.enc_hidden)).astype(np.float32)
        bits = oracle_mod.to_t(enc.reshape(streams * frames, -1), dtype).view(np.int16)
        dev = torch.from_numpy(bits).cuda().view(torch.bfloat16 if dtype == "bf16" else torch.float16)
        paths = state.decode_chunk(dev, frames)
        for s in range(streams):
            stats = ro.check_path(ref, enc[s], caches[s], paths[s])
            assert stats["mismatch"] == 0, (s, stats)
            decisions += stats["decisions"]
            differ += stats["differ"]
    assert differ <= max(1, decisions // 20), (differ, decisions)
    assert cq.device_status(0) == 0


def test_binding_checks_the_model_shape(cq, oracle_mod, tmp_path):
    from nemotron_cuda import CQError
    from nemotron_cuda.artifact import Artifact
    from nemotron_cuda.encoder import Encoder, EncoderConfig
    path = str(tmp_path / "artifact")
    ao.convert_tensors(path, "fixture/subsampling", ao.reference_fixture_specs())
    wider = dict(ao.REFERENCE_FIXTURE_CONFIG, hidden=256, ff=256, prompt_hidden=256)
    enc = Encoder(EncoderConfig.default(**wider), "f16")
    with Artifact(path) as art:
        with pytest.raises(CQError, match="invalid model shape"):
            enc.bind_artifact(art)
    two_layers = dict(ao.REFERENCE_FIXTURE_CONFIG, layers=2)
    enc = Encoder(EncoderConfig.default(**two_layers), "f16")
    with Artifact(path) as art:
        with pytest.raises(CQError, match="^missing artifact tensor encoder.layers.1"):
            enc.bind_artifact(art)
