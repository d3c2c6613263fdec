"""Pins the encoder oracle (CPU only) to the reference's own encoder tests.

Each test restates one test of crates/nemotron-mlx/tests/encoder_streaming.rs
or model_layers.rs with the same inputs, expected values and tolerances, run
against oracle/encoder_oracle.py.  The reference runs these ops in f16, so the
oracle runs them with T = f16 here.
"""
from __future__ import annotations

import numpy as np
import pytest

import encoder_oracle as eo


def identity(n):
    return np.eye(n, dtype=np.float32)


def test_causal_cache_prepends_previous_frames_and_updates_itself():
    """model_layers.rs:80-93."""
    cache = eo.CausalConv1dCache(2, 2)
    first = cache.prepend_and_update(np.array([1.0, 10.0]), 1)
    assert first.tolist() == [0.0, 0.0, 0.0, 0.0, 1.0, 10.0]
    assert cache.values.tolist() == [0.0, 0.0, 1.0, 10.0]
    second = cache.prepend_and_update(np.array([2.0, 20.0, 3.0, 30.0]), 2)
    assert second.tolist() == [0.0, 0.0, 1.0, 10.0, 2.0, 20.0, 3.0, 30.0]
    assert cache.values.tolist() == [2.0, 20.0, 3.0, 30.0]


def test_depthwise_conv_matches_causal_cross_correlation(oracle_mod):
    """model_layers.rs:95-112: kernel 3 over two channels, bias, tolerance 2e-3."""
    x = np.array([1.0, 10.0, 2.0, 20.0, 3.0, 30.0, 4.0, 40.0], np.float32).reshape(4, 2)
    layer = eo.DepthwiseConv1d(np.array([[1.0, 0.0, -1.0], [0.5, 0.25, 0.0]]),
                               np.array([0.5, -1.0]), "f16")
    got = layer.forward(x, eo.CausalConv1dCache(2, 2))
    want = np.array([-0.5, -1.0, -1.5, 1.5, -1.5, 9.0, -1.5, 16.5]).reshape(4, 2)
    assert got.shape == (4, 2)
    assert np.abs(got - want).max() <= 2e-3


def test_layer_norm_matches_cpu_reference(oracle_mod):
    """model_layers.rs:114-137: f16 inputs and affine parameters, tolerance 1e-3."""
    x = np.array([1.0, 2.0, 4.0, -1.0, 0.0, 3.0], np.float32).reshape(2, 3)
    w, b = np.array([1.0, 0.5, 2.0]), np.array([0.0, 1.0, -1.0])
    got = eo.layer_norm(x, w, b, 1e-5, "f16")
    mean = x.mean(1, keepdims=True)
    var = ((x - mean) ** 2).mean(1, keepdims=True)
    want = (x - mean) / np.sqrt(var + 1e-5) * w + b
    assert np.abs(got - want).max() <= 1e-3


def _conv2d_reference(values, time, freq, first):
    """encoder_streaming.rs:128-156 (the reference test's own direct sum)."""
    temporal = ([0.0] * (2 * freq) if first else []) + list(values)
    padded_time = len(temporal) // freq
    out_time = (padded_time - 3) // 2 + 1
    out_freq = (freq + 3 - 3) // 2 + 1
    out = []
    for t in range(out_time):
        for f in range(out_freq):
            s = 0.0
            for kt in range(3):
                for kf in range(3):
                    sf = f * 2 + kf
                    if 2 <= sf < 2 + freq:
                        s += temporal[(t * 2 + kt) * freq + sf - 2]
            out.append(s)
    return np.array(out)


def test_causal_conv2d_first_and_subsequent_chunks_use_exact_padding_cache(oracle_mod):
    """encoder_streaming.rs:94-126."""
    conv = eo.Conv2d(np.ones((1, 1, 3, 3)), np.zeros(1), 2, 1, "f16")
    cache = eo.CausalConv2dCache(4, 1, 1, 1)
    first = np.arange(1, 13, dtype=np.float32).reshape(3, 4, 1)
    out1 = conv.forward_causal(first, cache)
    assert out1.shape == (2, 3, 1)
    assert cache.values.ravel().tolist() == [9.0, 10.0, 11.0, 12.0]
    assert np.abs(out1.ravel() - _conv2d_reference(first.ravel(), 3, 4, True)).max() <= 1e-3
    second = np.arange(13, 21, dtype=np.float32).reshape(2, 4, 1)
    out2 = conv.forward_causal(second, cache)
    assert out2.shape == (1, 3, 1)
    assert cache.values.ravel().tolist() == [17.0, 18.0, 19.0, 20.0]
    cached = [9.0, 10.0, 11.0, 12.0] + second.ravel().tolist()
    assert np.abs(out2.ravel() - _conv2d_reference(cached, 3, 4, False)).max() <= 1e-3


def _tiny_subsampling(channels):
    """encoder_streaming.rs:210-262."""
    stem = eo.Conv2d(np.full((channels, 1, 3, 3), 0.01), np.zeros(channels), 2, 1, "f16")
    stages = []
    for _ in range(2):
        dw = eo.Conv2d(np.full((channels, 1, 3, 3), 0.01), np.zeros(channels), 2, channels, "f16")
        pw = eo.QLinear.from_f32(identity(channels), np.zeros(channels), 128, "f16")
        stages.append((dw, pw))
    w = np.zeros((channels, channels * 2), np.float32)
    for c in range(channels):
        w[c, c] = 0.5
        w[c, channels + c] = 0.5
    out = eo.QLinear.from_f32(w, np.zeros(channels), 128, "f16")
    return eo.Subsampling(stem, stages, out), eo.SubsamplingCache(8, channels, 3, 2, 3)


def test_factor_eight_subsampling_matches_one_shot_across_chunk_boundary(oracle_mod):
    """encoder_streaming.rs:158-208: 9 + 8 streamed frames equal 17 offline frames."""
    channels = 128
    x = ((np.arange(17 * 8) % 23).astype(np.float32) - 11.0) / 17.0
    x = x.reshape(17, 8)
    off_model, off_cache = _tiny_subsampling(channels)
    st_model, st_cache = _tiny_subsampling(channels)
    offline = off_model.forward(x, off_cache)
    first = st_model.forward(x[:9], st_cache)
    second = st_model.forward(x[9:], st_cache)
    assert offline.shape == (3, channels)
    assert first.shape == (2, channels)
    assert second.shape == (1, channels)
    assert np.all(np.abs(first[1:]) < 1e-6), "the extra ceil frame in the first chunk must be masked"
    streamed = np.concatenate([first, second])
    assert np.abs(streamed - offline).max() <= 3e-3


def test_attention_cache_returns_old_plus_current_and_retains_sliding_window():
    """encoder_streaming.rs:272-295."""
    cache = eo.AttentionKvCache(2, 2, 3)
    k1 = np.arange(8, dtype=np.float32)
    v1 = np.arange(100, 108, dtype=np.float32)
    frames, keys, _ = cache.update(k1, v1, 2)
    assert frames == 2 and keys.ravel().tolist() == k1.tolist() and cache.frames == 2
    k2 = np.arange(8, 16, dtype=np.float32)
    v2 = np.arange(108, 116, dtype=np.float32)
    frames, keys, _ = cache.update(k2, v2, 2)
    assert frames == 4 and keys.size == 16 and cache.frames == 3
    assert cache.keys.ravel().tolist() == [2.0, 3.0, 8.0, 9.0, 10.0, 11.0,
                                           6.0, 7.0, 12.0, 13.0, 14.0, 15.0]


def test_relative_positions_interleave_sine_and_cosine_in_transformers_order():
    """encoder_streaming.rs:312-333."""
    p = eo.relative_position_encoding(4, 2)
    s, c = np.sin, np.cos
    want = [s(1.0), c(1.0), s(0.01), c(0.01), 0.0, 1.0, 0.0, 1.0,
            -s(1.0), c(1.0), -s(0.01), c(0.01)]
    assert p.shape == (3, 4)
    assert np.abs(p.ravel() - np.array(want)).max() <= 1e-6


def test_relative_shift_matches_transformers_pad_view_slice_sequence():
    """encoder_streaming.rs:335-343."""
    got = eo.relative_shift(np.arange(10, dtype=np.float32), 2, 5)
    assert got.tolist() == [1.0, 2.0, 3.0, 4.0, 0.0, 5.0, 6.0, 7.0, 8.0, 9.0]


def test_relative_shift_equals_the_closed_form_index():
    """shifted[q][key] = raw[q][key + Q - 1 - q] for key < V <= P - Q + 1, the
    index map the CUDA attention kernel uses instead of the pad-and-slice."""
    rng = np.random.default_rng(0)
    for q_len, visible in ((14, 70), (14, 14), (3, 5), (1, 1)):
        p_len = 2 * visible - 1
        raw = rng.standard_normal((q_len, p_len))
        shifted = eo.relative_shift(raw, q_len, p_len).reshape(q_len, p_len)
        for q in range(q_len):
            for key in range(visible):
                assert shifted[q, key] == raw[q, key + q_len - 1 - q]


def _zero_sum_frames(hidden, magnitudes):
    return np.concatenate([np.concatenate([np.full(hidden // 2, m), np.full(hidden // 2, -m)])
                           for m in magnitudes]).astype(np.float32).reshape(len(magnitudes), hidden)


def test_relative_attention_averages_values_when_content_and_position_scores_are_zero(oracle_mod):
    """encoder_streaming.rs:345-403: zero scores -> plain average over the visible values."""
    hidden = 128
    const = np.full((hidden, hidden), 0.01, np.float32)
    lin = lambda w: eo.QLinear.from_f32(w, np.zeros(hidden), 128, "f16")  # noqa: E731
    att = eo.RelPosAttention(lin(const), lin(const), lin(identity(hidden)), lin(identity(hidden)),
                             lin(identity(hidden)), np.zeros(hidden), np.zeros(hidden), 2)
    cache = eo.AttentionKvCache(2, 64, 3)
    first = att.forward(_zero_sum_frames(hidden, [1.0, 2.0]), cache)
    assert first.shape == (2, hidden)
    for frame in first:
        assert abs(frame[0] - 1.5) <= 0.03 and abs(frame[-1] + 1.5) <= 0.03
    second = att.forward(_zero_sum_frames(hidden, [3.0]), cache)
    assert cache.frames == 3
    assert abs(second[0, 0] - 2.0) <= 0.03 and abs(second[0, -1] + 2.0) <= 0.03


def test_subsampling_flattens_channels_before_frequency_for_pytorch_linear():
    """encoder_streaming.rs:405-414."""
    x = np.arange(1, 7, dtype=np.float32).reshape(1, 2, 3)
    assert eo.channel_frequency_flatten(x).ravel().tolist() == [1.0, 4.0, 2.0, 5.0, 3.0, 6.0]


def test_prompt_projector_broadcasts_one_hot_over_time(oracle_mod):
    """encoder_streaming.rs:49-92 (prompt zh-TW = id 5), tolerance 0.04."""
    hidden = prompts = inter = 128
    w1 = np.zeros((inter, hidden + prompts), np.float32)
    w1[0, 0] = 1.0
    for p in range(prompts):
        w1[p, hidden + p] = 1.0
    w2 = identity(hidden)
    proj = eo.PromptProjector(eo.QLinear.from_f32(w1, np.zeros(inter), 128, "f16"),
                              eo.QLinear.from_f32(w2, np.zeros(hidden), 128, "f16"))
    x = np.zeros((2, hidden), np.float32)
    x[0, 0], x[1, 0] = 2.0, 3.0
    out = proj(x, 5)
    assert out.shape == (2, hidden)
    for got, want in ((out[0, 0], 2.0), (out[1, 0], 3.0), (out[0, 5], 1.0), (out[1, 5], 1.0)):
        assert abs(got - want) <= 0.04


def test_subsampling_cache_dimensions_of_the_checkpoint():
    """encoder.rs:12-35 with (128 mel bins, 256 channels, kernel 3, stride 2, 3 stages)."""
    cache = eo.SubsamplingCache(128, 256)
    assert [(c.frequency_bins, c.channels, c.left_frames, c.initial_extra_frames)
            for c in cache.layers] == [(128, 1, 1, 1), (65, 256, 1, 1), (33, 256, 1, 1)]
    assert eo.EncoderConfig().sub_freq == 17
    assert eo.EncoderConfig().cache_frames == 56


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_small_encoder_streams_fixed_chunk_shapes(oracle_mod, dtype):
    """A 2-layer encoder over three 112-frame chunks: 14 frames per chunk,
    the attention cache fills to its window, outputs stay finite."""
    cfg = eo.EncoderConfig(hidden=256, ff=512, layers=2, heads=2, sliding_window=21,
                           mel_bins=32, sub_channels=64, num_prompts=64, prompt_hidden=256)
    enc = eo.Encoder(cfg, eo.random_params(cfg, 1, dtype), dtype)
    cache = enc.new_cache()
    rng = np.random.default_rng(2)
    for chunk in range(3):
        y = enc.encode_chunk(rng.standard_normal((112, cfg.mel_bins)).astype(np.float32), 3, cache)
        assert y.shape == (14, cfg.hidden)
        assert np.all(np.isfinite(y))
        assert cache["layers"][0].attention.frames == min(14 * (chunk + 1), cfg.cache_frames)
