"""Pins the RNNT oracle (CPU only) to the reference's RNNT tests
(crates/nemotron-mlx/tests/rnnt_decode.rs), in f16 like the reference."""
from __future__ import annotations

import math

import numpy as np
import pytest

import rnnt_oracle as ro
from encoder_oracle import QLinear


def test_greedy_control_advances_only_on_blank_and_caps_symbols():
    """rnnt_decode.rs:9-36."""
    calls = []

    def score(frame, symbol):
        calls.append((frame, symbol))
        return {(0, 0): 4, (0, 1): 9}.get((frame, symbol), 5 if frame == 1 else 9)

    tokens = ro.greedy_decode_with(3, 9, 2, score)
    assert tokens == [(4, 0), (5, 1), (5, 1)]
    assert calls == [(0, 0), (0, 1), (1, 0), (1, 1), (2, 0)]


def test_lstm_cell_uses_pytorch_ifgo_gate_order(oracle_mod):
    """rnnt_decode.rs:38-59: zero input and state, candidate bias atanh(0.5)."""
    hidden = 128
    w = np.full((4 * hidden, hidden), 0.001, np.float32)
    bias = np.zeros(4 * hidden, np.float32)
    bias[2 * hidden:3 * hidden] = math.atanh(0.5)
    cell = ro.LstmCell(QLinear.from_f32(w, np.zeros(4 * hidden), 128, "f16"),
                       QLinear.from_f32(w, np.zeros(4 * hidden), 128, "f16"),
                       bias, np.zeros(4 * hidden), "f16")
    z = np.zeros(hidden, np.float32)
    h, c = cell.step(z, z, z)
    assert abs(c[0] - 0.25) <= 5e-4
    assert abs(h[0] - 0.5 * math.tanh(0.25)) <= 5e-4


def test_prediction_cache_does_not_advance_on_blank(oracle_mod):
    """rnnt_decode.rs:61-86."""
    hidden = 128
    emb_q = oracle_mod.quantize(np.full((4, hidden), 0.01, np.float32), 128, "f16")
    emb = oracle_mod.dequantize(*emb_q, 128, "f16")
    w = np.full((4 * hidden, hidden), 0.001, np.float32)
    bias = np.zeros(4 * hidden, np.float32)
    bias[2 * hidden:3 * hidden] = 0.2
    cell = ro.LstmCell(QLinear.from_f32(w, None, 128, "f16"), QLinear.from_f32(w, None, 128, "f16"),
                       bias, np.zeros(4 * hidden), "f16")
    proj = QLinear.from_f32(np.eye(hidden, dtype=np.float32), np.zeros(hidden), 128, "f16")
    net = ro.PredictionNetwork(emb, [cell], proj, 3)
    st = net.new_state()
    first = net.step(3, st)
    first_hidden = st["h"][0].copy()
    again = net.step(3, st)
    assert np.array_equal(again, first)
    assert np.array_equal(st["h"][0], first_hidden)
    net.step(1, st)
    assert not np.array_equal(st["h"][0], first_hidden)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_small_decoder_emits_bounded_symbols(oracle_mod, dtype):
    cfg = ro.RnntConfig(enc_hidden=256, pred_hidden=128, joint_hidden=128, vocab=65, max_symbols=3)
    dec = ro.RnntDecoder(cfg, ro.random_params(cfg, 4, dtype), dtype)
    st = dec.new_state()
    rng = np.random.default_rng(1)
    margins = []
    toks = dec.decode_frames(rng.standard_normal((5, 256)).astype(np.float32), st, margins)
    per_frame = np.bincount([f for _, f in toks], minlength=5)
    assert per_frame.max() <= cfg.max_symbols
    assert all(0 <= t < cfg.vocab and t != cfg.blank for t, _ in toks)
    assert len(margins) >= len(toks) and min(margins) >= 0


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_structured_decoder_has_wide_margins_and_early_ends(oracle_mod, dtype):
    """The wide-margin decoder used by the exact-token GPU test: every greedy
    decision clears the runner-up by at least 8 T ulps, most frames end at
    blank before the symbol cap, some run to the cap, and only active tokens
    are emitted."""
    cfg = ro.RnntConfig()
    params, tokens = ro.structured_params(cfg, 7, dtype)
    dec = ro.RnntDecoder(cfg, params, dtype)
    rng = np.random.default_rng(1)
    states = [dec.new_state() for _ in range(3)]
    margins, per_frame, emitted = [], [], set()
    for _ in range(2):
        x = ro.structured_frames(rng, 3, 14, cfg.enc_hidden, len(tokens))
        for s, st in enumerate(states):
            out = dec.decode_frames(x[s], st, margins)
            per_frame += list(np.bincount([f for _, f in out], minlength=14))
            emitted |= {t for t, _ in out}
    per_frame = np.array(per_frame)
    assert min(margins) >= 8.0, min(margins)
    assert np.mean(per_frame < cfg.max_symbols) > 0.5
    assert np.any(per_frame == cfg.max_symbols) and np.any(per_frame == 0)
    assert emitted <= set(tokens.tolist()) and len(emitted) > 10
