"""Batched RNNT greedy decoder on the GPU (include/cqrnnt.h) against the CPU
restatement in oracle/rnnt_oracle.py.

Two kinds of checks.  Free running (test_free_running_tokens_equal_the_oracle):
on a decoder built so that every greedy decision clears its runner-up by at
least 8 T ulps (asserted from the oracle's logits), the GPU's token stream --
tokens, frames and counts, chunk after chunk -- must equal the oracle's
exactly.  Teacher forced (random weights, where the top two logits are often
closer than the two sides' summation-order differences): the oracle replays
the GPU's tokens and checks every decision against its own argmax; a differing
choice must be a near tie (its logit within 8 T ulps of the oracle's maximum)
and such ties must stay rare; every other decision must be identical.
"""
from __future__ import annotations

import numpy as np
import pytest

import rnnt_oracle as ro

pytestmark = pytest.mark.gpu

SMALL = dict(enc_hidden=256, pred_hidden=128, joint_hidden=128, vocab=65, max_symbols=3,
             group_size=64)


def _ocfg(d):
    return ro.RnntConfig(enc_hidden=d["enc_hidden"], pred_hidden=d["pred_hidden"],
                         joint_hidden=d["joint_hidden"], vocab=d["vocab"],
                         max_symbols=d["max_symbols"], group=d["group_size"])


def _dev(torch, x_f32, dtype):
    import oracle
    bits = oracle.to_t(x_f32, dtype).view(np.int16)
    return torch.from_numpy(bits).cuda().view(torch.bfloat16 if dtype == "bf16" else torch.float16)


def _check_streams(torch, state, ref, caches, enc_f32, streams, frames, dtype, totals):
    paths = state.decode_chunk(_dev(torch, enc_f32.reshape(streams * frames, -1), dtype), frames)
    for s in range(streams):
        stats = ro.check_path(ref, enc_f32[s], caches[s], paths[s])
        assert stats["mismatch"] == 0, (s, stats, paths[s])
        totals["decisions"] += stats["decisions"]
        totals["differ"] += stats["differ"]
    return paths


def _bind(dec, params, cfg):
    for name, (n, k, has_bias) in ro.linear_names(cfg).items():
        q, s, b, bias = params[name]
        dec.set_linear(name, q, s, b, bias if has_bias else None, cfg.group)
    for name in ro.dense_names(cfg):
        dec.set_tensor(name, params[name])


@pytest.mark.parametrize("dtype,streams,chunks,persistent", [
    ("bf16", 1, 4, False), ("bf16", 64, 3, False), ("f16", 1, 4, False), ("f16", 64, 3, False),
    ("bf16", 1, 4, True)])
def test_free_running_tokens_equal_the_oracle(cq, oracle_mod, dtype, streams, chunks, persistent):
    """Full size (hidden 640, encoder 1024, vocab 1025, two LSTM layers, ten
    symbols per frame).  Greedy decoding runs free on both sides -- each side
    feeds its own tokens back -- over several chunks (the prediction state
    crosses chunk boundaries); the token streams must be identical.  The
    structured decoder (rnnt_oracle.structured_params) makes most frames end at
    blank early, some alternate or repeat up to the cap; every decision's
    top-1 / top-2 margin is at least 8 T ulps (asserted)."""
    import torch
    from nemotron_cuda.rnnt import Rnnt, RnntConfig
    cfg = ro.RnntConfig()
    params, tokens = ro.structured_params(cfg, 7, dtype)
    dec = Rnnt(RnntConfig.default(), dtype)
    _bind(dec, params, cfg)
    ref = ro.RnntDecoder(cfg, params, dtype)
    frames = 14
    state = dec.state(streams, frames)
    state.set_persistent(persistent)
    caches = [ref.new_state() for _ in range(streams)]
    rng = np.random.default_rng(100 + streams)
    margins, emitted, capped, early = [], 0, 0, 0
    for chunk in range(chunks):
        enc = ro.structured_frames(rng, streams, frames, cfg.enc_hidden, len(tokens))
        got = state.decode_chunk(_dev(torch, enc.reshape(streams * frames, -1), dtype), frames)
        for s in range(streams):
            want = ref.decode_frames(enc[s], caches[s], margins)
            assert got[s] == want, (chunk, s, got[s], want)
            per_frame = np.bincount([f for _, f in want], minlength=frames)
            emitted += len(want)
            capped += int((per_frame == cfg.max_symbols).sum())
            early += int((per_frame < cfg.max_symbols).sum())
    assert min(margins) >= 8.0, min(margins)
    assert emitted > 0 and capped > 0 and early > capped
    assert cq.device_status(0) == 0


@pytest.mark.parametrize("persistent", [False, True])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_small_decoder_greedy_paths_match_oracle(cq, oracle_mod, dtype, persistent):
    import torch
    from nemotron_cuda.rnnt import Rnnt, RnntConfig
    cfg = _ocfg(SMALL)
    params = ro.random_params(cfg, 21, dtype)
    dec = Rnnt(RnntConfig.default(**SMALL), dtype)
    for name, (n, k, has_bias) in ro.linear_names(cfg).items():
        q, s, b, bias = params[name]
        dec.set_linear(name, q, s, b, bias if has_bias else None, cfg.group)
    for name in ro.dense_names(cfg):
        dec.set_tensor(name, params[name])
    ref = ro.RnntDecoder(cfg, params, dtype)
    streams, frames = 3, 5
    state = dec.state(streams, frames)
    state.set_persistent(persistent)
    assert state.capacity == frames * cfg.max_symbols
    caches = [ref.new_state() for _ in range(streams)]
    rng = np.random.default_rng(3)
    totals = {"decisions": 0, "differ": 0}
    for _ in range(3):
        enc = rng.standard_normal((streams, frames, cfg.enc_hidden)).astype(np.float32)
        paths = _check_streams(torch, state, ref, caches, enc, streams, frames, dtype, totals)
        for p in paths:
            assert all(t != cfg.blank and 0 <= t < cfg.vocab for t, _ in p)
            assert max(np.bincount([f for _, f in p], minlength=frames)) <= cfg.max_symbols
    assert totals["differ"] <= max(1, totals["decisions"] // 20), totals
    if persistent:  # the encoder projector, the barrier reset, one cooperative launch
        assert 0 < state.kernels_per_chunk <= 5, state.kernels_per_chunk
    else:
        # launch per op: per frame one joint input, then per symbol head,
        # argmax, the LSTM layers, projector, joint input
        assert state.kernels_per_chunk > 60, state.kernels_per_chunk
    assert cq.device_status(0) == 0


@pytest.mark.parametrize("persistent", [False, True])
def test_full_size_decoder_device_weights(cq, oracle_mod, persistent):
    """Hidden 640, encoder 1024, vocab 1025, ten symbols per frame, two LSTM
    layers; device-generated weights read back for the oracle."""
    import torch
    from nemotron_cuda.rnnt import Rnnt
    dtype = "bf16"
    dec = Rnnt.random(None, seed=5, dtype=dtype)
    cfg = ro.RnntConfig()
    params = dec.export_params(ro.linear_names(cfg), ro.dense_names(cfg))
    ref = ro.RnntDecoder(cfg, params, dtype)
    streams, frames = 2, 14
    state = dec.state(streams, frames)
    state.set_persistent(persistent)
    caches = [ref.new_state() for _ in range(streams)]
    rng = np.random.default_rng(8)
    totals = {"decisions": 0, "differ": 0}
    enc = (rng.standard_normal((streams, frames, 1024)) * 0.5).astype(np.float32)
    _check_streams(torch, state, ref, caches, enc, streams, frames, dtype, totals)
    assert totals["differ"] <= max(2, totals["decisions"] // 20), totals


def test_persistent_path_skips_frames_that_end_in_blank(cq, oracle_mod):
    """A blank-favouring joint bias makes most frames end at their first
    symbol, so the persistent kernel's early exit is taken; its greedy paths
    still match the oracle decision by decision."""
    import torch
    import oracle
    from nemotron_cuda.rnnt import Rnnt, RnntConfig
    cfg = _ocfg(SMALL)
    params = ro.random_params(cfg, 12, "f16")
    q, s, b, bias = params["joint.head.weight"]
    rng = np.random.default_rng(6)
    encs = [rng.standard_normal((3, 6, cfg.enc_hidden)).astype(np.float32) for _ in range(3)]
    # the smallest blank bias (from a sweep on the oracle) under which most
    # frames end at blank before the symbol cap
    for blank_bias in (0.05, 0.1, 0.15, 0.2, 0.3, 0.45, 0.6):
        bias_f = oracle.from_t(bias, "f16")
        bias_f[cfg.blank] = blank_bias
        trial = dict(params)
        trial["joint.head.weight"] = (q, s, b, oracle.to_t(bias_f, "f16"))
        probe = ro.RnntDecoder(cfg, trial, "f16")
        st = probe.new_state()
        n = len(probe.decode_frames(encs[0][0], st))
        if n < 6 * cfg.max_symbols // 2:
            break
    params = trial
    dec = Rnnt(RnntConfig.default(**SMALL), "f16")
    for name, (n, k, has_bias) in ro.linear_names(cfg).items():
        q, s, b, bias = params[name]
        dec.set_linear(name, q, s, b, bias if has_bias else None, cfg.group)
    for name in ro.dense_names(cfg):
        dec.set_tensor(name, params[name])
    ref = ro.RnntDecoder(cfg, params, "f16")
    streams, frames = 3, 6
    state = dec.state(streams, frames)
    state.set_persistent(True)
    caches = [ref.new_state() for _ in range(streams)]
    totals = {"decisions": 0, "differ": 0}
    emitted = 0
    for enc in encs:
        paths = _check_streams(torch, state, ref, caches, enc, streams, frames, "f16", totals)
        emitted += sum(len(p) for p in paths)
    assert 0 < emitted < 3 * streams * frames * cfg.max_symbols
    assert totals["differ"] <= max(1, totals["decisions"] // 20), totals


def test_reset_replays_the_same_tokens(cq):
    import torch
    from nemotron_cuda.rnnt import Rnnt, RnntConfig
    dec = Rnnt.random(RnntConfig.default(**SMALL), seed=9, dtype="bf16")
    state = dec.state(4, 6)
    enc = torch.randn((4 * 6, SMALL["enc_hidden"]), device="cuda").to(torch.bfloat16)
    first = [state.decode_chunk(enc, 6) for _ in range(2)]
    state.reset()
    again = [state.decode_chunk(enc, 6) for _ in range(2)]
    assert first == again
    state.set_pdl(False)  # without programmatic dependent launch
    state.reset()
    assert [state.decode_chunk(enc, 6) for _ in range(2)] == first


def test_rnnt_binding_errors(cq):
    from nemotron_cuda import CQError
    from nemotron_cuda.rnnt import Rnnt, RnntConfig
    dec = Rnnt(RnntConfig.default(**SMALL), "f16")
    with pytest.raises(CQError, match="unknown RNNT tensor"):
        dec.set_tensor("decoder.lstm.bias_ih_l7", np.zeros(512))
    with pytest.raises(CQError, match="is not bound"):
        dec.state(1, 4)
    assert "decoder.embedding.weight" in dec.tensor_names()
    st = Rnnt.random(RnntConfig.default(**SMALL), seed=1, dtype="f16").state(65, 4)
    with pytest.raises(CQError, match="does not fit"):
        st.set_persistent(True)


@pytest.mark.parametrize("dtype,size,streams,frames", [
    ("bf16", "small", 3, 5), ("f16", "small", 3, 5),
    # full size at 64 streams: the second layer's step runs 80-row bands at two
    # CTAs per SM, the first layer's reads the per-token table (two per SM)
    ("bf16", "full", 64, 2)])
def test_one_launch_lstm_step_matches_separate_launches(cq, dtype, size, streams, frames):
    """The LSTM step as one launch (ih and hh products on a CTA pair, the cell in
    the leader's epilogue, gate-interleaved weights; layer 0's ih product from
    the per-token table) does K1's arithmetic and the cell kernel's: the greedy
    paths equal those of the separate ih, hh and cell launches
    (cq_rnnt_set_fused_lstm(0)) token for token."""
    import torch
    from nemotron_cuda.rnnt import Rnnt, RnntConfig
    cfg = RnntConfig.default(**(SMALL if size == "small" else {}))
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    outs = []
    for fused in (True, False):
        dec = Rnnt.random(cfg, seed=31, dtype=dtype)
        dec.set_fused_lstm(fused)
        st = dec.state(streams, frames)
        rng = np.random.default_rng(4)
        out = []
        for _ in range(3):
            enc = rng.standard_normal((streams * frames, cfg.enc_hidden)).astype(np.float32)
            out.append(st.decode_chunk(torch.from_numpy(enc).cuda().to(tdt), frames))
        outs.append(out)
        del st, dec
    assert outs[0] == outs[1]
    assert sum(len(p) for chunk in outs[0] for p in chunk) > 0
