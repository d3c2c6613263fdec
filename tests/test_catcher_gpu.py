"""The transcription ABI (include/catcher.h) end to end on the GPU.

A seeded two-block model (encoder d 256 + RNNT, vocabulary 65) is written as
a release artifact by the oracle's converter, with a tokenizer.json whose
piece for id i is "▁t<i>", so the transcript spells the token ids.  Audio is
the reference's synthetic log-mel test signal, 4.3 s at 16 kHz, pushed in the
reference test's ragged block sizes (127, 1024, 333, 2048; crates/catcher-ffi/
tests/ffi_lifecycle.rs:100-118) and in 1600-sample blocks.  Checks:

* the handle's token ids equal those of the same windows driven through the
  library's own log-mel, encoder and RNNT entry points (the same kernels:
  identical), whatever the block sizes;
* those entry points agree with the oracles: every window's encoder output
  within the encoder tolerance of the oracle's (oracle/encoder_oracle.py on
  the oracle's log-mel features), and the greedy tokens checked by teacher
  forcing against oracle/rnnt_oracle.py on the GPU's encoder output;
* the transcript is the oracle tokenizer's decode of the ids;
* text_before / finish_before keep the tokens that start before the cutoff;
* the session life cycle of ffi_lifecycle.rs:69-92.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

import artifact_oracle as ao
import encoder_oracle as eo
import logmel_oracle as lo
import rnnt_oracle as ro
import stream_oracle as so

pytestmark = pytest.mark.gpu

ENC = dict(hidden=256, ff=512, layers=2, heads=2, conv_kernel=9, sliding_window=21, mel_bins=128,
           sub_channels=64, num_prompts=128, prompt_hidden=256, group_size=64)
RNNT = dict(enc_hidden=256, pred_hidden=128, joint_hidden=128, vocab=65, max_symbols=10,
            group_size=64)
ENC_TOL = (4e-3, 1.6e-2)  # f16: rel-L2, max |diff| / max |ref| (tests/test_encoder_gpu.py)
LOOKAHEAD = 3
PROMPT = 0  # en-US


def _configs():
    ecfg = eo.EncoderConfig(hidden=ENC["hidden"], ff=ENC["ff"], layers=ENC["layers"], heads=ENC["heads"],
                            conv_kernel=ENC["conv_kernel"], sliding_window=ENC["sliding_window"],
                            mel_bins=ENC["mel_bins"], sub_channels=ENC["sub_channels"],
                            num_prompts=ENC["num_prompts"], prompt_hidden=ENC["prompt_hidden"],
                            group=ENC["group_size"])
    rcfg = ro.RnntConfig(enc_hidden=RNNT["enc_hidden"], pred_hidden=RNNT["pred_hidden"],
                         joint_hidden=RNNT["joint_hidden"], vocab=RNNT["vocab"],
                         max_symbols=RNNT["max_symbols"], group=RNNT["group_size"])
    return ecfg, rcfg


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    ecfg, rcfg = _configs()
    path = str(tmp_path_factory.mktemp("catcher") / "model")
    names = {**eo.linear_names(ecfg), **ro.linear_names(rcfg)}
    dense = {**eo.dense_names(ecfg), **ro.dense_names(rcfg)}
    # joint weights large enough that the audio, not the head's biases, picks
    # the tokens (with N(0, 0.02) everywhere one token wins every frame)
    std = {"encoder_projector.weight": 0.1, "decoder.decoder_projector.weight": 0.1,
           "joint.head.weight": 0.3}
    ao.convert_tensors(path, "fixture/catcher", ao.random_specs(names, dense, 64, seed=29, std=std))
    vocab = {f"▁t{i}": i for i in range(1, rcfg.vocab - 1)}
    tok = {"model": {"type": "BPE", "vocab": vocab},
           "added_tokens": [{"id": 0, "content": "<pad>", "special": True},
                            {"id": rcfg.blank, "content": "<blank>", "special": True}],
           "decoder": {"type": "Metaspace", "replacement": "▁"}}
    with open(f"{path}/tokenizer.json", "w", encoding="utf-8") as f:
        json.dump(tok, f)
    return path


def _ids(text: str) -> list[int]:
    return [int(w[1:]) for w in text.split()]


def _blocks(samples: np.ndarray, sizes):
    pos, k = 0, 0
    while pos < samples.size:
        n = sizes[k % len(sizes)]
        yield samples[pos:pos + n]
        pos += n
        k += 1


def _handle(model_dir):
    from nemotron_cuda.catcher import Catcher
    from nemotron_cuda.encoder import EncoderConfig
    from nemotron_cuda.rnnt import RnntConfig
    return Catcher(model_dir, "en-US", LOOKAHEAD, EncoderConfig.default(**ENC),
                   RnntConfig.default(**RNNT), "f16")


def _transcribe(h, audio, sizes):
    from nemotron_cuda import catcher as C
    assert h.start() == C.CATCHER_OK
    statuses = [h.push_audio(b) for b in _blocks(audio, sizes)]
    statuses.append(h.finish())
    assert all(s in (C.CATCHER_OK, C.CATCHER_NO_UPDATE) for s in statuses), (statuses, h.last_error())
    return h.text(), statuses


def _direct(model_dir, audio):
    """The same windows through the library's own log-mel, encoder and RNNT
    entry points: [(token, global frame)], per-window encoder outputs and
    the windows."""
    import torch
    from nemotron_cuda.artifact import Artifact
    from nemotron_cuda.catcher import ChunkScheduler
    from nemotron_cuda.encoder import Encoder, EncoderConfig
    from nemotron_cuda.logmel import LogMelFrontend
    from nemotron_cuda.rnnt import Rnnt, RnntConfig
    with Artifact(model_dir) as art:
        enc = Encoder.from_artifact(art, EncoderConfig.default(**ENC), "f16")
        dec = Rnnt.from_artifact(art, RnntConfig.default(**RNNT), "f16")
    sched = ChunkScheduler(LOOKAHEAD)
    windows = []
    for b in _blocks(audio, [1600]):
        windows += sched.push(b)
    tail = sched.finish()
    if tail is not None:
        windows.append(tail)
    est = enc.state(1, 8 * (LOOKAHEAD + 1))
    est.set_prompts([PROMPT])
    rst = dec.state(1, LOOKAHEAD + 1)
    rst.set_persistent(True)  # as the handle's single-stream decoder
    fe = LogMelFrontend.nemotron()
    mel = torch.empty((1, 8 * (LOOKAHEAD + 1), 128), device="cuda")
    out = torch.empty((LOOKAHEAD + 1, ENC["hidden"]), dtype=torch.float16, device="cuda")
    tokens, encoded, seen = [], [], 0
    for samples, center, mel_frames in windows:
        a = torch.from_numpy(samples).cuda()[None, :]
        m = mel[:, :mel_frames]
        fe.extract_raw(a, samples.size, center, m)
        q = est.output_frames(mel_frames)
        y = est.encode_chunk(m, out[:q])
        path = rst.decode_chunk(y, q)[0]
        encoded.append(y.float().cpu().numpy())
        tokens += [(t, f + seen) for t, f in path]
        seen += q
    return tokens, encoded, windows


def test_transcript_matches_the_library_pipeline_and_the_oracles(cq, oracle_mod, model_dir):
    from nemotron_cuda import catcher as C
    audio = lo.synthetic_audio(68_800)
    h = _handle(model_dir)
    text, statuses = _transcribe(h, audio, [127, 1024, 333, 2048])
    text_1600, _ = _transcribe(h, audio, [1600])
    assert text == text_1600
    tokens, encoded, windows = _direct(model_dir, audio)
    assert len(windows) >= 10
    ids = [t for t, _ in tokens]
    assert len(ids) > 0 and _ids(text) == ids
    assert C.CATCHER_OK in statuses
    tok = so.Tokenizer(f"{model_dir}/tokenizer.json", 0, RNNT["vocab"] - 1)
    assert text == tok.decode(ids)
    assert h.segments() == "[]" and h.warning() is None

    # the oracles, window by window
    ecfg, rcfg = _configs()
    oart = ao.Artifact(model_dir)
    oenc = eo.Encoder(ecfg, ao.model_params(oart, eo.linear_names(ecfg), eo.dense_names(ecfg), "f16"),
                      "f16")
    odec = ro.RnntDecoder(rcfg, ao.model_params(oart, ro.linear_names(rcfg), ro.dense_names(rcfg),
                                                "f16"), "f16")
    cache, st = oenc.new_cache(), odec.new_state()
    seen, decisions, differ = 0, 0, 0
    for (samples, center, mel_frames), enc_gpu in zip(windows, encoded):
        feats = lo.extract(samples, center)
        want = oenc.encode_chunk(feats, PROMPT, cache)
        assert want.shape == enc_gpu.shape
        diff = np.abs(enc_gpu.astype(np.float64) - want)
        rel_l2 = np.sqrt((diff ** 2).sum() / (want.astype(np.float64) ** 2).sum())
        assert rel_l2 <= ENC_TOL[0] and diff.max() / np.abs(want).max() <= ENC_TOL[1], rel_l2
        q = enc_gpu.shape[0]
        path = [(t, f - seen) for t, f in tokens if seen <= f < seen + q]
        stats = ro.check_path(odec, enc_gpu, st, path)
        assert stats["mismatch"] == 0, stats
        decisions += stats["decisions"]
        differ += stats["differ"]
        seen += q
    assert differ <= max(1, decisions // 20), (differ, decisions)
    assert cq.device_status(0) == 0


def test_text_before_and_finish_before_keep_tokens_before_the_cutoff(cq, model_dir):
    audio = lo.synthetic_audio(68_800)
    tokens, _, _ = _direct(model_dir, audio)
    last = max(f for _, f in tokens)
    cutoff_ms = 80 * (last // 2) + 40
    keep = [t for t, f in tokens if f * 80 < cutoff_ms]
    assert 0 < len(keep) < len(tokens)
    h = _handle(model_dir)
    _transcribe(h, audio, [1600])
    assert _ids(h.text_before(cutoff_ms)) == keep
    assert _ids(h.text()) == [t for t, _ in tokens]  # unchanged by text_before
    h.start()
    for b in _blocks(audio, [1600]):
        h.push_audio(b)
    h.finish_before(cutoff_ms)
    assert _ids(h.text()) == keep


def test_valid_handle_can_restart_without_reloading(cq, model_dir):
    """ffi_lifecycle.rs:69-92."""
    from nemotron_cuda import catcher as C
    h = _handle(model_dir)
    assert h.push_audio([]) == C.CATCHER_INVALID_STATE  # idle: not recording
    assert h.last_error() == "catcher session is not recording"
    assert h.start() == C.CATCHER_OK
    assert h.push_audio([]) == C.CATCHER_NO_UPDATE
    assert h.finish() == C.CATCHER_NO_UPDATE
    assert h.push_audio([]) == C.CATCHER_INVALID_STATE
    assert h.finish() == C.CATCHER_INVALID_STATE
    assert h.text() == ""
    assert h.start() == C.CATCHER_OK
    assert h.text() == ""
    # a short utterance (less than one window) is decoded from its padded tail
    h.push_audio(lo.synthetic_audio(3000))
    assert h.finish() in (C.CATCHER_OK, C.CATCHER_NO_UPDATE)
    assert cq.device_status(0) == 0
