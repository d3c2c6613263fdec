"""The transcription ABI's host side on CPU (include/catcher.h, include/cqstream.h).

* The window scheduler, through its C ABI and in the oracle, on the
  reference's own cases (crates/nemotron-mlx/tests/incremental_stream.rs).
* The tokenizer decode, both ways, on the reference's case
  (crates/nemotron-mlx/tests/tokenizer.rs) and on escapes a tokenizer.json
  may hold.
* catcher_* with NULL arguments (crates/catcher-ffi/tests/ffi_lifecycle.rs:
  36-67) and catcher_create's host-side errors, none of which touches a GPU.
"""
from __future__ import annotations

import ctypes
import json
import os

import numpy as np
import pytest

import artifact_oracle as ao
import stream_oracle as so


@pytest.fixture(params=["abi", "oracle"])
def scheduler(request, cq):
    if request.param == "abi":
        from nemotron_cuda.catcher import ChunkScheduler
        return ChunkScheduler(3)
    return so.ChunkScheduler(3)


def test_waits_for_complete_first_and_subsequent_windows(scheduler):
    """incremental_stream.rs:8-27."""
    assert scheduler.push(np.full(4039, 1.0)) == []
    first = scheduler.push([2.0])
    assert len(first) == 1
    samples, center, mel = first[0]
    assert samples.size == 4040 and center and mel == 25
    assert scheduler.push(np.full(5223, 3.0)) == []
    second = scheduler.push([4.0])
    assert len(second) == 1
    samples, center, mel = second[0]
    assert samples.size == 5520 and not center and mel == 32
    assert np.all(samples[:295] == 1.0) and samples[295] == 2.0


def test_finish_pads_at_most_one_tail_and_locks_the_scheduler(scheduler, cq):
    """incremental_stream.rs:29-43."""
    scheduler.push(np.full(4040, 1.0))
    tail = scheduler.finish()
    samples, center, mel = tail
    assert samples.size == 5520 and not center
    assert np.all(samples[:296] == 1.0) and np.all(samples[296:] == 0.0)
    with pytest.raises((ValueError, cq.CQError), match="already finished"):
        scheduler.finish()
    with pytest.raises((ValueError, cq.CQError), match="already finished"):
        scheduler.push([1.0])


def test_reset_clears_audio_and_lifecycle_state(scheduler):
    """incremental_stream.rs:45-57."""
    scheduler.push(np.full(4040, 1.0))
    scheduler.finish()
    scheduler.reset()
    assert scheduler.push(np.full(4039, 2.0)) == []
    first = scheduler.push([3.0])
    assert len(first) == 1 and first[0][1] and first[0][0][4039] == 3.0


def test_finishing_empty_audio_emits_nothing(scheduler):
    """incremental_stream.rs:59-63."""
    assert scheduler.finish() is None


@pytest.mark.parametrize("lookahead", [0, 3, 6, 13])
def test_scheduler_abi_matches_oracle_on_ragged_blocks(cq, lookahead):
    """Arbitrary block sizes: the same windows, sample for sample, then the
    same padded tail."""
    from nemotron_cuda.catcher import ChunkScheduler
    a, b = ChunkScheduler(lookahead), so.ChunkScheduler(lookahead)
    rng = np.random.default_rng(lookahead)
    audio = rng.standard_normal(5 * 16000).astype(np.float32)
    pos, sizes, total = 0, [127, 1024, 333, 2048, 1600, 1], 0
    while pos < audio.size:
        n = sizes[pos % len(sizes)]
        blk = audio[pos:pos + n]
        pos += n
        try:
            wa = a.push(blk)
        except cq.CQError as e:
            wa = str(e)
        try:
            wb = b.push(blk)
        except ValueError as e:
            wb = str(e)
        if isinstance(wa, str) or isinstance(wb, str):
            # lookahead 0: the reference's uncentered offset (1 frame * 160 -
            # 256 samples) underflows right after the first window, on both
            assert wa == wb == "streaming audio offset underflow" and lookahead == 0
            return
        assert len(wa) == len(wb)
        for (sa, ca, ma), (sb, cb, mb) in zip(wa, wb):
            assert ca == cb and ma == mb and np.array_equal(sa, sb)
        total += len(wa)
    assert total >= 3
    ta, tb = a.finish(), b.finish()
    assert (ta is None) == (tb is None)
    if ta is not None:
        assert ta[1] == tb[1] and ta[2] == tb[2] and np.array_equal(ta[0], tb[0])


def test_scheduler_rejects_unsupported_lookahead(cq):
    from nemotron_cuda.catcher import ChunkScheduler
    with pytest.raises(cq.CQError, match=r"unsupported lookahead 4; supported values are \[3, 0, 6, 13\]"):
        ChunkScheduler(4)


TOKENIZER_JSON = {
    "model": {"type": "BPE", "vocab": {"▁hello": 0, "世": 1, "界": 2}},
    "added_tokens": [
        {"id": 3, "content": "<en-US>", "special": True},
        {"id": 4, "content": "<pad>", "special": True},
        {"id": 5, "content": "<blank>", "special": True},
    ],
    "decoder": {"type": "Metaspace", "replacement": "▁", "prepend_scheme": "always",
                "split": True},
}


@pytest.mark.parametrize("impl", ["abi", "oracle"])
def test_tokenizer_decodes_bpe_metaspace_and_strips_control_ids(cq, tmp_path, impl):
    """tokenizer.rs:5-33 (pad 4, blank 5)."""
    path = tmp_path / "tokenizer.json"
    path.write_text(json.dumps(TOKENIZER_JSON))
    if impl == "abi":
        from nemotron_cuda.catcher import Tokenizer
        tok, err = Tokenizer(str(path), 4, 5), cq.CQError
    else:
        tok, err = so.Tokenizer(str(path), 4, 5), KeyError
    assert tok.decode([3, 0, 1, 2, 4, 5], True) == "hello世界"
    assert tok.decode([3, 0, 1, 2, 4, 5], False) == "<en-US> hello世界"
    with pytest.raises(err, match="token id 99 is absent from tokenizer.json"):
        tok.decode([99], True)


def test_tokenizer_reads_escapes_and_rejects_other_models(cq, tmp_path):
    from nemotron_cuda.catcher import Tokenizer
    # \u escapes, a surrogate pair (U+1F600) and a multi-byte replacement
    text = ('{"model":{"type":"BPE","vocab":{"\\u2581a":1,"\\ud83d\\ude00":2,"b\\"c":3}},'
            '"decoder":{"type":"Metaspace","replacement":"\\u2581"}}')
    path = tmp_path / "tokenizer.json"
    path.write_text(text)
    tok = Tokenizer(str(path), 0, 9)
    assert tok.decode([1, 2, 3, 1]) == "a\U0001F600b\"c a"
    assert tok.decode([0, 9]) == ""
    bad = dict(TOKENIZER_JSON, decoder={"type": "ByteLevel", "replacement": "x"})
    path.write_text(json.dumps(bad))
    with pytest.raises(cq.CQError, match="unsupported tokenizer model or decoder: BPE \\+ ByteLevel"):
        Tokenizer(str(path), 0, 9)


def test_null_arguments_report_errors_without_unwinding(cq):
    """ffi_lifecycle.rs:36-54."""
    from nemotron_cuda import catcher as C
    L = cq.lib()
    assert L.catcher_start(None) == C.CATCHER_INVALID_ARGUMENT
    assert L.catcher_push_audio(None, None, 0) == C.CATCHER_INVALID_ARGUMENT
    assert L.catcher_finish(None) == C.CATCHER_INVALID_ARGUMENT
    assert L.catcher_finish_before(None, 1000) == C.CATCHER_INVALID_ARGUMENT
    assert L.catcher_text(None) is None
    assert L.catcher_text_before(None, 1500) is None
    assert L.catcher_last_error(None) == b"catcher handle is null"
    L.catcher_destroy(None)
    assert L.catcher_push_audio(None, None, 5) == C.CATCHER_INVALID_ARGUMENT
    assert L.catcher_last_error(None) == b"samples is null while count is non-zero"


def test_null_handle_segments_and_warning_are_safe(cq):
    """ffi_lifecycle.rs:56-67."""
    L = cq.lib()
    assert L.catcher_segments(None) is None
    assert L.catcher_last_error(None) is not None
    assert L.catcher_warning(None) is None
    assert L.catcher_last_error(None) is not None


def _fixture_artifact(tmp_path) -> str:
    path = str(tmp_path / "artifact")
    ao.convert_tensors(path, "fixture/subsampling", ao.reference_fixture_specs())
    return path


def test_create_reports_host_side_errors_before_device_work(cq, tmp_path):
    L = cq.lib()
    path = _fixture_artifact(tmp_path)

    def create(p, lang, la, diar=None):
        h = L.catcher_create(None if p is None else p.encode(), diar, None if lang is None else lang.encode(), la)
        assert not h
        return L.catcher_last_error(None).decode()

    assert create(None, "en-US", 3) == "asr_model_path is null"
    assert create(path, None, 3) == "language is null"
    assert "cannot open" in create(str(tmp_path / "absent"), "en-US", 3)
    assert "diarization" in create(path, "en-US", 3, diar=b"/some/diarizer")
    assert create(path, "en-US", 4) == "unsupported lookahead 4; supported values are [3, 0, 6, 13]"
    assert create(path, "xx-XX", 3) == "unsupported language prompt: xx-XX"
    # the fixture is one block without an RNNT: the Nemotron geometry asks for its head
    assert create(path, "auto", 13) == "missing artifact tensor joint.head.weight"
    bad = L.catcher_create(path.encode(), None, b"en-\xff", 3)
    assert not bad and L.catcher_last_error(None) == b"language is not valid UTF-8"
