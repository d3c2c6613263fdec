"""CPU restatement of the streaming session behind catcher.h (TEST INFRASTRUCTURE).

Only the test suite uses this module; the CUDA library never calls it.  It
restates:

* ``AudioChunkScheduler`` (crates/nemotron-mlx/src/model/stream.rs:17-128)
  over ``StreamingChunkPlan`` (encoder.rs:941-994): a centered first window of
  (8 * lookahead) * 160 + 200 samples, then uncentered windows of
  8 * (lookahead + 1) * 160 + 400 samples starting 256 samples before their
  first frame; ``finish`` zero-pads at most one tail window;
* ``Tokenizer::decode`` (crates/nemotron-mlx/src/tokenizer.rs:69-87);
* ``StreamingTranscriber`` (stream.rs:130-236): every window through the
  log-mel, encoder and RNNT oracles, tokens offset by the encoder frames seen
  so far.

Pinned by the reference's own tests of the scheduler
(crates/nemotron-mlx/tests/incremental_stream.rs) and of the tokenizer
(crates/nemotron-mlx/tests/tokenizer.rs), rebuilt in tests/test_catcher.py.
"""
from __future__ import annotations

import json

import numpy as np

import logmel_oracle as lo

HOP = 160
FACTOR = 8


class ChunkScheduler:
    def __init__(self, lookahead: int):
        if lookahead not in (3, 0, 6, 13):
            raise ValueError(f"unsupported lookahead {lookahead}; supported values are [3, 0, 6, 13]")
        self.lookahead = lookahead
        self.reset()

    @property
    def first_mel(self) -> int:
        return 1 + FACTOR * self.lookahead

    @property
    def next_mel(self) -> int:
        return FACTOR * (self.lookahead + 1)

    @property
    def first_samples(self) -> int:
        return (self.first_mel - 1) * HOP + 200

    @property
    def next_samples(self) -> int:
        return self.next_mel * HOP + 400

    def reset(self) -> None:
        self.audio = np.zeros(0, np.float32)
        self.first_done = False
        self.mel_index = 0
        self.finished = False

    def _start(self) -> int:
        s = self.mel_index * HOP - 256
        if s < 0:
            raise ValueError("streaming audio offset underflow")
        return s

    def push(self, samples) -> list:
        if self.finished:
            raise ValueError("streaming audio session is already finished")
        self.audio = np.concatenate([self.audio, np.asarray(samples, np.float32)])
        out = []
        while True:
            if not self.first_done:
                n = self.first_samples
                if self.audio.size < n:
                    break
                out.append((self.audio[:n].copy(), True, self.first_mel))
                self.first_done = True
                self.mel_index = self.first_mel
                continue
            s, n = self._start(), self.next_samples
            if self.audio.size < s + n:
                break
            out.append((self.audio[s:s + n].copy(), False, self.next_mel))
            self.mel_index += self.next_mel
        return out

    def finish(self):
        if self.finished:
            raise ValueError("streaming audio session is already finished")
        self.finished = True
        if self.audio.size == 0:
            return None
        if not self.first_done:
            self.first_done = True
            self.mel_index = self.first_mel
            return (_padded(self.audio, 0, self.first_samples), True, self.first_mel)
        s = self._start()
        if s >= self.audio.size:
            return None
        self.mel_index += self.next_mel
        return (_padded(self.audio, s, self.next_samples), False, self.next_mel)


def _padded(audio: np.ndarray, start: int, n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    if start < audio.size:
        k = min(n, audio.size - start)
        out[:k] = audio[start:start + k]
    return out


class Tokenizer:
    def __init__(self, path: str, pad: int, blank: int):
        with open(path, encoding="utf-8") as f:
            doc = json.load(f)
        if doc["model"]["type"] != "BPE" or doc["decoder"]["type"] != "Metaspace":
            raise ValueError(f"unsupported tokenizer model or decoder: "
                             f"{doc['model']['type']} + {doc['decoder']['type']}")
        self.tokens = {int(i): t for t, i in doc["model"]["vocab"].items()}
        self.special = set()
        for t in doc.get("added_tokens", []):
            self.tokens[int(t["id"])] = t["content"]
            if t["special"]:
                self.special.add(int(t["id"]))
        self.replacement = doc["decoder"]["replacement"]
        self.pad, self.blank = pad, blank

    def decode(self, ids, strip_language_tag: bool = True) -> str:
        pieces = []
        for i in ids:
            if i in (self.pad, self.blank):
                continue
            if i not in self.tokens:
                raise KeyError(f"token id {i} is absent from tokenizer.json")
            if strip_language_tag and i in self.special:
                continue
            pieces.append(self.tokens[i])
        return "".join(pieces).replace(self.replacement, " ").lstrip(" ")


class Transcriber:
    """Windows -> log-mel -> encoder -> RNNT for one utterance; tokens carry
    their global encoder frame.  `trace` (a list) collects, per window, the
    encoder output and the decoder's state before it, for teacher-forced
    checks of another implementation's tokens."""

    def __init__(self, encoder, decoder, prompt_id: int, lookahead: int):
        self.encoder, self.decoder, self.prompt = encoder, decoder, prompt_id
        self.scheduler = ChunkScheduler(lookahead)
        self.reset()

    def reset(self) -> None:
        self.cache = self.encoder.new_cache()
        self.state = self.decoder.new_state()
        self.scheduler.reset()
        self.frames_seen = 0

    def _chunk(self, window, trace):
        samples, center, mel_frames = window
        feats = lo.extract(samples, center)
        assert feats.shape == (mel_frames, 128), feats.shape
        encoded = self.encoder.encode_chunk(feats, self.prompt, self.cache)
        offset = self.frames_seen
        self.frames_seen += encoded.shape[0]
        if trace is not None:
            import copy
            trace.append((encoded, copy.deepcopy(self.state), offset))
        return [(t, f + offset) for t, f in self.decoder.decode_frames(encoded, self.state)]

    def push(self, samples, trace=None) -> list:
        out = []
        for w in self.scheduler.push(samples):
            out += self._chunk(w, trace)
        return out

    def finish(self, trace=None) -> list:
        w = self.scheduler.finish()
        return [] if w is None else self._chunk(w, trace)
