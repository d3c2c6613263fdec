"""Python bindings of the transcription ABI (include/catcher.h) and of the
window scheduler and tokenizer it is built on (include/cqstream.h).

``Catcher`` mirrors the reference's C ABI handle
(crates/catcher-ffi/src/lib.rs:251-586): ``start``, ``push_audio``,
``finish``, ``finish_before``, ``text``, ``text_before``; statuses are
returned as the ABI returns them (CATCHER_OK, CATCHER_NO_UPDATE or a negative
error, whose message ``last_error`` holds).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import CQError, DTYPES, _check, lib

CATCHER_OK = 0
CATCHER_NO_UPDATE = 1
CATCHER_COMMAND_DETECTED = 2
CATCHER_INVALID_ARGUMENT = -1
CATCHER_INVALID_STATE = -2
CATCHER_RUNTIME_ERROR = -3


def global_error() -> str:
    return lib().catcher_last_error(None).decode()


class Catcher:
    """One transcription handle.  ``encoder`` / ``rnnt`` configurations (both
    or neither) select catcher_create_config; without them catcher_create
    loads the Nemotron 3.5 architecture."""

    def __init__(self, model_dir: str, language: str = "en-US", lookahead: int = 3,
                 encoder=None, rnnt=None, dtype: str = "f16", device: int = 0):
        if encoder is None:
            h = lib().catcher_create(model_dir.encode(), None, language.encode(), lookahead)
        else:
            h = lib().catcher_create_config(model_dir.encode(), language.encode(), lookahead,
                                            ctypes.byref(encoder), ctypes.byref(rnnt),
                                            DTYPES[dtype], device)
        if not h:
            raise CQError(CATCHER_RUNTIME_ERROR, global_error())
        self._h = ctypes.c_void_p(h)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                lib().catcher_destroy(h)
            except TypeError:  # interpreter shutdown
                pass
            self._h = None

    def start(self) -> int:
        return lib().catcher_start(self._h)

    def push_audio(self, samples) -> int:
        a = np.ascontiguousarray(np.asarray(samples, dtype=np.float32))
        ptr = ctypes.c_void_p(a.ctypes.data) if a.size else None
        return lib().catcher_push_audio(self._h, ptr, a.size)

    def finish(self) -> int:
        return lib().catcher_finish(self._h)

    def finish_before(self, cutoff_ms: int) -> int:
        return lib().catcher_finish_before(self._h, cutoff_ms)

    def text(self) -> str:
        return lib().catcher_text(self._h).decode()

    def text_before(self, cutoff_ms: int) -> str | None:
        t = lib().catcher_text_before(self._h, cutoff_ms)
        return None if t is None else t.decode()

    def segments(self) -> str:
        return lib().catcher_segments(self._h).decode()

    def warning(self) -> str | None:
        w = lib().catcher_warning(self._h)
        return None if w is None else w.decode()

    def last_error(self) -> str:
        return lib().catcher_last_error(self._h).decode()


class ChunkScheduler:
    """AudioChunkScheduler (cq_chunk_scheduler_*): push returns the windows a
    block completed as (samples, center, mel_frames) tuples."""

    def __init__(self, lookahead: int = 3):
        h = ctypes.c_void_p()
        _check(lib().cq_chunk_scheduler_create(lookahead, ctypes.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                lib().cq_chunk_scheduler_destroy(h)
            except TypeError:
                pass
            self._h = None

    def _windows(self, n: int) -> list:
        out = []
        for i in range(n):
            count = ctypes.c_size_t()
            _check(lib().cq_chunk_scheduler_window(self._h, i, None, 0, ctypes.byref(count), None, None))
            buf = np.empty(count.value, np.float32)
            center, mel = ctypes.c_int32(), ctypes.c_int32()
            _check(lib().cq_chunk_scheduler_window(self._h, i, ctypes.c_void_p(buf.ctypes.data),
                                                   buf.size, ctypes.byref(count), ctypes.byref(center),
                                                   ctypes.byref(mel)))
            out.append((buf, bool(center.value), mel.value))
        return out

    def push(self, samples) -> list:
        a = np.ascontiguousarray(np.asarray(samples, dtype=np.float32))
        n = ctypes.c_int32()
        _check(lib().cq_chunk_scheduler_push(self._h, ctypes.c_void_p(a.ctypes.data) if a.size else None,
                                             a.size, ctypes.byref(n)))
        return self._windows(n.value)

    def finish(self):
        n = ctypes.c_int32()
        _check(lib().cq_chunk_scheduler_finish(self._h, ctypes.byref(n)))
        w = self._windows(n.value)
        return w[0] if w else None

    def reset(self) -> None:
        _check(lib().cq_chunk_scheduler_reset(self._h))


class Tokenizer:
    """Tokenizer::from_json / decode (cq_tokenizer_*)."""

    def __init__(self, path: str, pad_token_id: int, blank_token_id: int):
        h = ctypes.c_void_p()
        _check(lib().cq_tokenizer_from_json(path.encode(), pad_token_id, blank_token_id,
                                            ctypes.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                lib().cq_tokenizer_destroy(h)
            except TypeError:
                pass
            self._h = None

    def decode(self, ids, strip_language_tag: bool = True) -> str:
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.uint32))
        out = ctypes.c_char_p()
        _check(lib().cq_tokenizer_decode(self._h, ctypes.c_void_p(a.ctypes.data) if a.size else None,
                                         a.size, int(strip_language_tag), ctypes.byref(out)))
        return out.value.decode()
