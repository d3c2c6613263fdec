"""Python bindings of the GPU log-mel frontend (include/cqlogmel.h).

Mirrors the reference's LogMelFrontend (crates/nemotron-mlx/src/audio/
log_mel.rs:8-108): ``LogMelFrontend.nemotron()`` is the published Nemotron
configuration; ``extract`` turns audio windows (one per stream, on the
device) into f32 log-mel frames [streams, frames, mel_bins], centered for a
first chunk, uncentered after it, as the reference's chunk scheduler cuts
them.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _check, _ptr, _stream_ptr, lib


class LogMelFrontend:
    def __init__(self, sample_rate: int = 16000, hop_length: int = 160, n_fft: int = 512,
                 win_length: int = 400, mel_bins: int = 128, preemphasis: float = 0.97,
                 device: int = 0):
        h = ctypes.c_void_p()
        _check(lib().cq_logmel_create(sample_rate, hop_length, n_fft, win_length, mel_bins,
                                      preemphasis, device, ctypes.byref(h)))
        self._h = h
        self.n_fft, self.hop_length, self.mel_bins = n_fft, hop_length, mel_bins

    @classmethod
    def nemotron(cls, device: int = 0) -> "LogMelFrontend":
        return cls(16000, 160, 512, 400, 128, 0.97, device)

    def close(self) -> None:
        if getattr(self, "_h", None):
            try:
                lib().cq_logmel_destroy(self._h)
            except TypeError:  # interpreter shutdown
                pass
            self._h = None

    def __del__(self):
        self.close()

    def frames(self, samples: int, center: bool) -> int:
        return int(lib().cq_logmel_frames(self._h, samples, int(center)))

    def window(self) -> np.ndarray:
        out = np.empty(self.n_fft, np.float32)
        _check(lib().cq_logmel_window(self._h, out.ctypes.data, out.size))
        return out

    def filters(self) -> np.ndarray:
        out = np.empty((self.mel_bins, self.n_fft // 2 + 1), np.float32)
        _check(lib().cq_logmel_filters(self._h, out.ctypes.data, out.size))
        return out

    def extract_raw(self, audio, samples: int, center: bool, out, stream=None) -> None:
        """audio: device f32 [streams, ld]; out: device f32 [streams, frames, mel_bins]."""
        _check(lib().cq_logmel_extract(self._h, _ptr(audio), audio.shape[0], samples, audio.stride(0),
                                       int(center), _ptr(out), _stream_ptr(stream)))

    def extract(self, audio, center: bool, stream=None):
        """audio torch f32 [streams, samples] on the device -> [streams, frames, mel_bins]."""
        import torch
        if audio.dim() == 1:
            audio = audio[None, :]
        frames = self.frames(audio.shape[1], center)
        out = torch.empty((audio.shape[0], frames, self.mel_bins), dtype=torch.float32,
                          device=audio.device)
        if frames:
            self.extract_raw(audio, audio.shape[1], center, out, stream)
        return out
