"""CPU oracle of the log-mel frontend -- test infrastructure only.

A numpy restatement of LogMelFrontend (crates/nemotron-mlx/src/audio/
log_mel.rs:8-173): preemphasis x[i] - p * x[i-1] per window (the first
sample kept), a win_length Hann window centred in n_fft (:37-42), the Slaney
mel filterbank (:124-149) on the Slaney mel scale (:151-173), the power
spectrum re.mul_add(re, im * im) (:92-94), the filter folded with mul_add in
bin order (:97-101) and ln(energy + 2^-24) (:102).  Every step the reference
takes in f32 is taken in f32 here (products rounded separately where the
reference rounds them separately; mul_add emulated exactly in float64, one
rounding to f32).  The FFT is float64 and its output rounded once to f32:
the exact spectrum, where the reference's rustfft adds its own summation
error (which the reference's tests allow 1e-3 for against NumPy/PyTorch).

Pinned by the reference's own tests (crates/nemotron-mlx/tests/log_mel.rs):
the published centered-frame values (:15-55, 1e-3), silence at the guard
(:57-65, 1e-5) and uncentered overlap = centered frame (:67-79, 2e-4).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

F32 = np.float32
LOG_ZERO_GUARD = F32(5.9604645e-8)  # 2^-24


@dataclass(frozen=True)
class LogMelConfig:
    sample_rate: int = 16000
    hop_length: int = 160
    n_fft: int = 512
    win_length: int = 400
    mel_bins: int = 128
    preemphasis: float = 0.97


NEMOTRON = LogMelConfig()


def frames(samples: int, center: bool, cfg: LogMelConfig = NEMOTRON) -> int:
    """log_mel.rs:64-70."""
    if center:
        return samples // cfg.hop_length
    return 0 if samples < cfg.n_fft else (samples - cfg.n_fft) // cfg.hop_length + 1


def hann_window(cfg: LogMelConfig = NEMOTRON) -> np.ndarray:
    """log_mel.rs:37-42: 0.5 - 0.5 cos(2 pi i / (win - 1)), f32, centred in n_fft."""
    w = np.zeros(cfg.n_fft, F32)
    left = (cfg.n_fft - cfg.win_length) // 2
    i = np.arange(cfg.win_length, dtype=F32)
    phase = (F32(2.0) * F32(np.pi) * i) / F32(cfg.win_length - 1)
    w[left:left + cfg.win_length] = F32(0.5) - F32(0.5) * np.cos(phase.astype(F32))
    return w


_FREQ_SPACING = F32(200.0) / F32(3.0)
_MIN_LOG_HZ = F32(1000.0)
_MIN_LOG_MEL = _MIN_LOG_HZ / _FREQ_SPACING
_LOG_STEP = F32(0.068751775)


def hz_to_mel(f):
    """log_mel.rs:151-161 (f32)."""
    f = F32(f)
    if f >= _MIN_LOG_HZ:
        return F32(_MIN_LOG_MEL + F32(np.log(F32(f / _MIN_LOG_HZ))) / _LOG_STEP)
    return F32(f / _FREQ_SPACING)


def mel_to_hz(m):
    """log_mel.rs:163-173 (f32)."""
    m = F32(m)
    if m >= _MIN_LOG_MEL:
        return F32(_MIN_LOG_HZ * F32(np.exp(F32(_LOG_STEP * F32(m - _MIN_LOG_MEL)))))
    return F32(m * _FREQ_SPACING)


def slaney_filters(cfg: LogMelConfig = NEMOTRON) -> np.ndarray:
    """log_mel.rs:124-149: [mel_bins][n_fft/2 + 1] f32."""
    min_mel = hz_to_mel(0.0)
    max_mel = hz_to_mel(F32(cfg.sample_rate) / F32(2.0))
    step = F32(F32(max_mel - min_mel) / F32(cfg.mel_bins + 1))
    edges = [mel_to_hz(F32(min_mel + F32(step * F32(i)))) for i in range(cfg.mel_bins + 2)]
    fft_step = F32(F32(cfg.sample_rate) / F32(cfg.n_fft))
    freq = (fft_step * np.arange(cfg.n_fft // 2 + 1, dtype=F32)).astype(F32)
    out = np.zeros((cfg.mel_bins, cfg.n_fft // 2 + 1), F32)
    for m in range(cfg.mel_bins):
        lower, center, upper = edges[m], edges[m + 1], edges[m + 2]
        norm = F32(F32(2.0) / F32(upper - lower))
        rising = ((freq - lower) / F32(center - lower)).astype(F32)
        falling = ((upper - freq) / F32(upper - center)).astype(F32)
        out[m] = (np.maximum(np.minimum(rising, falling), F32(0.0)) * norm).astype(F32)
    return out


def preemphasize(audio: np.ndarray, coef: float) -> np.ndarray:
    """log_mel.rs:110-122: first sample kept, then x[i] - coef * x[i-1] (two roundings)."""
    a = np.asarray(audio, F32)
    out = np.empty_like(a)
    if a.size:
        out[0] = a[0]
        out[1:] = a[1:] - (F32(coef) * a[:-1]).astype(F32)
    return out


def _fma_f32(a, b, c):
    """f32 mul_add: a*b + c rounded once (a*b is exact in float64)."""
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(F32)


def extract(audio: np.ndarray, center: bool, cfg: LogMelConfig = NEMOTRON,
            window: np.ndarray | None = None, filters: np.ndarray | None = None) -> np.ndarray:
    """LogMelFrontend::extract (log_mel.rs:63-107) -> f32 [frames, mel_bins]."""
    n = frames(len(audio), center, cfg)
    if n == 0:
        return np.zeros((0, cfg.mel_bins), F32)
    w = hann_window(cfg) if window is None else window
    fb = slaney_filters(cfg) if filters is None else filters
    e = preemphasize(audio, cfg.preemphasis)
    off = -(cfg.n_fft // 2) if center else 0
    idx = np.arange(n)[:, None] * cfg.hop_length + off + np.arange(cfg.n_fft)[None, :]
    valid = (idx >= 0) & (idx < len(e))
    seg = np.where(valid, e[np.clip(idx, 0, max(len(e) - 1, 0))], F32(0.0)).astype(F32)
    windowed = (seg * w[None, :]).astype(F32)
    spec = np.fft.rfft(windowed.astype(np.float64), axis=1)
    re, im = spec.real.astype(F32), spec.imag.astype(F32)
    power = _fma_f32(re, re, (im * im).astype(F32))  # [frames, bins]
    energy = np.zeros((n, cfg.mel_bins), F32)
    for k in range(power.shape[1]):
        energy = _fma_f32(np.broadcast_to(fb[:, k], energy.shape), np.broadcast_to(power[:, k:k + 1],
                                                                                   energy.shape), energy)
    return np.log((energy + LOG_ZERO_GUARD).astype(F32)).astype(F32)


def synthetic_audio(samples: int) -> np.ndarray:
    """The reference test's signal (tests/log_mel.rs:4-13): 440 Hz and 1200 Hz
    tones plus a 31-sample sawtooth, in f32."""
    i = np.arange(samples)
    t = (i.astype(F32) / F32(16000.0)).astype(F32)
    two_pi = F32(2.0) * F32(np.pi)
    a = (F32(0.3) * np.sin((two_pi * F32(440.0) * t).astype(F32))).astype(F32)
    b = (F32(0.1) * np.sin((two_pi * F32(1200.0) * t).astype(F32))).astype(F32)
    c = ((i % 31).astype(F32) - F32(15.0)) * F32(0.0005)
    return (a + b + c.astype(F32)).astype(F32)
