"""GPU log-mel frontend (include/cqlogmel.h) against the reference's published
values (crates/nemotron-mlx/tests/log_mel.rs) and the oracle.

The oracle is run with the library's own window and filterbank (made on the
host in f32; their agreement with the oracle's tables is a CPU test), so the
comparison isolates the kernel: the f64 FFT rounded to f32, then the
reference's f32 power, fma fold and log.  Both FFTs are f64, so the spectra
agree to far below an f32 ulp; what remains is logf against numpy's log, an
ulp or two of values near 10: every output within 1e-5 of the oracle.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import logmel_oracle as lo  # noqa: E402
from test_logmel import SILENCE, kat_error  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _oracle(fe, audio, center, cfg=lo.NEMOTRON):
    return lo.extract(audio, center, cfg, window=fe.window(), filters=fe.filters())


def _speechlike(rng, samples):
    t = np.arange(samples) / 16000.0
    x = np.zeros(samples)
    for _ in range(6):
        x += rng.uniform(0.01, 0.3) * np.sin(2 * np.pi * rng.uniform(60, 7000) * t + rng.uniform(0, 6.3))
    x += rng.standard_normal(samples) * 0.01
    gap = rng.integers(0, samples // 2)
    x[gap:gap + samples // 8] = 0.0  # a stretch of silence
    return x.astype(np.float32)


def test_published_values_and_oracle(cq):
    import torch
    from nemotron_cuda.logmel import LogMelFrontend
    fe = LogMelFrontend.nemotron()
    audio = lo.synthetic_audio(1600)
    got = fe.extract(torch.from_numpy(audio).cuda(), center=True)
    torch.cuda.synchronize()
    got = got.cpu().numpy()[0]
    assert got.shape == (10, 128)
    assert kat_error(got) <= 1e-3  # tests/log_mel.rs:54
    assert np.abs(got - _oracle(fe, audio, True)).max() <= TOL
    assert cq.device_status(0) == 0


def test_silence_is_the_log_zero_guard(cq):
    import torch
    from nemotron_cuda.logmel import LogMelFrontend
    fe = LogMelFrontend.nemotron()
    got = fe.extract(torch.zeros(1600, device="cuda"), center=True).cpu().numpy()
    assert np.allclose(got, SILENCE, atol=1e-5)


def test_streaming_windows_for_many_streams(cq):
    """The scheduler's windows (stream.rs:37-70): a centered first chunk of
    16840 samples (105 frames) and uncentered later chunks of 18320 samples
    (112 frames), five streams per launch, rows padded past the window."""
    import torch
    from nemotron_cuda.logmel import LogMelFrontend
    fe = LogMelFrontend.nemotron()
    rng = np.random.default_rng(5)
    for samples, center, frames in [(16840, True, 105), (18320, False, 112)]:
        audio = np.stack([_speechlike(rng, samples) for _ in range(5)])
        ld = samples + 37
        dev = torch.zeros((5, ld), device="cuda")
        dev[:, :samples] = torch.from_numpy(audio).cuda()
        dev[:, samples:] = 1.0e3  # past the window: must not be read
        out = torch.full((5, frames, 128), float("nan"), device="cuda")
        fe.extract_raw(dev, samples, center, out)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        for s in range(5):
            want = _oracle(fe, audio[s], center)
            assert want.shape == (frames, 128)
            assert np.abs(got[s] - want).max() <= TOL, (s, center)
    assert cq.device_status(0) == 0


def test_uncentered_overlap_reproduces_a_centered_frame(cq):
    """tests/log_mel.rs:67-79 on the GPU."""
    import torch
    from nemotron_cuda.logmel import LogMelFrontend
    fe = LogMelFrontend.nemotron()
    audio = lo.synthetic_audio(2000)
    centered = fe.extract(torch.from_numpy(audio).cuda(), center=True).cpu().numpy()[0]
    start = 4 * 160 - 512 // 2
    un = fe.extract(torch.from_numpy(audio[start:start + 512].copy()).cuda(), center=False).cpu().numpy()[0]
    assert un.shape == (1, 128)
    assert np.abs(un[0] - centered[4]).max() <= 2e-4


def test_another_configuration(cq):
    """LogMelFrontend::new with other sizes: 8 kHz, hop 80, n_fft 256, window
    200, 64 mel bins, preemphasis 0.9; and n_fft 2048 with 1024 threads."""
    import torch
    from nemotron_cuda.logmel import LogMelFrontend
    rng = np.random.default_rng(9)
    for args in [(8000, 80, 256, 200, 64, 0.9), (16000, 160, 2048, 1600, 80, 0.97)]:
        cfg = lo.LogMelConfig(*args)
        fe = LogMelFrontend(*args)
        audio = _speechlike(rng, 9000)
        for center in (True, False):
            got = fe.extract(torch.from_numpy(audio).cuda(), center=center).cpu().numpy()[0]
            want = _oracle(fe, audio, center, cfg)
            assert got.shape == want.shape
            assert np.abs(got - want).max() <= TOL, (args, center)


def test_short_windows_make_no_frames(cq):
    import torch
    from nemotron_cuda.logmel import LogMelFrontend
    fe = LogMelFrontend.nemotron()
    out = fe.extract(torch.zeros((3, 300), device="cuda"), center=False)
    assert tuple(out.shape) == (3, 0, 128)
    assert cq.device_status(0) == 0
