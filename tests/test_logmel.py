"""Log-mel frontend on CPU: the oracle against the reference's own tests
(crates/nemotron-mlx/tests/log_mel.rs), and the library's host tables
(window, Slaney filterbank) and frame counts against the oracle -- no GPU."""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import logmel_oracle as lo  # noqa: E402

# tests/log_mel.rs:23-41: frames 0, 1, 4, 9 of the centered extraction of 1600
# samples of synthetic_audio, at mel bins 0, 1, 5, 10, 20, 40, 80, 127
KAT_BINS = [0, 1, 5, 10, 20, 40, 80, 127]
KAT_FRAMES = [0, 1, 4, 9]
KAT_VALUES = [
    [-9.101493, -8.904302, -7.602791, -6.0763245, -2.515178, -10.496132, -7.321813, -8.829868],
    [-14.00288, -13.877358, -12.133504, -10.178206, -3.0286355, -11.540961, -9.994083, -9.654244],
    [-16.550058, -16.28926, -16.119799, -12.411482, -3.1358635, -11.955688, -10.157519, -9.673437],
    [-11.115188, -11.104209, -10.721158, -9.595677, -3.0761108, -11.387222, -9.937812, -9.673555],
]
SILENCE = -16.635532  # tests/log_mel.rs:63


def kat_error(frames: np.ndarray) -> float:
    got = frames[np.ix_(KAT_FRAMES, KAT_BINS)]
    return float(np.abs(got - np.array(KAT_VALUES, np.float32)).max())


def test_oracle_matches_the_published_frontend_values():
    """tests/log_mel.rs:15-55 (1e-3: FFT summation order differs between implementations)."""
    frames = lo.extract(lo.synthetic_audio(1600), center=True)
    assert frames.shape == (10, 128)
    assert kat_error(frames) <= 1e-3


def test_oracle_silence_is_the_log_zero_guard():
    """tests/log_mel.rs:57-65."""
    frames = lo.extract(np.zeros(1600, np.float32), center=True)
    assert np.allclose(frames, SILENCE, atol=1e-5)


def test_oracle_uncentered_overlap_reproduces_a_centered_frame():
    """tests/log_mel.rs:67-79."""
    audio = lo.synthetic_audio(2000)
    centered = lo.extract(audio, center=True)
    start = 4 * 160 - 512 // 2
    un = lo.extract(audio[start:start + 512], center=False)
    assert un.shape == (1, 128)
    assert np.abs(un[0] - centered[4]).max() <= 2e-4


def test_frame_counts_follow_the_reference():
    """log_mel.rs:64-70, and the chunk windows of the streaming scheduler
    (encoder.rs:961-978: 105 centered frames from 16840 samples, then 112
    uncentered frames from 18320)."""
    assert lo.frames(1600, True) == 10
    assert lo.frames(512, False) == 1
    assert lo.frames(511, False) == 0
    assert lo.frames(16840, True) == 105
    assert lo.frames(18320, False) == 112


@pytest.fixture(scope="module")
def frontend(cq):
    from nemotron_cuda.logmel import LogMelFrontend
    return LogMelFrontend.nemotron()  # no device work until extract


def test_library_tables_match_the_oracle(frontend):
    w = frontend.window()
    assert np.abs(w - lo.hann_window()).max() <= 1e-7  # libm vs numpy cos: an ulp at most
    f = frontend.filters()
    ref = lo.slaney_filters()
    assert f.shape == ref.shape == (128, 257)
    # the band edges come from f32 exp/log (libm here, numpy's own there), an
    # ulp apart; near a triangle's corners that moves a small weight by a
    # larger fraction of itself, but by under 1e-5 of the filter's peak (a mel
    # energy by under 1e-5, relative)
    rowmax = np.abs(ref).max(axis=1, keepdims=True)
    assert (np.abs(f - ref) / rowmax).max() <= 2e-5
    assert np.array_equal(f != 0, ref != 0)


def test_library_frame_counts(frontend):
    for samples, center in [(1600, True), (512, False), (511, False), (16840, True), (18320, False),
                            (0, True), (159, True)]:
        assert frontend.frames(samples, center) == lo.frames(samples, center)


def test_library_rejects_bad_configurations(cq):
    from nemotron_cuda import CQError
    from nemotron_cuda.logmel import LogMelFrontend
    with pytest.raises(CQError, match="longer than n_fft"):
        LogMelFrontend(16000, 160, 512, 600, 128, 0.97)
    with pytest.raises(CQError, match="power of two"):
        LogMelFrontend(16000, 160, 500, 400, 128, 0.97)
    with pytest.raises(CQError, match="positive"):
        LogMelFrontend(16000, 0, 512, 400, 128, 0.97)
    L = cq.lib()
    assert L.cq_logmel_extract(None, None, 1, 1600, 1600, 1, None, None) == cq.CQ_INVALID_ARGUMENT
    assert L.cq_logmel_frames(None, 1600, 1) == -1
    h = ctypes.c_void_p()
    assert L.cq_logmel_create_nemotron(0, ctypes.byref(h)) == cq.CQ_OK
    assert L.cq_logmel_mel_bins(h) == 128
    buf = np.empty(10, np.float32)
    assert L.cq_logmel_window(h, buf.ctypes.data, buf.size) == cq.CQ_INVALID_ARGUMENT
    L.cq_logmel_destroy(h)
