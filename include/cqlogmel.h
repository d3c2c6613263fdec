/*
 * cqlogmel.h - C ABI of the GPU log-mel frontend.
 *
 * Stands in for LogMelFrontend (crates/nemotron-mlx/src/audio/log_mel.rs:8-108):
 * preemphasis, Hann-windowed STFT power spectrum, Slaney mel filterbank and
 * natural log with the 2^-24 guard, for many audio windows at once.  The
 * windows are the ones the reference's AudioChunkScheduler cuts
 * (crates/nemotron-mlx/src/model/stream.rs:37-100): a centered first chunk,
 * uncentered later chunks; each window is preemphasised on its own, as
 * LogMelFrontend::extract does.  Conventions are those of cqlinear.h.
 */
#ifndef CQLOGMEL_H
#define CQLOGMEL_H

#include <stddef.h>
#include <stdint.h>

#include "cqlinear.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cq_logmel cq_logmel;

/* LogMelFrontend::new (log_mel.rs:26-55).  n_fft must be a power of two in
 * [4, 2048], win_length <= n_fft, every size > 0.  No device work: the
 * tables go to `device` at the first extract. */
cq_status cq_logmel_create(int32_t sample_rate, int32_t hop_length, int32_t n_fft, int32_t win_length,
                           int32_t mel_bins, float preemphasis, int32_t device, cq_logmel **out);

/* LogMelFrontend::nemotron (log_mel.rs:21-23): 16 kHz, hop 160, n_fft 512,
 * window 400, 128 mel bins, preemphasis 0.97. */
cq_status cq_logmel_create_nemotron(int32_t device, cq_logmel **out);

/* Frames extract() makes from `samples` samples (log_mel.rs:64-70):
 * centered samples / hop, else (samples - n_fft) / hop + 1 (0 if shorter). */
int64_t cq_logmel_frames(const cq_logmel *fe, int64_t samples, int32_t center);
int32_t cq_logmel_mel_bins(const cq_logmel *fe);

/* Host copies of the tables: the n_fft-long window and the [mel_bins][n_fft/2+1]
 * filterbank, computed in f32 as the reference computes them. */
cq_status cq_logmel_window(const cq_logmel *fe, float *out, size_t len);
cq_status cq_logmel_filters(const cq_logmel *fe, float *out, size_t len);

/* LogMelFrontend::extract (log_mel.rs:63-107) of `streams` windows at once:
 * audio is device f32 [streams][ld] (the first `samples` of each row used),
 * out device f32 [streams][frames][mel_bins] with frames = cq_logmel_frames.
 * Asynchronous on `stream`; nothing is written when frames is 0. */
cq_status cq_logmel_extract(cq_logmel *fe, const float *audio, int32_t streams, int64_t samples, int64_t ld,
                            int32_t center, float *out, void *stream);

void cq_logmel_destroy(cq_logmel *fe);

#ifdef __cplusplus
}
#endif

#endif /* CQLOGMEL_H */
