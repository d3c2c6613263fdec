// extern "C" entry points of include/cqlogmel.h over LogMelFrontend.
#include <memory>

#include "capi_guard.hpp"
#include "cqlogmel.h"
#include "logmel.hpp"

using nemotron_cuda::guarded;
using nemotron_cuda::LogMelFrontend;
using nemotron_cuda::need_handle;

struct cq_logmel {
  std::unique_ptr<LogMelFrontend> impl;
};

extern "C" {

cq_status cq_logmel_create(int32_t sample_rate, int32_t hop_length, int32_t n_fft, int32_t win_length,
                           int32_t mel_bins, float preemphasis, int32_t device, cq_logmel** out) {
  return guarded([&] {
    need_handle(out, "out");
    *out = nullptr;
    auto h = std::make_unique<cq_logmel>();
    h->impl = std::make_unique<LogMelFrontend>(sample_rate, hop_length, n_fft, win_length, mel_bins,
                                               preemphasis, device);
    *out = h.release();
  });
}

cq_status cq_logmel_create_nemotron(int32_t device, cq_logmel** out) {
  return cq_logmel_create(16000, 160, 512, 400, 128, 0.97f, device, out);
}

int64_t cq_logmel_frames(const cq_logmel* fe, int64_t samples, int32_t center) {
  return fe ? fe->impl->frames(samples, center != 0) : -1;
}

int32_t cq_logmel_mel_bins(const cq_logmel* fe) { return fe ? fe->impl->mel_bins() : -1; }

cq_status cq_logmel_window(const cq_logmel* fe, float* out, size_t len) {
  return guarded([&] {
    need_handle(fe, "frontend");
    need_handle(out, "out");
    const auto& w = fe->impl->window();
    if (len != w.size()) nemotron_cuda::throw_invalid("window buffer must hold n_fft values");
    std::copy(w.begin(), w.end(), out);
  });
}

cq_status cq_logmel_filters(const cq_logmel* fe, float* out, size_t len) {
  return guarded([&] {
    need_handle(fe, "frontend");
    need_handle(out, "out");
    const auto& f = fe->impl->filters();
    if (len != f.size()) nemotron_cuda::throw_invalid("filter buffer must hold mel_bins * (n_fft / 2 + 1) values");
    std::copy(f.begin(), f.end(), out);
  });
}

cq_status cq_logmel_extract(cq_logmel* fe, const float* audio, int32_t streams, int64_t samples, int64_t ld,
                            int32_t center, float* out, void* stream) {
  return guarded([&] {
    need_handle(fe, "frontend");
    fe->impl->extract(audio, streams, samples, ld, center != 0, out, static_cast<cudaStream_t>(stream));
  });
}

void cq_logmel_destroy(cq_logmel* fe) { delete fe; }

}  // extern "C"
