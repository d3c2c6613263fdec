// Host side of the GPU log-mel frontend: the counterpart of LogMelFrontend
// (crates/nemotron-mlx/src/audio/log_mel.rs:8-108).  The window and the
// Slaney filterbank are computed on the host in f32 exactly as the reference
// computes them; the device gets them (and the FFT twiddles) at the first
// extract, so a frontend can be made and inspected without a GPU.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "device_buffer.hpp"

namespace nemotron_cuda {

class LogMelFrontend {
 public:
  LogMelFrontend(int sample_rate, int hop_length, int n_fft, int win_length, int mel_bins,
                 float preemphasis, int device);
  static LogMelFrontend nemotron(int device) { return LogMelFrontend(16000, 160, 512, 400, 128, 0.97f, device); }

  int64_t frames(int64_t samples, bool center) const;
  int mel_bins() const { return mel_bins_; }
  int n_fft() const { return n_fft_; }
  const std::vector<float>& window() const { return window_; }
  const std::vector<float>& filters() const { return filters_; }  // [mel][n_fft/2+1]

  // audio: device f32 [streams][ld]; out: device f32 [streams][frames][mel_bins]
  void extract(const float* audio, int streams, int64_t samples, int64_t ld, bool center, float* out,
               cudaStream_t stream);

 private:
  void upload();

  int sample_rate_, hop_, n_fft_, win_length_, mel_bins_;
  float preemphasis_;
  int device_;
  std::vector<float> window_, filters_;
  std::vector<int> support_;  // [mel][2]: first and one-past-last nonzero bin
  bool uploaded_ = false;
  DeviceBuffer d_window_, d_twiddle_, d_filters_, d_support_;
};

}  // namespace nemotron_cuda
