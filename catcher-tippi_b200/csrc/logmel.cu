// GPU log-mel frontend: LogMelFrontend::extract
// (crates/nemotron-mlx/src/audio/log_mel.rs:63-107) for many audio windows in
// one launch.
//
// One CTA per (frame, stream), n_fft / 2 threads.  The frame's samples are
// preemphasised and windowed with the reference's separate f32 roundings
// (x[i] - p * x[i-1], then * w[i]), written in bit-reversed order into shared
// memory, and transformed by an in-place radix-2 FFT in double (a few hundred
// MFLOP per 64-stream chunk): each spectrum value is the exact DFT rounded
// once to f32, where the reference's f32 FFT (rustfft) adds its own
// summation-order error -- which, in low-energy bins, is what separates
// rustfft from the NumPy/PyTorch FFTs its test values come from.  From there
// the reference's f32 steps: the power spectrum in mul_add form, each mel
// energy folding the filter over its nonzero bins with fma in bin order (the
// reference folds over every bin; the zero weights add nothing), and
// ln(energy + 2^-24).
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdint>
#include <string>

#include "common.cuh"
#include "logmel.hpp"
#include "qlinear.hpp"

namespace nemotron_cuda {

namespace {

constexpr float kLogZeroGuard = 5.9604645e-8f;  // 2^-24

struct LogMelArgs {
  const float* audio;
  int64_t ld, samples;
  int64_t offset;  // sample index of frame 0's first FFT input: -n_fft/2 centered, else 0
  int hop, n_fft, log2n, mel_bins, frames;
  float preemphasis;
  const float* window;    // [n_fft]
  const double2* twiddle;  // [n_fft / 2]: (cos, -sin)(2 pi k / n_fft)
  const float* filters;   // [mel_bins][n_fft / 2 + 1]
  const int2* support;    // [mel_bins]: first and one-past-last nonzero bin
  float* out;             // [streams][frames][mel_bins]
};

__device__ __forceinline__ float emphasized(const float* a, int64_t idx, int64_t samples, float p) {
  if (idx < 0 || idx >= samples) return 0.0f;
  if (idx == 0) return a[0];
  return __fsub_rn(a[idx], __fmul_rn(p, a[idx - 1]));
}

__global__ void __launch_bounds__(1024) logmel_kernel(const LogMelArgs a) {
  extern __shared__ double sm[];
  const int N = a.n_fft, half_n = N >> 1;
  double* re = sm;
  double* im = sm + N;
  float* power = reinterpret_cast<float*>(sm + 2 * N);  // [N/2 + 1]
  const int tid = threadIdx.x;
  const int frame = blockIdx.x, s = blockIdx.y;
  const float* row = a.audio + static_cast<size_t>(s) * a.ld;
  const int64_t start = static_cast<int64_t>(frame) * a.hop + a.offset;

  // windowed samples into bit-reversed positions
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int i = tid + h * half_n;
    const float v = __fmul_rn(emphasized(row, start + i, a.samples, a.preemphasis), a.window[i]);
    const int r = static_cast<int>(__brev(static_cast<unsigned>(i)) >> (32 - a.log2n));
    re[r] = static_cast<double>(v);
    im[r] = 0.0;
  }
  __syncthreads();

  // radix-2 decimation in time, one butterfly per thread and stage
  for (int st = 1; st <= a.log2n; ++st) {
    const int half = 1 << (st - 1);
    const int pos = tid & (half - 1);
    const int i = ((tid >> (st - 1)) << st) + pos;
    const int j = i + half;
    const double2 w = a.twiddle[pos << (a.log2n - st)];
    const double xr = re[j], xi = im[j];
    const double tr = fma(w.x, xr, -w.y * xi);
    const double ti = fma(w.x, xi, w.y * xr);
    const double ur = re[i], ui = im[i];
    re[j] = ur - tr;
    im[j] = ui - ti;
    re[i] = ur + tr;
    im[i] = ui + ti;
    __syncthreads();
  }

  // power spectrum of bins 0 .. N/2 from the f32 spectrum: re.mul_add(re, im * im)
  for (int k = tid; k <= half_n; k += half_n) {
    const float xr = __double2float_rn(re[k]), xi = __double2float_rn(im[k]);
    power[k] = fmaf(xr, xr, __fmul_rn(xi, xi));
  }
  __syncthreads();

  const int bins = half_n + 1;
  float* out = a.out + (static_cast<size_t>(s) * a.frames + frame) * a.mel_bins;
  for (int m = tid; m < a.mel_bins; m += half_n) {
    const int2 sup = a.support[m];
    const float* f = a.filters + static_cast<size_t>(m) * bins;
    float energy = 0.0f;
    for (int k = sup.x; k < sup.y; ++k) energy = fmaf(f[k], power[k], energy);
    out[m] = logf(__fadd_rn(energy, kLogZeroGuard));
  }
}

// Slaney mel scale (log_mel.rs:151-173), f32 throughout.
constexpr float kFreqSpacing = 200.0f / 3.0f;
constexpr float kMinLogHz = 1000.0f;
constexpr float kMinLogMel = kMinLogHz / kFreqSpacing;
constexpr float kLogStep = 0.068751775f;

float hz_to_mel(float f) {
  return f >= kMinLogHz ? kMinLogMel + std::log(f / kMinLogHz) / kLogStep : f / kFreqSpacing;
}

float mel_to_hz(float m) {
  return m >= kMinLogMel ? kMinLogHz * std::exp(kLogStep * (m - kMinLogMel)) : m * kFreqSpacing;
}

}  // namespace

LogMelFrontend::LogMelFrontend(int sample_rate, int hop_length, int n_fft, int win_length, int mel_bins,
                               float preemphasis, int device)
    : sample_rate_(sample_rate),
      hop_(hop_length),
      n_fft_(n_fft),
      win_length_(win_length),
      mel_bins_(mel_bins),
      preemphasis_(preemphasis),
      device_(device) {
  if (sample_rate <= 0 || hop_length <= 0 || n_fft <= 0 || mel_bins <= 0 || win_length <= 0)
    throw_invalid("log-mel frontend sizes must be positive");
  if (win_length > n_fft) throw_invalid("log-mel window is longer than n_fft");
  if (n_fft < 4 || n_fft > 2048 || (n_fft & (n_fft - 1)) != 0)
    throw_invalid("log-mel n_fft must be a power of two in [4, 2048]");
  if (mel_bins > 4096) throw_invalid("log-mel frontend supports at most 4096 mel bins");

  // Hann window of win_length samples centred in n_fft (log_mel.rs:37-42)
  window_.assign(n_fft, 0.0f);
  const int left = (n_fft - win_length) / 2;
  const float pi = 3.14159265358979323846f;
  for (int i = 0; i < win_length; ++i) {
    const float phase = 2.0f * pi * static_cast<float>(i) / static_cast<float>(win_length - 1);
    window_[left + i] = 0.5f - 0.5f * std::cos(phase);
  }

  // Slaney filterbank (log_mel.rs:124-149)
  const int bins = n_fft / 2 + 1;
  const float min_mel = hz_to_mel(0.0f);
  const float max_mel = hz_to_mel(static_cast<float>(sample_rate) / 2.0f);
  const float mel_step = (max_mel - min_mel) / static_cast<float>(mel_bins + 1);
  std::vector<float> edges(mel_bins + 2);
  for (int i = 0; i < mel_bins + 2; ++i) edges[i] = mel_to_hz(min_mel + mel_step * static_cast<float>(i));
  const float fft_step = static_cast<float>(sample_rate) / static_cast<float>(n_fft);
  filters_.assign(static_cast<size_t>(mel_bins) * bins, 0.0f);
  support_.assign(2 * mel_bins, 0);
  for (int m = 0; m < mel_bins; ++m) {
    const float lower = edges[m], center = edges[m + 1], upper = edges[m + 2];
    const float norm = 2.0f / (upper - lower);
    int first = bins, last = 0;
    for (int b = 0; b < bins; ++b) {
      const float freq = fft_step * static_cast<float>(b);
      const float rising = (freq - lower) / (center - lower);
      const float falling = (upper - freq) / (upper - center);
      const float w = std::fmax(std::fmin(rising, falling), 0.0f) * norm;
      filters_[static_cast<size_t>(m) * bins + b] = w;
      if (w != 0.0f) {
        first = std::min(first, b);
        last = b + 1;
      }
    }
    support_[2 * m] = first < last ? first : 0;
    support_[2 * m + 1] = first < last ? last : 0;
  }
}

int64_t LogMelFrontend::frames(int64_t samples, bool center) const {
  if (samples < 0) return 0;
  if (center) return samples / hop_;
  return samples < n_fft_ ? 0 : (samples - n_fft_) / hop_ + 1;
}

void LogMelFrontend::upload() {
  if (uploaded_) return;
  DeviceGuard guard(device_);
  const int half = n_fft_ / 2;
  std::vector<double2> tw(half);
  for (int k = 0; k < half; ++k) {
    const double ang = 2.0 * 3.14159265358979323846 * static_cast<double>(k) / static_cast<double>(n_fft_);
    tw[k] = make_double2(std::cos(ang), -std::sin(ang));
  }
  d_window_ = DeviceBuffer(window_.size() * sizeof(float));
  d_twiddle_ = DeviceBuffer(tw.size() * sizeof(double2));
  d_filters_ = DeviceBuffer(filters_.size() * sizeof(float));
  d_support_ = DeviceBuffer(support_.size() * sizeof(int));
  check_cuda(cudaMemcpy(d_window_.get(), window_.data(), d_window_.bytes(), cudaMemcpyHostToDevice), "window");
  check_cuda(cudaMemcpy(d_twiddle_.get(), tw.data(), d_twiddle_.bytes(), cudaMemcpyHostToDevice), "twiddles");
  check_cuda(cudaMemcpy(d_filters_.get(), filters_.data(), d_filters_.bytes(), cudaMemcpyHostToDevice),
             "mel filters");
  check_cuda(cudaMemcpy(d_support_.get(), support_.data(), d_support_.bytes(), cudaMemcpyHostToDevice),
             "mel supports");
  uploaded_ = true;
}

void LogMelFrontend::extract(const float* audio, int streams, int64_t samples, int64_t ld, bool center,
                             float* out, cudaStream_t stream) {
  if (streams <= 0) throw_invalid("log-mel extract needs at least one stream");
  if (streams > 65535) throw_invalid("log-mel extract takes at most 65535 streams per call");
  if (samples < 0 || ld < samples) throw_invalid("log-mel audio row stride is smaller than the window");
  const int64_t nf = frames(samples, center);
  if (nf == 0) return;
  if (nf > INT32_MAX) throw_invalid("log-mel window is too long");
  if (audio == nullptr || out == nullptr) throw_invalid("audio and out must not be null");
  upload();
  DeviceGuard guard(device_);
  LogMelArgs a{};
  a.audio = audio;
  a.ld = ld;
  a.samples = samples;
  a.offset = center ? -(n_fft_ / 2) : 0;
  a.hop = hop_;
  a.n_fft = n_fft_;
  a.log2n = 0;
  while ((1 << a.log2n) < n_fft_) ++a.log2n;
  a.mel_bins = mel_bins_;
  a.frames = static_cast<int>(nf);
  a.preemphasis = preemphasis_;
  a.window = d_window_.as<float>();
  a.twiddle = d_twiddle_.as<double2>();
  a.filters = d_filters_.as<float>();
  a.support = d_support_.as<int2>();
  a.out = out;
  const size_t smem = 2 * static_cast<size_t>(n_fft_) * sizeof(double) + (n_fft_ / 2 + 1) * sizeof(float);
  logmel_kernel<<<dim3(static_cast<unsigned>(nf), static_cast<unsigned>(streams)), n_fft_ / 2, smem, stream>>>(a);
  check_cuda(cudaGetLastError(), "log-mel kernel");
}

}  // namespace nemotron_cuda
