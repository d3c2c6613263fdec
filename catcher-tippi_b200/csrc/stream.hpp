// Streaming session of one mono 16 kHz utterance on the GPU: the pieces
// behind the catcher.h C ABI.
//
//  * ChunkScheduler -- AudioChunkScheduler
//    (crates/nemotron-mlx/src/model/stream.rs:17-128): buffers arbitrary
//    microphone blocks and cuts the exact cache-aware model windows (a
//    centered first window of 1 + 8 * lookahead mel frames, then uncentered
//    windows of 8 * (lookahead + 1) frames that overlap the previous one by
//    n_fft / 2 samples; StreamingChunkPlan, encoder.rs:941-994).
//  * Tokenizer -- the decode-only Metaspace BPE tokenizer
//    (crates/nemotron-mlx/src/tokenizer.rs:25-87).
//  * StreamingTranscriber -- StreamingTranscriber (stream.rs:130-236): every
//    window goes through the GPU log-mel frontend, the cache-aware encoder and
//    the batched RNNT greedy decoder (one stream), and the emitted tokens carry
//    their global encoder-frame index.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "cqencoder.h"
#include "cqrnnt.h"
#include "device_buffer.hpp"
#include "encoder.hpp"
#include "logmel.hpp"
#include "rnnt.hpp"

namespace nemotron_cuda {

class Artifact;

// One exact audio window for the log-mel frontend (stream.rs:9-15).
struct AudioChunk {
  std::vector<float> samples;
  bool center = false;
  int mel_frames = 0;
};

// An emitted token and its encoder frame in the whole utterance (80 ms each).
struct TimedToken {
  uint32_t id;
  uint64_t frame;
};

// Lookahead values the checkpoint was trained for (encoder.rs:933); others
// are rejected with the reference's message.
bool supported_lookahead(int lookahead);
void check_lookahead(int lookahead);

class ChunkScheduler {
 public:
  explicit ChunkScheduler(int lookahead);

  int first_mel_frames() const { return 1 + kFactor * lookahead_; }
  int subsequent_mel_frames() const { return kFactor * (lookahead_ + 1); }
  size_t first_audio_samples() const { return static_cast<size_t>(first_mel_frames() - 1) * kHop + 200; }
  size_t subsequent_audio_samples() const {
    return static_cast<size_t>(subsequent_mel_frames()) * kHop + 400;
  }

  // Appends samples and returns every window completed by them.
  std::vector<AudioChunk> push(const float* samples, size_t count);
  // Zero-pads and returns the last incomplete window; false when there is
  // none.  The scheduler is closed afterwards until reset().
  bool finish(AudioChunk* out);
  void reset();

 private:
  static constexpr int kFactor = 8;    // encoder subsampling
  static constexpr size_t kHop = 160;  // 10 ms at 16 kHz
  void ensure_open() const;
  size_t next_start() const;  // absolute sample index of the next uncentered window
  void drop_before(size_t absolute);

  int lookahead_;
  std::vector<float> audio_;  // samples from absolute index base_ on
  size_t base_ = 0;
  bool first_processed_ = false;
  size_t mel_frame_index_ = 0;
  bool finished_ = false;
};

class Tokenizer {
 public:
  // tokenizer.json with a BPE model and a Metaspace decoder.
  Tokenizer(const std::string& path, uint32_t pad_token_id, uint32_t blank_token_id);
  // Token ids -> text: pad and blank are skipped, special tokens too when
  // strip_special; the pieces are joined, the Metaspace replacement becomes a
  // space and leading spaces are trimmed.
  std::string decode(const uint32_t* ids, size_t count, bool strip_special) const;

 private:
  std::unordered_map<uint32_t, std::string> tokens_;
  std::unordered_set<uint32_t> special_;
  std::string replacement_;
  uint32_t pad_, blank_;
};

// Encoder and RNNT configuration of a release artifact: the Nemotron 3.5
// architecture (EncoderConfig::nemotron_3_5, encoder.rs:922-937; the RNNT's
// hidden sizes and ten symbols per frame), with the group size and the
// vocabulary read from the artifact's manifest.
void nemotron_configs(const Artifact& art, cq_encoder_config* enc, cq_rnnt_config* dec);

class StreamingTranscriber {
 public:
  StreamingTranscriber(const Artifact& art, const cq_encoder_config& ecfg, const cq_rnnt_config& rcfg,
                       cq_dtype dtype, int lookahead, int prompt_id, int device);
  ~StreamingTranscriber();
  StreamingTranscriber(const StreamingTranscriber&) = delete;
  StreamingTranscriber& operator=(const StreamingTranscriber&) = delete;

  std::vector<TimedToken> push_samples(const float* samples, size_t count);
  std::vector<TimedToken> finish();
  void reset();
  int lookahead() const { return lookahead_; }

 private:
  std::vector<TimedToken> decode_chunk(const AudioChunk& chunk);

  int lookahead_, prompt_id_, device_;
  ChunkScheduler scheduler_;
  LogMelFrontend frontend_;
  Encoder encoder_;
  RnntDecoder decoder_;
  std::unique_ptr<EncoderState> enc_state_;
  std::unique_ptr<RnntState> dec_state_;
  DeviceBuffer audio_, mel_, encoded_, tokens_, token_frames_, counts_;
  std::vector<int> host_tokens_, host_frames_;
  cudaStream_t stream_ = nullptr;
  uint64_t frames_seen_ = 0;
};

}  // namespace nemotron_cuda
