// Streaming session of one utterance on the GPU: window scheduler, tokenizer
// decode and the log-mel -> encoder -> RNNT transcriber (stream.hpp).
#include "stream.hpp"

#include <algorithm>
#include <fstream>
#include <sstream>

#include "artifact.hpp"
#include "json.hpp"
#include "qlinear.hpp"

namespace nemotron_cuda {

// ------------------------------------------------------------------ plan

bool supported_lookahead(int lookahead) {
  return lookahead == 3 || lookahead == 0 || lookahead == 6 || lookahead == 13;
}

void check_lookahead(int lookahead) {
  // the message of ModelError::UnsupportedLookahead (model/mod.rs:46)
  if (!supported_lookahead(lookahead))
    throw_invalid("unsupported lookahead " + std::to_string(lookahead) +
                  "; supported values are [3, 0, 6, 13]");
}

// ------------------------------------------------------------------ scheduler

ChunkScheduler::ChunkScheduler(int lookahead) : lookahead_(lookahead) { check_lookahead(lookahead); }

void ChunkScheduler::ensure_open() const {
  if (finished_) throw_invalid("streaming audio session is already finished");
}

size_t ChunkScheduler::next_start() const {
  // an uncentered window starts n_fft / 2 samples before its first frame
  const size_t at = mel_frame_index_ * kHop;
  if (at < 512 / 2) throw_invalid("streaming audio offset underflow");
  return at - 512 / 2;
}

void ChunkScheduler::drop_before(size_t absolute) {
  // samples before the next window's start are never read again
  if (absolute <= base_) return;
  const size_t n = std::min(absolute - base_, audio_.size());
  audio_.erase(audio_.begin(), audio_.begin() + static_cast<std::ptrdiff_t>(n));
  base_ += n;
}

std::vector<AudioChunk> ChunkScheduler::push(const float* samples, size_t count) {
  ensure_open();
  if (count > 0 && samples == nullptr) throw_invalid("samples is null while count is non-zero");
  audio_.insert(audio_.end(), samples, samples + count);
  std::vector<AudioChunk> out;
  while (true) {
    if (!first_processed_) {
      const size_t n = first_audio_samples();
      if (base_ + audio_.size() < n) break;
      AudioChunk c;
      c.samples.assign(audio_.begin(), audio_.begin() + static_cast<std::ptrdiff_t>(n));
      c.center = true;
      c.mel_frames = first_mel_frames();
      out.push_back(std::move(c));
      first_processed_ = true;
      mel_frame_index_ = static_cast<size_t>(first_mel_frames());
      drop_before(next_start());
      continue;
    }
    const size_t start = next_start(), n = subsequent_audio_samples();
    if (base_ + audio_.size() < start + n) break;
    const size_t off = start - base_;
    AudioChunk c;
    c.samples.assign(audio_.begin() + static_cast<std::ptrdiff_t>(off),
                     audio_.begin() + static_cast<std::ptrdiff_t>(off + n));
    c.center = false;
    c.mel_frames = subsequent_mel_frames();
    out.push_back(std::move(c));
    mel_frame_index_ += static_cast<size_t>(subsequent_mel_frames());
    drop_before(next_start());
  }
  return out;
}

bool ChunkScheduler::finish(AudioChunk* out) {
  ensure_open();
  finished_ = true;
  if (base_ + audio_.size() == 0) return false;  // nothing was ever pushed
  size_t start = 0, n = 0;
  if (!first_processed_) {
    first_processed_ = true;
    mel_frame_index_ = static_cast<size_t>(first_mel_frames());
    n = first_audio_samples();
    out->center = true;
    out->mel_frames = first_mel_frames();
  } else {
    start = next_start();
    if (start >= base_ + audio_.size()) return false;
    mel_frame_index_ += static_cast<size_t>(subsequent_mel_frames());
    n = subsequent_audio_samples();
    out->center = false;
    out->mel_frames = subsequent_mel_frames();
  }
  // the window from `start`, zero-padded past the end of the audio
  out->samples.assign(n, 0.0f);
  const size_t off = start - base_;
  const size_t avail = std::min(n, audio_.size() - off);
  std::copy(audio_.begin() + static_cast<std::ptrdiff_t>(off),
            audio_.begin() + static_cast<std::ptrdiff_t>(off + avail), out->samples.begin());
  return true;
}

void ChunkScheduler::reset() {
  audio_.clear();
  base_ = 0;
  first_processed_ = false;
  mel_frame_index_ = 0;
  finished_ = false;
}

// ------------------------------------------------------------------ tokenizer

Tokenizer::Tokenizer(const std::string& path, uint32_t pad_token_id, uint32_t blank_token_id)
    : pad_(pad_token_id), blank_(blank_token_id) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw Error(CQ_INVALID_ARGUMENT, "cannot open " + path);
  std::ostringstream ss;
  ss << f.rdbuf();
  const std::string text = ss.str();
  const Json doc = JsonParser(text.data(), text.size(), "tokenizer.json").parse();
  const Json* model = doc.get("model");
  const Json* decoder = doc.get("decoder");
  auto kind_of = [](const Json* j) -> std::string {
    const Json* t = j != nullptr ? j->get("type") : nullptr;
    return t != nullptr && t->kind == Json::kStr ? t->str : std::string();
  };
  if (model == nullptr || decoder == nullptr)
    throw_invalid("invalid tokenizer.json: expected model and decoder");
  if (kind_of(model) != "BPE" || kind_of(decoder) != "Metaspace")
    throw_invalid("unsupported tokenizer model or decoder: " + kind_of(model) + " + " + kind_of(decoder));
  const Json* vocab = model->get("vocab");
  const Json* repl = decoder->get("replacement");
  if (vocab == nullptr || vocab->kind != Json::kObj || repl == nullptr || repl->kind != Json::kStr)
    throw_invalid("invalid tokenizer.json: expected model.vocab and decoder.replacement");
  for (const auto& kv : vocab->obj) {
    if (kv.second.kind != Json::kNum || kv.second.num < 0)
      throw_invalid("invalid tokenizer.json: bad id of " + kv.first);
    tokens_[static_cast<uint32_t>(kv.second.num)] = kv.first;
  }
  if (const Json* added = doc.get("added_tokens")) {
    if (added->kind != Json::kArr) throw_invalid("invalid tokenizer.json: added_tokens");
    for (const Json& t : added->arr) {
      const Json* id = t.get("id");
      const Json* content = t.get("content");
      const Json* special = t.get("special");
      if (id == nullptr || id->kind != Json::kNum || content == nullptr || content->kind != Json::kStr ||
          special == nullptr || special->kind != Json::kBool)
        throw_invalid("invalid tokenizer.json: bad added token");
      const uint32_t i = static_cast<uint32_t>(id->num);
      tokens_[i] = content->str;
      if (special->b) special_.insert(i);
    }
  }
  replacement_ = repl->str;
}

std::string Tokenizer::decode(const uint32_t* ids, size_t count, bool strip_special) const {
  std::string pieces;
  for (size_t i = 0; i < count; ++i) {
    const uint32_t id = ids[i];
    if (id == pad_ || id == blank_) continue;
    auto it = tokens_.find(id);
    if (it == tokens_.end())
      throw_invalid("token id " + std::to_string(id) + " is absent from tokenizer.json");
    if (strip_special && special_.count(id) != 0) continue;
    pieces += it->second;
  }
  std::string out;
  out.reserve(pieces.size());
  if (replacement_.empty()) {
    out = pieces;
  } else {
    for (size_t i = 0; i < pieces.size();) {
      if (pieces.compare(i, replacement_.size(), replacement_) == 0) {
        out.push_back(' ');
        i += replacement_.size();
      } else {
        out.push_back(pieces[i++]);
      }
    }
  }
  const size_t first = out.find_first_not_of(' ');
  return first == std::string::npos ? std::string() : out.substr(first);
}

// ------------------------------------------------------------------ transcriber

void nemotron_configs(const Artifact& art, cq_encoder_config* enc, cq_rnnt_config* dec) {
  cq_encoder_default_config(enc);
  cq_rnnt_default_config(dec);
  auto group_of = [&](const std::string& name) {
    const ArtifactTensorInfo* t = art.tensor_info(name);
    if (t == nullptr) throw_invalid("missing artifact tensor " + name);
    if (t->storage != ArtifactTensorInfo::Storage::kInt8Affine)
      throw_invalid("artifact tensor " + name + " is not Int8Affine");
    return t->group_size;
  };
  enc->group_size = group_of("encoder.layers.0.feed_forward1.linear1.weight");
  dec->group_size = group_of("joint.head.weight");
  const ArtifactTensorInfo* head = art.tensor_info("joint.head.weight");
  if (head->shape.size() != 2) throw_invalid("invalid model shape: joint.head.weight must have rank 2");
  dec->vocab = static_cast<int32_t>(head->shape[0]);
  dec->blank = dec->vocab - 1;
}

StreamingTranscriber::StreamingTranscriber(const Artifact& art, const cq_encoder_config& ecfg,
                                           const cq_rnnt_config& rcfg, cq_dtype dtype, int lookahead,
                                           int prompt_id, int device)
    : lookahead_(lookahead),
      prompt_id_(prompt_id),
      device_(device),
      scheduler_(lookahead),
      frontend_(LogMelFrontend::nemotron(device)),
      encoder_(ecfg, dtype, device),
      decoder_(rcfg, dtype, device) {
  if (ecfg.mel_bins != frontend_.mel_bins())
    throw_invalid("the encoder takes " + std::to_string(ecfg.mel_bins) + " mel bins; the frontend makes " +
                  std::to_string(frontend_.mel_bins()));
  if (prompt_id < 0 || prompt_id >= ecfg.num_prompts)
    throw_invalid("language prompt " + std::to_string(prompt_id) + " is outside the model's " +
                  std::to_string(ecfg.num_prompts) + " prompts");
  load_encoder_artifact(encoder_, art);
  load_rnnt_artifact(decoder_, art);
  DeviceGuard guard(device);
  const int max_mel = std::max(scheduler_.first_mel_frames(), scheduler_.subsequent_mel_frames());
  enc_state_ = std::make_unique<EncoderState>(encoder_, 1, max_mel);
  enc_state_->set_prompts(&prompt_id_, 1);
  const int max_frames = lookahead + 1;  // encoder frames of one window
  dec_state_ = std::make_unique<RnntState>(decoder_, 1, max_frames);
  // one stream whose frames mostly end at their first symbol: the persistent
  // decode (one launch per chunk, frames skipped once every stream emitted
  // blank) is the faster path here -- measured 1.64 against 2.25 ms per
  // 14-frame chunk at one stream; it loses at 16 streams and more.  Models
  // whose weights do not fit it resident keep the per-step launches.
  try {
    dec_state_->set_persistent(true);
  } catch (const Error&) {
  }
  const size_t max_samples = std::max(scheduler_.first_audio_samples(), scheduler_.subsequent_audio_samples());
  audio_ = DeviceBuffer(max_samples * sizeof(float));
  mel_ = DeviceBuffer(static_cast<size_t>(max_mel) * ecfg.mel_bins * sizeof(float));
  encoded_ = DeviceBuffer(static_cast<size_t>(max_frames) * ecfg.hidden * 2);
  const size_t cap = static_cast<size_t>(dec_state_->capacity());
  tokens_ = DeviceBuffer(cap * sizeof(int));
  token_frames_ = DeviceBuffer(cap * sizeof(int));
  counts_ = DeviceBuffer(sizeof(int));
  host_tokens_.resize(cap);
  host_frames_.resize(cap);
  check_cuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "transcriber stream");
}

StreamingTranscriber::~StreamingTranscriber() {
  if (stream_ != nullptr) {
    cudaStreamSynchronize(stream_);
    cudaStreamDestroy(stream_);
  }
}

std::vector<TimedToken> StreamingTranscriber::push_samples(const float* samples, size_t count) {
  std::vector<TimedToken> out;
  for (const AudioChunk& c : scheduler_.push(samples, count)) {
    std::vector<TimedToken> t = decode_chunk(c);
    out.insert(out.end(), t.begin(), t.end());
  }
  return out;
}

std::vector<TimedToken> StreamingTranscriber::finish() {
  AudioChunk c;
  if (!scheduler_.finish(&c)) return {};
  return decode_chunk(c);
}

void StreamingTranscriber::reset() {
  DeviceGuard guard(device_);
  check_cuda(cudaStreamSynchronize(stream_), "transcriber reset");
  enc_state_->reset();
  dec_state_->reset();
  scheduler_.reset();
  frames_seen_ = 0;
}

std::vector<TimedToken> StreamingTranscriber::decode_chunk(const AudioChunk& chunk) {
  DeviceGuard guard(device_);
  const int64_t n = static_cast<int64_t>(chunk.samples.size());
  const int64_t frames = frontend_.frames(n, chunk.center);
  if (frames != chunk.mel_frames)
    throw_invalid("audio frontend produced " + std::to_string(frames) + " frames, expected " +
                  std::to_string(chunk.mel_frames) + "x" + std::to_string(frontend_.mel_bins()));
  check_cuda(cudaMemcpyAsync(audio_.get(), chunk.samples.data(), static_cast<size_t>(n) * sizeof(float),
                             cudaMemcpyHostToDevice, stream_),
             "upload audio");
  frontend_.extract(audio_.as<float>(), 1, n, n, chunk.center, mel_.as<float>(), stream_);
  const int enc_frames = enc_state_->output_frames(chunk.mel_frames);
  enc_state_->encode_chunk(mel_.as<float>(), chunk.mel_frames, encoded_.get(), stream_);
  // the encoder caches have consumed this window whatever the decoder does
  // next, so the utterance's frame clock advances here (stream.rs:222-227)
  const uint64_t offset = frames_seen_;
  frames_seen_ += static_cast<uint64_t>(enc_frames);
  dec_state_->decode_chunk(encoded_.get(), encoder_.config().hidden, enc_frames, tokens_.as<int>(),
                           token_frames_.as<int>(), counts_.as<int>(), stream_);
  int count = 0, status = 0;
  check_cuda(cudaMemcpyAsync(&count, counts_.get(), sizeof(int), cudaMemcpyDeviceToHost, stream_),
             "read token count");
  // the device watchdog word (bounded waits that ran out set it)
  check_cuda(cudaMemcpyAsync(&status, device_context(device_).status, sizeof(int),
                             cudaMemcpyDeviceToHost, stream_),
             "read device status");
  check_cuda(cudaStreamSynchronize(stream_), "decode chunk");
  if (status != 0)
    throw Error(CQ_RUNTIME_ERROR, "device watchdog reported a timeout while decoding a chunk");
  const int cap = dec_state_->capacity();
  count = std::min(count, cap);
  std::vector<TimedToken> out;
  if (count > 0) {
    check_cuda(cudaMemcpy(host_tokens_.data(), tokens_.get(), static_cast<size_t>(count) * sizeof(int),
                          cudaMemcpyDeviceToHost),
               "read tokens");
    check_cuda(cudaMemcpy(host_frames_.data(), token_frames_.get(),
                          static_cast<size_t>(count) * sizeof(int), cudaMemcpyDeviceToHost),
               "read token frames");
    for (int i = 0; i < count; ++i)
      out.push_back(TimedToken{static_cast<uint32_t>(host_tokens_[i]),
                               offset + static_cast<uint64_t>(host_frames_[i])});
  }
  return out;
}

}  // namespace nemotron_cuda
