// extern "C" layer of catcher.h (the transcription ABI) and cqstream.h (the
// window scheduler and the tokenizer).  Every catcher_* entry keeps the
// reference's contract (crates/catcher-ffi/src/lib.rs:251-586): argument
// checks before anything else, a NULL handle reported through the
// thread-local error, the session's Idle -> Started -> Finished states, and
// no exception crossing the boundary.
#include <climits>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "artifact.hpp"
#include "capi_guard.hpp"
#include "catcher.h"
#include "cqstream.h"
#include "stream.hpp"

using nemotron_cuda::Artifact;
using nemotron_cuda::AudioChunk;
using nemotron_cuda::ChunkScheduler;
using nemotron_cuda::StreamingTranscriber;
using nemotron_cuda::TimedToken;
using nemotron_cuda::Tokenizer;

namespace {

constexpr uint64_t kFrameMs = 80;  // one encoder frame (lib.rs:28)

// Language prompt codes of the checkpoint's processor_config.json and their
// prompt slots (LanguagePrompt::from_code, crates/nemotron-mlx/src/model/
// prompt.rs:14-20, 143-265): the same aliases must resolve to the same slots.
struct PromptCode {
  const char* code;
  int id;
};
constexpr PromptCode kPrompts[] = {
    {"af-ZA", 54}, {"am-ET", 49}, {"ar", 7}, {"ar-AR", 7}, {"auto", 101}, {"ay-BO", 81},
    {"az-AZ", 66}, {"bg", 30}, {"bg-BG", 30}, {"bn-IN", 36}, {"cs", 22}, {"cs-CZ", 22},
    {"da", 25}, {"da-DK", 25}, {"de", 9}, {"de-DE", 9}, {"el", 21}, {"el-GR", 21},
    {"en", 0}, {"en-GB", 1}, {"en-US", 0}, {"enGB", 1}, {"es", 3}, {"es-ES", 2},
    {"es-US", 3}, {"esES", 2}, {"et", 60}, {"et-EE", 60}, {"fa-IR", 38}, {"fi", 26},
    {"fi-FI", 26}, {"fr", 8}, {"fr-CA", 100}, {"fr-FR", 8}, {"gn-PY", 82}, {"gu-IN", 42},
    {"ha-NG", 50}, {"haw-US", 97}, {"he-IL", 64}, {"hi", 6}, {"hi-HI", 6}, {"hi-IN", 6},
    {"hr", 29}, {"hr-HR", 29}, {"hu", 23}, {"hu-HU", 23}, {"hy-AM", 68}, {"id-ID", 34},
    {"ig-NG", 53}, {"it", 15}, {"it-IT", 15}, {"ja-JA", 10}, {"ja-JP", 10}, {"ka-GE", 67},
    {"km-KH", 47}, {"kn-IN", 43}, {"ko", 14}, {"ko-KO", 14}, {"ko-KR", 14}, {"ku-TR", 65},
    {"ky-KG", 71}, {"ln-CD", 58}, {"lt", 31}, {"lt-LT", 31}, {"lv", 61}, {"lv-LV", 61},
    {"mi-NZ", 96}, {"ml-IN", 44}, {"mr-IN", 41}, {"ms-MY", 35}, {"mt-MT", 102},
    {"nah-MX", 83}, {"nb", 103}, {"nb-NO", 103}, {"ne-NP", 46}, {"nl", 16}, {"nl-NL", 16},
    {"nn", 104}, {"nn-NO", 104}, {"no", 27}, {"no-NO", 27}, {"ny-MW", 57}, {"or-KE", 59},
    {"pl", 17}, {"pl-PL", 17}, {"pt", 13}, {"pt-BR", 12}, {"pt-PT", 13}, {"qu-PE", 80},
    {"ro", 20}, {"ro-RO", 20}, {"ru", 11}, {"ru-RU", 11}, {"rw-RW", 55}, {"si-LK", 45},
    {"sk", 28}, {"sk-SK", 28}, {"sl", 62}, {"sl-SI", 62}, {"sm-WS", 98}, {"so-SO", 56},
    {"sv", 24}, {"sv-SE", 24}, {"sw-KE", 48}, {"ta-IN", 39}, {"te-IN", 40}, {"tg-TJ", 70},
    {"th-TH", 32}, {"to-TO", 99}, {"tr", 18}, {"tr-TR", 18}, {"uk", 19}, {"uk-UA", 19},
    {"ur-PK", 37}, {"uz-UZ", 69}, {"vi-VN", 33}, {"yo-NG", 52}, {"zh-CN", 4}, {"zh-TW", 5},
    {"zh-ZH", 4}, {"zu-ZA", 51},
};

int prompt_id(const std::string& code) {
  for (const PromptCode& p : kPrompts)
    if (code == p.code) return p.id;
  nemotron_cuda::throw_invalid("unsupported language prompt: " + code);
}

// A C string for the ABI: interior NUL bytes become U+FFFD (lib.rs:760-762).
std::string safe(const std::string& s) {
  if (s.find('\0') == std::string::npos) return s;
  std::string out;
  for (char c : s) {
    if (c == '\0') out += "\xEF\xBF\xBD";
    else out.push_back(c);
  }
  return out;
}

std::string& global_error() {
  thread_local std::string message;
  return message;
}
void set_global_error(const std::string& m) { global_error() = safe(m); }

bool valid_utf8(const char* s) {
  const unsigned char* p = reinterpret_cast<const unsigned char*>(s);
  while (*p) {
    int n = 0;
    unsigned cp = 0;
    if (*p < 0x80) { ++p; continue; }
    if ((*p & 0xE0) == 0xC0) { n = 1; cp = *p & 0x1F; }
    else if ((*p & 0xF0) == 0xE0) { n = 2; cp = *p & 0x0F; }
    else if ((*p & 0xF8) == 0xF0) { n = 3; cp = *p & 0x07; }
    else return false;
    ++p;
    for (int i = 0; i < n; ++i, ++p) {
      if ((*p & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (*p & 0x3F);
    }
    if ((n == 1 && cp < 0x80) || (n == 2 && cp < 0x800) || (n == 3 && (cp < 0x10000 || cp > 0x10FFFF)) ||
        (cp >= 0xD800 && cp < 0xE000))
      return false;
  }
  return true;
}

std::string required_string(const char* p, const char* name) {
  if (p == nullptr) nemotron_cuda::throw_invalid(std::string(name) + " is null");
  if (!valid_utf8(p)) nemotron_cuda::throw_invalid(std::string(name) + " is not valid UTF-8");
  return std::string(p);
}

// An error with the catcher status it maps to.
struct CatcherError {
  catcher_status_t status;
  std::string message;
};

}  // namespace

struct catcher_handle {
  std::unique_ptr<StreamingTranscriber> transcriber;
  std::unique_ptr<Tokenizer> tokenizer;
  std::vector<TimedToken> timed;
  std::string text, text_before, last_error;
  enum State { kIdle, kStarted, kFinished } state = kIdle;
};

namespace {

catcher_handle_t* create_handle(const char* asr_model_path, const char* language, uint32_t lookahead,
                                const cq_encoder_config* ecfg, const cq_rnnt_config* rcfg,
                                cq_dtype dtype, int device, const char* diar_model_path) {
  try {
    const std::string path = required_string(asr_model_path, "asr_model_path");
    const std::string lang = required_string(language, "language");
    if (diar_model_path != nullptr) {
      required_string(diar_model_path, "diar_model_path");
      nemotron_cuda::throw_invalid(
          "speaker diarization is not part of this library; pass a NULL diar_model_path for "
          "ASR-only transcription");
    }
    // host-side checks, then the device
    auto art = std::make_unique<Artifact>(path);
    const int la = lookahead > static_cast<uint32_t>(INT_MAX) ? -1 : static_cast<int>(lookahead);
    if (la < 0)
      nemotron_cuda::throw_invalid("unsupported lookahead " + std::to_string(lookahead) +
                                   "; supported values are [3, 0, 6, 13]");
    nemotron_cuda::check_lookahead(la);
    const int pid = prompt_id(lang);
    cq_encoder_config e{};
    cq_rnnt_config r{};
    if (ecfg != nullptr && rcfg != nullptr) {
      e = *ecfg;
      r = *rcfg;
    } else {
      nemotron_cuda::nemotron_configs(*art, &e, &r);
    }
    auto h = std::make_unique<catcher_handle>();
    h->tokenizer = std::make_unique<Tokenizer>(path + "/tokenizer.json", 0u,
                                               static_cast<uint32_t>(r.blank));
    h->transcriber = std::make_unique<StreamingTranscriber>(*art, e, r, dtype, la, pid, device);
    return h.release();
  } catch (const std::exception& ex) {
    set_global_error(ex.what());
  } catch (...) {
    set_global_error("unknown error in catcher_create");
  }
  return nullptr;
}

template <class F>
catcher_status_t with_handle(catcher_handle_t* h, F&& op) {
  if (h == nullptr) {
    set_global_error("catcher handle is null");
    return CATCHER_INVALID_ARGUMENT;
  }
  try {
    return op(*h);
  } catch (const CatcherError& e) {
    h->last_error = safe(e.message);
    return e.status;
  } catch (const std::exception& e) {
    h->last_error = safe(e.what());
    return CATCHER_RUNTIME_ERROR;
  } catch (...) {
    h->last_error = "unknown error";
    return CATCHER_RUNTIME_ERROR;
  }
}

std::string decode_ids(const catcher_handle_t& h, const std::vector<TimedToken>& tokens,
                       uint64_t cutoff_ms, bool all) {
  std::vector<uint32_t> ids;
  ids.reserve(tokens.size());
  for (const TimedToken& t : tokens) {
    // frame * 80 ms, saturating (lib.rs:606-611)
    const uint64_t start_ms = t.frame > UINT64_MAX / kFrameMs ? UINT64_MAX : t.frame * kFrameMs;
    if (all || start_ms < cutoff_ms) ids.push_back(t.id);
  }
  return h.tokenizer->decode(ids.data(), ids.size(), true);
}

// Runs a transcriber call; its failures are runtime errors (lib.rs:382-385).
template <class F>
std::vector<TimedToken> transcribe(F&& f) {
  try {
    return f();
  } catch (const std::exception& e) {
    throw CatcherError{CATCHER_RUNTIME_ERROR, e.what()};
  }
}

void rebuild_text(catcher_handle_t& h) {
  try {
    h.text = safe(decode_ids(h, h.timed, 0, true));
  } catch (const std::exception& e) {
    throw CatcherError{CATCHER_RUNTIME_ERROR, e.what()};
  }
}

catcher_status_t finish_session(catcher_handle_t& h, bool cut, uint64_t cutoff_ms) {
  if (h.state != catcher_handle::kStarted)
    throw CatcherError{CATCHER_INVALID_STATE, "catcher session is not recording"};
  std::vector<TimedToken> tokens = transcribe([&] { return h.transcriber->finish(); });
  const bool fresh = !tokens.empty();
  h.timed.insert(h.timed.end(), tokens.begin(), tokens.end());
  if (cut) {
    std::vector<TimedToken> kept;
    for (const TimedToken& t : h.timed) {
      const uint64_t start_ms = t.frame > UINT64_MAX / kFrameMs ? UINT64_MAX : t.frame * kFrameMs;
      if (start_ms < cutoff_ms) kept.push_back(t);
    }
    h.timed.swap(kept);
  }
  h.state = catcher_handle::kFinished;
  rebuild_text(h);
  return fresh ? CATCHER_OK : CATCHER_NO_UPDATE;
}

}  // namespace

extern "C" {

catcher_handle_t* catcher_create(const char* asr_model_path, const char* diar_model_path,
                                 const char* language, uint32_t lookahead) {
  return create_handle(asr_model_path, language, lookahead, nullptr, nullptr, CQ_F16, 0,
                       diar_model_path);
}

catcher_handle_t* catcher_create_config(const char* asr_model_path, const char* language,
                                        uint32_t lookahead, const cq_encoder_config* encoder,
                                        const cq_rnnt_config* rnnt, cq_dtype dtype, int32_t device) {
  if (encoder == nullptr || rnnt == nullptr) {
    set_global_error("encoder and rnnt configurations must not be null");
    return nullptr;
  }
  return create_handle(asr_model_path, language, lookahead, encoder, rnnt, dtype, device, nullptr);
}

catcher_status_t catcher_start(catcher_handle_t* handle) {
  return with_handle(handle, [](catcher_handle_t& h) {
    try {
      h.transcriber->reset();
    } catch (const std::exception& e) {
      throw CatcherError{CATCHER_RUNTIME_ERROR, e.what()};
    }
    h.timed.clear();
    h.text.clear();
    h.text_before.clear();
    h.state = catcher_handle::kStarted;
    return static_cast<catcher_status_t>(CATCHER_OK);
  });
}

catcher_status_t catcher_push_audio(catcher_handle_t* handle, const float* samples, size_t count) {
  if (count > 0 && samples == nullptr) {
    set_global_error("samples is null while count is non-zero");
    return CATCHER_INVALID_ARGUMENT;
  }
  return with_handle(handle, [&](catcher_handle_t& h) {
    if (h.state != catcher_handle::kStarted)
      throw CatcherError{CATCHER_INVALID_STATE, "catcher session is not recording"};
    std::vector<TimedToken> tokens =
        transcribe([&] { return h.transcriber->push_samples(samples, count); });
    const bool fresh = !tokens.empty();
    if (fresh) {
      h.timed.insert(h.timed.end(), tokens.begin(), tokens.end());
      rebuild_text(h);
    }
    return static_cast<catcher_status_t>(fresh ? CATCHER_OK : CATCHER_NO_UPDATE);
  });
}

catcher_status_t catcher_finish(catcher_handle_t* handle) {
  return with_handle(handle, [](catcher_handle_t& h) { return finish_session(h, false, 0); });
}

catcher_status_t catcher_finish_before(catcher_handle_t* handle, uint64_t cutoff_ms) {
  return with_handle(handle, [&](catcher_handle_t& h) { return finish_session(h, true, cutoff_ms); });
}

const char* catcher_text(const catcher_handle_t* handle) {
  if (handle == nullptr) {
    set_global_error("catcher handle is null");
    return nullptr;
  }
  return handle->text.c_str();
}

const char* catcher_text_before(catcher_handle_t* handle, uint64_t cutoff_ms) {
  if (handle == nullptr) {
    set_global_error("catcher handle is null");
    return nullptr;
  }
  try {
    handle->text_before = safe(decode_ids(*handle, handle->timed, cutoff_ms, false));
    return handle->text_before.c_str();
  } catch (const std::exception& e) {
    handle->last_error = safe(e.what());
  } catch (...) {
    handle->last_error = "unknown error";
  }
  return nullptr;
}

const char* catcher_segments(const catcher_handle_t* handle) {
  if (handle == nullptr) {
    set_global_error("catcher handle is null");
    return nullptr;
  }
  return "[]";
}

const char* catcher_warning(const catcher_handle_t* handle) {
  if (handle == nullptr) set_global_error("catcher handle is null");
  return nullptr;
}

const char* catcher_last_error(const catcher_handle_t* handle) {
  if (handle == nullptr) return global_error().c_str();
  return handle->last_error.c_str();
}

void catcher_destroy(catcher_handle_t* handle) {
  try {
    delete handle;
  } catch (...) {
    set_global_error("error while releasing a catcher handle");
  }
}

// ------------------------------------------------------------------ cqstream.h

}  // extern "C"

struct cq_chunk_scheduler {
  std::unique_ptr<ChunkScheduler> impl;
  std::vector<AudioChunk> windows;
};

struct cq_tokenizer {
  std::unique_ptr<Tokenizer> impl;
  std::string text;
};

extern "C" {

using nemotron_cuda::guarded;
using nemotron_cuda::need_handle;

cq_status cq_chunk_scheduler_create(int32_t lookahead, cq_chunk_scheduler** out) {
  return guarded([&] {
    need_handle(out, "out");
    *out = nullptr;
    auto s = std::make_unique<cq_chunk_scheduler>();
    s->impl = std::make_unique<ChunkScheduler>(lookahead);
    *out = s.release();
  });
}

cq_status cq_chunk_scheduler_push(cq_chunk_scheduler* s, const float* samples, size_t count,
                                  int32_t* windows) {
  return guarded([&] {
    need_handle(s, "scheduler");
    s->windows = s->impl->push(samples, count);
    if (windows != nullptr) *windows = static_cast<int32_t>(s->windows.size());
  });
}

cq_status cq_chunk_scheduler_finish(cq_chunk_scheduler* s, int32_t* windows) {
  return guarded([&] {
    need_handle(s, "scheduler");
    s->windows.clear();
    AudioChunk c;
    if (s->impl->finish(&c)) s->windows.push_back(std::move(c));
    if (windows != nullptr) *windows = static_cast<int32_t>(s->windows.size());
  });
}

cq_status cq_chunk_scheduler_window(const cq_chunk_scheduler* s, int32_t index, float* samples,
                                    size_t capacity, size_t* count, int32_t* center,
                                    int32_t* mel_frames) {
  return guarded([&] {
    need_handle(s, "scheduler");
    if (index < 0 || static_cast<size_t>(index) >= s->windows.size())
      nemotron_cuda::throw_invalid("window " + std::to_string(index) + " of " +
                                   std::to_string(s->windows.size()));
    const AudioChunk& c = s->windows[static_cast<size_t>(index)];
    if (count != nullptr) *count = c.samples.size();
    if (samples != nullptr) {
      std::memcpy(samples, c.samples.data(), std::min(capacity, c.samples.size()) * sizeof(float));
      if (center != nullptr) *center = c.center ? 1 : 0;
      if (mel_frames != nullptr) *mel_frames = c.mel_frames;
    }
  });
}

cq_status cq_chunk_scheduler_reset(cq_chunk_scheduler* s) {
  return guarded([&] {
    need_handle(s, "scheduler");
    s->impl->reset();
    s->windows.clear();
  });
}

void cq_chunk_scheduler_destroy(cq_chunk_scheduler* s) { delete s; }

cq_status cq_tokenizer_from_json(const char* path, uint32_t pad_token_id, uint32_t blank_token_id,
                                 cq_tokenizer** out) {
  return guarded([&] {
    need_handle(path, "path");
    need_handle(out, "out");
    *out = nullptr;
    auto t = std::make_unique<cq_tokenizer>();
    t->impl = std::make_unique<Tokenizer>(path, pad_token_id, blank_token_id);
    *out = t.release();
  });
}

cq_status cq_tokenizer_decode(cq_tokenizer* t, const uint32_t* ids, size_t count,
                              int32_t strip_special, const char** text) {
  return guarded([&] {
    need_handle(t, "tokenizer");
    need_handle(text, "text");
    if (count > 0 && ids == nullptr) nemotron_cuda::throw_invalid("ids is null while count is non-zero");
    t->text = t->impl->decode(ids, count, strip_special != 0);
    *text = t->text.c_str();
  });
}

void cq_tokenizer_destroy(cq_tokenizer* t) { delete t; }

}  // extern "C"
