// extern "C" boundary of the streaming encoder (include/cqencoder.h).
#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>

#include "capi_guard.hpp"
#include "cqencoder.h"
#include "encoder.hpp"

struct cq_encoder {
  std::unique_ptr<nemotron_cuda::Encoder> impl;
  std::map<std::string, std::unique_ptr<cq_linear>> borrowed;  // cq_encoder_linear handles
};

struct cq_encoder_state {
  std::unique_ptr<nemotron_cuda::EncoderState> impl;
};

namespace {

using nemotron_cuda::guarded;
using nemotron_cuda::need_handle;

std::string name_of(const char* name) {
  need_handle(name, "name");
  return std::string(name);
}

}  // namespace

extern "C" {

void cq_encoder_default_config(cq_encoder_config* cfg) {
  if (cfg == nullptr) return;
  cfg->hidden = 1024;
  cfg->ff = 4096;
  cfg->layers = 24;
  cfg->heads = 8;
  cfg->conv_kernel = 9;
  cfg->sliding_window = 57;
  cfg->mel_bins = 128;
  cfg->sub_channels = 256;
  cfg->num_prompts = 128;
  cfg->prompt_hidden = 2048;
  cfg->group_size = 64;
}

cq_status cq_encoder_create(const cq_encoder_config* cfg, cq_dtype dtype, int32_t device,
                            cq_encoder** out) {
  return guarded([&] {
    need_handle(cfg, "config");
    need_handle(out, "out");
    *out = nullptr;
    auto h = std::make_unique<cq_encoder>();
    h->impl = std::make_unique<nemotron_cuda::Encoder>(*cfg, dtype, device);
    *out = h.release();
  });
}

cq_status cq_encoder_set_linear(cq_encoder* enc, const char* name, const uint32_t* qweight,
                                const void* scales, const void* biases, const void* bias_or_null,
                                int32_t output_dims, int32_t input_dims, int32_t group_size) {
  return guarded([&] {
    need_handle(enc, "encoder");
    const std::string n = name_of(name);
    enc->borrowed.erase(n);
    enc->impl->set_linear(n, qweight, scales, biases, bias_or_null, output_dims, input_dims,
                          group_size);
  });
}

cq_status cq_encoder_set_tensor(cq_encoder* enc, const char* name, const float* values, size_t len) {
  return guarded([&] {
    need_handle(enc, "encoder");
    enc->impl->set_tensor(name_of(name), values, len);
  });
}

cq_status cq_encoder_bind_artifact(cq_encoder* enc, const cq_artifact* art) {
  return guarded([&] {
    need_handle(enc, "encoder");
    need_handle(art, "artifact");
    enc->borrowed.clear();
    nemotron_cuda::load_encoder_artifact(*enc->impl, *art->impl);
  });
}

cq_status cq_encoder_get_tensor(const cq_encoder* enc, const char* name, float* values, size_t len) {
  return guarded([&] {
    need_handle(enc, "encoder");
    need_handle(values, "values");
    enc->impl->get_tensor(name_of(name), values, len);
  });
}

const cq_linear* cq_encoder_linear(const cq_encoder* enc, const char* name) {
  if (enc == nullptr || name == nullptr) return nullptr;
  nemotron_cuda::QuantizedLinear* L = enc->impl->linear(name);
  if (L == nullptr) return nullptr;
  auto& slot = const_cast<cq_encoder*>(enc)->borrowed[name];
  if (!slot || slot->impl != L) {
    slot = std::make_unique<cq_linear>();
    slot->impl = L;
    slot->borrowed = true;
  }
  return slot.get();
}

cq_status cq_encoder_init_random(cq_encoder* enc, uint64_t seed) {
  return guarded([&] {
    need_handle(enc, "encoder");
    enc->borrowed.clear();
    enc->impl->init_random(seed);
  });
}

int32_t cq_encoder_tensor_count(const cq_encoder* enc) {
  return enc ? static_cast<int32_t>(enc->impl->specs().size()) : -1;
}

const char* cq_encoder_tensor_name(const cq_encoder* enc, int32_t index) {
  if (enc == nullptr || index < 0 || index >= static_cast<int32_t>(enc->impl->specs().size()))
    return nullptr;
  return enc->impl->specs()[index].name.c_str();
}

void cq_encoder_destroy(cq_encoder* enc) { delete enc; }

cq_status cq_encoder_state_create(cq_encoder* enc, int32_t streams, int32_t max_mel_frames,
                                  cq_encoder_state** out) {
  return guarded([&] {
    need_handle(enc, "encoder");
    need_handle(out, "out");
    *out = nullptr;
    auto h = std::make_unique<cq_encoder_state>();
    h->impl = std::make_unique<nemotron_cuda::EncoderState>(*enc->impl, streams, max_mel_frames);
    *out = h.release();
  });
}

cq_status cq_encoder_state_set_prompts(cq_encoder_state* st, const int32_t* prompt_ids,
                                       int32_t count) {
  return guarded([&] {
    need_handle(st, "state");
    st->impl->set_prompts(prompt_ids, count);
  });
}

int32_t cq_encoder_state_output_frames(const cq_encoder_state* st, int32_t mel_frames) {
  return st ? st->impl->output_frames(mel_frames) : 0;
}

cq_status cq_encoder_encode_chunk(cq_encoder_state* st, const float* mel, int32_t mel_frames,
                                  void* out, void* stream) {
  return guarded([&] {
    need_handle(st, "state");
    st->impl->encode_chunk(mel, mel_frames, out, static_cast<cudaStream_t>(stream));
  });
}

int32_t cq_encoder_state_chunks(const cq_encoder_state* st) { return st ? st->impl->chunks() : -1; }

int32_t cq_encoder_state_kernels_per_chunk(const cq_encoder_state* st) {
  return st ? st->impl->launches_per_chunk() : -1;
}

cq_status cq_encoder_state_set_pdl(cq_encoder_state* st, int32_t enable) {
  return guarded([&] {
    need_handle(st, "state");
    st->impl->set_pdl(enable != 0);
  });
}

cq_status cq_encoder_state_reset(cq_encoder_state* st) {
  return guarded([&] {
    need_handle(st, "state");
    st->impl->reset();
  });
}

void cq_encoder_state_destroy(cq_encoder_state* st) { delete st; }

}  // extern "C"
