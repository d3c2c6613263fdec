// extern "C" boundary of the batched RNNT decoder (include/cqrnnt.h).
#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>

#include "capi_guard.hpp"
#include "cqrnnt.h"
#include "rnnt.hpp"

struct cq_rnnt {
  std::unique_ptr<nemotron_cuda::RnntDecoder> impl;
  std::map<std::string, std::unique_ptr<cq_linear>> borrowed;
};

struct cq_rnnt_state {
  std::unique_ptr<nemotron_cuda::RnntState> impl;
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

void cq_rnnt_default_config(cq_rnnt_config* cfg) {
  if (cfg == nullptr) return;
  cfg->enc_hidden = 1024;
  cfg->pred_hidden = 640;
  cfg->joint_hidden = 640;
  cfg->vocab = 1025;
  cfg->blank = 1024;
  cfg->lstm_layers = 2;
  cfg->max_symbols = 10;
  cfg->group_size = 64;
}

cq_status cq_rnnt_create(const cq_rnnt_config* cfg, cq_dtype dtype, int32_t device, cq_rnnt** out) {
  return guarded([&] {
    need_handle(cfg, "config");
    need_handle(out, "out");
    *out = nullptr;
    auto h = std::make_unique<cq_rnnt>();
    h->impl = std::make_unique<nemotron_cuda::RnntDecoder>(*cfg, dtype, device);
    *out = h.release();
  });
}

cq_status cq_rnnt_set_linear(cq_rnnt* dec, const char* name, const uint32_t* qweight,
                             const void* scales, const void* biases, const void* bias_or_null,
                             int32_t output_dims, int32_t input_dims, int32_t group_size) {
  return guarded([&] {
    need_handle(dec, "decoder");
    const std::string n = name_of(name);
    dec->borrowed.erase(n);
    dec->impl->set_linear(n, qweight, scales, biases, bias_or_null, output_dims, input_dims, group_size);
  });
}

cq_status cq_rnnt_set_tensor(cq_rnnt* dec, const char* name, const float* values, size_t len) {
  return guarded([&] {
    need_handle(dec, "decoder");
    dec->impl->set_tensor(name_of(name), values, len);
  });
}

cq_status cq_rnnt_bind_artifact(cq_rnnt* dec, const cq_artifact* art) {
  return guarded([&] {
    need_handle(dec, "decoder");
    need_handle(art, "artifact");
    dec->borrowed.clear();
    nemotron_cuda::load_rnnt_artifact(*dec->impl, *art->impl);
  });
}

cq_status cq_rnnt_get_tensor(const cq_rnnt* dec, const char* name, float* values, size_t len) {
  return guarded([&] {
    need_handle(dec, "decoder");
    need_handle(values, "values");
    dec->impl->get_tensor(name_of(name), values, len);
  });
}

const cq_linear* cq_rnnt_linear(const cq_rnnt* dec, const char* name) {
  if (dec == nullptr || name == nullptr) return nullptr;
  nemotron_cuda::QuantizedLinear* L = dec->impl->linear(name);
  if (L == nullptr) return nullptr;
  auto& slot = const_cast<cq_rnnt*>(dec)->borrowed[name];
  if (!slot || slot->impl != L) {
    slot = std::make_unique<cq_linear>();
    slot->impl = L;
    slot->borrowed = true;
  }
  return slot.get();
}

cq_status cq_rnnt_init_random(cq_rnnt* dec, uint64_t seed) {
  return guarded([&] {
    need_handle(dec, "decoder");
    dec->borrowed.clear();
    dec->impl->init_random(seed);
  });
}

cq_status cq_rnnt_set_fused_lstm(cq_rnnt* dec, int32_t enable) {
  return guarded([&] {
    need_handle(dec, "decoder");
    dec->impl->set_fused_lstm(enable != 0);
  });
}

int32_t cq_rnnt_tensor_count(const cq_rnnt* dec) {
  return dec ? static_cast<int32_t>(dec->impl->specs().size()) : -1;
}

const char* cq_rnnt_tensor_name(const cq_rnnt* dec, int32_t index) {
  if (dec == nullptr || index < 0 || index >= static_cast<int32_t>(dec->impl->specs().size()))
    return nullptr;
  return dec->impl->specs()[index].name.c_str();
}

void cq_rnnt_destroy(cq_rnnt* dec) { delete dec; }

cq_status cq_rnnt_state_create(cq_rnnt* dec, int32_t streams, int32_t max_frames, cq_rnnt_state** out) {
  return guarded([&] {
    need_handle(dec, "decoder");
    need_handle(out, "out");
    *out = nullptr;
    auto h = std::make_unique<cq_rnnt_state>();
    h->impl = std::make_unique<nemotron_cuda::RnntState>(*dec->impl, streams, max_frames);
    *out = h.release();
  });
}

int32_t cq_rnnt_state_capacity(const cq_rnnt_state* st) { return st ? st->impl->capacity() : -1; }

cq_status cq_rnnt_decode_chunk(cq_rnnt_state* st, const void* encoded, int32_t ld, int32_t frames,
                               int32_t* tokens, int32_t* token_frames, int32_t* counts, void* stream) {
  return guarded([&] {
    need_handle(st, "state");
    st->impl->decode_chunk(encoded, ld, frames, tokens, token_frames, counts,
                           static_cast<cudaStream_t>(stream));
  });
}

cq_status cq_rnnt_state_set_persistent(cq_rnnt_state* st, int32_t enable) {
  return guarded([&] {
    need_handle(st, "state");
    st->impl->set_persistent(enable != 0);
  });
}

cq_status cq_rnnt_state_set_pdl(cq_rnnt_state* st, int32_t enable) {
  return guarded([&] {
    need_handle(st, "state");
    st->impl->set_pdl(enable != 0);
  });
}

int32_t cq_rnnt_state_kernels_per_chunk(const cq_rnnt_state* st) {
  return st ? st->impl->launches_per_chunk() : -1;
}

cq_status cq_rnnt_state_reset(cq_rnnt_state* st) {
  return guarded([&] {
    need_handle(st, "state");
    st->impl->reset();
  });
}

void cq_rnnt_state_destroy(cq_rnnt_state* st) { delete st; }

}  // extern "C"
