// extern "C" boundary of the artifact reader (include/cqartifact.h).
#include <cstring>
#include <memory>
#include <string>

#include "artifact.hpp"
#include "capi_guard.hpp"
#include "cqartifact.h"

namespace {

using nemotron_cuda::guarded;
using nemotron_cuda::need_handle;

const nemotron_cuda::ArtifactTensorInfo& info_of(const cq_artifact* art, const char* name) {
  need_handle(art, "artifact");
  need_handle(name, "name");
  const nemotron_cuda::ArtifactTensorInfo* t = art->impl->tensor_info(name);
  if (t == nullptr) nemotron_cuda::throw_invalid(std::string("missing artifact tensor ") + name);
  return *t;
}

}  // namespace

extern "C" {

cq_status cq_artifact_open(const char* dir, cq_artifact** out) {
  return guarded([&] {
    need_handle(dir, "dir");
    need_handle(out, "out");
    *out = nullptr;
    auto h = std::make_unique<cq_artifact>();
    h->impl = std::make_unique<nemotron_cuda::Artifact>(dir);
    for (const auto& kv : h->impl->tensors()) h->names.push_back(kv.first);
    *out = h.release();
  });
}

void cq_artifact_close(cq_artifact* art) { delete art; }

const char* cq_artifact_model_id(const cq_artifact* art) {
  return art == nullptr ? nullptr : art->impl->model_id().c_str();
}

int32_t cq_artifact_format_version(const cq_artifact* art) {
  return art == nullptr ? 0 : art->impl->format_version();
}

int32_t cq_artifact_tensor_count(const cq_artifact* art) {
  return art == nullptr ? 0 : static_cast<int32_t>(art->names.size());
}

const char* cq_artifact_tensor_name(const cq_artifact* art, int32_t index) {
  if (art == nullptr || index < 0 || index >= static_cast<int32_t>(art->names.size())) return nullptr;
  return art->names[index].c_str();
}

cq_status cq_artifact_tensor_info(const cq_artifact* art, const char* name, int32_t* rank,
                                  int64_t* shape, int32_t max_rank, int32_t* storage,
                                  int32_t* group_size) {
  return guarded([&] {
    const nemotron_cuda::ArtifactTensorInfo& t = info_of(art, name);
    if (rank != nullptr) *rank = static_cast<int32_t>(t.shape.size());
    if (shape != nullptr)
      for (int32_t i = 0; i < max_rank && i < static_cast<int32_t>(t.shape.size()); ++i)
        shape[i] = static_cast<int64_t>(t.shape[i]);
    using S = nemotron_cuda::ArtifactTensorInfo::Storage;
    if (storage != nullptr)
      *storage = t.storage == S::kInt8Affine ? CQ_STORAGE_INT8_AFFINE
                 : t.storage == S::kF16      ? CQ_STORAGE_F16
                 : t.storage == S::kF32      ? CQ_STORAGE_F32
                                             : CQ_STORAGE_I32;
    if (group_size != nullptr) *group_size = t.storage == S::kInt8Affine ? t.group_size : 0;
  });
}

cq_status cq_artifact_f16_to_f32(const cq_artifact* art, const char* name, float* values,
                                 size_t len) {
  return guarded([&] {
    need_handle(art, "artifact");
    need_handle(name, "name");
    need_handle(values, "values");
    const std::vector<float> v = art->impl->f16_to_f32(name);
    if (v.size() != len)
      nemotron_cuda::throw_invalid(std::string("tensor ") + name + " has " + std::to_string(v.size()) +
                                   " values, the buffer holds " + std::to_string(len));
    std::memcpy(values, v.data(), len * sizeof(float));
  });
}

cq_status cq_linear_from_artifact(const cq_artifact* art, const char* weight_name,
                                  const char* bias_name_or_null, cq_dtype dtype, int32_t device,
                                  cq_linear** out) {
  return guarded([&] {
    need_handle(art, "artifact");
    need_handle(weight_name, "weight name");
    need_handle(out, "out");
    *out = nullptr;
    const std::string bn = bias_name_or_null ? bias_name_or_null : "";
    const nemotron_cuda::ArtifactLinear L = nemotron_cuda::artifact_linear(
        *art->impl, weight_name, bias_name_or_null ? &bn : nullptr, dtype);
    auto h = std::make_unique<cq_linear>();
    h->owned = nemotron_cuda::QuantizedLinear::from_packed(
        L.qweight, L.scales.data(), L.biases.data(), L.bias.empty() ? nullptr : L.bias.data(), L.out,
        L.in, L.group, dtype, device);
    h->impl = h->owned.get();
    *out = h.release();
  });
}

}  // extern "C"
