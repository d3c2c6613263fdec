// Reader of the reference's MLX release artifact (a directory holding
// manifest.json and weights.safetensors; crates/nemotron-mlx/src/weights/
// artifact.rs:156-240, manifest.rs) and the binding of its tensors into an
// Encoder or RnntDecoder by name.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "cqlinear.h"

namespace nemotron_cuda {

class Encoder;
class RnntDecoder;

// Manifest entry (ArtifactTensorInfo): runtime shape and storage policy.
struct ArtifactTensorInfo {
  std::vector<size_t> shape;
  enum class Storage { kInt8Affine, kF16, kF32, kI32 } storage = Storage::kF16;
  int group_size = 0;  // kInt8Affine only
};

// One array of weights.safetensors (memory-mapped, read-only).
struct SafetensorsArray {
  std::string dtype;  // "F16", "U32", "F32", ...
  std::vector<size_t> shape;
  const uint8_t* data = nullptr;
  size_t bytes = 0;
};

class Artifact {
 public:
  // Artifact::load: parses manifest.json and maps weights.safetensors.
  explicit Artifact(const std::string& dir);
  ~Artifact();
  Artifact(const Artifact&) = delete;
  Artifact& operator=(const Artifact&) = delete;

  const std::string& model_id() const { return model_id_; }
  int format_version() const { return format_version_; }
  const ArtifactTensorInfo* tensor_info(const std::string& name) const;
  const SafetensorsArray* array(const std::string& name) const;
  const std::map<std::string, ArtifactTensorInfo>& tensors() const { return tensors_; }

  // The "{name}.__qweight/__scales/__biases" triple of an Int8Affine tensor
  // (Artifact::quantized_arrays, artifact.rs:222-240); throws the reference's
  // errors for missing tensors/arrays and incompatible storage.
  struct Quantized {
    const SafetensorsArray *qweight, *scales, *biases;
    int group_size;
    std::vector<size_t> shape;
  };
  Quantized quantized(const std::string& name) const;
  // An F16 tensor widened to f32 (Artifact::f16_to_f32, artifact.rs:200-212).
  std::vector<float> f16_to_f32(const std::string& name) const;

 private:
  void index_safetensors(const std::string& path);  // parses the mapped header

  std::string model_id_;
  int format_version_ = 0;
  std::map<std::string, ArtifactTensorInfo> tensors_;
  std::map<std::string, SafetensorsArray> arrays_;
  void* map_ = nullptr;
  size_t map_bytes_ = 0;
};

// Host arrays of one quantized linear read from an artifact, with the F16
// scales, quantization biases and output bias converted to the element type T
// (QuantizedLinear::from_artifact, crates/nemotron-mlx/src/model/layers.rs:
// 222-256).  qweight points into the mapped file.
struct ArtifactLinear {
  const uint32_t* qweight = nullptr;
  std::vector<uint16_t> scales, biases, bias;  // bias empty: no output bias
  int out = 0, in = 0, group = 0;
};
ArtifactLinear artifact_linear(const Artifact& art, const std::string& weight_name,
                               const std::string* bias_name, cq_dtype dtype);

// StreamingEncoder::from_artifact / StreamingRnntDecoder::from_artifact:
// binds every tensor the model's configuration names.
void load_encoder_artifact(Encoder& enc, const Artifact& art);
void load_rnnt_artifact(RnntDecoder& dec, const Artifact& art);

}  // namespace nemotron_cuda
