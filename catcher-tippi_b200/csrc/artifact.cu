// MLX release artifact reader: manifest.json (serde_json of ArtifactManifest,
// crates/nemotron-mlx/src/weights/artifact.rs:91-103) and weights.safetensors
// (8-byte little-endian header length, JSON header of {dtype, shape,
// data_offsets} per array, then the data), memory-mapped.  Binds an Encoder or
// RnntDecoder tensor by tensor, as StreamingEncoder::from_artifact and
// StreamingRnntDecoder::from_artifact do.  Host code only.
#include "artifact.hpp"
#include "json.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <fstream>
#include <limits>
#include <sstream>

#include "encoder.hpp"
#include "qlinear.hpp"
#include "rnnt.hpp"

namespace nemotron_cuda {

namespace {



std::vector<size_t> shape_of(const Json* j, const std::string& what) {
  if (j == nullptr || j->kind != Json::kArr) throw_invalid("invalid " + what + ": missing shape");
  std::vector<size_t> s;
  for (const Json& d : j->arr) {
    if (d.kind != Json::kNum || d.num < 0) throw_invalid("invalid " + what + ": bad dimension");
    s.push_back(static_cast<size_t>(d.num));
  }
  return s;
}

size_t product(const std::vector<size_t>& s) {
  size_t p = 1;
  for (size_t d : s) p *= d;
  return p;
}

std::string storage_text(const ArtifactTensorInfo& t) {
  switch (t.storage) {
    case ArtifactTensorInfo::Storage::kInt8Affine:
      return "Int8Affine { group_size: " + std::to_string(t.group_size) + " }";
    case ArtifactTensorInfo::Storage::kF16: return "F16";
    case ArtifactTensorInfo::Storage::kF32: return "F32";
    default: return "I32";
  }
}

// IEEE half -> float and float -> bfloat16 (round to nearest even), host side.
float half_to_float(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  const int exp = (h >> 10) & 0x1F;
  const uint32_t man = h & 0x3FFu;
  float f;
  if (exp == 0) {
    f = std::ldexp(static_cast<float>(man), -24);
  } else if (exp == 31) {
    f = man ? std::numeric_limits<float>::quiet_NaN() : std::numeric_limits<float>::infinity();
  } else {
    f = std::ldexp(static_cast<float>(man | 0x400u), exp - 25);
  }
  uint32_t u;
  std::memcpy(&u, &f, 4);
  u |= sign;
  std::memcpy(&f, &u, 4);
  return f;
}

uint16_t float_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return static_cast<uint16_t>(((u >> 16) & 0x8000u) | 0x7FC0u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

// F16 artifact values in the model's element type T (bit patterns).
std::vector<uint16_t> to_t_bits(const SafetensorsArray& a, cq_dtype dtype) {
  const size_t n = a.bytes / 2;
  std::vector<uint16_t> out(n);
  const uint16_t* src = reinterpret_cast<const uint16_t*>(a.data);
  if (dtype == CQ_F16) {
    std::memcpy(out.data(), src, n * 2);
  } else {
    for (size_t i = 0; i < n; ++i) out[i] = float_to_bf16(half_to_float(src[i]));
  }
  return out;
}

std::string bias_name_of(const std::string& weight_name) {
  const std::string suffix = ".weight";
  if (weight_name.size() > suffix.size() &&
      weight_name.compare(weight_name.size() - suffix.size(), suffix.size(), suffix) == 0)
    return weight_name.substr(0, weight_name.size() - suffix.size()) + ".bias";
  return weight_name + ".bias";
}

std::string read_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw Error(CQ_INVALID_ARGUMENT, "cannot open " + path);
  std::ostringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

}  // namespace

// ------------------------------------------------------------------ Artifact

Artifact::Artifact(const std::string& dir) {
  // manifest.json
  const std::string text = read_file(dir + "/manifest.json");
  const Json m = JsonParser(text.data(), text.size(), "artifact manifest").parse();
  const Json* fv = m.get("format_version");
  const Json* id = m.get("model_id");
  const Json* ts = m.get("tensors");
  if (fv == nullptr || fv->kind != Json::kNum || ts == nullptr || ts->kind != Json::kObj)
    throw_invalid("invalid artifact manifest: expected format_version and tensors");
  format_version_ = static_cast<int>(fv->num);
  if (format_version_ != 1)
    throw_invalid("unsupported artifact format_version " + std::to_string(format_version_));
  model_id_ = (id != nullptr && id->kind == Json::kStr) ? id->str : "";
  for (const auto& kv : ts->obj) {
    ArtifactTensorInfo t;
    t.shape = shape_of(kv.second.get("shape"), "artifact manifest entry " + kv.first);
    const Json* st = kv.second.get("storage");
    if (st == nullptr) throw_invalid("invalid artifact manifest: " + kv.first + " has no storage");
    if (st->kind == Json::kStr) {
      if (st->str == "F16") t.storage = ArtifactTensorInfo::Storage::kF16;
      else if (st->str == "F32") t.storage = ArtifactTensorInfo::Storage::kF32;
      else if (st->str == "I32") t.storage = ArtifactTensorInfo::Storage::kI32;
      else throw_invalid("invalid artifact manifest: unknown storage " + st->str);
    } else if (const Json* q = st->get("Int8Affine")) {
      const Json* g = q->get("group_size");
      if (g == nullptr || g->kind != Json::kNum)
        throw_invalid("invalid artifact manifest: " + kv.first + " has no group_size");
      t.storage = ArtifactTensorInfo::Storage::kInt8Affine;
      t.group_size = static_cast<int>(g->num);
    } else {
      throw_invalid("invalid artifact manifest: unknown storage of " + kv.first);
    }
    tensors_[kv.first] = t;
  }

  // weights.safetensors, mapped
  const std::string path = dir + "/weights.safetensors";
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw Error(CQ_INVALID_ARGUMENT, "cannot open " + path);
  struct stat sb {};
  if (::fstat(fd, &sb) != 0 || sb.st_size < 8) {
    ::close(fd);
    throw_invalid("invalid safetensors file " + path);
  }
  map_bytes_ = static_cast<size_t>(sb.st_size);
  map_ = ::mmap(nullptr, map_bytes_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) {
    map_ = nullptr;
    throw Error(CQ_RUNTIME_ERROR, "cannot map " + path);
  }
  // a constructor that throws runs no destructor: unmap on every error below
  try {
    index_safetensors(path);
  } catch (...) {
    ::munmap(map_, map_bytes_);
    map_ = nullptr;
    arrays_.clear();
    throw;
  }
}

void Artifact::index_safetensors(const std::string& path) {
  const uint8_t* base = static_cast<const uint8_t*>(map_);
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | base[i];
  if (hlen > map_bytes_ - 8) throw_invalid("invalid safetensors header in " + path);
  const Json h = JsonParser(reinterpret_cast<const char*>(base + 8), hlen, "safetensors header").parse();
  const uint8_t* data = base + 8 + hlen;
  const size_t data_bytes = map_bytes_ - 8 - hlen;
  for (const auto& kv : h.obj) {
    if (kv.first == "__metadata__") continue;
    SafetensorsArray a;
    const Json* dt = kv.second.get("dtype");
    const Json* off = kv.second.get("data_offsets");
    if (dt == nullptr || dt->kind != Json::kStr || off == nullptr || off->kind != Json::kArr ||
        off->arr.size() != 2)
      throw_invalid("invalid safetensors entry " + kv.first);
    a.dtype = dt->str;
    a.shape = shape_of(kv.second.get("shape"), "safetensors entry " + kv.first);
    // offsets are JSON numbers (doubles): accept only non-negative integers
    // that a double represents exactly, before any conversion
    for (const Json& o : off->arr)
      if (o.kind != Json::kNum || !(o.num >= 0.0) || o.num > 9007199254740992.0 ||
          o.num != std::floor(o.num))
        throw_invalid("invalid safetensors entry " + kv.first + ": bad data_offsets");
    const size_t b0 = static_cast<size_t>(off->arr[0].num), b1 = static_cast<size_t>(off->arr[1].num);
    if (b1 < b0 || b1 > data_bytes) throw_invalid("safetensors entry " + kv.first + " lies outside the file");
    a.data = data + b0;
    a.bytes = b1 - b0;
    arrays_[kv.first] = a;
  }
}

Artifact::~Artifact() {
  if (map_ != nullptr) ::munmap(map_, map_bytes_);
}

const ArtifactTensorInfo* Artifact::tensor_info(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

const SafetensorsArray* Artifact::array(const std::string& name) const {
  auto it = arrays_.find(name);
  return it == arrays_.end() ? nullptr : &it->second;
}

Artifact::Quantized Artifact::quantized(const std::string& name) const {
  const ArtifactTensorInfo* t = tensor_info(name);
  if (t == nullptr) throw_invalid("missing artifact tensor " + name);
  if (t->storage != ArtifactTensorInfo::Storage::kInt8Affine)
    throw_invalid("tensor " + name + " has incompatible storage " + storage_text(*t));
  Quantized q{};
  const std::string parts[3] = {name + ".__qweight", name + ".__scales", name + ".__biases"};
  const SafetensorsArray* arr[3];
  for (int i = 0; i < 3; ++i) {
    arr[i] = array(parts[i]);
    if (arr[i] == nullptr) throw_invalid("missing artifact array " + parts[i]);
  }
  if (t->shape.size() != 2)
    throw_invalid("invalid model shape: linear artifact " + name + " must have rank 2");
  const size_t N = t->shape[0], K = t->shape[1], g = static_cast<size_t>(t->group_size);
  if (g == 0 || K % g != 0 || K % 4 != 0) throw_invalid("artifact tensor " + name + " has an invalid group size");
  if (arr[0]->dtype != "U32" || arr[0]->bytes != N * K)
    throw_invalid("artifact array " + parts[0] + " must be U32 [" + std::to_string(N) + ", " +
                  std::to_string(K / 4) + "]");
  for (int i = 1; i < 3; ++i)
    if (arr[i]->dtype != "F16" || arr[i]->bytes != N * (K / g) * 2)
      throw_invalid("artifact array " + parts[i] + " must be F16 [" + std::to_string(N) + ", " +
                    std::to_string(K / g) + "]");
  q.qweight = arr[0];
  q.scales = arr[1];
  q.biases = arr[2];
  q.group_size = t->group_size;
  q.shape = t->shape;
  return q;
}

std::vector<float> Artifact::f16_to_f32(const std::string& name) const {
  const ArtifactTensorInfo* t = tensor_info(name);
  if (t == nullptr) throw_invalid("missing artifact tensor " + name);
  if (t->storage != ArtifactTensorInfo::Storage::kF16)
    throw_invalid("tensor " + name + " has incompatible storage " + storage_text(*t));
  const SafetensorsArray* a = array(name);
  if (a == nullptr) throw_invalid("missing artifact array " + name);
  if (a->dtype != "F16" || a->bytes != product(t->shape) * 2)
    throw_invalid("artifact array " + name + " must be F16 with " + std::to_string(product(t->shape)) +
                  " values");
  std::vector<float> out(a->bytes / 2);
  const uint16_t* src = reinterpret_cast<const uint16_t*>(a->data);
  for (size_t i = 0; i < out.size(); ++i) out[i] = half_to_float(src[i]);
  return out;
}

// ------------------------------------------------------------------ binding

ArtifactLinear artifact_linear(const Artifact& art, const std::string& weight_name,
                               const std::string* bias_name, cq_dtype dtype) {
  if (dtype != CQ_F16 && dtype != CQ_BF16) throw_invalid("artifact linears load as f16 or bf16");
  const Artifact::Quantized q = art.quantized(weight_name);
  ArtifactLinear L;
  L.qweight = reinterpret_cast<const uint32_t*>(q.qweight->data);
  L.out = static_cast<int>(q.shape[0]);
  L.in = static_cast<int>(q.shape[1]);
  L.group = q.group_size;
  L.scales = to_t_bits(*q.scales, dtype);
  L.biases = to_t_bits(*q.biases, dtype);
  if (bias_name != nullptr) {
    // the F16 output bias must exist (Artifact::f16_array, artifact.rs:242-251)
    const std::vector<float> bf = art.f16_to_f32(*bias_name);
    if (bf.size() != static_cast<size_t>(L.out))
      throw_invalid("invalid model shape: linear bias " + *bias_name + " must have shape [" +
                    std::to_string(L.out) + "]");
    L.bias = to_t_bits(*art.array(*bias_name), dtype);
  }
  return L;
}


namespace {

template <class Model>
void bind_linear(Model& model, const Artifact& art, const std::string& name, int out, int in,
                 bool has_bias) {
  const std::string bn = bias_name_of(name);
  const ArtifactLinear L = artifact_linear(art, name, has_bias ? &bn : nullptr, model.dtype());
  if (L.out != out || L.in != in)
    throw_invalid("invalid model shape: artifact tensor " + name + " is " + std::to_string(L.out) + "x" +
                  std::to_string(L.in) + ", the model needs " + std::to_string(out) + "x" +
                  std::to_string(in));
  model.set_linear(name, L.qweight, L.scales.data(), L.biases.data(),
                   L.bias.empty() ? nullptr : L.bias.data(), out, in, L.group);
}

}  // namespace

void load_encoder_artifact(Encoder& enc, const Artifact& art) {
  for (const Encoder::Spec& s : enc.specs()) {
    if (s.kind == Encoder::Kind::kLinear) {
      bind_linear(enc, art, s.name, s.out, s.in, s.has_bias);
    } else {
      const std::vector<float> v = art.f16_to_f32(s.name);
      enc.set_tensor(s.name, v.data(), v.size());
    }
  }
}

void load_rnnt_artifact(RnntDecoder& dec, const Artifact& art) {
  for (const RnntDecoder::Spec& s : dec.specs()) {
    if (s.linear) {
      bind_linear(dec, art, s.name, s.out, s.in, s.has_bias);
    } else {
      const std::vector<float> v = art.f16_to_f32(s.name);
      dec.set_tensor(s.name, v.data(), v.size());
    }
  }
}

}  // namespace nemotron_cuda
