// Streaming FastConformer encoder: tensor binding by artifact name, synthetic
// weights, per-stream caches and the launch sequence of one chunk, replayed
// as a CUDA graph after the first chunk.  See encoder.hpp.
#include "encoder.hpp"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <sstream>

#include "common.cuh"
#include "encoder_ops.hpp"
#include "qops.hpp"

namespace nemotron_cuda {

namespace {

// Output length of the stride-2 kernel-3 convolution over `combined` frames
// (MLX conv2d without time padding).
int conv_out(int combined) { return combined < 3 ? 0 : (combined - 3) / 2 + 1; }

// Fp16Conv2d::streaming_output_length (layers.rs:38-45) for kernel 3, stride 2.
int streaming_len(int frames) { return frames + 1 < 3 ? 0 : (frames + 1 - 3) / 2 + 1; }

}  // namespace

// ------------------------------------------------------------------ DeviceBuffer

DeviceBuffer::DeviceBuffer(size_t bytes) : n_(bytes) {
  if (bytes > 0) check_cuda(cudaMalloc(&p_, bytes), "cudaMalloc(encoder buffer)");
}

DeviceBuffer::~DeviceBuffer() {
  if (p_ != nullptr) cudaFree(p_);
}

DeviceBuffer::DeviceBuffer(DeviceBuffer&& o) noexcept : p_(o.p_), n_(o.n_) {
  o.p_ = nullptr;
  o.n_ = 0;
}

DeviceBuffer& DeviceBuffer::operator=(DeviceBuffer&& o) noexcept {
  if (this != &o) {
    if (p_ != nullptr) cudaFree(p_);
    p_ = o.p_;
    n_ = o.n_;
    o.p_ = nullptr;
    o.n_ = 0;
  }
  return *this;
}

// ------------------------------------------------------------------ Encoder

Encoder::Encoder(const cq_encoder_config& cfg, cq_dtype dtype, int device)
    : cfg_(cfg), dtype_(dtype), device_(device) {
  if (dtype != CQ_F16 && dtype != CQ_BF16) throw_invalid("encoder dtype must be f16 or bf16");
  const auto& c = cfg;
  if (c.hidden <= 0 || c.heads <= 0 || c.hidden % c.heads != 0)
    throw_invalid("invalid model shape: relative attention dimensions are inconsistent");
  const int hd = c.hidden / c.heads;
  if (hd > 128 || c.hidden % 8 != 0 || c.hidden > 4096)
    throw_invalid("encoder hidden size must be a multiple of 8 up to 4096 with heads of at most 128");
  if (c.ff <= 0 || c.layers <= 0 || c.conv_kernel < 2 || c.sliding_window < 2)
    throw_invalid("invalid model shape: streaming encoder needs layers and at least one cached frame");
  if (c.mel_bins <= 0 || c.sub_channels <= 0 || c.sub_channels % 8 != 0 || c.num_prompts < 0 ||
      c.prompt_hidden <= 0)
    throw_invalid("invalid subsampling or prompt dimensions");
  // the Conv2D kernels keep a thread on one group of 8 channels
  if (!cq::conv2d_channels_ok(c.sub_channels))
    throw_invalid("subsampling channels must be 8 times a power of two up to 2048");
  device_context(device);
  DeviceGuard guard(device);

  const int d = c.hidden, ch = c.sub_channels;
  int f = c.mel_bins;
  for (int i = 0; i < 3; ++i) f = f / 2 + 1;  // (f + 2 + 1 - 3) / 2 + 1
  auto lin = [&](const std::string& n, int out, int in, bool bias) {
    Spec s;
    s.name = n;
    s.kind = Kind::kLinear;
    s.out = out;
    s.in = in;
    s.has_bias = bias;
    s.init = Init::kLinear;
    specs_.push_back(s);
  };
  auto dense = [&](const std::string& n, size_t len, Init init, bool f32 = false) {
    Spec s;
    s.name = n;
    s.kind = Kind::kDense;
    s.len = len;
    s.init = init;
    s.f32_storage = f32;
    specs_.push_back(s);
  };
  // linears (weight_manifest order: subsampling, layers, prompt)
  lin("encoder.subsampling.layers.0.pointwise_conv.weight", ch, ch, true);
  lin("encoder.subsampling.layers.1.pointwise_conv.weight", ch, ch, true);
  lin("encoder.subsampling.linear.weight", d, ch * f, true);
  for (int i = 0; i < c.layers; ++i) {
    const std::string p = "encoder.layers." + std::to_string(i);
    lin(p + ".feed_forward1.linear1.weight", c.ff, d, false);
    lin(p + ".feed_forward1.linear2.weight", d, c.ff, false);
    for (const char* proj : {"q_proj", "k_proj", "v_proj", "o_proj", "relative_k_proj"})
      lin(p + ".self_attn." + proj + ".weight", d, d, false);
    lin(p + ".conv.pointwise_conv1.weight", 2 * d, d, false);
    lin(p + ".conv.pointwise_conv2.weight", d, d, false);
    lin(p + ".feed_forward2.linear1.weight", c.ff, d, false);
    lin(p + ".feed_forward2.linear2.weight", d, c.ff, false);
  }
  lin("prompt_projector.linear_1.weight", c.prompt_hidden, d + c.num_prompts, true);
  lin("prompt_projector.linear_2.weight", d, c.prompt_hidden, true);
  // unquantised tensors
  dense("encoder.subsampling.conv_in.weight", static_cast<size_t>(ch) * 9, Init::kKernel);
  dense("encoder.subsampling.conv_in.bias", ch, Init::kSmall);
  for (int s = 0; s < 2; ++s) {
    const std::string p = "encoder.subsampling.layers." + std::to_string(s);
    dense(p + ".depthwise_conv.weight", static_cast<size_t>(ch) * 9, Init::kKernel);
    dense(p + ".depthwise_conv.bias", ch, Init::kSmall);
  }
  for (int i = 0; i < c.layers; ++i) {
    const std::string p = "encoder.layers." + std::to_string(i);
    dense(p + ".conv.depthwise_conv.weight", static_cast<size_t>(d) * c.conv_kernel, Init::kKernel);
    for (const char* n : {"conv.norm", "norm_feed_forward1", "norm_self_att", "norm_conv",
                          "norm_feed_forward2", "norm_out"}) {
      dense(p + "." + n + ".weight", d, Init::kNormWeight);
      dense(p + "." + n + ".bias", d, Init::kSmall);
    }
    dense(p + ".self_attn.bias_u", d, Init::kSmall, true);
    dense(p + ".self_attn.bias_v", d, Init::kSmall, true);
  }
  for (size_t i = 0; i < specs_.size(); ++i) index_[specs_[i].name] = i;
  // the checkpoint's depthwise convolutions carry no bias (encoder.rs:357-361)
  zero_dw_bias_ = DeviceBuffer(static_cast<size_t>(d) * 2);
  check_cuda(cudaMemset(zero_dw_bias_.get(), 0, zero_dw_bias_.bytes()), "zero depthwise bias");
}

const Encoder::Spec& Encoder::spec(const std::string& name, Kind kind) const {
  auto it = index_.find(name);
  if (it == index_.end()) throw_invalid("unknown encoder tensor \"" + name + "\"");
  const Spec& s = specs_[it->second];
  if (s.kind != kind)
    throw_invalid("encoder tensor \"" + name + "\" is " +
                  (s.kind == Kind::kLinear ? "a quantized linear" : "an unquantised tensor"));
  return s;
}

void Encoder::set_linear(const std::string& name, const uint32_t* q, const void* scales,
                         const void* biases, const void* bias, int out, int in, int group) {
  const Spec& s = spec(name, Kind::kLinear);
  if (out != s.out || in != s.in) {
    std::ostringstream os;
    os << "invalid model shape: " << name << " must be " << s.out << "x" << s.in << ", got " << out
       << "x" << in;
    throw_invalid(os.str());
  }
  linears_[name] = QuantizedLinear::from_packed(q, scales, biases, bias, out, in, group, dtype_,
                                                device_);
  finalized_ = false;
}

void Encoder::bind_dense_device(const Spec& s, const float* dvalues) {
  DeviceGuard guard(device_);
  const size_t es = s.f32_storage ? 4 : 2;
  DeviceBuffer buf(s.len * es);
  if (s.f32_storage) {
    // f32 storage of T values: round through T (the artifact holds f16)
    DeviceBuffer tmp(s.len * 2);
    check_cuda(cq::launch_f32_to_t(dtype_, dvalues, s.len, tmp.get(), nullptr), "round tensor");
    check_cuda(cq::launch_t_to_f32(dtype_, tmp.get(), s.len, buf.as<float>(), nullptr),
               "widen tensor");
    check_cuda(cudaDeviceSynchronize(), "bind tensor");
  } else {
    check_cuda(cq::launch_f32_to_t(dtype_, dvalues, s.len, buf.get(), nullptr), "round tensor");
    check_cuda(cudaDeviceSynchronize(), "bind tensor");
  }
  dense_[s.name] = std::move(buf);
  finalized_ = false;
}

void Encoder::set_tensor(const std::string& name, const float* values, size_t len) {
  const Spec& s = spec(name, Kind::kDense);
  if (len != s.len)
    throw_invalid("invalid model shape: " + name + " has " + std::to_string(len) +
                  " values, expected " + std::to_string(s.len));
  if (values == nullptr) throw_invalid("tensor values must not be null");
  DeviceGuard guard(device_);
  DeviceBuffer tmp(len * 4);
  check_cuda(cudaMemcpy(tmp.get(), values, len * 4, cudaMemcpyDefault), "upload tensor");
  bind_dense_device(s, tmp.as<float>());
}

void Encoder::get_tensor(const std::string& name, float* values, size_t len) const {
  const Spec& s = spec(name, Kind::kDense);
  if (len != s.len)
    throw_invalid(name + " has " + std::to_string(s.len) + " values, not " + std::to_string(len));
  auto it = dense_.find(name);
  if (it == dense_.end()) throw_invalid("encoder tensor \"" + name + "\" is not bound");
  DeviceGuard guard(device_);
  if (s.f32_storage) {
    check_cuda(cudaMemcpy(values, it->second.get(), len * 4, cudaMemcpyDeviceToHost), "read tensor");
    return;
  }
  DeviceBuffer tmp(len * 4);
  check_cuda(cq::launch_t_to_f32(dtype_, it->second.get(), len, tmp.as<float>(), nullptr),
             "widen tensor");
  check_cuda(cudaMemcpy(values, tmp.get(), len * 4, cudaMemcpyDeviceToHost), "read tensor");
}

QuantizedLinear* Encoder::linear(const std::string& name) const {
  auto it = linears_.find(name);
  return it == linears_.end() ? nullptr : it->second.get();
}

const void* Encoder::tensor(const std::string& name) const {
  auto it = dense_.find(name);
  if (it == dense_.end()) throw_invalid("encoder tensor \"" + name + "\" is not bound");
  return it->second.get();
}

void Encoder::init_random(uint64_t seed) {
  DeviceGuard guard(device_);
  size_t max_w = 0, max_d = 0;
  for (const Spec& s : specs_) {
    if (s.kind == Kind::kLinear) max_w = std::max(max_w, static_cast<size_t>(s.out) * s.in);
    else max_d = std::max(max_d, s.len);
  }
  DeviceBuffer w(max_w * 4), q(max_w), sc(max_w / 32 * 2 + 256), bi(max_w / 32 * 2 + 256);
  DeviceBuffer bias32(std::max<size_t>(max_d, 65536) * 4), bias16(std::max<size_t>(max_d, 65536) * 2);
  const int g = cfg_.group_size;
  for (size_t i = 0; i < specs_.size(); ++i) {
    const Spec& s = specs_[i];
    const uint64_t sub = seed * 1000003ull + i;
    if (s.kind == Kind::kLinear) {
      const size_t n = static_cast<size_t>(s.out) * s.in;
      check_cuda(cq::launch_fill_normal(w.as<float>(), n, sub, 0.0f, 0.02f, nullptr), "fill");
      check_cuda(cq::launch_quantize(dtype_, w.as<float>(), s.out, s.in, g, true, q.as<uint8_t>(),
                                     sc.get(), bi.get(), nullptr),
                 "quantize");
      const void* bias = nullptr;
      if (s.has_bias) {
        check_cuda(cq::launch_fill_normal(bias32.as<float>(), s.out, sub ^ 0x5bd1e995ull, 0.0f,
                                          0.02f, nullptr),
                   "fill bias");
        check_cuda(cq::launch_f32_to_t(dtype_, bias32.as<float>(), s.out, bias16.get(), nullptr),
                   "round bias");
        bias = bias16.get();
      }
      check_cuda(cudaDeviceSynchronize(), "synthetic linear");
      set_linear(s.name, reinterpret_cast<const uint32_t*>(q.get()), sc.get(), bi.get(), bias,
                 s.out, s.in, g);
    } else {
      float mean = 0.0f, std = 0.02f;
      if (s.init == Init::kNormWeight) {
        mean = 1.0f;
        std = 0.1f;
      } else if (s.init == Init::kKernel) {
        std = 1.0f / 3.0f;
      }
      check_cuda(cq::launch_fill_normal(bias32.as<float>(), s.len, sub, mean, std, nullptr), "fill");
      bind_dense_device(s, bias32.as<float>());
    }
  }
  check_cuda(cudaDeviceSynchronize(), "synthetic weights");
}

void Encoder::finalize() {
  if (finalized_) return;
  for (const Spec& s : specs_) {
    const bool bound = s.kind == Kind::kLinear ? linears_.count(s.name) != 0 : dense_.count(s.name) != 0;
    if (!bound) throw_invalid("encoder tensor \"" + s.name + "\" is not bound");
  }
  DeviceGuard guard(device_);
  fused_qkv_.clear();
  blocks_.clear();
  dw_wt_.clear();
  const int D = cfg_.hidden, K = cfg_.conv_kernel;
  std::vector<float> w(static_cast<size_t>(D) * K), wt(w.size());
  for (int i = 0; i < cfg_.layers; ++i) {
    const std::string p = "encoder.layers." + std::to_string(i);
    // one N = 3 * hidden projection: output columns are independent, so the
    // fused weight gives the q, k and v results bit for bit
    fused_qkv_.push_back(QuantizedLinear::concat({linear(p + ".self_attn.q_proj.weight"),
                                                  linear(p + ".self_attn.k_proj.weight"),
                                                  linear(p + ".self_attn.v_proj.weight")}));
    Block b{};
    b.ff1a = linear(p + ".feed_forward1.linear1.weight");
    b.ff1b = linear(p + ".feed_forward1.linear2.weight");
    b.qkv = fused_qkv_.back().get();
    b.o = linear(p + ".self_attn.o_proj.weight");
    b.pos = linear(p + ".self_attn.relative_k_proj.weight");
    b.pw1 = linear(p + ".conv.pointwise_conv1.weight");
    b.pw2 = linear(p + ".conv.pointwise_conv2.weight");
    b.ff2a = linear(p + ".feed_forward2.linear1.weight");
    b.ff2b = linear(p + ".feed_forward2.linear2.weight");
    b.norm_ff1_w = tensor(p + ".norm_feed_forward1.weight");
    b.norm_ff1_b = tensor(p + ".norm_feed_forward1.bias");
    b.norm_att_w = tensor(p + ".norm_self_att.weight");
    b.norm_att_b = tensor(p + ".norm_self_att.bias");
    b.norm_conv_w = tensor(p + ".norm_conv.weight");
    b.norm_conv_b = tensor(p + ".norm_conv.bias");
    b.norm_ff2_w = tensor(p + ".norm_feed_forward2.weight");
    b.norm_ff2_b = tensor(p + ".norm_feed_forward2.bias");
    b.norm_out_w = tensor(p + ".norm_out.weight");
    b.norm_out_b = tensor(p + ".norm_out.bias");
    b.conv_norm_w = tensor(p + ".conv.norm.weight");
    b.conv_norm_b = tensor(p + ".conv.norm.bias");
    // [D, 1, K] -> [K][D]: the conv kernel reads eight channels of one tap per load
    get_tensor(p + ".conv.depthwise_conv.weight", w.data(), w.size());
    for (int c = 0; c < D; ++c)
      for (int k = 0; k < K; ++k) wt[static_cast<size_t>(k) * D + c] = w[static_cast<size_t>(c) * K + k];
    DeviceBuffer f32(wt.size() * 4), tbuf(wt.size() * 2);
    check_cuda(cudaMemcpy(f32.get(), wt.data(), wt.size() * 4, cudaMemcpyHostToDevice), "upload kernel");
    check_cuda(cq::launch_f32_to_t(dtype_, f32.as<float>(), wt.size(), tbuf.get(), nullptr), "round kernel");
    check_cuda(cudaDeviceSynchronize(), "transpose depthwise kernel");
    dw_wt_.push_back(std::move(tbuf));
    b.dw_wt = dw_wt_.back().get();
    b.dw_b = zero_dw_bias_.get();
    b.bias_u = static_cast<const float*>(tensor(p + ".self_attn.bias_u"));
    b.bias_v = static_cast<const float*>(tensor(p + ".self_attn.bias_v"));
    blocks_.push_back(b);
  }
  finalized_ = true;
}

// ------------------------------------------------------------------ EncoderState

EncoderState::Geometry EncoderState::geometry(int mel_frames, bool first) const {
  const auto& c = enc_.config();
  const int extra = first ? 1 : 0;  // CausalConv2dCache initial extra frame (cache.rs:94-104)
  Geometry g{};
  g.time = mel_frames;
  g.F1 = c.mel_bins / 2 + 1;
  g.F2 = g.F1 / 2 + 1;
  g.F3 = g.F2 / 2 + 1;
  g.T1 = conv_out(mel_frames + 1 + extra);
  g.T2 = conv_out(g.T1 + 1 + extra);
  g.T3 = conv_out(g.T2 + 1 + extra);
  g.valid1 = streaming_len(mel_frames);
  g.valid2 = streaming_len(g.valid1);
  g.valid3 = streaming_len(g.valid2);
  return g;
}

EncoderState::EncoderState(Encoder& enc, int streams, int max_mel_frames)
    : enc_(enc), S_(streams), max_mel_(max_mel_frames) {
  if (streams <= 0) throw_invalid("encoder state needs at least one stream");
  enc_.finalize();
  const auto& c = enc_.config();
  const Geometry gmax = geometry(max_mel_frames, true);
  if (gmax.T3 <= 0)
    throw_invalid("chunks of " + std::to_string(max_mel_frames) + " mel frames produce no encoder frame");
  qmax_ = std::max(gmax.T3, geometry(max_mel_frames, false).T3);
  const int cache_frames = c.sliding_window - 1;
  ring_ = cache_frames + qmax_;
  vmax_ = cache_frames + qmax_;
  pmax_ = vmax_ + qmax_ - 1;
  const size_t smem = cq::attention_smem_bytes(qmax_, vmax_, c.hidden / c.heads);
  if (smem > 227 * 1024)
    throw_invalid("attention window of " + std::to_string(vmax_) + " frames exceeds shared memory");

  DeviceGuard guard(enc_.device());
  num_sms_ = device_context(enc_.device()).num_sms;
  const size_t S = S_, D = c.hidden, C = c.sub_channels, L = c.layers, Q = qmax_;
  const size_t es = 2;
  hid_width_ = std::max<size_t>({static_cast<size_t>(c.ff), 2 * D, static_cast<size_t>(c.prompt_hidden)});
  counters_ = DeviceBuffer(cq::kNumCounters * sizeof(int));
  prompts_ = DeviceBuffer(S * sizeof(int));
  res_ = DeviceBuffer(S * Q * D * 4);
  xn_ = DeviceBuffer(S * Q * D * es);
  hid_ = DeviceBuffer(S * Q * hid_width_ * es);
  y_ = DeviceBuffer(S * Q * D * es);
  att_ = DeviceBuffer(S * Q * D * es);
  x16_ = DeviceBuffer(S * Q * D * 2);
  scale16_ = DeviceBuffer(S * Q * sizeof(float));
  qkv_ = DeviceBuffer(S * Q * 3 * D * es);
  pin_ = DeviceBuffer(S * Q * (D + c.num_prompts) * es);
  relk_ = DeviceBuffer(L * static_cast<size_t>(pmax_) * D * es);  // per layer, projected once
  pos_table_ = DeviceBuffer(static_cast<size_t>(pmax_) * D * es);
  kring_ = DeviceBuffer(L * S * ring_ * D * es);
  vring_ = DeviceBuffer(L * S * ring_ * D * es);
  conv_cache_ = DeviceBuffer(L * 2 * S * (c.conv_kernel - 1) * D * es);
  stem_out_ = DeviceBuffer(S * gmax.T1 * gmax.F1 * C * es);
  dw1_out_ = DeviceBuffer(S * gmax.T2 * gmax.F2 * C * es);
  pw1_out_ = DeviceBuffer(S * gmax.T2 * gmax.F2 * C * es);
  dw2_out_ = DeviceBuffer(S * gmax.T3 * gmax.F3 * C * es);
  pw2_out_ = DeviceBuffer(S * gmax.T3 * gmax.F3 * C * es);
  flat_ = DeviceBuffer(S * Q * C * gmax.F3 * es);
  sub_cache_[0] = DeviceBuffer(2 * S * c.mel_bins * es);
  sub_cache_[1] = DeviceBuffer(2 * S * gmax.F1 * C * es);
  sub_cache_[2] = DeviceBuffer(2 * S * gmax.F2 * C * es);

  // scratch for the batched bf16 GEMM's f16 staging, sized for the widest call
  size_t need = 0;
  const int rows_main = S_ * qmax_;
  auto want = [&](const QuantizedLinear* Lp, int rows) { need = std::max(need, Lp->scratch_bytes_for(rows)); };
  want(enc_.linear("encoder.subsampling.layers.0.pointwise_conv.weight"), S_ * gmax.T2 * gmax.F2);
  want(enc_.linear("encoder.subsampling.layers.1.pointwise_conv.weight"), S_ * gmax.T3 * gmax.F3);
  want(enc_.linear("encoder.subsampling.linear.weight"), rows_main);
  want(enc_.linear("prompt_projector.linear_1.weight"), rows_main);
  want(enc_.linear("prompt_projector.linear_2.weight"), rows_main);
  for (const auto& b : enc_.blocks()) {
    for (const QuantizedLinear* Lp : {b.ff1a, b.ff1b, b.qkv, b.o, b.pw1, b.pw2, b.ff2a, b.ff2b})
      want(Lp, rows_main);
    want(b.pos, pmax_);
  }
  scratch_ = DeviceBuffer(std::max<size_t>(need, 256));

  // relative_position_encoding (encoder.rs:864-884) for positions vmax-1 .. -(qmax-1),
  // in the reference's f32 arithmetic
  std::vector<float> table(static_cast<size_t>(pmax_) * D);
  for (int i = 0; i < pmax_; ++i) {
    const float pos = static_cast<float>(vmax_ - 1 - i);
    for (size_t k = 0; k < D / 2; ++k) {
      const float exponent = static_cast<float>(2 * k) / static_cast<float>(D);
      const float angle = pos / std::pow(10000.0f, exponent);
      table[i * D + 2 * k] = std::sin(angle);
      table[i * D + 2 * k + 1] = std::cos(angle);
    }
  }
  DeviceBuffer tmp(table.size() * 4);
  check_cuda(cudaMemcpy(tmp.get(), table.data(), table.size() * 4, cudaMemcpyHostToDevice),
             "upload positions");
  check_cuda(cq::launch_f32_to_t(enc_.dtype(), tmp.as<float>(), table.size(), pos_table_.get(), nullptr),
             "round positions");
  // relative_k_proj of the position table (encoder.rs:262-264): the table
  // depends only on the position values and the weights are fixed once a
  // state exists, so every layer's projection is made here, once, instead of
  // in every chunk (same kernel and inputs: the same bits)
  for (size_t l = 0; l < L; ++l)
    enc_.blocks()[l].pos->forward_array(pos_table_.get(), static_cast<int>(D), pmax_,
                                        static_cast<char*>(relk_.get()) + l * pmax_ * D * es,
                                        static_cast<int>(D), CQ_ACT_NONE, nullptr);
  check_cuda(cudaDeviceSynchronize(), "position projections");
  check_cuda(cudaStreamCreateWithFlags(&capture_stream_, cudaStreamNonBlocking), "capture stream");
  reset();
  std::vector<int> ids(S_, c.num_prompts > 101 ? 101 : 0);
  set_prompts(ids.data(), S_);
}

EncoderState::~EncoderState() {
  for (auto& g : graphs_) cudaGraphExecDestroy(g.exec);
  if (capture_stream_ != nullptr) cudaStreamDestroy(capture_stream_);
}

void EncoderState::set_pdl(bool on) {
  if (on == pdl_) return;
  DeviceGuard guard(enc_.device());
  check_cuda(cudaDeviceSynchronize(), "switch PDL");
  for (auto& g : graphs_) cudaGraphExecDestroy(g.exec);
  graphs_.clear();
  pdl_ = on;
}

void EncoderState::reset() {
  DeviceGuard guard(enc_.device());
  check_cuda(cudaDeviceSynchronize(), "reset");
  for (DeviceBuffer* b : {&counters_, &kring_, &vring_, &conv_cache_, &sub_cache_[0], &sub_cache_[1],
                          &sub_cache_[2]})
    check_cuda(cudaMemset(b->get(), 0, b->bytes()), "zero cache");
  check_cuda(cudaDeviceSynchronize(), "reset");
  chunks_ = 0;
}

void EncoderState::set_prompts(const int* ids, int count) {
  if (count != S_) throw_invalid("expected " + std::to_string(S_) + " prompt ids, got " + std::to_string(count));
  if (ids == nullptr) throw_invalid("prompt ids must not be null");
  const int np = enc_.config().num_prompts;
  for (int i = 0; i < count; ++i)
    if (ids[i] < 0 || ids[i] >= np)
      throw_invalid("invalid model shape: prompt " + std::to_string(ids[i]) + " is not below " +
                    std::to_string(np));
  DeviceGuard guard(enc_.device());
  check_cuda(cudaDeviceSynchronize(), "set prompts");
  check_cuda(cudaMemcpy(prompts_.get(), ids, count * sizeof(int), cudaMemcpyHostToDevice), "prompts");
}

int EncoderState::output_frames(int mel_frames) const {
  if (mel_frames <= 0 || mel_frames > max_mel_) return 0;
  return geometry(mel_frames, chunks_ == 0).T3;
}

void EncoderState::linear(QuantizedLinear* L, const void* x, int ldx, int rows, void* y, int ldy,
                          int act, cudaStream_t stream) {
  L->forward_array_in_scratch(x, ldx, rows, y, ldy, act, stream, scratch_.get(), scratch_.bytes());
}

void EncoderState::launch_chunk(const float* mel, const Geometry& g, void* out, cudaStream_t st) {
  const auto& c = enc_.config();
  const int dt = enc_.dtype() == CQ_BF16 ? cq::kBF16 : cq::kF16;
  const bool pdl = pdl_;
  PdlScope pdl_scope(pdl_);  // the linears follow the state's setting
  const int S = S_, D = c.hidden, C = c.sub_channels, Q = g.T3, rows = S * Q;
  const int P = c.num_prompts;
  int* ctr = counters_.as<int>();
  const size_t es = 2;

  // ---- Conv2dSubsampling::forward (encoder.rs:767-802)
  cq::Conv2dArgs a{};
  a.in = mel;
  a.Tin = g.time;
  a.Fin = c.mel_bins;
  a.valid_in = g.time;
  a.w = enc_.tensor("encoder.subsampling.conv_in.weight");
  a.b = enc_.tensor("encoder.subsampling.conv_in.bias");
  a.cache = sub_cache_[0].get();
  a.out = stem_out_.get();
  a.Tout = g.T1;
  a.Fout = g.F1;
  a.valid_out = g.valid1;
  a.counters = ctr;
  a.S = S;
  a.C = C;
  check_cuda(cq::launch_stem_conv(dt, a, st, pdl), "stem conv");

  const void* stage_in = stem_out_.get();
  int tin = g.T1, fin = g.F1, vin = g.T1;  // the stem already zeroed its invalid frames
  void* dw_out[2] = {dw1_out_.get(), dw2_out_.get()};
  void* pw_out[2] = {pw1_out_.get(), pw2_out_.get()};
  const int tout[2] = {g.T2, g.T3}, fout[2] = {g.F2, g.F3}, vout[2] = {g.valid2, g.valid3};
  for (int s = 0; s < 2; ++s) {
    const std::string p = "encoder.subsampling.layers." + std::to_string(s);
    cq::Conv2dArgs d{};
    d.in = stage_in;
    d.Tin = tin;
    d.Fin = fin;
    d.valid_in = vin;
    d.w = enc_.tensor(p + ".depthwise_conv.weight");
    d.b = enc_.tensor(p + ".depthwise_conv.bias");
    d.cache = sub_cache_[s + 1].get();
    d.out = dw_out[s];
    d.Tout = tout[s];
    d.Fout = fout[s];
    d.valid_out = tout[s];
    d.counters = ctr;
    d.S = S;
    d.C = C;
    check_cuda(cq::launch_depthwise_conv2d(dt, d, st, pdl), "depthwise conv2d");
    // pointwise linear with its bias; ReLU fused (masking is applied by the reader)
    linear(enc_.linear(p + ".pointwise_conv.weight"), dw_out[s], C, S * tout[s] * fout[s], pw_out[s], C,
           CQ_ACT_RELU, st);
    stage_in = pw_out[s];
    tin = tout[s];
    fin = fout[s];
    vin = vout[s];
  }
  check_cuda(cq::launch_flatten_cf(dt, pw2_out_.get(), flat_.get(), S, g.T3, g.F3, C, g.valid3, st, pdl),
             "flatten");
  linear(enc_.linear("encoder.subsampling.linear.weight"), flat_.get(), C * g.F3, rows, y_.get(), D,
         CQ_ACT_NONE, st);

  // ---- FastConformerLayer::forward x layers (encoder.rs:498-535)
  const auto& blocks = enc_.blocks();
  cq::LnArgs ln{};
  ln.res = res_.as<float>();
  ln.y = y_.get();
  ln.ldy = D;
  ln.rows = rows;
  ln.D = D;
  ln.eps = 1e-5f;
  ln.ldo = D;
  ln.out = xn_.get();
  ln.prompt_ids = prompts_.as<int>();
  ln.num_prompts = P;
  ln.rows_per_stream = Q;
  // LayerNorm / conv outputs that feed a tensor-core GEMM also leave its f16
  // activations, so those linears skip their prepass
  const bool prescale = enc_.dtype() == CQ_BF16 && blocks[0].ff1a->gemm_for(rows);
  void* x16 = prescale ? x16_.get() : nullptr;
  float* s16 = prescale ? scale16_.as<float>() : nullptr;
  auto block_linear = [&](QuantizedLinear* L, const void* x, int ldx, void* y, int ldy, int act) {
    if (prescale) L->forward_prescaled(x16, s16, rows, y, ldy, act, st);
    else linear(L, x, ldx, rows, y, ldy, act, st);
  };
  ln.out16 = x16;
  ln.scale16 = s16;
  // residual stream = subsampling output; first block's feed-forward norm
  ln.mode = 1;
  ln.scale = 1.0f;
  ln.w1 = blocks[0].norm_ff1_w;
  ln.b1 = blocks[0].norm_ff1_b;
  check_cuda(cq::launch_layernorm(dt, ln, st, pdl), "layernorm");

  const int cache_frames = c.sliding_window - 1;
  const int hd = D / c.heads;
  for (int l = 0; l < c.layers; ++l) {
    const auto& b = blocks[l];
    auto add_ln = [&](float scale, const void* w, const void* bias) {
      cq::LnArgs x = ln;
      x.mode = 0;
      x.scale = scale;
      x.w1 = w;
      x.b1 = bias;
      x.w2 = nullptr;
      x.b2 = nullptr;
      x.out_kind = 0;
      x.out = xn_.get();
      x.ldo = D;
      check_cuda(cq::launch_layernorm(dt, x, st, pdl), "layernorm");
    };
    // feed-forward 1 (half-step residual)
    block_linear(b.ff1a, xn_.get(), D, hid_.get(), c.ff, CQ_ACT_SILU);
    linear(b.ff1b, hid_.get(), c.ff, rows, y_.get(), D, CQ_ACT_NONE, st);
    add_ln(0.5f, b.norm_att_w, b.norm_att_b);
    // self-attention
    block_linear(b.qkv, xn_.get(), D, qkv_.get(), 3 * D, CQ_ACT_NONE);
    cq::AttnArgs at{};
    at.qkv = qkv_.get();
    at.ldqkv = 3 * D;
    at.relk = static_cast<const char*>(relk_.get()) + static_cast<size_t>(l) * pmax_ * D * es;
    at.bias_u = b.bias_u;
    at.bias_v = b.bias_v;
    at.kring = static_cast<char*>(kring_.get()) + static_cast<size_t>(l) * S * ring_ * D * es;
    at.vring = static_cast<char*>(vring_.get()) + static_cast<size_t>(l) * S * ring_ * D * es;
    at.out = att_.get();
    at.counters = ctr;
    at.S = S;
    at.Q = Q;
    at.D = D;
    at.heads = c.heads;
    at.head_dim = hd;
    at.ring = ring_;
    at.cache_frames = cache_frames;
    at.vmax = vmax_;
    at.qsplit = cq::attention_qsplit(S, c.heads, Q, num_sms_);
    at.scale = 1.0f / std::sqrt(static_cast<float>(hd));
    check_cuda(cq::launch_attention(dt, at, st, pdl), "attention");
    linear(b.o, att_.get(), D, rows, y_.get(), D, CQ_ACT_NONE, st);
    add_ln(1.0f, b.norm_conv_w, b.norm_conv_b);
    // convolution module
    block_linear(b.pw1, xn_.get(), D, hid_.get(), 2 * D, CQ_ACT_NONE);
    cq::ConvArgs cv{};
    cv.pw1 = hid_.get();
    cv.ldp = 2 * D;
    cv.dw_wt = b.dw_wt;
    cv.dw_b = b.dw_b;
    cv.ln_w = b.conv_norm_w;
    cv.ln_b = b.conv_norm_b;
    cv.cache = static_cast<char*>(conv_cache_.get()) +
               static_cast<size_t>(l) * 2 * S * (c.conv_kernel - 1) * D * es;
    cv.out = att_.get();
    cv.counters = ctr;
    cv.S = S;
    cv.Q = Q;
    cv.D = D;
    cv.K = c.conv_kernel;
    cv.eps = 1e-5f;
    cv.out16 = x16;
    cv.scale16 = s16;
    check_cuda(cq::launch_conv_module(dt, cv, st, pdl), "conv module");
    block_linear(b.pw2, att_.get(), D, y_.get(), D, CQ_ACT_NONE);
    add_ln(1.0f, b.norm_ff2_w, b.norm_ff2_b);
    // feed-forward 2 (half-step residual), then norm_out and the next block's first norm
    block_linear(b.ff2a, xn_.get(), D, hid_.get(), c.ff, CQ_ACT_SILU);
    linear(b.ff2b, hid_.get(), c.ff, rows, y_.get(), D, CQ_ACT_NONE, st);
    cq::LnArgs x = ln;
    x.mode = 0;
    x.scale = 0.5f;
    x.w1 = b.norm_out_w;
    x.b1 = b.norm_out_b;
    const bool last = l + 1 == c.layers;
    if (last) {
      x.w2 = nullptr;
      x.b2 = nullptr;
      x.out16 = nullptr;  // the projector's input is D + prompts wide: it keeps its prepass
      x.scale16 = nullptr;
      x.out_kind = 1;  // [block output | one-hot prompt] for the prompt projector
      x.out = pin_.get();
      x.ldo = D + P;
    } else {
      x.w2 = blocks[l + 1].norm_ff1_w;
      x.b2 = blocks[l + 1].norm_ff1_b;
      x.out_kind = 0;
      x.out = xn_.get();
      x.ldo = D;
    }
    check_cuda(cq::launch_layernorm(dt, x, st, pdl), "layernorm");
  }

  // ---- PromptProjector::forward_f32 (prompt.rs:110-140)
  linear(enc_.linear("prompt_projector.linear_1.weight"), pin_.get(), D + P, rows, hid_.get(),
         c.prompt_hidden, CQ_ACT_RELU, st);
  linear(enc_.linear("prompt_projector.linear_2.weight"), hid_.get(), c.prompt_hidden, rows, out, D,
         CQ_ACT_NONE, st);
  check_cuda(cq::launch_advance_counters(ctr, Q, st, pdl), "advance counters");
}

void EncoderState::encode_chunk(const float* mel, int mel_frames, void* out, cudaStream_t stream) {
  if (mel == nullptr || out == nullptr) throw_invalid("mel and out must not be null");
  if (mel_frames <= 0 || mel_frames > max_mel_)
    throw_invalid("chunk of " + std::to_string(mel_frames) + " mel frames; this state takes 1.." +
                  std::to_string(max_mel_));
  if ((reinterpret_cast<uintptr_t>(out) & 15) != 0) throw_invalid("out must be 16-byte aligned");
  const bool first = chunks_ == 0;
  const Geometry g = geometry(mel_frames, first);
  if (g.T3 <= 0)
    throw_invalid("chunk of " + std::to_string(mel_frames) + " mel frames produces no encoder frame");
  DeviceGuard guard(enc_.device());
  if (first) {
    launch_chunk(mel, g, out, stream);
  } else {
    cudaGraphExec_t exec = nullptr;
    for (auto& e : graphs_)
      if (e.mel_frames == mel_frames && e.mel == mel && e.out == out) exec = e.exec;
    if (exec == nullptr) {
      // capture the whole chunk once; kernels read the per-chunk counters from
      // device memory, so replays advance the streams correctly
      cudaGraph_t graph = nullptr;
      check_cuda(cudaStreamBeginCapture(capture_stream_, cudaStreamCaptureModeThreadLocal),
                 "begin capture");
      try {
        launch_chunk(mel, g, out, capture_stream_);
      } catch (...) {
        cudaStreamEndCapture(capture_stream_, &graph);
        if (graph != nullptr) cudaGraphDestroy(graph);
        throw;
      }
      check_cuda(cudaStreamEndCapture(capture_stream_, &graph), "end capture");
      size_t nodes = 0;
      if (cudaGraphGetNodes(graph, nullptr, &nodes) == cudaSuccess) launches_ = static_cast<int>(nodes);
      cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      check_cuda(e, "instantiate chunk graph");
      if (graphs_.size() >= 4) {
        cudaGraphExecDestroy(graphs_.front().exec);
        graphs_.erase(graphs_.begin());
      }
      graphs_.push_back({mel_frames, mel, out, exec});
    }
    check_cuda(cudaGraphLaunch(exec, stream), "launch chunk graph");
  }
  ++chunks_;
}

}  // namespace nemotron_cuda
