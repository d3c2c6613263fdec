// Batched RNNT greedy decoder: tensor binding, synthetic weights, prediction
// state and the launch sequence of one chunk (replayed as a CUDA graph).
// See rnnt.hpp.
#include "rnnt.hpp"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <sstream>

#include "common.cuh"
#include "encoder_ops.hpp"
#include "qops.hpp"
#include "rnnt_ops.hpp"

namespace nemotron_cuda {

namespace {

// A copy of a [4H, K] gate weight with rows interleaved: row 4j + q holds
// gate q of hidden unit j (source row q * H + j); same codes, scales, biases.
std::unique_ptr<QuantizedLinear> interleave_gates(const QuantizedLinear& L, int H, cq_dtype dtype,
                                                  int device) {
  const int N = L.output_dims(), K = L.input_dims(), g = L.group_size();
  const size_t gpr = static_cast<size_t>(K / g);
  std::vector<uint8_t> q(static_cast<size_t>(N) * K), qi(q.size());
  std::vector<uint16_t> sc(N * gpr), bi(N * gpr), sci(sc.size()), bii(bi.size());
  check_cuda(cudaMemcpy(q.data(), L.qweight(), q.size(), cudaMemcpyDeviceToHost), "read weights");
  check_cuda(cudaMemcpy(sc.data(), L.scales(), sc.size() * 2, cudaMemcpyDeviceToHost), "read scales");
  check_cuda(cudaMemcpy(bi.data(), L.biases(), bi.size() * 2, cudaMemcpyDeviceToHost), "read biases");
  for (int j = 0; j < H; ++j)
    for (int gq = 0; gq < 4; ++gq) {
      const size_t dst = static_cast<size_t>(4 * j + gq), src = static_cast<size_t>(gq * H + j);
      std::memcpy(&qi[dst * K], &q[src * K], K);
      std::memcpy(&sci[dst * gpr], &sc[src * gpr], gpr * 2);
      std::memcpy(&bii[dst * gpr], &bi[src * gpr], gpr * 2);
    }
  return QuantizedLinear::from_packed(reinterpret_cast<const uint32_t*>(qi.data()), sci.data(),
                                      bii.data(), nullptr, N, K, g, dtype, device);
}

}  // namespace

RnntDecoder::RnntDecoder(const cq_rnnt_config& cfg, cq_dtype dtype, int device)
    : cfg_(cfg), dtype_(dtype), device_(device) {
  if (dtype != CQ_F16 && dtype != CQ_BF16) throw_invalid("RNNT dtype must be f16 or bf16");
  const auto& c = cfg;
  if (c.enc_hidden <= 0 || c.pred_hidden <= 0 || c.joint_hidden <= 0 || c.vocab <= 1 ||
      c.lstm_layers <= 0 || c.max_symbols <= 0)
    throw_invalid("invalid model shape: RNNT dimensions must be positive");
  if (c.blank < 0 || c.blank >= c.vocab)
    throw_invalid("blank id " + std::to_string(c.blank) + " is outside the vocabulary");
  device_context(device);
  const int H = c.pred_hidden, J = c.joint_hidden;
  auto lin = [&](const std::string& n, int out, int in, bool bias) {
    specs_.push_back(Spec{n, true, out, in, bias, 0});
  };
  lin("encoder_projector.weight", J, c.enc_hidden, true);
  lin("decoder.embedding.weight", c.vocab, H, false);
  for (int l = 0; l < c.lstm_layers; ++l) {
    lin("decoder.lstm.weight_ih_l" + std::to_string(l), 4 * H, H, false);
    lin("decoder.lstm.weight_hh_l" + std::to_string(l), 4 * H, H, false);
  }
  lin("decoder.decoder_projector.weight", J, H, true);
  lin("joint.head.weight", c.vocab, J, true);
  for (int l = 0; l < c.lstm_layers; ++l)
    for (const char* k : {"ih", "hh"})
      specs_.push_back(Spec{"decoder.lstm.bias_" + std::string(k) + "_l" + std::to_string(l), false,
                            0, 0, false, static_cast<size_t>(4 * H)});
  for (size_t i = 0; i < specs_.size(); ++i) index_[specs_[i].name] = i;
}

const RnntDecoder::Spec& RnntDecoder::spec(const std::string& name, bool linear) const {
  auto it = index_.find(name);
  if (it == index_.end()) throw_invalid("unknown RNNT tensor \"" + name + "\"");
  const Spec& s = specs_[it->second];
  if (s.linear != linear)
    throw_invalid("RNNT tensor \"" + name + "\" is " +
                  (s.linear ? "quantized" : "an unquantised tensor"));
  return s;
}

void RnntDecoder::set_linear(const std::string& name, const uint32_t* q, const void* scales,
                             const void* biases, const void* bias, int out, int in, int group) {
  const Spec& s = spec(name, true);
  if (out != s.out || in != s.in) {
    std::ostringstream os;
    os << "invalid model shape: " << name << " must be " << s.out << "x" << s.in << ", got " << out
       << "x" << in;
    throw_invalid(os.str());
  }
  linears_[name] = QuantizedLinear::from_packed(q, scales, biases, bias, out, in, group, dtype_, device_);
  finalized_ = false;
}

void RnntDecoder::bind_dense_device(const Spec& s, const float* dvalues) {
  DeviceGuard guard(device_);
  // stored as f32 holding T values (the artifact's f16)
  DeviceBuffer tmp(s.len * 2), buf(s.len * 4);
  check_cuda(cq::launch_f32_to_t(dtype_, dvalues, s.len, tmp.get(), nullptr), "round tensor");
  check_cuda(cq::launch_t_to_f32(dtype_, tmp.get(), s.len, buf.as<float>(), nullptr), "widen tensor");
  check_cuda(cudaDeviceSynchronize(), "bind tensor");
  dense_[s.name] = std::move(buf);
  finalized_ = false;
}

void RnntDecoder::set_tensor(const std::string& name, const float* values, size_t len) {
  const Spec& s = spec(name, false);
  if (len != s.len)
    throw_invalid("invalid model shape: " + name + " has " + std::to_string(len) +
                  " values, expected " + std::to_string(s.len));
  if (values == nullptr) throw_invalid("tensor values must not be null");
  DeviceGuard guard(device_);
  DeviceBuffer tmp(len * 4);
  check_cuda(cudaMemcpy(tmp.get(), values, len * 4, cudaMemcpyDefault), "upload tensor");
  bind_dense_device(s, tmp.as<float>());
}

void RnntDecoder::get_tensor(const std::string& name, float* values, size_t len) const {
  const Spec& s = spec(name, false);
  if (len != s.len) throw_invalid(name + " has " + std::to_string(s.len) + " values, not " + std::to_string(len));
  auto it = dense_.find(name);
  if (it == dense_.end()) throw_invalid("RNNT tensor \"" + name + "\" is not bound");
  DeviceGuard guard(device_);
  check_cuda(cudaMemcpy(values, it->second.get(), len * 4, cudaMemcpyDeviceToHost), "read tensor");
}

QuantizedLinear* RnntDecoder::linear(const std::string& name) const {
  auto it = linears_.find(name);
  return it == linears_.end() ? nullptr : it->second.get();
}

QuantizedLinear* RnntDecoder::ih(int l) const {
  return linear("decoder.lstm.weight_ih_l" + std::to_string(l));
}

QuantizedLinear* RnntDecoder::hh(int l) const {
  return linear("decoder.lstm.weight_hh_l" + std::to_string(l));
}

void RnntDecoder::init_random(uint64_t seed) {
  DeviceGuard guard(device_);
  size_t max_w = 0, max_n = 0;
  for (const Spec& s : specs_) {
    if (s.linear) {
      max_w = std::max(max_w, static_cast<size_t>(s.out) * s.in);
      max_n = std::max(max_n, static_cast<size_t>(s.out));
    } else {
      max_n = std::max(max_n, s.len);
    }
  }
  const int g = cfg_.group_size;
  DeviceBuffer w(max_w * 4), q(max_w), sc(max_w / 32 * 2 + 256), bi(max_w / 32 * 2 + 256);
  DeviceBuffer v32(max_n * 4), v16(max_n * 2);
  for (size_t i = 0; i < specs_.size(); ++i) {
    const Spec& s = specs_[i];
    const uint64_t sub = seed * 1000003ull + 7919 + i;
    if (s.linear) {
      const size_t n = static_cast<size_t>(s.out) * s.in;
      const float std = s.name == "decoder.embedding.weight" ? 1.0f : 0.02f;
      check_cuda(cq::launch_fill_normal(w.as<float>(), n, sub, 0.0f, std, nullptr), "fill");
      check_cuda(cq::launch_quantize(dtype_, w.as<float>(), s.out, s.in, g, true, q.as<uint8_t>(),
                                     sc.get(), bi.get(), nullptr),
                 "quantize");
      const void* bias = nullptr;
      if (s.has_bias) {
        check_cuda(cq::launch_fill_normal(v32.as<float>(), s.out, sub ^ 0x5bd1e995ull, 0.0f, 0.02f,
                                          nullptr),
                   "fill bias");
        check_cuda(cq::launch_f32_to_t(dtype_, v32.as<float>(), s.out, v16.get(), nullptr), "round bias");
        bias = v16.get();
      }
      check_cuda(cudaDeviceSynchronize(), "synthetic linear");
      set_linear(s.name, reinterpret_cast<const uint32_t*>(q.get()), sc.get(), bi.get(), bias, s.out,
                 s.in, g);
    } else {
      check_cuda(cq::launch_fill_normal(v32.as<float>(), s.len, sub, 0.0f, 0.02f, nullptr), "fill");
      bind_dense_device(s, v32.as<float>());
    }
  }
  check_cuda(cudaDeviceSynchronize(), "synthetic weights");
}

void RnntDecoder::finalize() {
  if (finalized_) return;
  for (const Spec& s : specs_) {
    const bool bound = s.linear ? linears_.count(s.name) != 0 : dense_.count(s.name) != 0;
    if (!bound) throw_invalid("RNNT tensor \"" + s.name + "\" is not bound");
  }
  DeviceGuard guard(device_);
  const int V = cfg_.vocab, H = cfg_.pred_hidden;
  // QuantizedEmbedding: dequantised once, lookups read T rows
  const QuantizedLinear* E = linear("decoder.embedding.weight");
  DeviceBuffer w32(static_cast<size_t>(V) * H * 4);
  embedding_ = DeviceBuffer(static_cast<size_t>(V) * H * 2);
  check_cuda(cq::launch_dequantize(dtype_, static_cast<const uint8_t*>(E->qweight()), E->scales(),
                                   E->biases(), V, H, E->group_size(), w32.as<float>(), nullptr),
             "dequantize embedding");
  check_cuda(cq::launch_f32_to_t(dtype_, w32.as<float>(), static_cast<size_t>(V) * H, embedding_.get(),
                                 nullptr),
             "round embedding");
  // LstmCell::from_artifact: bias = bias_ih + bias_hh, added in T
  lstm_bias_.clear();
  std::vector<float> bih(4 * H), bhh(4 * H), sum(4 * H);
  for (int l = 0; l < cfg_.lstm_layers; ++l) {
    get_tensor("decoder.lstm.bias_ih_l" + std::to_string(l), bih.data(), bih.size());
    get_tensor("decoder.lstm.bias_hh_l" + std::to_string(l), bhh.data(), bhh.size());
    for (int i = 0; i < 4 * H; ++i) sum[i] = bih[i] + bhh[i];  // both exact T values
    DeviceBuffer f32(sum.size() * 4), t(sum.size() * 2);
    check_cuda(cudaMemcpy(f32.get(), sum.data(), sum.size() * 4, cudaMemcpyHostToDevice), "upload bias");
    check_cuda(cq::launch_f32_to_t(dtype_, f32.as<float>(), sum.size(), t.get(), nullptr), "round bias");
    check_cuda(cudaDeviceSynchronize(), "lstm bias");
    lstm_bias_.push_back(std::move(t));
  }
  // gate-interleaved LSTM weights for the one-launch step (rnnt_lstm.cu)
  ih_il_.clear();
  hh_il_.clear();
  gate_bias_il_.clear();
  const int g = ih(0)->group_size();
  bool fits = cq::lstm_step_fits(H, g) && fused_lstm_;
  for (int l = 0; l < cfg_.lstm_layers && fits; ++l)
    fits = ih(l)->group_size() == g && hh(l)->group_size() == g && ih(l)->input_dims() == H;
  if (fits) {
    for (int l = 0; l < cfg_.lstm_layers; ++l) {
      ih_il_.push_back(interleave_gates(*ih(l), H, dtype_, device_));
      hh_il_.push_back(interleave_gates(*hh(l), H, dtype_, device_));
      std::vector<uint16_t> b(4 * H), bi(4 * H);
      check_cuda(cudaMemcpy(b.data(), lstm_bias_[l].get(), b.size() * 2, cudaMemcpyDeviceToHost),
                 "read gate bias");
      for (int j = 0; j < H; ++j)
        for (int q = 0; q < 4; ++q) bi[4 * j + q] = b[q * H + j];
      DeviceBuffer t(bi.size() * 2);
      check_cuda(cudaMemcpy(t.get(), bi.data(), bi.size() * 2, cudaMemcpyHostToDevice), "gate bias");
      gate_bias_il_.push_back(std::move(t));
    }
    lstm_m5_.clear();
    if ((4 * H) % 80 == 0)
      for (int l = 0; l < cfg_.lstm_layers; ++l)
        for (const auto* w : {ih_il_[l].get(), hh_il_[l].get()})
          lstm_m5_.push_back(make_map_2d(w->qweight(), 1, 4 * H, H, H, 80, 64, CU_TENSOR_MAP_SWIZZLE_NONE));
    // layer 0's ih product of every embedding row, by the step kernel's own
    // arithmetic (the W_hh half of the launch multiplies the same rows and is
    // discarded)
    ih0_table_ = DeviceBuffer(static_cast<size_t>(V) * 4 * H * 2);
    cq::LstmMaps maps;
    maps.m[0] = ih_il_[0]->gemv_map(4);
    maps.m[1] = hh_il_[0]->gemv_map(4);
    maps.has_m5 = 0;
    cq::LstmStepArgs a{};
    a.x = embedding_.get();
    a.h_prev = embedding_.get();
    a.scales_ih = ih_il_[0]->scales();
    a.biases_ih = ih_il_[0]->biases();
    a.scales_hh = hh_il_[0]->scales();
    a.biases_hh = hh_il_[0]->biases();
    a.gate_bias = gate_bias_il_[0].get();
    a.all = 1;
    a.status = device_context(device_).status;
    a.S = V;
    a.H = H;
    a.gi_out = ih0_table_.get();
    const int dt = dtype_ == CQ_BF16 ? cq::kBF16 : cq::kF16;
    check_cuda(cq::launch_lstm_step(dt, g, maps, a, nullptr, false), "layer-0 ih table");
  }
  check_cuda(cudaDeviceSynchronize(), "finalize RNNT");
  finalized_ = true;
}

// ------------------------------------------------------------------ RnntState

RnntState::RnntState(RnntDecoder& dec, int streams, int max_frames)
    : dec_(dec), S_(streams), max_frames_(max_frames) {
  if (streams <= 0 || max_frames <= 0) throw_invalid("RNNT state needs streams and frames");
  dec_.finalize();
  const auto& c = dec_.config();
  DeviceGuard guard(dec_.device());
  const size_t S = S_, H = c.pred_hidden, J = c.joint_hidden, V = c.vocab;
  ep_ = DeviceBuffer(S * max_frames * J * 2);
  dec_out_ = DeviceBuffer(S * J * 2);
  dec_new_ = DeviceBuffer(S * J * 2);
  fused_ = DeviceBuffer(S * J * 2);
  logits_ = DeviceBuffer(S * V * 2);
  x_ = DeviceBuffer(S * H * 2);
  gi_ = DeviceBuffer(S * 4 * H * 2);
  gh_ = DeviceBuffer(static_cast<size_t>(c.lstm_layers) * S * 4 * H * 2);  // one slice per layer
  active_ = DeviceBuffer(S * sizeof(int));
  for (int l = 0; l < c.lstm_layers; ++l) {
    h_.emplace_back(S * H * 2);
    c_.emplace_back(S * H * 2);
  }
  hpar_.assign(c.lstm_layers, 0);
  lstm_fused_ = dec_.lstm_fused() && S_ < cq::kGemmMinRows;
  if (lstm_fused_)
    for (int l = 0; l < c.lstm_layers; ++l) h_next_.emplace_back(S * H * 2);
  fused_epi_ = lstm_fused_ && H % 8 == 0 && dec_.head()->rnnt_epilogue_fits(S_) &&
               dec_.dec_proj()->rnnt_epilogue_fits(S_);
  if (fused_epi_) {
    best_ = DeviceBuffer(S * sizeof(unsigned long long));
    done_ = DeviceBuffer(static_cast<size_t>((S_ + 15) / 16) * sizeof(unsigned));
    check_cuda(cudaMemset(best_.get(), 0, best_.bytes()), "greedy keys");
    check_cuda(cudaMemset(done_.get(), 0, done_.bytes()), "greedy counter");
    ih0_from_table_ = dec_.ih0_table() != nullptr;
    if (ih0_from_table_) last_token_ = DeviceBuffer(S * sizeof(int));
    defer_greedy_ = ih0_from_table_ && c.lstm_layers >= 2;
  }
  size_t need = dec_.enc_proj()->scratch_bytes_for(S_ * max_frames);
  for (const QuantizedLinear* L : {dec_.head(), dec_.dec_proj()}) need = std::max(need, L->scratch_bytes_for(S_));
  for (int l = 0; l < c.lstm_layers; ++l)
    need = std::max({need, dec_.ih(l)->scratch_bytes_for(S_), dec_.hh(l)->scratch_bytes_for(S_)});
  scratch_ = DeviceBuffer(std::max<size_t>(need, 256));

  // One persistent launch per chunk when the shapes fit its tiling (64-wide
  // sub-blocks, one group size >= 64 for all of its linears, <= 64 streams).
  const int g = dec_.head()->group_size();
  bool fits = S_ <= 64 && c.lstm_layers <= cq::kRnntMaxLayers &&
              H % 64 == 0 && J % 64 == 0 && g % 64 == 0 && dec_.dec_proj()->group_size() == g;
  for (int l = 0; l < c.lstm_layers && fits; ++l)
    fits = dec_.ih(l)->group_size() == g && dec_.hh(l)->group_size() == g;
  if (fits) {
    const int dt = dec_.dtype() == CQ_BF16 ? cq::kBF16 : cq::kF16;
    grid_ = cq::rnnt_chunk_grid(dt, S_, static_cast<int>(H), static_cast<int>(J), static_cast<int>(V),
                                c.lstm_layers, device_context(dec_.device()).num_sms);
  }
  if (grid_ > 0) {
    for (int l = 0; l < c.lstm_layers; ++l) h_alt_.emplace_back(S * H * 2);
    part_ = DeviceBuffer(static_cast<size_t>((V + 15) / 16) * S * sizeof(float2));
    barrier_ = DeviceBuffer(2 * sizeof(unsigned));
  }
  check_cuda(cudaStreamCreateWithFlags(&capture_stream_, cudaStreamNonBlocking), "capture stream");
  reset();
}

RnntState::~RnntState() {
  for (auto& g : graphs_) cudaGraphExecDestroy(g.exec);
  if (capture_stream_ != nullptr) cudaStreamDestroy(capture_stream_);
}

void RnntState::linear(QuantizedLinear* L, const void* x, int ldx, int rows, void* y, int ldy, int act,
                       cudaStream_t stream) {
  L->forward_array_in_scratch(x, ldx, rows, y, ldy, act, stream, scratch_.get(), scratch_.bytes());
}

// PredictionNetwork::step for the streams whose flag is set (or all): the
// LSTM stack on x, then the decoder projector into dec_new.
void RnntState::prediction_step(bool all, cudaStream_t st, const cq::RnntEpilogue* proj_epi) {
  const auto& c = dec_.config();
  const int dt = dec_.dtype() == CQ_BF16 ? cq::kBF16 : cq::kF16;
  const bool pdl = pdl_;
  PdlScope pdl_scope(pdl_);  // the linears follow the state's setting
  const int H = c.pred_hidden;
  if (lstm_fused_) {
    const void* in = x_.get();
    const int g = dec_.ih(0)->group_size();
    for (int l = 0; l < c.lstm_layers; ++l) {
      const QuantizedLinear* wi = dec_.ih_interleaved(l);
      const QuantizedLinear* wh = dec_.hh_interleaved(l);
      cq::LstmMaps maps;
      maps.m[0] = wi->gemv_map(4);
      maps.m[1] = wh->gemv_map(4);
      maps.has_m5 = dec_.has_lstm_m5() ? 1 : 0;
      if (maps.has_m5) {
        maps.m5[0] = dec_.lstm_m5(l, 0);
        maps.m5[1] = dec_.lstm_m5(l, 1);
      }
      cq::LstmStepArgs a{};
      a.x = in;
      a.h_prev = h_cur(l);
      a.h_out = h_other(l);
      a.c = c_[l].get();
      a.scales_ih = wi->scales();
      a.biases_ih = wi->biases();
      a.scales_hh = wh->scales();
      a.biases_hh = wh->biases();
      a.gate_bias = dec_.gate_bias_interleaved(l);
      a.active = active_.as<int>();
      a.all = all ? 1 : 0;
      a.status = device_context(dec_.device()).status;
      a.S = S_;
      a.H = H;
      if (l == 0 && ih0_from_table_) {
        a.gi_table = dec_.ih0_table();
        a.gi_token = last_token_.as<int>();
      }
      if (proj_epi != nullptr && proj_epi->defer) {
        // the greedy choice the head deferred (launch_chunk)
        if (l == 0) {
          a.greedy_best = proj_epi->best;
          a.greedy_active = proj_epi->active;
          a.greedy_blank = proj_epi->blank;
          a.tokens = proj_epi->tokens;
          a.token_frames = proj_epi->token_frames;
          a.counts = proj_epi->counts;
          a.cap = proj_epi->cap;
          a.frame = proj_epi->frame;
        } else if (l == 1) {
          a.clear_best = proj_epi->best;
        }
      }
      check_cuda(cq::launch_lstm_step(dt, g, maps, a, st, pdl), "lstm step");
      hpar_[l] ^= 1;
      in = h_cur(l);
    }
    if (proj_epi != nullptr)
      dec_.dec_proj()->forward_rnnt(in, H, S_, dec_new_.get(), c.joint_hidden, cq::kGemvJointInput,
                                    *proj_epi, st);
    else
      linear(dec_.dec_proj(), in, H, S_, dec_new_.get(), c.joint_hidden, CQ_ACT_NONE, st);
    return;
  }
  const void* in = x_.get();
  auto gh = [&](int l) { return static_cast<char*>(gh_.get()) + static_cast<size_t>(l) * S_ * 4 * H * 2; };
  // ih of layer 0 and hh of every layer read only what the previous step
  // left: one grouped launch; ih of the later layers waits for its cell.
  const bool grouped = S_ < cq::kGemmMinRows && c.lstm_layers + 1 <= cq::kGemvMaxGroup;
  if (grouped) {
    QuantizedLinear::GroupCall calls[cq::kGemvMaxGroup];
    calls[0] = {dec_.ih(0), in, H, gi_.get(), 4 * H};
    for (int l = 0; l < c.lstm_layers; ++l) calls[l + 1] = {dec_.hh(l), h_[l].get(), H, gh(l), 4 * H};
    QuantizedLinear::forward_group(calls, c.lstm_layers + 1, S_, CQ_ACT_NONE, st);
  }
  for (int l = 0; l < c.lstm_layers; ++l) {
    if (!grouped || l > 0) linear(dec_.ih(l), in, H, S_, gi_.get(), 4 * H, CQ_ACT_NONE, st);
    if (!grouped) linear(dec_.hh(l), h_[l].get(), H, S_, gh(l), 4 * H, CQ_ACT_NONE, st);
    check_cuda(cq::launch_lstm_cell(dt, gi_.get(), gh(l), dec_.lstm_bias(l), h_[l].get(), c_[l].get(),
                                    active_.as<int>(), S_, H, all, st, pdl),
               "lstm cell");
    in = h_[l].get();
  }
  linear(dec_.dec_proj(), in, H, S_, dec_new_.get(), c.joint_hidden, CQ_ACT_NONE, st);
}

void RnntState::normalize_h(cudaStream_t stream) {
  const size_t bytes = static_cast<size_t>(S_) * dec_.config().pred_hidden * 2;
  for (size_t l = 0; l < hpar_.size(); ++l) {
    if (!hpar_[l]) continue;
    check_cuda(cudaMemcpyAsync(h_[l].get(), h_next_[l].get(), bytes, cudaMemcpyDeviceToDevice, stream),
               "hidden state");
    hpar_[l] = 0;
  }
}

void RnntState::reset() {
  const auto& c = dec_.config();
  DeviceGuard guard(dec_.device());
  check_cuda(cudaDeviceSynchronize(), "reset");
  for (auto* v : {&h_, &c_})
    for (auto& b : *v) check_cuda(cudaMemset(b.get(), 0, b.bytes()), "zero LSTM state");
  // the first PredictionNetwork::step(blank) of every stream
  check_cuda(cq::launch_broadcast_row(dec_.embedding(), c.blank, c.pred_hidden, x_.get(), S_, nullptr),
             "blank embedding");
  if (ih0_from_table_) {
    const std::vector<int> blank(S_, c.blank);
    check_cuda(cudaMemcpy(last_token_.get(), blank.data(), blank.size() * sizeof(int), cudaMemcpyHostToDevice),
               "blank token");
  }
  std::fill(hpar_.begin(), hpar_.end(), 0);
  prediction_step(true, nullptr);
  normalize_h(nullptr);
  check_cuda(cudaMemcpy(dec_out_.get(), dec_new_.get(), dec_out_.bytes(), cudaMemcpyDeviceToDevice),
             "initial decoder output");
  check_cuda(cudaDeviceSynchronize(), "reset");
}

void RnntState::launch_chunk(const void* encoded, int ld, int frames, int* tokens, int* token_frames,
                             int* counts, cudaStream_t st) {
  const auto& c = dec_.config();
  const int dt = dec_.dtype() == CQ_BF16 ? cq::kBF16 : cq::kF16;
  const bool pdl = pdl_;
  PdlScope pdl_scope(pdl_);  // the linears follow the state's setting
  const int J = c.joint_hidden, V = c.vocab, H = c.pred_hidden;
  const int cap = capacity();
  if (use_persistent_) {
    // encoder projector over every frame of every stream, then the whole greedy
    // loop of the chunk in one cooperative launch (rnnt_persistent.cu)
    linear(dec_.enc_proj(), encoded, ld, S_ * frames, ep_.get(), J, CQ_ACT_NONE, st);
    check_cuda(cq::launch_zero_ints(barrier_.as<int>(), 2, st), "zero barrier");
    cq::RnntChunkArgs a{};
    const QuantizedLinear* head = dec_.head();
    const QuantizedLinear* proj = dec_.dec_proj();
    a.head_q = static_cast<const uint8_t*>(head->qweight());
    a.head_s = head->scales();
    a.head_b = head->biases();
    a.head_bias = head->bias();
    for (int l = 0; l < c.lstm_layers; ++l) {
      a.ih_q[l] = static_cast<const uint8_t*>(dec_.ih(l)->qweight());
      a.ih_s[l] = dec_.ih(l)->scales();
      a.ih_b[l] = dec_.ih(l)->biases();
      a.hh_q[l] = static_cast<const uint8_t*>(dec_.hh(l)->qweight());
      a.hh_s[l] = dec_.hh(l)->scales();
      a.hh_b[l] = dec_.hh(l)->biases();
      a.lstm_bias[l] = dec_.lstm_bias(l);
      a.h[l][0] = h_[l].get();
      a.h[l][1] = h_alt_[l].get();
      a.c[l] = c_[l].get();
    }
    a.proj_q = static_cast<const uint8_t*>(proj->qweight());
    a.proj_s = proj->scales();
    a.proj_b = proj->biases();
    a.proj_bias = proj->bias();
    a.emb = dec_.embedding();
    a.ep = ep_.get();
    a.dec = dec_out_.get();
    a.fused = fused_.get();
    a.part = part_.as<float2>();
    a.tokens = tokens;
    a.token_frames = token_frames;
    a.counts = counts;
    a.cap = cap;
    a.barrier = barrier_.as<unsigned>();
    a.status = device_context(dec_.device()).status;
    a.S = S_;
    a.Q = frames;
    a.H = H;
    a.J = J;
    a.V = V;
    a.blank = c.blank;
    a.max_symbols = c.max_symbols;
    a.layers = c.lstm_layers;
    a.group = head->group_size();
    check_cuda(cq::launch_rnnt_chunk(dt, a, grid_, st), "persistent RNNT chunk");
    return;
  }
  check_cuda(cq::launch_zero_ints(counts, S_, st), "zero counts");
  // encoder projector over every frame of every stream (row = stream * frames + frame)
  linear(dec_.enc_proj(), encoded, ld, S_ * frames, ep_.get(), J, CQ_ACT_NONE, st);
  for (int f = 0; f < frames; ++f) {
    const void* enc_f = static_cast<const char*>(ep_.get()) + static_cast<size_t>(f) * J * 2;
    check_cuda(cq::launch_joint_input(dt, enc_f, frames * J, nullptr, dec_out_.get(), fused_.get(),
                                      active_.as<int>(), S_, J, false, true, st, pdl),
               "joint input");
    for (int sym = 0; sym < c.max_symbols && fused_epi_; ++sym) {
      // head + greedy choice, then the prediction step whose projector
      // updates the joint input: four launches per symbol
      cq::RnntEpilogue e{};
      e.active = active_.as<int>();
      e.enc = enc_f;
      e.ld_enc = frames * J;
      e.dec = dec_out_.get();
      e.fused = fused_.get();
      e.best = best_.as<unsigned long long>();
      e.done = done_.as<unsigned>();
      e.blank = c.blank;
      e.emb = dec_.embedding();
      e.H = H;
      e.x = x_.get();
      e.last_token = ih0_from_table_ ? last_token_.as<int>() : nullptr;
      e.defer = defer_greedy_ ? 1 : 0;
      e.tokens = tokens;
      e.token_frames = token_frames;
      e.counts = counts;
      e.cap = cap;
      e.frame = f;
      dec_.head()->forward_rnnt(fused_.get(), J, S_, logits_.get(), V, cq::kGemvGreedy, e, st);
      prediction_step(false, st, &e);
    }
    for (int sym = 0; sym < c.max_symbols && !fused_epi_; ++sym) {
      linear(dec_.head(), fused_.get(), J, S_, logits_.get(), V, CQ_ACT_NONE, st);
      check_cuda(cq::launch_argmax_emit(dt, logits_.get(), V, V, c.blank, active_.as<int>(),
                                        dec_.embedding(), H, x_.get(), tokens, token_frames, counts, cap,
                                        f, S_, st, pdl),
                 "argmax");
      prediction_step(false, st);
      check_cuda(cq::launch_joint_input(dt, enc_f, frames * J, dec_new_.get(), dec_out_.get(),
                                        fused_.get(), active_.as<int>(), S_, J, true, false, st, pdl),
                 "joint input");
    }
  }
  normalize_h(st);  // the chunk ends with the state in h_, whatever its step count
}

void RnntState::set_pdl(bool on) {
  if (on == pdl_) return;
  DeviceGuard guard(dec_.device());
  check_cuda(cudaDeviceSynchronize(), "switch PDL");
  for (auto& g : graphs_) cudaGraphExecDestroy(g.exec);
  graphs_.clear();
  pdl_ = on;
}

void RnntState::set_persistent(bool on) {
  if (on && grid_ == 0)
    throw_invalid("the persistent RNNT kernel does not fit this state (at most 64 streams, hidden sizes "
                  "multiple of 64, one group size >= 64 for the head, LSTM and projector)");
  if (on == use_persistent_) return;
  DeviceGuard guard(dec_.device());
  check_cuda(cudaDeviceSynchronize(), "switch RNNT path");
  for (auto& g : graphs_) cudaGraphExecDestroy(g.exec);
  graphs_.clear();
  launches_ = 0;
  use_persistent_ = on;
}

void RnntState::decode_chunk(const void* encoded, int ld, int frames, int* tokens, int* token_frames,
                             int* counts, cudaStream_t stream) {
  const auto& c = dec_.config();
  if (encoded == nullptr || tokens == nullptr || token_frames == nullptr || counts == nullptr)
    throw_invalid("encoded, tokens, token_frames and counts must not be null");
  if (frames <= 0 || frames > max_frames_)
    throw_invalid("chunk of " + std::to_string(frames) + " frames; this state takes 1.." +
                  std::to_string(max_frames_));
  if (ld < c.enc_hidden) throw_invalid("encoder row stride is smaller than enc_hidden");
  DeviceGuard guard(dec_.device());
  cudaGraphExec_t exec = nullptr;
  for (auto& e : graphs_)
    if (e.encoded == encoded && e.ld == ld && e.frames == frames && e.tokens == tokens &&
        e.token_frames == token_frames && e.counts == counts)
      exec = e.exec;
  if (exec == nullptr) {
    cudaGraph_t graph = nullptr;
    check_cuda(cudaStreamBeginCapture(capture_stream_, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
      launch_chunk(encoded, ld, frames, tokens, token_frames, counts, capture_stream_);
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
    check_cuda(e, "instantiate decode graph");
    if (graphs_.size() >= 4) {
      cudaGraphExecDestroy(graphs_.front().exec);
      graphs_.erase(graphs_.begin());
    }
    graphs_.push_back({encoded, ld, frames, tokens, token_frames, counts, exec});
  }
  check_cuda(cudaGraphLaunch(exec, stream), "launch decode graph");
}

}  // namespace nemotron_cuda
