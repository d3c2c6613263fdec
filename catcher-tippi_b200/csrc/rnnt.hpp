// C++ host layer of the batched RNNT greedy decoder: the counterpart of the
// reference's StreamingRnntDecoder, PredictionNetwork, LstmCell,
// QuantizedEmbedding and JointNetwork (crates/nemotron-mlx/src/model/rnnt.rs).
// The C ABI in include/cqrnnt.h wraps these classes.
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "cqrnnt.h"
#include "device_buffer.hpp"
#include "qgemv.hpp"
#include "qlinear.hpp"

namespace nemotron_cuda {

class RnntDecoder {
 public:
  struct Spec {
    std::string name;
    bool linear;
    int out = 0, in = 0;
    bool has_bias = false;
    size_t len = 0;
  };

  RnntDecoder(const cq_rnnt_config& cfg, cq_dtype dtype, int device);

  const cq_rnnt_config& config() const { return cfg_; }
  cq_dtype dtype() const { return dtype_; }
  int device() const { return device_; }
  const std::vector<Spec>& specs() const { return specs_; }

  void set_linear(const std::string& name, const uint32_t* q, const void* scales,
                  const void* biases, const void* bias, int out, int in, int group);
  void set_tensor(const std::string& name, const float* values, size_t len);
  void get_tensor(const std::string& name, float* values, size_t len) const;
  QuantizedLinear* linear(const std::string& name) const;
  void init_random(uint64_t seed);

  // Checks every tensor is bound; dequantises the embedding and adds the LSTM
  // bias pairs.
  void finalize();
  // The one-launch LSTM step (default on where the shapes fit it); off, each
  // step runs the ih and hh products and the cell as separate launches.
  // Takes effect for states created afterwards.
  void set_fused_lstm(bool on) {
    fused_lstm_ = on;
    finalized_ = false;
  }
  QuantizedLinear* enc_proj() const { return linear("encoder_projector.weight"); }
  QuantizedLinear* dec_proj() const { return linear("decoder.decoder_projector.weight"); }
  QuantizedLinear* head() const { return linear("joint.head.weight"); }
  QuantizedLinear* ih(int l) const;
  QuantizedLinear* hh(int l) const;
  const void* embedding() const { return embedding_.get(); }  // T [vocab, pred_hidden]
  const void* lstm_bias(int l) const { return lstm_bias_[l].get(); }  // T [4 * pred_hidden]
  // Gate-interleaved copies (row 4j + q = gate q of hidden unit j) of the LSTM
  // weights and summed biases for the one-launch LSTM step; empty when the
  // shapes do not fit it.
  bool lstm_fused() const { return !ih_il_.empty(); }
  const QuantizedLinear* ih_interleaved(int l) const { return ih_il_[l].get(); }
  const QuantizedLinear* hh_interleaved(int l) const { return hh_il_[l].get(); }
  const void* gate_bias_interleaved(int l) const { return gate_bias_il_[l].get(); }
  // T(W_ih emb[v]) of layer 0 for every token v, gate-interleaved: T [vocab, 4 H]
  // (nullptr when the one-launch LSTM step is off)
  const void* ih0_table() const { return ih0_table_.get(); }
  // interleaved W_ih / W_hh of layer l with 80-row TMA boxes (has_lstm_m5())
  bool has_lstm_m5() const { return !lstm_m5_.empty(); }
  const CUtensorMap& lstm_m5(int l, int which) const { return lstm_m5_[2 * l + which]; }

 private:
  const Spec& spec(const std::string& name, bool linear) const;
  void bind_dense_device(const Spec& s, const float* dvalues);

  cq_rnnt_config cfg_;
  cq_dtype dtype_;
  int device_;
  std::vector<Spec> specs_;
  std::map<std::string, size_t> index_;
  std::map<std::string, std::unique_ptr<QuantizedLinear>> linears_;
  std::map<std::string, DeviceBuffer> dense_;  // f32 copies of the LSTM biases
  DeviceBuffer embedding_, ih0_table_;
  std::vector<CUtensorMap> lstm_m5_;
  std::vector<DeviceBuffer> lstm_bias_;
  std::vector<std::unique_ptr<QuantizedLinear>> ih_il_, hh_il_;
  std::vector<DeviceBuffer> gate_bias_il_;
  bool finalized_ = false;
  bool fused_lstm_ = true;
};

class RnntState {
 public:
  RnntState(RnntDecoder& dec, int streams, int max_frames);
  ~RnntState();
  RnntState(const RnntState&) = delete;
  RnntState& operator=(const RnntState&) = delete;

  int capacity() const { return max_frames_ * dec_.config().max_symbols; }
  void reset();
  void decode_chunk(const void* encoded, int ld, int frames, int* tokens, int* token_frames,
                    int* counts, cudaStream_t stream);
  int launches_per_chunk() const { return launches_; }
  // Chunks as one persistent cooperative launch (true) or as a graph of one
  // launch per op (false, the default).  Throws if the persistent kernel does
  // not fit this state's shapes.
  void set_persistent(bool on);
  // Programmatic dependent launch between this state's kernels (default:
  // on).  Changing it drops the captured chunk graphs.
  void set_pdl(bool on);
  bool pdl() const { return pdl_; }
  bool persistent() const { return use_persistent_; }

 private:
  void launch_chunk(const void* encoded, int ld, int frames, int* tokens, int* token_frames,
                    int* counts, cudaStream_t stream);
  // proj_epi: the decoder projector also updates the joint input (active
  // streams' decoder output and relu(enc + dec)) in its epilogue
  void prediction_step(bool all, cudaStream_t stream, const cq::RnntEpilogue* proj_epi = nullptr);
  // the one-launch LSTM step writes each layer's new hidden state into the
  // other of two buffers; these give the current / other one and bring the
  // state back into h_ (at chunk ends, so captured graphs replay alike)
  void* h_cur(int l) { return hpar_[l] ? h_next_[l].get() : h_[l].get(); }
  void* h_other(int l) { return hpar_[l] ? h_[l].get() : h_next_[l].get(); }
  void normalize_h(cudaStream_t stream);
  void linear(QuantizedLinear* L, const void* x, int ldx, int rows, void* y, int ldy, int act,
              cudaStream_t stream);

  RnntDecoder& dec_;
  int S_, max_frames_;
  int launches_ = 0;
  bool pdl_ = pdl_default();
  DeviceBuffer ep_, dec_out_, dec_new_, fused_, logits_, x_, gi_, gh_, active_;
  std::vector<DeviceBuffer> h_, c_;
  bool lstm_fused_ = false;
  // head and projector carry the greedy choice and the joint input in their
  // epilogues (per-stream argmax keys and a CTA counter, zero between calls)
  bool fused_epi_ = false;
  DeviceBuffer best_, done_;
  // layer 0 reads T(W_ih emb[token]) from the decoder's table: the token each
  // stream feeds its prediction network next (the greedy epilogue writes it)
  bool ih0_from_table_ = false;
  DeviceBuffer last_token_;
  // the head only folds logits into best_; layer 0's step decodes the tokens
  // and records them, layer 1's clears best_ (two or more layers)
  bool defer_greedy_ = false;
  std::vector<DeviceBuffer> h_next_;
  std::vector<int> hpar_;
  // persistent path: second hidden-state buffer per layer, head partials, barrier
  std::vector<DeviceBuffer> h_alt_;
  DeviceBuffer part_, barrier_;
  int grid_ = 0;  // persistent grid size, 0 if the kernel does not fit
  bool use_persistent_ = false;
  DeviceBuffer scratch_;

  struct GraphEntry {
    const void* encoded;
    int ld, frames;
    const int *tokens, *token_frames, *counts;
    cudaGraphExec_t exec;
  };
  std::vector<GraphEntry> graphs_;
  cudaStream_t capture_stream_ = nullptr;
};

}  // namespace nemotron_cuda
