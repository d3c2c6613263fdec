// C++ host layer of the streaming FastConformer encoder: the counterpart of
// the reference's StreamingEncoder and its layers
// (crates/nemotron-mlx/src/model/encoder.rs, layers.rs, cache.rs, prompt.rs).
// The C ABI in include/cqencoder.h wraps these classes.
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "cqencoder.h"
#include "device_buffer.hpp"
#include "qlinear.hpp"

namespace nemotron_cuda {

class Encoder {
 public:
  enum class Kind { kLinear, kDense };
  enum class Init { kLinear, kNormWeight, kKernel, kSmall };
  struct Spec {
    std::string name;
    Kind kind;
    int out = 0, in = 0;  // linear
    bool has_bias = false;
    size_t len = 0;  // dense element count
    bool f32_storage = false;
    Init init = Init::kSmall;
  };

  // Device pointers of one FastConformer block (valid after finalize()).
  struct Block {
    QuantizedLinear *ff1a, *ff1b, *qkv, *o, *pos, *pw1, *pw2, *ff2a, *ff2b;
    const void *norm_ff1_w, *norm_ff1_b, *norm_att_w, *norm_att_b, *norm_conv_w, *norm_conv_b;
    const void *norm_ff2_w, *norm_ff2_b, *norm_out_w, *norm_out_b;
    const void *conv_norm_w, *conv_norm_b, *dw_wt, *dw_b;  // dw_wt: [K][D]
    const float *bias_u, *bias_v;
  };

  Encoder(const cq_encoder_config& cfg, cq_dtype dtype, int device);

  const cq_encoder_config& config() const { return cfg_; }
  cq_dtype dtype() const { return dtype_; }
  int device() const { return device_; }

  void set_linear(const std::string& name, const uint32_t* q, const void* scales,
                  const void* biases, const void* bias, int out, int in, int group);
  void set_tensor(const std::string& name, const float* values, size_t len);
  void get_tensor(const std::string& name, float* values, size_t len) const;
  QuantizedLinear* linear(const std::string& name) const;
  void init_random(uint64_t seed);
  const std::vector<Spec>& specs() const { return specs_; }

  // Checks every tensor is bound and builds the fused q|k|v projections.
  void finalize();
  const std::vector<Block>& blocks() const { return blocks_; }
  const void* tensor(const std::string& name) const;

 private:
  const Spec& spec(const std::string& name, Kind kind) const;
  void bind_dense_device(const Spec& s, const float* dvalues);

  cq_encoder_config cfg_;
  cq_dtype dtype_;
  int device_;
  std::vector<Spec> specs_;
  std::map<std::string, size_t> index_;
  std::map<std::string, std::unique_ptr<QuantizedLinear>> linears_;
  std::map<std::string, DeviceBuffer> dense_;
  std::vector<std::unique_ptr<QuantizedLinear>> fused_qkv_;
  DeviceBuffer zero_dw_bias_;
  std::vector<DeviceBuffer> dw_wt_;  // depthwise kernels transposed to [K][D]
  std::vector<Block> blocks_;
  bool finalized_ = false;
};

// Streaming state of S lock-step streams plus the chunk workspaces.
class EncoderState {
 public:
  EncoderState(Encoder& enc, int streams, int max_mel_frames);
  ~EncoderState();
  EncoderState(const EncoderState&) = delete;
  EncoderState& operator=(const EncoderState&) = delete;

  void set_prompts(const int* ids, int count);
  int output_frames(int mel_frames) const;
  void encode_chunk(const float* mel, int mel_frames, void* out, cudaStream_t stream);
  void reset();
  // Programmatic dependent launch between this state's kernels (default:
  // on).  Changing it drops the captured chunk graphs.
  void set_pdl(bool on);
  bool pdl() const { return pdl_; }
  int chunks() const { return chunks_; }
  // Kernel launches of one chunk (the node count of the last captured chunk
  // graph, or the launches of the last eager chunk).
  int launches_per_chunk() const { return launches_; }
  int streams() const { return S_; }

  // Frame counts of one chunk through the subsampling (encoder.rs:767-802).
  struct Geometry {
    int time;
    int T1, F1, valid1;  // stem
    int T2, F2, valid2;  // stage 1
    int T3, F3, valid3;  // stage 2 = encoder frames of the chunk
  };
  Geometry geometry(int mel_frames, bool first) const;

 private:
  void launch_chunk(const float* mel, const Geometry& g, void* out, cudaStream_t stream);
  void linear(QuantizedLinear* L, const void* x, int ldx, int rows, void* y, int ldy, int act,
              cudaStream_t stream);

  Encoder& enc_;
  int S_, max_mel_, qmax_, ring_, vmax_, pmax_;
  int chunks_ = 0;
  int launches_ = 0;
  bool pdl_ = pdl_default();
  DeviceBuffer counters_, prompts_;
  DeviceBuffer res_, xn_, hid_, y_, att_, qkv_, pin_, relk_, pos_table_;
  // f16 copy + per-row scales of the LayerNorm / conv outputs that feed a
  // tensor-core GEMM (bf16, rows >= the GEMM threshold): the GEMM's prepass
  // done by the producer
  DeviceBuffer x16_, scale16_;
  DeviceBuffer kring_, vring_, conv_cache_;
  DeviceBuffer stem_out_, dw1_out_, pw1_out_, dw2_out_, pw2_out_, flat_;
  DeviceBuffer sub_cache_[3];
  DeviceBuffer scratch_;
  size_t hid_width_ = 0;
  int num_sms_ = 148;

  struct GraphEntry {
    int mel_frames;
    const void* mel;
    void* out;
    cudaGraphExec_t exec;
  };
  std::vector<GraphEntry> graphs_;
  cudaStream_t capture_stream_ = nullptr;
};

}  // namespace nemotron_cuda
