// Host side of the persistent linear-chain executor: a fixed sequence of
// quantized-linear calls (layer, input, output, activation) on small token
// counts, planned once and run as one cooperative launch per call of run().
// The counterpart of calling QuantizedLinear::forward_array
// (crates/nemotron-mlx/src/model/layers.rs:298-310) for each step in order.
#pragma once

#include <cuda_runtime.h>

#include <vector>

#include "device_buffer.hpp"
#include "qchain.hpp"
#include "qlinear.hpp"

namespace nemotron_cuda {

struct ChainStepSpec {
  const QuantizedLinear* layer;
  const void* x;
  int ldx, rows;
  void* y;
  int ldy, act;
};

class LinearChain {
 public:
  // Steps run as if issued one after another on one stream.  Dependencies are
  // derived from the buffers: a step waits for the latest earlier step that
  // writes memory it reads (read after write), reads memory it writes (write
  // after read) or writes memory it writes (write after write).
  explicit LinearChain(const std::vector<ChainStepSpec>& steps);

  void run(cudaStream_t stream);
  // Per-item %globaltimer stamps of later runs (cq::kChainTraceStamps each).
  void set_profile(bool on);
  void read_profile(uint64_t* host, size_t len) const;

  int steps() const { return static_cast<int>(host_.size()); }
  int grid() const { return grid_; }
  int items() const { return items_; }
  int device() const { return device_; }
  // Steps that read their producer's tagged output instead of waiting for it.
  int tagged_reads() const { return tagged_reads_; }
  int tagged_source(int i) const { return tagged_src_.at(i); }
  // Work decomposition of one step: weight rows per item, K sub-blocks of 64
  // per item, K slices, and the steps it waits for.
  const cq::ChainStep& step_plan(int i) const { return host_.at(i); }

 private:
  int device_ = 0;
  int dtype_ = 0, group_ = 0;
  int grid_ = 0, items_ = 0, narrive_ = 0;
  std::vector<cq::ChainStep> host_;
  DeviceBuffer steps_, maps_, partial_, arrive_, done_, exit_, abort_, trace_, tagged_, epoch_;
  int tagged_reads_ = 0;
  std::vector<int> tagged_src_;
};

}  // namespace nemotron_cuda
