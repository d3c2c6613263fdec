// C++ host layer of the B200 quantized linear: the counterpart of the
// reference's Rust `QuantizedLinear` (crates/nemotron-mlx/src/model/layers.rs:208-319),
// `PointwiseConv1d` (layers.rs:321-352) and `backend::quantized_matmul`
// (crates/nemotron-mlx/src/backend/mod.rs:41-94).  The C ABI in
// include/cqlinear.h wraps these classes; errors are C++ exceptions inside the
// library and status codes at the ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "cqlinear.h"
#include "qgemm.hpp"
#include "qgemv.hpp"

namespace nemotron_cuda {

// Error carrying the ABI status.  Shape errors use the reference's texts
// (ModelError::InvalidShape prints "invalid model shape: ...",
// BackendError::InvalidShape prints "invalid matrix shape: ...").
class Error : public std::runtime_error {
 public:
  Error(cq_status status, const std::string& msg) : std::runtime_error(msg), status_(status) {}
  cq_status status() const { return status_; }

 private:
  cq_status status_;
};

[[noreturn]] void throw_invalid(const std::string& msg);
void check_cuda(cudaError_t e, const char* what);

// Per-device state: SM count and the device watchdog word.
struct DeviceContext {
  int device = 0;
  int num_sms = 0;
  int* status = nullptr;  // device int, see cq_device_status
};
DeviceContext& device_context(int device);

// Restores the caller's current device on scope exit.
class DeviceGuard {
 public:
  explicit DeviceGuard(int device);
  ~DeviceGuard();

 private:
  int prev_ = -1;
};

// 2-D tiled tensor map over a row-major [rows, cols] matrix of 1- or 2-byte
// elements (row stride in elements), box [box_rows, box_cols].
CUtensorMap make_map_2d(const void* base, int elem_bytes, int rows, int cols, int ld,
                        int box_rows, int box_cols, CUtensorMapSwizzle swizzle);

// The K2 GEMM's activation maps over f16 [rows, K] with row stride ld.
cq::GemmActMaps make_act_maps(const void* base, int rows, int K, int ld, int tn);

// Programmatic dependent launch (PDL) on this thread's kernel launches: on,
// or as the innermost live PdlScope says.  Encoder and RNNT
// states set it per chunk (streams that overlap on one GPU can run faster
// without it: CTAs launched early wait on the GPU holding their SM's room).
bool pdl_default();
bool pdl_enabled();
class PdlScope {
 public:
  explicit PdlScope(bool on);
  ~PdlScope();
  PdlScope(const PdlScope&) = delete;
  PdlScope& operator=(const PdlScope&) = delete;

 private:
  int prev_;
};

class QuantizedLinear {
 public:
  // Packed arrays in host memory -> owned device copy (from_artifact).
  static std::unique_ptr<QuantizedLinear> from_packed(const uint32_t* qweight, const void* scales,
                                                      const void* biases, const void* bias,
                                                      int output_dims, int input_dims, int group,
                                                      cq_dtype dtype, int device);
  // f32 weight in host memory, quantised on the device (from_f32).
  static std::unique_ptr<QuantizedLinear> from_f32(const float* weight, size_t weight_len,
                                                   int output_dims, int input_dims,
                                                   const float* bias, size_t bias_len, int group,
                                                   cq_dtype dtype, int device);
  static std::unique_ptr<QuantizedLinear> concat(const std::vector<const QuantizedLinear*>& parts);

  ~QuantizedLinear();
  QuantizedLinear(const QuantizedLinear&) = delete;
  QuantizedLinear& operator=(const QuantizedLinear&) = delete;

  // Device pointers in T, asynchronous (forward_array).
  void forward_array(const void* x, int ldx, int rows, void* y, int ldy, int act,
                     cudaStream_t stream) const;
  // Host f32 in / out, synchronous (forward_f32).
  void forward_f32(const float* input, size_t input_len, int rows, float* output,
                   size_t output_len);
  // Allocates the batched-path workspace for up to `max_rows` rows now, so
  // later calls of that size allocate nothing (e.g. before graph capture).
  void reserve(int max_rows);
  // True when batched calls run on the tensor-core GEMM (K2).
  bool gemm_enabled() const { return gemm_ok_; }
  // forward_array that never allocates device memory: the batched bf16 path
  // stages its f16 activations in the caller-provided device scratch instead
  // of the layer's workspace; every other path needs no scratch.  Throws
  // invalid-argument if the scratch is smaller than scratch_bytes_for(rows).
  void forward_array_in_scratch(const void* x, int ldx, int rows, void* y, int ldy, int act,
                                cudaStream_t stream, void* scratch, size_t scratch_bytes);
  size_t scratch_bytes_for(int rows) const;

  // Several calls of same-shape layers (N, K, group, dtype, device) on the
  // same number of rows below the GEMM threshold, as one K1 launch whose CTAs
  // span every member's bands (e.g. the independent ih / hh products of an
  // LSTM step).  Asynchronous on `stream`.
  // True when a call on `rows` rows runs the tensor-core GEMM on f16
  // activations converted by its prepass (bf16 layers), i.e. when
  // forward_prescaled can take a producer's converted copy instead.
  bool gemm_for(int rows) const;
  // forward_array for such a call, given the activations already converted:
  // x16 f16 [rows, K] (row stride K) and the per-row inverse scales.
  void forward_prescaled(const void* x16, const float* row_scale, int rows, void* y, int ldy,
                         int act, cudaStream_t stream);
  // The conversion forward_array does before such a call: x bf16 [rows, ldx]
  // -> x16 f16 [rows, K] (row stride K) and row_scale [rows], for producers
  // that hand forward_prescaled their own copy.  Same restriction.
  void prescale(const void* x, int ldx, int rows, void* x16, float* row_scale,
                cudaStream_t stream);

  // forward_array on the GEMV with one of the RNNT decoder's epilogues
  // (cq::kGemvJointInput / kGemvGreedy, see qgemv.hpp); rows below the GEMM
  // threshold and K within one CTA, else invalid-argument.
  void forward_rnnt(const void* x, int ldx, int rows, void* y, int ldy, int mode,
                    const cq::RnntEpilogue& epi, cudaStream_t stream) const;
  bool rnnt_epilogue_fits(int rows) const;

  struct GroupCall {
    const QuantizedLinear* layer;
    const void* x;
    int ldx;
    void* y;
    int ldy;
  };
  static void forward_group(const GroupCall* calls, int count, int rows, int act,
                            cudaStream_t stream);

  int input_dims() const { return K_; }
  int output_dims() const { return N_; }
  int group_size() const { return group_; }
  cq_dtype dtype() const { return dtype_; }
  int device() const { return device_; }
  const void* qweight() const { return q_; }
  const void* scales() const { return scales_; }
  const void* biases() const { return biases_; }
  const void* bias() const { return bias_; }
  // K1 weight map with a (64 k x 16*rt rows) box, rt in {1, 2, 4}.
  const CUtensorMap& gemv_map(int rt) const { return wmap_rt_[rt == 1 ? 0 : rt == 2 ? 1 : 2]; }

 private:
  QuantizedLinear(int N, int K, int group, cq_dtype dtype, int device);
  void allocate(bool with_bias);
  void finalize();  // plan + tensor map once the arrays are in place

  int N_, K_, group_;
  cq_dtype dtype_;
  int device_;
  uint8_t* q_ = nullptr;
  void* scales_ = nullptr;
  void* biases_ = nullptr;
  void* bias_ = nullptr;
  cq::GemvPlan plan_{};
  CUtensorMap wmap_{};
  CUtensorMap wmap_rt_[3]{};  // weight maps with 16, 32 and 64-row boxes (plan_gemv_rows)
  // K2: packed weights with a 128-byte swizzle; scales/biases fit f16
  CUtensorMap qmap_gemm_{};
  bool gemm_ok_ = false;
  void* sb_tiles_ = nullptr;  // (scale, bias) pairs in the GEMM's k-tile order
  // K2 workspace (bf16 layers): f16 activations [rows, K] + row scales [rows]
  std::mutex ws_mu_;
  void* ws_ = nullptr;
  size_t ws_bytes_ = 0;
  int ws_rows_ = 0;
  // cached activation tensor maps
  cq::GemmActMaps amap_{};
  const void* amap_ptr_ = nullptr;
  int amap_ld_ = 0, amap_rows_ = 0;
  void forward_gemm(const void* x, int ldx, int rows, void* y, int ldy, int act,
                    cudaStream_t stream);
  // activation tensor map of the scratch-staged path, cached separately
  cq::GemmActMaps amap_scratch_{};
  const void* amap_scratch_ptr_ = nullptr;
  int amap_scratch_rows_ = 0;
  // activation tensor map of the prescaled path, cached separately
  cq::GemmActMaps amap_pre_{};
  const void* amap_pre_ptr_ = nullptr;
  int amap_pre_rows_ = 0;
  bool check_f16_range() const;

  // Scratch of the synchronous host-f32 path, grown on demand.
  std::mutex host_mu_;
  void* host_scratch_ = nullptr;
  size_t host_scratch_bytes_ = 0;
};

size_t dtype_size(cq_dtype dtype);

// Device scratch of the no-allocation entry point (noalloc.cu).
size_t noalloc_scratch_capacity();
void* noalloc_scratch_address(int device, cudaStream_t stream);

// backend::quantized_matmul: quantise the f32 weight (f32 scales) on the
// device and return input . dequant(weight)^T as f32.
void quantized_matmul(const float* input, size_t input_len, size_t rows, size_t input_dims,
                      const float* weight, size_t weight_len, size_t output_dims,
                      size_t group_size, float* output, size_t output_len);

}  // namespace nemotron_cuda
