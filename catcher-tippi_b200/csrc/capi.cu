// extern "C" boundary (include/cqlinear.h) over the C++ host layer.  Every
// entry catches exceptions and maps them to a status plus a thread-local
// message, the way catcher-ffi wraps its Rust calls
// (crates/catcher-ffi/src/lib.rs:703-722, :779-786).
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "capi_guard.hpp"
#include "cqlinear.h"
#include "qlinear.hpp"
#include "qops.hpp"

namespace {

using nemotron_cuda::guarded;
using nemotron_cuda::need_handle;

cq_linear* wrap(std::unique_ptr<nemotron_cuda::QuantizedLinear> p) {
  cq_linear* h = new cq_linear;
  h->owned = std::move(p);
  h->impl = h->owned.get();
  return h;
}

}  // namespace

extern "C" {

const char* cq_last_error(void) { return nemotron_cuda::last_error_slot().c_str(); }

const char* cq_version(void) { return "cqlinear 0.1.0 (sm_100a)"; }

int32_t cq_is_device_available(void) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  for (int d = 0; d < count; ++d) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d) == cudaSuccess &&
        major == 10)
      return 1;
  }
  return 0;
}

cq_status cq_linear_create(const uint32_t* qweight, const void* scales, const void* biases,
                           const void* bias_or_null, int32_t output_dims, int32_t input_dims,
                           int32_t group_size, cq_dtype dtype, int32_t device, cq_linear** out) {
  return guarded([&] {
    need_handle(out, "out");
    *out = nullptr;
    *out = wrap(nemotron_cuda::QuantizedLinear::from_packed(qweight, scales, biases, bias_or_null,
                                                           output_dims, input_dims, group_size,
                                                           dtype, device));
  });
}

cq_status cq_linear_create_from_f32(const float* weight, size_t weight_len, int32_t output_dims,
                                    int32_t input_dims, const float* bias, size_t bias_len,
                                    int32_t group_size, cq_dtype dtype, int32_t device,
                                    cq_linear** out) {
  return guarded([&] {
    need_handle(out, "out");
    *out = nullptr;
    *out = wrap(nemotron_cuda::QuantizedLinear::from_f32(weight, weight_len, output_dims,
                                                        input_dims, bias, bias_len, group_size,
                                                        dtype, device));
  });
}

cq_status cq_linear_concat(cq_linear* const* parts, int32_t count, cq_linear** out) {
  return guarded([&] {
    need_handle(out, "out");
    *out = nullptr;
    if (parts == nullptr || count <= 0) nemotron_cuda::throw_invalid("concat needs layers");
    std::vector<const nemotron_cuda::QuantizedLinear*> v;
    for (int i = 0; i < count; ++i) {
      need_handle(parts[i], "layer");
      v.push_back(parts[i]->impl);
    }
    *out = wrap(nemotron_cuda::QuantizedLinear::concat(v));
  });
}

cq_status cq_linear_forward(cq_linear* layer, const void* x, int32_t rows, void* y, void* stream) {
  return guarded([&] {
    need_handle(layer, "layer");
    const auto& L = *layer->impl;
    L.forward_array(x, L.input_dims(), rows, y, L.output_dims(), CQ_ACT_NONE,
                    static_cast<cudaStream_t>(stream));
  });
}

cq_status cq_linear_forward_ex(cq_linear* layer, const void* x, int32_t ldx, int32_t rows, void* y,
                               int32_t ldy, cq_act act, void* stream) {
  return guarded([&] {
    need_handle(layer, "layer");
    layer->impl->forward_array(x, ldx, rows, y, ldy, act, static_cast<cudaStream_t>(stream));
  });
}

cq_status cq_linear_prescale_activations(cq_linear* layer, const void* x, int32_t ldx,
                                         int32_t rows, void* x16, float* row_scale, void* stream) {
  return guarded([&] {
    need_handle(layer, "layer");
    layer->impl->prescale(x, ldx, rows, x16, row_scale, static_cast<cudaStream_t>(stream));
  });
}

cq_status cq_linear_forward_prescaled(cq_linear* layer, const void* x16, const float* row_scale,
                                      int32_t rows, void* y, int32_t ldy, cq_act act,
                                      void* stream) {
  return guarded([&] {
    need_handle(layer, "layer");
    layer->impl->forward_prescaled(x16, row_scale, rows, y, ldy, act,
                                   static_cast<cudaStream_t>(stream));
  });
}

cq_status cq_linear_forward_f32(cq_linear* layer, const float* input, size_t input_len,
                                int32_t rows, float* output, size_t output_len) {
  return guarded([&] {
    need_handle(layer, "layer");
    layer->impl->forward_f32(input, input_len, rows, output, output_len);
  });
}

cq_status cq_linear_forward_noalloc(cq_linear* layer, const void* x, int32_t ldx, int32_t rows,
                                   void* y, int32_t ldy, cq_act act, void* stream) {
  return guarded([&] {
    need_handle(layer, "layer");
    auto& L = *layer->impl;
    const size_t cap = nemotron_cuda::noalloc_scratch_capacity();
    if (rows > 0 && L.scratch_bytes_for(rows) > cap)
      nemotron_cuda::throw_invalid(
          "rows x input_dims = " + std::to_string(rows) + "x" + std::to_string(L.input_dims()) +
          " exceeds the no-allocation scratch of " + std::to_string(cap) + " bytes");
    void* scratch = rows > 0 && L.scratch_bytes_for(rows) > 0
                        ? nemotron_cuda::noalloc_scratch_address(L.device(),
                                                                static_cast<cudaStream_t>(stream))
                        : nullptr;
    L.forward_array_in_scratch(x, ldx, rows, y, ldy, act, static_cast<cudaStream_t>(stream),
                               scratch, cap);
  });
}

cq_status cq_linear_reserve(cq_linear* layer, int32_t max_rows) {
  return guarded([&] {
    need_handle(layer, "layer");
    layer->impl->reserve(max_rows);
  });
}

int32_t cq_linear_input_dims(const cq_linear* layer) {
  return layer ? layer->impl->input_dims() : -1;
}
int32_t cq_linear_output_dims(const cq_linear* layer) {
  return layer ? layer->impl->output_dims() : -1;
}
int32_t cq_linear_group_size(const cq_linear* layer) {
  return layer ? layer->impl->group_size() : -1;
}
cq_dtype cq_linear_dtype(const cq_linear* layer) { return layer ? layer->impl->dtype() : -1; }

cq_status cq_linear_device_arrays(const cq_linear* layer, const void** qweight,
                                  const void** scales, const void** biases, const void** bias) {
  return guarded([&] {
    need_handle(layer, "layer");
    const auto& L = *layer->impl;
    if (qweight) *qweight = L.qweight();
    if (scales) *scales = L.scales();
    if (biases) *biases = L.biases();
    if (bias) *bias = L.bias();
  });
}

cq_status cq_linear_copy_arrays(const cq_linear* layer, uint32_t* qweight, void* scales,
                                void* biases, void* bias) {
  return guarded([&] {
    need_handle(layer, "layer");
    const auto& L = *layer->impl;
    nemotron_cuda::DeviceGuard guard(L.device());
    const size_t n = static_cast<size_t>(L.output_dims()), k = static_cast<size_t>(L.input_dims());
    const size_t es = nemotron_cuda::dtype_size(L.dtype());
    const size_t groups = n * (k / L.group_size());
    if (qweight)
      nemotron_cuda::check_cuda(cudaMemcpy(qweight, L.qweight(), n * k, cudaMemcpyDefault), "copy qweight");
    if (scales)
      nemotron_cuda::check_cuda(cudaMemcpy(scales, L.scales(), groups * es, cudaMemcpyDefault), "copy scales");
    if (biases)
      nemotron_cuda::check_cuda(cudaMemcpy(biases, L.biases(), groups * es, cudaMemcpyDefault), "copy biases");
    if (bias) {
      if (L.bias() != nullptr) {
        nemotron_cuda::check_cuda(cudaMemcpy(bias, L.bias(), n * es, cudaMemcpyDefault), "copy bias");
      } else {
        const std::vector<unsigned char> zeros(n * es, 0);  // host or device destination
        nemotron_cuda::check_cuda(cudaMemcpy(bias, zeros.data(), n * es, cudaMemcpyDefault),
                                  "zero bias");
      }
    }
  });
}

void cq_linear_destroy(cq_linear* layer) {
  // borrowed handles (cq_encoder_linear) belong to their encoder
  if (layer != nullptr && !layer->borrowed) delete layer;
}

cq_status cq_quantized_matmul(const float* input, size_t input_len, size_t rows,
                              size_t input_dims, const float* weight, size_t weight_len,
                              size_t output_dims, size_t group_size, float* output,
                              size_t output_len) {
  return guarded([&] {
    nemotron_cuda::quantized_matmul(input, input_len, rows, input_dims, weight, weight_len,
                                    output_dims, group_size, output, output_len);
  });
}

cq_status cq_quantize(const float* w, int32_t rows, int32_t cols, int32_t group_size,
                      cq_dtype dtype, int32_t round_input, uint32_t* qweight, void* scales,
                      void* biases, void* stream) {
  return guarded([&] {
    if (dtype != CQ_F16 && dtype != CQ_BF16 && dtype != CQ_F32)
      nemotron_cuda::throw_invalid("unknown dtype " + std::to_string(dtype));
    if (group_size != 32 && group_size != 64 && group_size != 128)
      nemotron_cuda::throw_invalid("group size " + std::to_string(group_size) +
                                   " is not supported; supported group sizes are 32, 64 and 128");
    if (rows < 0 || cols < 0 || cols % group_size != 0)
      nemotron_cuda::throw_invalid("invalid matrix shape: " + std::to_string(rows) + "x" +
                                   std::to_string(cols) + " with group size " +
                                   std::to_string(group_size));
    if (rows == 0 || cols == 0) return;
    if (!w || !qweight || !scales || !biases)
      nemotron_cuda::throw_invalid("quantize pointers must not be null");
    nemotron_cuda::check_cuda(
        cq::launch_quantize(dtype, w, rows, cols, group_size, round_input != 0,
                            reinterpret_cast<uint8_t*>(qweight), scales, biases,
                            static_cast<cudaStream_t>(stream)),
        "quantize");
  });
}

cq_status cq_dequantize(const uint32_t* qweight, const void* scales, const void* biases,
                        int32_t rows, int32_t cols, int32_t group_size, cq_dtype dtype, float* w,
                        void* stream) {
  return guarded([&] {
    if (dtype != CQ_F16 && dtype != CQ_BF16 && dtype != CQ_F32)
      nemotron_cuda::throw_invalid("unknown dtype " + std::to_string(dtype));
    if (group_size != 32 && group_size != 64 && group_size != 128)
      nemotron_cuda::throw_invalid("group size " + std::to_string(group_size) +
                                   " is not supported; supported group sizes are 32, 64 and 128");
    if (rows < 0 || cols < 0 || cols % group_size != 0)
      nemotron_cuda::throw_invalid("invalid matrix shape: " + std::to_string(rows) + "x" +
                                   std::to_string(cols) + " with group size " +
                                   std::to_string(group_size));
    if (rows == 0 || cols == 0) return;
    if (!w || !qweight || !scales || !biases)
      nemotron_cuda::throw_invalid("dequantize pointers must not be null");
    nemotron_cuda::check_cuda(
        cq::launch_dequantize(dtype, reinterpret_cast<const uint8_t*>(qweight), scales, biases,
                              rows, cols, group_size, w, static_cast<cudaStream_t>(stream)),
        "dequantize");
  });
}

cq_status cq_device_status(int32_t device, int32_t* status) {
  return guarded([&] {
    if (status == nullptr) nemotron_cuda::throw_invalid("status must not be null");
    nemotron_cuda::DeviceContext& ctx = nemotron_cuda::device_context(device);
    nemotron_cuda::DeviceGuard guard(device);
    nemotron_cuda::check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    int v = 0;
    nemotron_cuda::check_cuda(cudaMemcpy(&v, ctx.status, sizeof(int), cudaMemcpyDeviceToHost),
                              "read status");
    nemotron_cuda::check_cuda(cudaMemset(ctx.status, 0, sizeof(int)), "clear status");
    *status = v;
  });
}

}  // extern "C"
