// Host-side interface of the supporting device ops (qops.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace cq {

cudaError_t launch_quantize(int dtype, const float* w, int N, int K, int g, bool round_input,
                            uint8_t* q, void* scales, void* biases, cudaStream_t stream);
cudaError_t launch_dequantize(int dtype, const uint8_t* q, const void* scales, const void* biases,
                              int N, int K, int g, float* w, cudaStream_t stream);
cudaError_t launch_f32_to_t(int dtype, const float* in, size_t n, void* out, cudaStream_t stream);
cudaError_t launch_t_to_f32(int dtype, const void* in, size_t n, float* out, cudaStream_t stream);
cudaError_t launch_qmatmul_f32(const float* x, int M, int K, const uint8_t* q, const float* s,
                               const float* b, int N, int g, float* y, cudaStream_t stream);

}  // namespace cq
