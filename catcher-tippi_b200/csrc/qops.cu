// Supporting device ops around the quantized linear:
//  * affine 8-bit quantisation (MLX `quantize(w, g, 8)`, used by
//    QuantizedLinear::from_f32 at crates/nemotron-mlx/src/model/layers.rs:249-280
//    and backend::quantized_matmul at crates/nemotron-mlx/src/backend/mod.rs:81);
//  * dequantisation to fp32 (Artifact::dequantize_to_f32,
//    crates/nemotron-mlx/src/weights/artifact.rs:183-200);
//  * element conversions f32 <-> T for the host-f32 forward path;
//  * the fp32 quantized matmul of backend::quantized_matmul, where scales,
//    biases and activations stay f32 (backend/mod.rs:78-93).
#include "common.cuh"
#include "qops.hpp"

namespace cq {
namespace {

// One warp per (row, group), MLX's edge/sign form of affine quantisation:
// the group's extreme of larger magnitude (the edge) becomes the bias and is
// represented exactly; step = max((max - min) / 255, 1e-7) takes the edge's
// sign, q0 = round(edge / step), and when q0 != 0 the scale is edge / q0 (else
// the scale stays step and the bias is 0).  Codes are
// clamp(round((w - bias) / scale), 0, 255) from the fp32 scale and bias, which
// are rounded to T only when stored.  round = half to even; every operation is
// an IEEE single-rounded fp32 operation, so the result is bit-identical to the
// CPU restatement.
template <int DT>
__global__ void quantize_kernel(const float* __restrict__ w, int N, int K, int g, int round_input,
                                uint8_t* __restrict__ q, void* __restrict__ scales,
                                void* __restrict__ biases) {
  const int groups = K / g;
  const long long item = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (item >= static_cast<long long>(N) * groups) return;
  const int n = static_cast<int>(item / groups), j = static_cast<int>(item % groups);
  const float* src = w + static_cast<size_t>(n) * K + static_cast<size_t>(j) * g;
  const int per = g / 32;  // 1, 2 or 4 values per lane
  float v[4];
  float lo = INFINITY, hi = -INFINITY;
  for (int i = 0; i < per; ++i) {
    float t = src[lane * per + i];
    if (round_input) t = round_t<DT>(t);
    v[i] = t;
    lo = fminf(lo, t);
    hi = fmaxf(hi, t);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xFFFFFFFFu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xFFFFFFFFu, hi, o));
  }
  const bool low_edge = fabsf(lo) > fabsf(hi);
  const float step = fmaxf(__fdiv_rn(__fsub_rn(hi, lo), 255.0f), 1e-7f);
  float scale = low_edge ? step : -step;
  const float edge = low_edge ? lo : hi;
  const float q0 = rintf(__fdiv_rn(edge, scale));
  float bias = 0.0f;
  if (q0 != 0.0f) {
    scale = __fdiv_rn(edge, q0);
    bias = edge;
  }
  uint8_t* dst = q + static_cast<size_t>(n) * K + static_cast<size_t>(j) * g;
  for (int i = 0; i < per; ++i) {
    float cdx = rintf(__fdiv_rn(__fsub_rn(v[i], bias), scale));
    cdx = fminf(fmaxf(cdx, 0.0f), 255.0f);
    dst[lane * per + i] = static_cast<uint8_t>(cdx);
  }
  if (lane == 0) {
    st_t<DT>(scales, item, scale);
    st_t<DT>(biases, item, bias);
  }
}

template <int DT>
__global__ void dequantize_kernel(const uint8_t* __restrict__ q, const void* __restrict__ scales,
                                  const void* __restrict__ biases, int N, int K, int g,
                                  float* __restrict__ w) {
  const size_t total = static_cast<size_t>(N) * K;
  const int groups = K / g;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t n = i / K, k = i % K;
    const size_t gi = n * groups + k / g;
    // scale * q + bias with two roundings (no contraction), as the formula reads
    w[i] = __fadd_rn(__fmul_rn(ld_t<DT>(scales, gi), static_cast<float>(q[i])), ld_t<DT>(biases, gi));
  }
}

template <int DT>
__global__ void f32_to_t_kernel(const float* __restrict__ in, size_t n, void* __restrict__ out) {
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    st_t<DT>(out, i, in[i]);
}

template <int DT>
__global__ void t_to_f32_kernel(const void* __restrict__ in, size_t n, float* __restrict__ out) {
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = ld_t<DT>(in, i);
}

// fp32 affine INT8 matmul, one warp per output row n and 32-lane strided K.
// Used for the f32 backend path only (tests); the T paths use K1 / K2.
__global__ void qmatmul_f32_kernel(const float* __restrict__ x, int M, int K,
                                   const uint8_t* __restrict__ q, const float* __restrict__ s,
                                   const float* __restrict__ b, int N, int g,
                                   float* __restrict__ y) {
  const int n = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  const int groups = K / g;
  const uint8_t* qr = q + static_cast<size_t>(n) * K;
  for (int m = 0; m < M; ++m) {
    const float* xr = x + static_cast<size_t>(m) * K;
    float acc = 0.f;
    for (int k = lane; k < K; k += 32) {
      const int gi = n * groups + k / g;
      acc = fmaf(xr[k], fmaf(s[gi], static_cast<float>(qr[k]), b[gi]), acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    if (lane == 0) y[static_cast<size_t>(m) * N + n] = acc;
  }
}

inline int grid_for(size_t n, int block) {
  size_t g = (n + block - 1) / block;
  return static_cast<int>(g > 65535 * 16 ? 65535 * 16 : (g == 0 ? 1 : g));
}

}  // namespace

cudaError_t launch_quantize(int dtype, const float* w, int N, int K, int g, bool round_input,
                            uint8_t* q, void* scales, void* biases, cudaStream_t stream) {
  const long long warps = static_cast<long long>(N) * (K / g);
  const int block = 256;
  const int grid = static_cast<int>((warps * 32 + block - 1) / block);
  if (grid == 0) return cudaSuccess;
  if (dtype == kF16)
    quantize_kernel<kF16><<<grid, block, 0, stream>>>(w, N, K, g, round_input, q, scales, biases);
  else if (dtype == kBF16)
    quantize_kernel<kBF16><<<grid, block, 0, stream>>>(w, N, K, g, round_input, q, scales, biases);
  else
    quantize_kernel<kF32><<<grid, block, 0, stream>>>(w, N, K, g, round_input, q, scales, biases);
  return cudaGetLastError();
}

cudaError_t launch_dequantize(int dtype, const uint8_t* q, const void* scales, const void* biases,
                              int N, int K, int g, float* w, cudaStream_t stream) {
  const size_t total = static_cast<size_t>(N) * K;
  if (total == 0) return cudaSuccess;
  const int block = 256, grid = grid_for(total, block);
  if (dtype == kF16)
    dequantize_kernel<kF16><<<grid, block, 0, stream>>>(q, scales, biases, N, K, g, w);
  else if (dtype == kBF16)
    dequantize_kernel<kBF16><<<grid, block, 0, stream>>>(q, scales, biases, N, K, g, w);
  else
    dequantize_kernel<kF32><<<grid, block, 0, stream>>>(q, scales, biases, N, K, g, w);
  return cudaGetLastError();
}

cudaError_t launch_f32_to_t(int dtype, const float* in, size_t n, void* out, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const int block = 256, grid = grid_for(n, block);
  if (dtype == kF16) f32_to_t_kernel<kF16><<<grid, block, 0, stream>>>(in, n, out);
  else if (dtype == kBF16) f32_to_t_kernel<kBF16><<<grid, block, 0, stream>>>(in, n, out);
  else f32_to_t_kernel<kF32><<<grid, block, 0, stream>>>(in, n, out);
  return cudaGetLastError();
}

cudaError_t launch_t_to_f32(int dtype, const void* in, size_t n, float* out, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const int block = 256, grid = grid_for(n, block);
  if (dtype == kF16) t_to_f32_kernel<kF16><<<grid, block, 0, stream>>>(in, n, out);
  else if (dtype == kBF16) t_to_f32_kernel<kBF16><<<grid, block, 0, stream>>>(in, n, out);
  else t_to_f32_kernel<kF32><<<grid, block, 0, stream>>>(in, n, out);
  return cudaGetLastError();
}

cudaError_t launch_qmatmul_f32(const float* x, int M, int K, const uint8_t* q, const float* s,
                               const float* b, int N, int g, float* y, cudaStream_t stream) {
  if (M == 0 || N == 0) return cudaSuccess;
  const int block = 256;
  const int grid = (N * 32 + block - 1) / block;
  qmatmul_f32_kernel<<<grid, block, 0, stream>>>(x, M, K, q, s, b, N, g, y);
  return cudaGetLastError();
}

}  // namespace cq
