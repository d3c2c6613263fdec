// Host-side interface of the K2 tensor-core dequant-GEMM (qgemm.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace cq {

constexpr int kGemmBN = 128;       // output columns per CTA
constexpr int kGemmMinRows = 128;  // below this the GEMV (K1) is used

struct GemmArgs {
  const float* row_scale;  // [M] per-row scale of the f16 activations, or nullptr
  const void* scales;      // T [N, K/g]
  const void* biases;      // T [N, K/g]
  const void* bias;        // T [N] or nullptr
  void* y;                 // T [M, ldy]
  int* status;             // device status word (watchdog)
  int M, N, K, ldy;
  int act;                 // cq::Act
};

// amap: f16 activations [M, K] (box 64 x 128, 128B swizzle);
// qmap: packed weights u8 [N, K] (box 64 x 128, 64B swizzle).
cudaError_t launch_gemm(int dtype, int group, const CUtensorMap& amap, const CUtensorMap& qmap,
                        const GemmArgs& args, cudaStream_t stream, bool pdl);
// bf16 [M, ldx] -> f16 [M, ldo] with row_scale[m] = 2^e (power-of-two per row).
cudaError_t launch_gemm_prepass(const void* x, int ldx, int M, int K, void* xo, int ldo,
                                float* row_scale, cudaStream_t stream, bool pdl);
size_t gemm_smem_bytes();

}  // namespace cq
