// Host-side interface of the K2 tensor-core dequant-GEMM (qgemm.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace cq {

constexpr int kGemmBN = 128;       // output columns (weight rows) per CTA
constexpr int kGemmTN = 224;       // rows (tokens) per CTA: 896 = 4 x 224
constexpr int kGemmTNSmall = 128;  // the narrower tile for layers whose kGemmTN tiles leave SMs idle
constexpr int kGemmMinRows = 256;  // below this the GEMV (K1) is used

struct GemmArgs {
  const float* row_scale;  // [M] per-row scale of the f16 activations, or nullptr
  const void* sb_tiles;    // f16 (scale, bias) pairs in k-tile order (build_sb_tiles)
  const void* bias;        // T [N] or nullptr
  void* y;                 // T [M, ldy]
  int* status;             // device status word (watchdog)
  int M, N, K, ldy;
  int act;                 // cq::Act
  int splits;              // K split over a (1, 1, splits) cluster: 1, 2 or 4
  int pair_tiles;          // full 64-wide k-tiles the `pair` activation map covers (0: none)
  int tn;                  // tokens per CTA: kGemmTN or kGemmTNSmall (gemm_tile_tokens)
};

// The activation maps the GEMM reads (f16 [M, K], 128B swizzle): `tile`
// copies one 64-wide k-tile of `tn` rows (2-D, zero past K and M);
// `pair` copies two consecutive full k-tiles in one copy (3-D view
// {64, M, K / 64} with the k-tile stride 128 bytes).
struct GemmActMaps {
  CUtensorMap tile;
  CUtensorMap pair;
  int pair_tiles;  // K / 64 when K >= 128, else 0 (`pair` unused)
  int tn;          // rows per box: the call's GemmArgs::tn
};

// K split that fills the GPU when the output tiles alone leave most SMs idle:
// the CTAs of one cluster accumulate disjoint k ranges and reduce through
// distributed shared memory (gemm_splits returns 1, 2 or 4).
int gemm_splits(int M, int N, int K, int num_sms, int tn);
// Tokens per CTA for an M x N x K call: kGemmTNSmall when its tiles fit one
// wave of num_sms CTAs and the wide tile cannot split K four ways, else
// kGemmTN.
int gemm_tile_tokens(int M, int N, int K, int num_sms);

// qmap: packed weights u8 [N, K] (box 128 x kGemmBN, 128B swizzle: two
// k-tiles per copy).
cudaError_t launch_gemm(int dtype, int group, const GemmActMaps& amaps, const CUtensorMap& qmap,
                        const GemmArgs& args, cudaStream_t stream, bool pdl);
// bf16 [M, ldx] -> f16 [M, ldo] with row_scale[m] = 2^e (power-of-two per row).
cudaError_t launch_gemm_prepass(const void* x, int ldx, int M, int K, void* xo, int ldo,
                                float* row_scale, cudaStream_t stream, bool pdl);
// Repacks T scales/biases [N, K/g] into the f16 (scale, bias) pair order the
// GEMM streams per k-tile: [ceil(N/kGemmBN)][ceil(K/64)][kGemmBN][g == 32 ? 2 : 1].
size_t sb_tiles_bytes(int N, int K, int group);
cudaError_t build_sb_tiles(int dtype, const void* scales, const void* biases, int N, int K,
                           int group, void* out, cudaStream_t stream);

}  // namespace cq
