// Host-side interface of the encoder's supporting kernels (encoder_ops.cu):
// everything in a FastConformer chunk that is not a quantized linear.  All
// kernels are launched with programmatic dependent launch when `pdl` is set
// and then wait for their predecessor before touching its output.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace cq {

// Device counters of one encoder state (advanced once per chunk on the
// device, so a captured chunk graph replays correctly).
enum EncoderCounter : int {
  kCtrFramesSeen = 0,  // encoder frames processed before the current chunk
  kCtrChunk = 1,       // chunks processed before the current chunk
  kNumCounters = 4,
};

// Residual add + LayerNorm over rows of the f32 residual stream.
//   mode 0: res += scale * y     mode 1: res = y     mode 2: res unchanged
//   r = res;  o1 = T(LN1(T(r)))
//   second stage absent:   res = r, out = o1
//   second stage present:  res = o1 (the block output), then
//     out_kind 0: out = T(LN2(o1))
//     out_kind 1: out[:, :D] = o1, out[:, D + prompt] = 1, other prompt columns 0
struct LnArgs {
  float* res;
  const void* y;
  int ldy;
  float scale;
  int mode;
  const void* w1;
  const void* b1;
  const void* w2;  // second LayerNorm (nullptr: none)
  const void* b2;
  void* out;
  int ldo;
  int out_kind;
  const int* prompt_ids;  // [streams], out_kind 1
  int num_prompts;
  int rows_per_stream;
  int rows, D;
  float eps;
  // bf16 only, out_kind 0: also the f16 copy [rows, D] and per-row scales the
  // tensor-core GEMM takes as its activations (what qgemm_prepass computes
  // from `out`), so the next linear skips its prepass.  nullptr: none.
  void* out16;
  float* scale16;
};
cudaError_t launch_layernorm(int dtype, const LnArgs& a, cudaStream_t stream, bool pdl);

// Relative-position multi-head attention core for one chunk of every stream,
// with the sliding K/V window kept as a ring of `ring` frames per stream.
struct AttnArgs {
  const void* qkv;  // [S*Q, 3D] T: q | k | v
  int ldqkv;
  const void* relk;      // [vmax + Qmax - 1, D] T; row i holds position (vmax - 1 - i)
  const float* bias_u;   // [D]
  const float* bias_v;   // [D]
  void* kring;           // [S][ring][D] T
  void* vring;           // [S][ring][D] T
  void* out;             // [S*Q, D] T
  const int* counters;
  int S, Q, D, heads, head_dim, ring, cache_frames, vmax;
  int qsplit;  // CTAs per (stream, head), each taking ceil(Q / qsplit) queries
  float scale;
};
// Dynamic shared memory of one attention CTA holding `rows_q` queries.
size_t attention_smem_bytes(int rows_q, int vmax, int head_dim);
// Query groups per (stream, head): one CTA per 16 queries (the MMA row tile).
int attention_qsplit(int streams, int heads, int Q, int num_sms);
cudaError_t launch_attention(int dtype, const AttnArgs& a, cudaStream_t stream, bool pdl);

// Conformer convolution core: GLU -> causal depthwise conv (K taps, cache of
// K-1 frames, ping-pong by chunk parity) -> LayerNorm -> SiLU.
struct ConvArgs {
  const void* pw1;  // [S*Q, 2D] T
  int ldp;
  const void* dw_wt;  // [K][D] T (the artifact's [D, 1, K] kernel transposed)
  const void* dw_b;  // [D] T
  const void* ln_w;
  const void* ln_b;
  void* cache;  // [2][S][K-1][D] T
  void* out;    // [S*Q, D] T
  const int* counters;
  int S, Q, D, K;
  float eps;  void* out16;     // bf16 only: f16 copy of `out` + per-row scales for the next GEMM
  float* scale16;  // (nullptr: none)
};
cudaError_t launch_conv_module(int dtype, const ConvArgs& a, cudaStream_t stream, bool pdl);

// Causal stride-2 3x3 Conv2D of the subsampling: the stem (one input channel,
// f32 log-mel input) or a depthwise stage (groups = channels).  The time cache
// holds one input frame per stream (ping-pong by chunk parity); the first
// chunk also sees one extra leading zero frame.
struct Conv2dArgs {
  const void* in;  // stem: f32 [S][Tin][Fin]; depthwise: T [S][Tin][Fin][C]
  int Tin, Fin, valid_in;  // input frames >= valid_in read as zero
  const void* w;           // [C][3][3] T
  const void* b;           // [C] T
  void* cache;             // [2][S][Fin][Cin] T
  void* out;               // [S][Tout][Fout][C] T
  int Tout, Fout, valid_out;  // stem: frames >= valid_out written as zero, then ReLU
  const int* counters;
  int S, C;
};
// C / 8 divides the Conv2D kernels' 256 threads (C = 8, 16, ..., 2048).
bool conv2d_channels_ok(int C);
cudaError_t launch_stem_conv(int dtype, const Conv2dArgs& a, cudaStream_t stream, bool pdl);
cudaError_t launch_depthwise_conv2d(int dtype, const Conv2dArgs& a, cudaStream_t stream, bool pdl);

// [S*T*F, C] -> [S*T, C*F] (channel-major flattening); frames >= valid -> 0.
cudaError_t launch_flatten_cf(int dtype, const void* in, void* out, int S, int T, int F, int C,
                              int valid, cudaStream_t stream, bool pdl);

// counters[frames_seen] += frames, counters[chunk] += 1.
cudaError_t launch_advance_counters(int* counters, int frames, cudaStream_t stream, bool pdl);

// Seeded N(mean, std) fill of an f32 device buffer (synthetic weights).
cudaError_t launch_fill_normal(float* out, size_t n, uint64_t seed, float mean, float std,
                               cudaStream_t stream);

}  // namespace cq
