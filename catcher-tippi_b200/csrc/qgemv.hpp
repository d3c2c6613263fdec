// Host-side interface of the K1 dequant-GEMV (qgemv.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace cq {

struct GemvArgs {
  const void* x;       // T [M, ldx], 16-byte aligned rows
  const void* scales;  // T [N, K/g]
  const void* biases;  // T [N, K/g]
  const void* bias;    // T [N] or nullptr
  void* y;             // T [M, ldy]
  int* status;         // device status word (watchdog)
  int M, N, K, ldx, ldy;
  int sb_per_cta;      // 64-wide K sub-blocks per CTA
  int act;             // cq::Act
  int mode;            // kGemvPlain, kGemvJointInput or kGemvGreedy (RnntEpilogue)
};

// Epilogues of the batched RNNT decoder's two per-symbol linears
// (StreamingRnntDecoder::decode_frames, rnnt.rs:364-388), so that the joint
// input and the greedy choice need no launches of their own:
//  * kGemvJointInput (decoder projector, y = dec_new): active streams take
//    dec = y, then fused = T(relu(enc + dec)) for every stream;
//  * kGemvGreedy (vocabulary head; no logits are stored): each CTA folds its
//    logits into a per-stream 64-bit maximum of (ordered value, ~index) --
//    the first index of the largest logit, MLX argmax.  Unless `defer` hands
//    the choice to the next launch, the last CTA to finish records the token
//    (or retires the stream on blank) and either writes its id to last_token
//    or gathers the next embedding row into x.
enum GemvMode : int { kGemvPlain = 0, kGemvJointInput = 1, kGemvGreedy = 2 };
struct RnntEpilogue {
  int* active;  // [S] stream still emitting on this frame
  // joint input
  const void* enc;  // T: this frame's encoder projection, row s at enc + s * ld_enc
  int ld_enc;
  void* dec;    // T [S, ldy]: decoder output kept per stream
  void* fused;  // T [S, ldy]: relu(enc + dec), the head's input
  // greedy choice
  unsigned long long* best;  // [S] (zero between calls)
  unsigned* done;            // [M / 16] CTAs finished per token tile (zero between calls)
  int blank;
  const void* emb;  // T [V, H] dequantised embedding
  int H;
  void* x;  // T [S, H]: the prediction network's next input
  // When set, the emitted token id goes here instead of its embedding row
  // into x (layer 0 then reads its ih product from a per-token table).
  int* last_token;  // [S] or nullptr
  // Deferred: the head only folds its logits into `best`; the next LSTM step
  // decodes the tokens and updates the flags (no arrival counter, no finish).
  int defer;
  int* tokens;
  int* token_frames;
  int* counts;
  int cap, frame;
};

// Work decomposition: RB = 16*rt weight rows per CTA, K split across a
// cluster of `ksplit` CTAs, each owning `sb_per_cta` sub-blocks of 64.
struct GemvPlan {
  int rt;
  int ksplit;
  int sb_per_cta;
  int num_sms;  // of the device the plan is for (bounds grid.z to one wave)
};

// Up to kGemvMaxGroup linears of one shape (N, K, M, group, plan) in one
// launch: grid.y runs over the bands of every member, each member with its own
// weights, scales, input and output (e.g. an LSTM step's independent ih / hh).
constexpr int kGemvMaxGroup = 4;
struct GemvMaps {
  CUtensorMap m[kGemvMaxGroup];
};
struct GemvGroup {
  GemvArgs a[kGemvMaxGroup];
  int count;
};

GemvPlan plan_gemv(int N, int K, int num_sms);
// The plan for a call with M rows: the base plan (chosen for one 16-row token
// tile) unless several token tiles would not fit one wave of two CTAs per SM;
// then taller weight bands (32 or 64 rows) leave room for the tiles to run
// side by side on grid.z, so each CTA reads its tokens' activations once.
GemvPlan plan_gemv_rows(const GemvPlan& base, int N, int M);
cudaError_t launch_gemv(int dtype, int group, const GemvPlan& plan, const CUtensorMap& wmap,
                        const GemvArgs& args, cudaStream_t stream, bool pdl);
cudaError_t launch_gemv_group(int dtype, int group, const GemvPlan& plan, const GemvMaps& maps,
                              const GemvGroup& g, cudaStream_t stream, bool pdl,
                              const RnntEpilogue* epi = nullptr);

}  // namespace cq
