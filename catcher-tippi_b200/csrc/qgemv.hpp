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
size_t gemv_smem_bytes(const GemvPlan& plan, int group);
cudaError_t launch_gemv(int dtype, int group, const GemvPlan& plan, const CUtensorMap& wmap,
                        const GemvArgs& args, cudaStream_t stream, bool pdl);
cudaError_t launch_gemv_group(int dtype, int group, const GemvPlan& plan, const GemvMaps& maps,
                              const GemvGroup& g, cudaStream_t stream, bool pdl);

}  // namespace cq
