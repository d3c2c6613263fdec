// Device interface of the persistent linear-chain executor (qchain.cu): a
// sequence of small-M quantized linears, each possibly reading the output of
// earlier ones, run as ONE cooperative launch.  Every CTA streams the weight
// tiles of its share of all steps through a ring of shared-memory slots ahead
// of time (weights do not depend on activations), and waits only for the
// completion counters of the steps whose outputs it reads.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace cq {

constexpr int kChainMaxDeps = 3;

struct ChainStep {
  const CUtensorMap* wmap;  // device copy; box 64 k x 16*rt rows, no swizzle
  const void* scales;       // T [N, K/g]
  const void* biases;       // T [N, K/g]
  const void* bias;         // T [N] or nullptr
  const void* x;            // T [M, ldx]
  void* y;                  // T [M, ldy]
  float* partial;           // [units][kslices][16*rt][16] f32 when kslices > 1
  unsigned* arrive;         // [units] K-split arrival counters when kslices > 1
  int ldx, ldy, M, N, K, act;
  int rt;                   // weight rows per item = 16 * rt (1 or 2)
  int sb_per_item;          // 64-wide K sub-blocks per item
  int kslices, bands, mtiles;
  int item_base, items;     // global item range of this step
  int units;                // bands * mtiles completions finish the step
  int dep[kChainMaxDeps];   // earlier steps whose completion this one awaits (-1: none)
  int evict_first;          // weights are read by one item only
  int signal;               // some later step waits for this one's completion count
  // Tagged copies: a word holds two adjacent output values (low 32 bits) and
  // the launch's tag (high 32 bits), stored as one 8-byte write, so a reader
  // that sees the tag sees the values -- no separate completion flag.
  const unsigned long long* x_tagged;  // the producer's tagged output this step reads, or null
  int x_tagged_ld;                     // words per row
  int x_tagged_col;                    // word of column 0 of x
  unsigned long long* y_tagged;        // tagged copy of this step's output, or null
  int y_tagged_ld;                     // words per row
};

struct ChainArgs {
  const ChainStep* steps;
  int nsteps;
  int total_items;
  unsigned* done;        // [nsteps] completed units per step (zero between launches)
  unsigned* arrive;      // [narrive] every step's K-split arrival counters
  int narrive;
  unsigned* exit_count;  // CTAs that left the launch (wraps at the grid size)
  int* abort_flag;       // set by a CTA whose bounded wait ran out
  int* status;           // device status word (watchdog)
  unsigned* epoch;       // launches so far; this launch tags its words epoch + 1
  // Optional profile: per item, %globaltimer (ns) when the producer issued its
  // weight copies, when the consumers started it, had their inputs, had the
  // weights, released the slot and finished it.  nullptr: not recorded.
  unsigned long long* trace;  // [total_items][kChainTraceStamps]
};

constexpr int kChainTraceStamps = 6;

constexpr int kChainSlotBytes = 32768;  // weight bytes one item may hold

size_t chain_smem_bytes();
int chain_threads();
cudaError_t chain_set_smem(int dtype, int group);
cudaError_t launch_chain(int dtype, int group, const ChainArgs& args, int grid,
                         cudaStream_t stream);

}  // namespace cq
