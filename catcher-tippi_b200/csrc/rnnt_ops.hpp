// Host-side interface of the RNNT decoder's supporting kernels (rnnt_ops.cu).
#pragma once

#include <cuda.h>

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace cq {

// fused[s] = T(relu(enc[s] + dec[s])) over J columns; `update`: active
// streams first copy dec_new into dec; `reset`: every stream becomes active.
cudaError_t launch_joint_input(int dtype, const void* enc, int ld_enc, const void* dec_new, void* dec,
                               void* fused, int* active, int S, int J, bool update, bool reset,
                               cudaStream_t stream, bool pdl);

// Per active stream: token = argmax(logits[s]); blank clears `active`,
// otherwise the token (and `frame`) is appended to the stream's list and its
// embedding row is copied to x[s].
cudaError_t launch_argmax_emit(int dtype, const void* logits, int ld, int V, int blank, int* active,
                               const void* emb, int H, void* x, int* tokens, int* frames,
                               int* counts, int cap, int frame, int S, cudaStream_t stream,
                               bool pdl);

// LSTM cell update from the two projections' outputs (active streams, or all).
cudaError_t launch_lstm_cell(int dtype, const void* gi, const void* gh, const void* bias, void* h,
                             void* c, const int* active, int S, int H, bool all, cudaStream_t stream,
                             bool pdl);

// p[0..n) = 0 (a kernel node, so the next launch may depend on it programmatically).
cudaError_t launch_zero_ints(int* p, int n, cudaStream_t stream);

// x[s] = table[row] for every stream (16-bit elements).
cudaError_t launch_broadcast_row(const void* table, int row, int H, void* x, int S,
                                 cudaStream_t stream);

// ---------------------------------------------------------------- persistent chunk kernel

constexpr int kRnntMaxLayers = 4;

// Everything one cooperative launch needs to decode a whole chunk
// (rnnt_persistent.cu).  Weights in the MLX layout (u8 [N, K], T scales and
// biases [N, K/g]); activations and state T.
struct RnntChunkArgs {
  const uint8_t* head_q;
  const void *head_s, *head_b, *head_bias;  // [V, J]
  const uint8_t* ih_q[kRnntMaxLayers];
  const void *ih_s[kRnntMaxLayers], *ih_b[kRnntMaxLayers];  // [4H, H]
  const uint8_t* hh_q[kRnntMaxLayers];
  const void *hh_s[kRnntMaxLayers], *hh_b[kRnntMaxLayers];
  const void* lstm_bias[kRnntMaxLayers];  // [4H], bias_ih + bias_hh in T
  const uint8_t* proj_q;
  const void *proj_s, *proj_b, *proj_bias;  // [J, H]
  const void* emb;                          // [V, H] dequantised
  const void* ep;                           // [S * Q, J] encoder projection of the chunk
  void* h[kRnntMaxLayers][2];               // [S, H] ping-pong; buffer 0 holds the state between chunks
  void* c[kRnntMaxLayers];                  // [S, H]
  void* dec;                                // [S, J] decoder output
  void* fused;                              // [S, J] joint input
  float2* part;                             // [ceil(V/16), S] per-tile (max logit, index)
  int *tokens, *token_frames, *counts;
  int cap;
  unsigned* barrier;  // {count, abort}, zero before the launch
  int* status;
  int S, Q, H, J, V, blank, max_symbols, layers, group;
};

// Grid size (CTAs) for S streams, 0 if the kernel cannot be used (shared
// memory or co-residency); smem bytes for that grid.
int rnnt_chunk_grid(int dtype, int S, int H, int J, int V, int layers, int num_sms);
size_t rnnt_chunk_smem_bytes(int S, int H, int J, int V, int layers, int grid);
cudaError_t launch_rnnt_chunk(int dtype, const RnntChunkArgs& a, int grid, cudaStream_t stream);

// One LSTM layer of a prediction step in one launch (rnnt_lstm.cu): the ih and
// hh products of a 64-row band of gate-interleaved weights (row 4j + q = gate
// q of hidden unit j) on a two-CTA cluster, then the cell.
struct LstmMaps {
  CUtensorMap m[2];   // interleaved W_ih, W_hh: box 64 k x 64 rows
  CUtensorMap m5[2];  // the same with box 64 k x 80 rows (valid if has_m5)
  int has_m5;
};
struct LstmStepArgs {
  const void* x;       // T [S, H]: the layer input
  const void* h_prev;  // T [S, H]: the layer's hidden state before the step
  void* h_out;         // T [S, H]: after the step (not h_prev)
  void* c;             // T [S, H]: cell state, updated in place
  const void* scales_ih;  // T [4H, H/g], interleaved rows
  const void* biases_ih;
  const void* scales_hh;
  const void* biases_hh;
  const void* gate_bias;  // T [4H] interleaved, T(b_ih) + T(b_hh) rounded to T
  const int* active;      // [S]
  int all;                // update every stream
  int* status;
  int S, H;
  // Layer 0's input is always an embedding row, so its ih product is a
  // function of the token: with gi_table set, a launch reads
  // gi_table[gi_token[s]] (T [V, 4H], interleaved) instead of multiplying,
  // one CTA per band and no cluster.  With gi_out set, a launch only writes
  // T(W_ih x) (T [S, 4H], interleaved) -- how the table is made, by the same
  // arithmetic -- and leaves the state alone.
  const void* gi_table;
  const int* gi_token;  // [S]
  void* gi_out;
  // Greedy choice deferred from the head (layer 0 with gi_table): the token
  // of stream s decodes from greedy_best[s] (ordered logit << 32 | ~index,
  // 0: index 0); a stream steps if it was active and the token is not blank.
  // The CTAs of band 0 record it: active, tokens, token_frames, counts.
  const unsigned long long* greedy_best;  // [S] or nullptr
  int* greedy_active;                     // [S]
  int greedy_blank;
  int* tokens;        // [S, cap]
  int* token_frames;  // [S, cap]
  int* counts;        // [S]
  int cap, frame;
  // A later layer's band 0 zeroes the keys for the next head (or nullptr).
  unsigned long long* clear_best;
};
bool lstm_step_fits(int H, int group);
cudaError_t launch_lstm_step(int dtype, int group, const LstmMaps& maps, const LstmStepArgs& a,
                             cudaStream_t stream, bool pdl);

}  // namespace cq
