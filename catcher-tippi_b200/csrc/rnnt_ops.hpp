// Host-side interface of the RNNT decoder's supporting kernels (rnnt_ops.cu).
#pragma once

#include <cuda_runtime.h>

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

}  // namespace cq
