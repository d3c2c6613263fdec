// Elementwise and selection kernels of the batched RNNT greedy decoder
// (crates/nemotron-mlx/src/model/rnnt.rs).  The quantized linears in between
// (encoder / decoder projectors, LSTM input and recurrent projections, joint
// head) run through QuantizedLinear.  Streams advance in lock step over the
// frames of a chunk; a per-stream `active` flag stands for "has not emitted
// blank on this frame yet", so every stream follows its own greedy path while
// the launch sequence stays fixed (and graph-capturable).
#include "common.cuh"
#include "rnnt_ops.hpp"

namespace cq {
namespace {

template <typename Kern, typename... Args>
cudaError_t launch_ex(Kern kern, dim3 grid, dim3 block, cudaStream_t stream, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// fused[s] = T(relu(enc[s] + dec[s])): JointNetwork::score adds the two
// projections in f32 and applies ReLU (rnnt.rs:321-333); the head linear then
// casts to T.  With `update`, active streams first take dec = dec_new (the
// projector output of their new token); with `reset`, every stream becomes
// active (a new frame).
template <int DT>
__global__ void joint_input_kernel(const void* enc, int ld_enc, const void* dec_new, void* dec,
                                   void* fused, int* active, int S, int J, int update, int reset) {
  pdl_wait();
  pdl_launch_dependents();
  const int s = blockIdx.x;
  if (s >= S) return;
  const bool act = reset ? true : active[s] != 0;
  for (int j = threadIdx.x; j < J; j += blockDim.x) {
    const size_t o = static_cast<size_t>(s) * J + j;
    float d;
    if (update && act) {
      d = ld_t<DT>(dec_new, o);
      st_t<DT>(dec, o, d);
    } else {
      d = ld_t<DT>(dec, o);
    }
    const float e = ld_t<DT>(enc, static_cast<size_t>(s) * ld_enc + j);
    st_t<DT>(fused, o, fmaxf(e + d, 0.0f));
  }
  if (reset && threadIdx.x == 0) active[s] = 1;
}

// Greedy choice of one stream: the first index of the largest logit (MLX
// argmax).  Blank ends the stream's frame; any other token is recorded and its
// embedding row becomes the prediction network's next input.
template <int DT>
__global__ void __launch_bounds__(256)
    argmax_emit_kernel(const void* logits, int ld, int V, int blank, int* active, const void* emb,
                       int H, void* x, int* tokens, int* frames, int* counts, int cap, int frame) {
  __shared__ float best_v[8];
  __shared__ int best_i[8];
  pdl_wait();
  pdl_launch_dependents();
  const int s = blockIdx.x;
  if (!active[s]) return;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = ld_t<DT>(logits, static_cast<size_t>(s) * ld + i);
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    best_v[warp] = bv;
    best_i[warp] = bi;
  }
  __syncthreads();
  bv = best_v[0];
  bi = best_i[0];
  for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
    if (best_v[w] > bv || (best_v[w] == bv && best_i[w] < bi)) {
      bv = best_v[w];
      bi = best_i[w];
    }
  if (bi >= V) bi = 0;  // every logit NaN: MLX returns index 0
  if (bi == blank) {
    __syncthreads();
    if (threadIdx.x == 0) active[s] = 0;
    return;
  }
  const int n = counts[s];
  if (threadIdx.x == 0) {
    if (n < cap) {
      tokens[static_cast<size_t>(s) * cap + n] = bi;
      frames[static_cast<size_t>(s) * cap + n] = frame;
    }
    counts[s] = n + 1;
  }
  const uint16_t* src = static_cast<const uint16_t*>(emb) + static_cast<size_t>(bi) * H;
  uint16_t* dst = static_cast<uint16_t*>(x) + static_cast<size_t>(s) * H;
  for (int j = threadIdx.x; j < H; j += blockDim.x) dst[j] = src[j];
}

// LstmCell::step_f32 (rnnt.rs:113-148) for active streams: every MLX op
// rounds to T.  gates = (ih + hh) + bias; i, f, o = sigmoid, g = tanh (PyTorch
// order i, f, g, o); c = f*c + i*g; h = o * tanh(c).
template <int DT>
__global__ void lstm_cell_kernel(const void* gi, const void* gh, const void* bias, void* h, void* c,
                                 const int* active, int S, int H, int all) {
  pdl_wait();
  pdl_launch_dependents();
  const int s = blockIdx.y;
  if (!all && !active[s]) return;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < H; j += gridDim.x * blockDim.x) {
    const size_t g0 = static_cast<size_t>(s) * 4 * H;
    float gate[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const size_t o = g0 + static_cast<size_t>(q) * H + j;
      gate[q] = round_t<DT>(round_t<DT>(ld_t<DT>(gi, o) + ld_t<DT>(gh, o)) +
                            ld_t<DT>(bias, static_cast<size_t>(q) * H + j));
    }
    const float i = round_t<DT>(1.0f / (1.0f + expf(-gate[0])));
    const float f = round_t<DT>(1.0f / (1.0f + expf(-gate[1])));
    const float g = round_t<DT>(tanhf(gate[2]));
    const float o = round_t<DT>(1.0f / (1.0f + expf(-gate[3])));
    const size_t hj = static_cast<size_t>(s) * H + j;
    const float c_prev = ld_t<DT>(c, hj);
    const float c_new = round_t<DT>(round_t<DT>(f * c_prev) + round_t<DT>(i * g));
    const float h_new = round_t<DT>(o * round_t<DT>(tanhf(c_new)));
    st_t<DT>(c, hj, c_new);
    st_t<DT>(h, hj, h_new);
  }
}

// Every stream's prediction input = the blank embedding row (the first
// PredictionNetwork::step of a new utterance, rnnt.rs:273-290).
__global__ void broadcast_row_kernel(const uint16_t* emb, int row, int H, uint16_t* x, int S) {
  const int s = blockIdx.x;
  for (int j = threadIdx.x; j < H; j += blockDim.x)
    x[static_cast<size_t>(s) * H + j] = emb[static_cast<size_t>(row) * H + j];
}

__global__ void zero_ints_kernel(int* p, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = 0;
}

}  // namespace

cudaError_t launch_zero_ints(int* p, int n, cudaStream_t stream) {
  zero_ints_kernel<<<(n + 255) / 256, 256, 0, stream>>>(p, n);
  return cudaGetLastError();
}

cudaError_t launch_joint_input(int dtype, const void* enc, int ld_enc, const void* dec_new, void* dec,
                               void* fused, int* active, int S, int J, bool update, bool reset,
                               cudaStream_t stream, bool pdl) {
  auto k = dtype == kBF16 ? joint_input_kernel<kBF16> : joint_input_kernel<kF16>;
  return launch_ex(k, dim3(S), dim3(128), stream, pdl, enc, ld_enc, dec_new, dec, fused, active, S, J,
                   update ? 1 : 0, reset ? 1 : 0);
}

cudaError_t launch_argmax_emit(int dtype, const void* logits, int ld, int V, int blank, int* active,
                               const void* emb, int H, void* x, int* tokens, int* frames,
                               int* counts, int cap, int frame, int S, cudaStream_t stream,
                               bool pdl) {
  auto k = dtype == kBF16 ? argmax_emit_kernel<kBF16> : argmax_emit_kernel<kF16>;
  return launch_ex(k, dim3(S), dim3(256), stream, pdl, logits, ld, V, blank, active, emb, H, x,
                   tokens, frames, counts, cap, frame);
}

cudaError_t launch_lstm_cell(int dtype, const void* gi, const void* gh, const void* bias, void* h,
                             void* c, const int* active, int S, int H, bool all, cudaStream_t stream,
                             bool pdl) {
  auto k = dtype == kBF16 ? lstm_cell_kernel<kBF16> : lstm_cell_kernel<kF16>;
  const int bx = (H + 255) / 256;
  return launch_ex(k, dim3(bx, S), dim3(256), stream, pdl, gi, gh, bias, h, c, active, S, H,
                   all ? 1 : 0);
}

cudaError_t launch_broadcast_row(const void* table, int row, int H, void* x, int S,
                                 cudaStream_t stream) {
  broadcast_row_kernel<<<S, 128, 0, stream>>>(static_cast<const uint16_t*>(table), row, H,
                                              static_cast<uint16_t*>(x), S);
  return cudaGetLastError();
}

}  // namespace cq
