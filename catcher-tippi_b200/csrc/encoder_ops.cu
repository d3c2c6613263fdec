// Supporting kernels of the streaming FastConformer encoder on sm_100a:
// residual + LayerNorm, the relative-position attention core with its K/V
// ring, the conformer convolution core, the subsampling convolutions and the
// channel-major flatten.  They restate, with the same rounding points (every
// value handed between the reference's ops is a T value widened to f32):
//   LayerNorm::forward_f32            crates/nemotron-mlx/src/model/layers.rs:492-507
//   DepthwiseConv1d::forward_f32      layers.rs:418-455
//   Fp16Conv2d::forward_causal        layers.rs:142-205
//   RelativePositionAttention         crates/nemotron-mlx/src/model/encoder.rs:183-259
//   ConformerConvolution::forward     encoder.rs:376-397
//   residual_add / silu_in_place      encoder.rs:538-558
//   mask_invalid_time, channel_frequency_flatten  encoder.rs:805-833
//   AttentionKvCache / CausalConv*Cache           crates/nemotron-mlx/src/model/cache.rs
// Everything here is small next to the quantized linears (HBM-bound at one
// stream, tensor-bound at many); the kernels are written for coalesced 2- and
// 16-byte accesses and a short dependent chain (PDL) rather than peak FLOPs.
#include "common.cuh"
#include "encoder_ops.hpp"

namespace cq {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxPerThread = 16;  // rows up to 16 * 256 = 4096 wide

template <typename Kern, typename... Args>
cudaError_t launch_ex(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
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

// Sum over the block; every thread returns the same value (same order).
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();  // red may still be read by a previous reduction
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.0f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

// LayerNorm of one row held in registers (v[k] for column threadIdx.x + k*256,
// already T values); returns T-rounded outputs in o[].
template <int DT>
__device__ __forceinline__ void layernorm_regs(const float (&v)[kMaxPerThread], float (&o)[kMaxPerThread],
                                               int D, const void* w, const void* b, float eps,
                                               float* red) {
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < kMaxPerThread; ++k) {
    const int i = threadIdx.x + k * kThreads;
    if (i < D) s += v[k];
  }
  const float mean = block_sum(s, red) / static_cast<float>(D);
  float sq = 0.0f;
#pragma unroll
  for (int k = 0; k < kMaxPerThread; ++k) {
    const int i = threadIdx.x + k * kThreads;
    if (i < D) {
      const float d = v[k] - mean;
      sq += d * d;
    }
  }
  const float var = block_sum(sq, red) / static_cast<float>(D);
  const float rstd = 1.0f / sqrtf(var + eps);
#pragma unroll
  for (int k = 0; k < kMaxPerThread; ++k) {
    const int i = threadIdx.x + k * kThreads;
    if (i < D) o[k] = round_t<DT>((v[k] - mean) * rstd * ld_t<DT>(w, i) + ld_t<DT>(b, i));
  }
}

// ------------------------------------------------------------------ LayerNorm

template <int DT>
__global__ void __launch_bounds__(kThreads) layernorm_kernel(const LnArgs a) {
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int D = a.D;
  float* res = a.res + static_cast<size_t>(row) * D;
  float r[kMaxPerThread], t[kMaxPerThread], o[kMaxPerThread];
#pragma unroll
  for (int k = 0; k < kMaxPerThread; ++k) {
    const int i = threadIdx.x + k * kThreads;
    r[k] = 0.0f;
    if (i < D) {
      if (a.mode == 1) {
        r[k] = ld_t<DT>(a.y, static_cast<size_t>(row) * a.ldy + i);
      } else {
        r[k] = res[i];
        // residual_add: left + scale * right in f32 (scale 0.5 or 1: the
        // product is exact, so a fused multiply-add rounds identically)
        if (a.mode == 0) r[k] = r[k] + a.scale * ld_t<DT>(a.y, static_cast<size_t>(row) * a.ldy + i);
      }
    }
    t[k] = round_t<DT>(r[k]);  // LayerNorm casts its f32 input to T
  }
  layernorm_regs<DT>(t, o, D, a.w1, a.b1, a.eps, red);
  const bool second = a.w2 != nullptr || a.out_kind == 1;
  if (!second) {
#pragma unroll
    for (int k = 0; k < kMaxPerThread; ++k) {
      const int i = threadIdx.x + k * kThreads;
      if (i < D) {
        if (a.mode != 2) res[i] = r[k];
        st_t<DT>(a.out, static_cast<size_t>(row) * a.ldo + i, o[k]);
      }
    }
    return;
  }
  // o is the block output (norm_out): it becomes the residual stream
#pragma unroll
  for (int k = 0; k < kMaxPerThread; ++k) {
    const int i = threadIdx.x + k * kThreads;
    if (i < D) res[i] = o[k];
  }
  if (a.out_kind == 1) {
#pragma unroll
    for (int k = 0; k < kMaxPerThread; ++k) {
      const int i = threadIdx.x + k * kThreads;
      if (i < D) st_t<DT>(a.out, static_cast<size_t>(row) * a.ldo + i, o[k]);
    }
    const int prompt = a.prompt_ids[row / a.rows_per_stream];
    for (int j = threadIdx.x; j < a.num_prompts; j += kThreads)
      st_t<DT>(a.out, static_cast<size_t>(row) * a.ldo + D + j, j == prompt ? 1.0f : 0.0f);
    return;
  }
  float o2[kMaxPerThread];
  layernorm_regs<DT>(o, o2, D, a.w2, a.b2, a.eps, red);
#pragma unroll
  for (int k = 0; k < kMaxPerThread; ++k) {
    const int i = threadIdx.x + k * kThreads;
    if (i < D) st_t<DT>(a.out, static_cast<size_t>(row) * a.ldo + i, o2[k]);
  }
}

// ------------------------------------------------------------------ attention

struct AttnSmem {
  float *qu, *qv, *k, *v, *r, *p;
};

__host__ __device__ inline size_t attn_floats(int Q, int vmax, int hd, AttnSmem* s, float* base) {
  const int hdp = hd + 1;  // padded rows: row-parallel dot products hit distinct banks
  size_t off = 0;
  auto take = [&](float** dst, size_t n) {
    if (s != nullptr) *dst = base + off;
    off += n;
  };
  float* dummy = nullptr;
  take(s ? &s->qu : &dummy, static_cast<size_t>(Q) * hd);
  take(s ? &s->qv : &dummy, static_cast<size_t>(Q) * hd);
  take(s ? &s->k : &dummy, static_cast<size_t>(vmax) * hdp);
  take(s ? &s->v : &dummy, static_cast<size_t>(vmax) * hd);
  take(s ? &s->r : &dummy, static_cast<size_t>(vmax + Q - 1) * hdp);
  take(s ? &s->p : &dummy, static_cast<size_t>(Q) * vmax);
  return off;
}

// One CTA per (stream, head).  With V visible frames (cached + current) and
// position rows ordered from V-1 down to -(V-1), the reference's relative
// shift (pad, flatten, drop Q entries) reads raw[q][key + Q - 1 - q]; the
// kernel reads that row directly.  Position rows depend only on the position
// value, so one table of vmax + Q - 1 rows serves every V.
template <int DT>
__global__ void __launch_bounds__(kThreads) attention_kernel(const AttnArgs a) {
  extern __shared__ float smem[];
  const int s = blockIdx.x / a.heads;
  const int h = blockIdx.x % a.heads;
  const int hd = a.head_dim, hdp = hd + 1, Q = a.Q, D = a.D, vmax = a.vmax;
  AttnSmem sm;
  attn_floats(Q, vmax, hd, &sm, smem);
  pdl_wait();
  pdl_launch_dependents();
  const int n_prev = a.counters[kCtrFramesSeen];
  const int cached = min(n_prev, a.cache_frames);
  const int V = cached + Q;
  const int col = h * hd;
  const size_t row0 = static_cast<size_t>(s) * Q;

  for (int i = threadIdx.x; i < Q * hd; i += kThreads) {
    const int q = i / hd, d = i % hd;
    const float x = ld_t<DT>(a.qkv, (row0 + q) * a.ldqkv + col + d);
    sm.qu[i] = x + a.bias_u[col + d];
    sm.qv[i] = x + a.bias_v[col + d];
  }
  for (int i = threadIdx.x; i < V * hd; i += kThreads) {
    const int j = i / hd, d = i % hd;
    float kx, vx;
    if (j < cached) {
      const int slot = (n_prev - cached + j) % a.ring;
      const size_t off = (static_cast<size_t>(s) * a.ring + slot) * D + col + d;
      kx = ld_t<DT>(a.kring, off);
      vx = ld_t<DT>(a.vring, off);
    } else {
      const size_t off = (row0 + (j - cached)) * a.ldqkv + col + d;
      kx = ld_t<DT>(a.qkv, off + D);
      vx = ld_t<DT>(a.qkv, off + 2 * static_cast<size_t>(D));
    }
    sm.k[j * hdp + d] = kx;
    sm.v[j * hd + d] = vx;
  }
  const int np = V + Q - 1;
  const int rbase = vmax - V;  // table row of position V-1
  for (int i = threadIdx.x; i < np * hd; i += kThreads) {
    const int p = i / hd, d = i % hd;
    sm.r[p * hdp + d] = ld_t<DT>(a.relk, static_cast<size_t>(rbase + p) * D + col + d);
  }
  __syncthreads();

  // scores[q][key] = ((q + bias_u) . k + (q + bias_v) . rel[key + Q - 1 - q]) * scale
  for (int pr = threadIdx.x; pr < Q * V; pr += kThreads) {
    const int q = pr / V, j = pr % V;
    const float* qu = sm.qu + q * hd;
    const float* qv = sm.qv + q * hd;
    const float* kr = sm.k + j * hdp;
    const float* rr = sm.r + (j + Q - 1 - q) * hdp;
    float c = 0.0f, r = 0.0f;
#pragma unroll 8
    for (int d = 0; d < hd; ++d) {
      c = fmaf(qu[d], kr[d], c);
      r = fmaf(qv[d], rr[d], r);
    }
    sm.p[q * vmax + j] = (c + r) * a.scale;
  }
  __syncthreads();

  // softmax_in_place per query row (encoder.rs:278-288)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int q = warp; q < Q; q += kThreads / 32) {
    float* row = sm.p + q * vmax;
    float m = -INFINITY;
    for (int j = lane; j < V; j += 32) m = fmaxf(m, row[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float tot = 0.0f;
    for (int j = lane; j < V; j += 32) {
      const float e = expf(row[j] - m);
      row[j] = e;
      tot += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    for (int j = lane; j < V; j += 32) row[j] = row[j] / tot;
  }
  __syncthreads();

  for (int o = threadIdx.x; o < Q * hd; o += kThreads) {
    const int q = o / hd, d = o % hd;
    const float* pr = sm.p + q * vmax;
    float acc = 0.0f;
    for (int j = 0; j < V; ++j) acc = fmaf(pr[j], sm.v[j * hd + d], acc);
    st_t<DT>(a.out, (row0 + q) * D + col + d, acc);
  }

  // Append this chunk's keys and values to the window (AttentionKvCache::update).
  // The ring holds cache_frames + Q frames, so these slots are not the ones read above.
  const uint16_t* src = reinterpret_cast<const uint16_t*>(a.qkv);
  uint16_t* kr = reinterpret_cast<uint16_t*>(a.kring);
  uint16_t* vr = reinterpret_cast<uint16_t*>(a.vring);
  for (int i = threadIdx.x; i < Q * hd; i += kThreads) {
    const int t = i / hd, d = i % hd;
    const int slot = (n_prev + t) % a.ring;
    const size_t dst = (static_cast<size_t>(s) * a.ring + slot) * D + col + d;
    const size_t off = (row0 + t) * a.ldqkv + col + d;
    kr[dst] = src[off + D];
    vr[dst] = src[off + 2 * static_cast<size_t>(D)];
  }
}

// ------------------------------------------------------------------ conv module

template <int DT>
__global__ void __launch_bounds__(kThreads) conv_module_kernel(const ConvArgs a) {
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int s = row / a.Q, t = row % a.Q;
  const int D = a.D, K = a.K, Q = a.Q;
  const int par = a.counters[kCtrChunk] & 1;
  const size_t per_stream = static_cast<size_t>(K - 1) * D;
  const uint16_t* old_c =
      reinterpret_cast<const uint16_t*>(a.cache) + (static_cast<size_t>(par) * a.S + s) * per_stream;
  uint16_t* new_c =
      reinterpret_cast<uint16_t*>(a.cache) + (static_cast<size_t>(1 - par) * a.S + s) * per_stream;
  float dv[kMaxPerThread], o[kMaxPerThread];
#pragma unroll
  for (int k = 0; k < kMaxPerThread; ++k) {
    const int i = threadIdx.x + k * kThreads;
    dv[k] = 0.0f;
    if (i < D) {
      float acc = 0.0f, g_t = 0.0f;
      for (int tap = 0; tap < K; ++tap) {
        const int f = t - (K - 1) + tap;
        float g;
        if (f >= 0) {
          // GLU: first / (1 + exp(-gate)) in f32, cast to T by the convolution
          const size_t off = (static_cast<size_t>(s) * Q + f) * a.ldp;
          const float first = ld_t<DT>(a.pw1, off + i);
          const float gate = ld_t<DT>(a.pw1, off + D + i);
          g = round_t<DT>(first / (1.0f + expf(-gate)));
        } else {
          g = ld_t<DT>(old_c, static_cast<size_t>(K - 1 + f) * D + i);
        }
        acc = fmaf(ld_t<DT>(a.dw_w, static_cast<size_t>(i) * K + tap), g, acc);
        g_t = g;
      }
      dv[k] = round_t<DT>(round_t<DT>(acc) + ld_t<DT>(a.dw_b, i));
      // new cache = last K-1 frames of (old cache ++ this chunk)
      if (t >= Q - (K - 1)) st_t<DT>(new_c, static_cast<size_t>(t - Q + K - 1) * D + i, g_t);
      if (t == 0)
        for (int j = 0; j < K - 1 - Q; ++j)
          new_c[static_cast<size_t>(j) * D + i] = old_c[static_cast<size_t>(Q + j) * D + i];
    }
  }
  layernorm_regs<DT>(dv, o, D, a.ln_w, a.ln_b, a.eps, red);
#pragma unroll
  for (int k = 0; k < kMaxPerThread; ++k) {
    const int i = threadIdx.x + k * kThreads;
    if (i < D) {
      const float n = o[k];
      st_t<DT>(a.out, static_cast<size_t>(row) * D + i, n / (1.0f + expf(-n)));
    }
  }
}

// ------------------------------------------------------------------ subsampling

// Combined-frame index jc (0-based over [extra zeros | cache | input]) of the
// causal time axis -> -2: zero, -1: cache frame, >= 0: input frame.
__device__ __forceinline__ int time_source(int jc, bool first) {
  if (first) {
    if (jc == 0) return -2;
    jc -= 1;
  }
  return jc == 0 ? -1 : jc - 1;
}

template <int DT>
__global__ void __launch_bounds__(kThreads) stem_conv_kernel(const Conv2dArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int chunk = a.counters[kCtrChunk];
  const bool first = chunk == 0;
  const int par = chunk & 1;
  const int CG = a.C / 8;
  const float* mel = static_cast<const float*>(a.in);
  const size_t total = static_cast<size_t>(a.S) * a.Tout * a.Fout * CG;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += stride) {
    const int cg = static_cast<int>(idx % CG);
    size_t rest = idx / CG;
    const int f = static_cast<int>(rest % a.Fout);
    rest /= a.Fout;
    const int t = static_cast<int>(rest % a.Tout);
    const int s = static_cast<int>(rest / a.Tout);
    float x[9];
#pragma unroll
    for (int kt = 0; kt < 3; ++kt) {
      const int src = time_source(2 * t + kt, first);
#pragma unroll
      for (int kf = 0; kf < 3; ++kf) {
        const int bin = 2 * f + kf - 2;  // frequency padded 2 left, 1 right
        float v = 0.0f;
        if (src != -2 && bin >= 0 && bin < a.Fin) {
          if (src == -1) {
            v = ld_t<DT>(a.cache, (static_cast<size_t>(par) * a.S + s) * a.Fin + bin);
          } else if (src < a.valid_in) {
            v = round_t<DT>(mel[(static_cast<size_t>(s) * a.Tin + src) * a.Fin + bin]);
          }
        }
        x[kt * 3 + kf] = v;
      }
    }
    const int c0 = cg * 8;
    uint16_t packed[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float acc = 0.0f;
#pragma unroll
      for (int tap = 0; tap < 9; ++tap)
        acc = fmaf(ld_t<DT>(a.w, static_cast<size_t>(c0 + c) * 9 + tap), x[tap], acc);
      float o = round_t<DT>(round_t<DT>(acc) + ld_t<DT>(a.b, c0 + c));
      if (t >= a.valid_out) o = 0.0f;  // mask_invalid_time, then ReLU
      o = o > 0.0f ? o : 0.0f;
      if constexpr (DT == kBF16) packed[c] = __bfloat16_as_ushort(__float2bfloat16_rn(o));
      else packed[c] = __half_as_ushort(__float2half_rn(o));
    }
    uint4 w;
    w.x = packed[0] | (static_cast<uint32_t>(packed[1]) << 16);
    w.y = packed[2] | (static_cast<uint32_t>(packed[3]) << 16);
    w.z = packed[4] | (static_cast<uint32_t>(packed[5]) << 16);
    w.w = packed[6] | (static_cast<uint32_t>(packed[7]) << 16);
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) +
                              ((static_cast<size_t>(s) * a.Tout + t) * a.Fout + f) * a.C + c0) = w;
  }
  // next chunk's cache: the last input frame
  const size_t ncache = static_cast<size_t>(a.S) * a.Fin;
  for (size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < ncache;
       idx += stride) {
    const int s = static_cast<int>(idx / a.Fin), bin = static_cast<int>(idx % a.Fin);
    const int fr = a.Tin - 1;
    const float v = fr < a.valid_in ? round_t<DT>(mel[(static_cast<size_t>(s) * a.Tin + fr) * a.Fin + bin]) : 0.0f;
    st_t<DT>(a.cache, (static_cast<size_t>(1 - par) * a.S + s) * a.Fin + bin, v);
  }
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&x)[8], int DT) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint16_t lo = static_cast<uint16_t>(w[i] & 0xFFFFu), hi = static_cast<uint16_t>(w[i] >> 16);
    if (DT == kBF16) {
      x[2 * i] = __uint_as_float(static_cast<uint32_t>(lo) << 16);
      x[2 * i + 1] = __uint_as_float(static_cast<uint32_t>(hi) << 16);
    } else {
      x[2 * i] = __half2float(__ushort_as_half(lo));
      x[2 * i + 1] = __half2float(__ushort_as_half(hi));
    }
  }
}

template <int DT>
__global__ void __launch_bounds__(kThreads) depthwise_conv2d_kernel(const Conv2dArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int chunk = a.counters[kCtrChunk];
  const bool first = chunk == 0;
  const int par = chunk & 1;
  const int C = a.C, CG = C / 8;
  const uint16_t* in = static_cast<const uint16_t*>(a.in);
  uint16_t* cache = static_cast<uint16_t*>(a.cache);
  const size_t total = static_cast<size_t>(a.S) * a.Tout * a.Fout * CG;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += stride) {
    const int cg = static_cast<int>(idx % CG);
    size_t rest = idx / CG;
    const int f = static_cast<int>(rest % a.Fout);
    rest /= a.Fout;
    const int t = static_cast<int>(rest % a.Tout);
    const int s = static_cast<int>(rest / a.Tout);
    const int c0 = cg * 8;
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
#pragma unroll
    for (int kt = 0; kt < 3; ++kt) {
      const int src = time_source(2 * t + kt, first);
#pragma unroll
      for (int kf = 0; kf < 3; ++kf) {
        const int bin = 2 * f + kf - 2;
        if (src == -2 || bin < 0 || bin >= a.Fin) continue;
        const uint16_t* p;
        if (src == -1) {
          p = cache + ((static_cast<size_t>(par) * a.S + s) * a.Fin + bin) * C + c0;
        } else if (src < a.valid_in) {
          p = in + ((static_cast<size_t>(s) * a.Tin + src) * a.Fin + bin) * C + c0;
        } else {
          continue;
        }
        float x[8];
        unpack8(*reinterpret_cast<const uint4*>(p), x, DT);
#pragma unroll
        for (int c = 0; c < 8; ++c)
          acc[c] = fmaf(ld_t<DT>(a.w, static_cast<size_t>(c0 + c) * 9 + kt * 3 + kf), x[c], acc[c]);
      }
    }
    uint16_t packed[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float o = round_t<DT>(round_t<DT>(acc[c]) + ld_t<DT>(a.b, c0 + c));
      if constexpr (DT == kBF16) packed[c] = __bfloat16_as_ushort(__float2bfloat16_rn(o));
      else packed[c] = __half_as_ushort(__float2half_rn(o));
    }
    uint4 w;
    w.x = packed[0] | (static_cast<uint32_t>(packed[1]) << 16);
    w.y = packed[2] | (static_cast<uint32_t>(packed[3]) << 16);
    w.z = packed[4] | (static_cast<uint32_t>(packed[5]) << 16);
    w.w = packed[6] | (static_cast<uint32_t>(packed[7]) << 16);
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) +
                              ((static_cast<size_t>(s) * a.Tout + t) * a.Fout + f) * C + c0) = w;
  }
  // next chunk's cache: the last input frame (zero if masked)
  const size_t ncache = static_cast<size_t>(a.S) * a.Fin * CG;
  for (size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < ncache;
       idx += stride) {
    const int cg = static_cast<int>(idx % CG);
    const size_t sb = idx / CG;  // s * Fin + bin
    const int s = static_cast<int>(sb / a.Fin), bin = static_cast<int>(sb % a.Fin);
    const int fr = a.Tin - 1;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (fr < a.valid_in)
      v = *reinterpret_cast<const uint4*>(in + ((static_cast<size_t>(s) * a.Tin + fr) * a.Fin + bin) * C +
                                          cg * 8);
    *reinterpret_cast<uint4*>(cache + ((static_cast<size_t>(1 - par) * a.S + s) * a.Fin + bin) * C +
                              cg * 8) = v;
  }
}

__global__ void __launch_bounds__(kThreads)
    flatten_cf_kernel(const uint16_t* in, uint16_t* out, int S, int T, int F, int C, int valid) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t width = static_cast<size_t>(C) * F;
  const size_t total = static_cast<size_t>(S) * T * width;
  for (size_t o = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; o < total;
       o += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = o / width;
    const int col = static_cast<int>(o % width);
    const int c = col / F, f = col % F;
    const int t = static_cast<int>(row % T);
    out[o] = t < valid ? in[(row * F + f) * C + c] : static_cast<uint16_t>(0);
  }
}

__global__ void advance_counters_kernel(int* counters, int frames) {
  pdl_wait();
  if (threadIdx.x == 0) {
    counters[kCtrFramesSeen] += frames;
    counters[kCtrChunk] += 1;
  }
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Box-Muller over a counter-based hash: element i depends only on (seed, i).
__global__ void fill_normal_kernel(float* out, size_t n, uint64_t seed, float mean, float std) {
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint64_t h = splitmix64(seed * 0x2545F4914F6CDD1Dull + i);
    const float u1 = (static_cast<float>(h >> 40) + 1.0f) * (1.0f / 16777216.0f);  // (0, 1]
    const float u2 = static_cast<float>((h >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
    out[i] = mean + std * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
  }
}

int grid_for(size_t work) {
  const size_t blocks = (work + kThreads - 1) / kThreads;
  return static_cast<int>(blocks < 148 * 16 ? (blocks == 0 ? 1 : blocks) : 148 * 16);
}

}  // namespace

cudaError_t launch_layernorm(int dtype, const LnArgs& a, cudaStream_t stream, bool pdl) {
  if (a.D > kMaxPerThread * kThreads || a.rows <= 0) return cudaErrorInvalidValue;
  auto k = dtype == kBF16 ? layernorm_kernel<kBF16> : layernorm_kernel<kF16>;
  return launch_ex(k, dim3(a.rows), dim3(kThreads), 0, stream, pdl, a);
}

size_t attention_smem_bytes(int Q, int vmax, int head_dim) {
  return attn_floats(Q, vmax, head_dim, nullptr, nullptr) * sizeof(float);
}

cudaError_t launch_attention(int dtype, const AttnArgs& a, cudaStream_t stream, bool pdl) {
  const size_t smem = attention_smem_bytes(a.Q, a.vmax, a.head_dim);
  auto k = dtype == kBF16 ? attention_kernel<kBF16> : attention_kernel<kF16>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  return launch_ex(k, dim3(a.S * a.heads), dim3(kThreads), smem, stream, pdl, a);
}

cudaError_t launch_conv_module(int dtype, const ConvArgs& a, cudaStream_t stream, bool pdl) {
  if (a.D > kMaxPerThread * kThreads) return cudaErrorInvalidValue;
  auto k = dtype == kBF16 ? conv_module_kernel<kBF16> : conv_module_kernel<kF16>;
  return launch_ex(k, dim3(a.S * a.Q), dim3(kThreads), 0, stream, pdl, a);
}

cudaError_t launch_stem_conv(int dtype, const Conv2dArgs& a, cudaStream_t stream, bool pdl) {
  if (a.C % 8) return cudaErrorInvalidValue;
  auto k = dtype == kBF16 ? stem_conv_kernel<kBF16> : stem_conv_kernel<kF16>;
  const size_t work = static_cast<size_t>(a.S) * a.Tout * a.Fout * (a.C / 8);
  return launch_ex(k, dim3(grid_for(work)), dim3(kThreads), 0, stream, pdl, a);
}

cudaError_t launch_depthwise_conv2d(int dtype, const Conv2dArgs& a, cudaStream_t stream, bool pdl) {
  if (a.C % 8) return cudaErrorInvalidValue;
  auto k = dtype == kBF16 ? depthwise_conv2d_kernel<kBF16> : depthwise_conv2d_kernel<kF16>;
  const size_t work = static_cast<size_t>(a.S) * a.Tout * a.Fout * (a.C / 8);
  return launch_ex(k, dim3(grid_for(work)), dim3(kThreads), 0, stream, pdl, a);
}

cudaError_t launch_flatten_cf(int dtype, const void* in, void* out, int S, int T, int F, int C,
                              int valid, cudaStream_t stream, bool pdl) {
  (void)dtype;  // a 16-bit copy: the element type does not matter
  const size_t work = static_cast<size_t>(S) * T * F * C;
  return launch_ex(flatten_cf_kernel, dim3(grid_for(work)), dim3(kThreads), 0, stream, pdl,
                   static_cast<const uint16_t*>(in), static_cast<uint16_t*>(out), S, T, F, C, valid);
}

cudaError_t launch_advance_counters(int* counters, int frames, cudaStream_t stream, bool pdl) {
  return launch_ex(advance_counters_kernel, dim3(1), dim3(32), 0, stream, pdl, counters, frames);
}

cudaError_t launch_fill_normal(float* out, size_t n, uint64_t seed, float mean, float std,
                               cudaStream_t stream) {
  fill_normal_kernel<<<grid_for(n), kThreads, 0, stream>>>(out, n, seed, mean, std);
  return cudaGetLastError();
}

}  // namespace cq
