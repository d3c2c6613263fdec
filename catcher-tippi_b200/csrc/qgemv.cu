// K1: affine INT8 dequant-GEMV for small token counts (the batch-1 streaming
// chunk, M = lookahead + 1 <= 16 rows per call; larger M loops over 16-row
// token tiles).
//
// Computes y[m, n] = sum_k x[m, k] * (s[n, k/g] * q[n, k] + b[n, k/g]) with the
// MLX affine INT8 layout (q: u32 [N, K/4] == u8 [N, K]; s, b: T [N, K/g]) --
// the operation behind QuantizedLinear::forward_array
// (crates/nemotron-mlx/src/model/layers.rs:298-310).
//
// Design (sm_100a):
//  * Each CTA owns a band of RB = 16*RT weight rows and a K-range of
//    `sb_per_cta` 64-wide sub-blocks.  Its whole weight tile is requested up
//    front with 2-D TMA bulk-tensor loads (one mbarrier per sub-block, L2
//    evict-first), and the group scales/biases are loaded, BEFORE
//    griddepcontrol.wait: under programmatic dependent launch the weight
//    stream of this linear overlaps the previous kernel.
//  * After the wait the critical path is short: every warp owns at most two
//    sub-blocks and issues all of its activation loads at once (one L2 round
//    trip), runs the MMAs on them as loaded, and the K-split partials are
//    reduced.
//  * The K-split CTAs of one band form a thread-block cluster: each pushes its
//    fp32 partial into the leader CTA's shared memory (distributed shared
//    memory stores), one cluster barrier, and the leader finishes the
//    epilogue.  No global scratch, no atomics, deterministic order.
//  * Tensor cores via mma.m16n8k16 in the activations' type on an exact
//    image o + q of each weight byte (f16: 1024 + q; bf16: 128 + q in two
//    fragments), with the offset folded into the group bias term; the
//    per-sub-block arithmetic lives in gemv_core.cuh.
#include "common.cuh"
#include "gemv_core.cuh"
#include "qgemv.hpp"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>

namespace cq {

namespace {

constexpr int kNW = 8;  // warps per CTA
constexpr int kThreads = kNW * 32;
constexpr int kMaxSubBlocks = 16;               // sub-blocks (of 64 k) per CTA
constexpr int kSbPerWarp = kMaxSubBlocks / kNW;  // at most two per warp
constexpr int kMaxSbPerThread = (kMaxSubBlocks * 2 * 64 + kThreads - 1) / kThreads;
// K <= 8192 (checked when a linear is created) keeps the K-split cluster
// within the portable 8 CTAs: ceil(8192 / 64 / 16) = 8.
static_assert((8192 / 64 + kMaxSubBlocks - 1) / kMaxSubBlocks <= 8, "K-split cluster above 8 CTAs");

struct GemvSmem {
  size_t wt, bars, sbsm, biasm, red, fin, total;
};

__host__ __device__ inline GemvSmem gemv_smem_layout(int rt, int sb_per_cta, int subg,
                                                     int ksplit) {
  const int rb = 16 * rt;
  GemvSmem L{};
  size_t off = 0;
  L.wt = off;  // [sb_per_cta][rb][64] u8, TMA destination
  off += static_cast<size_t>(sb_per_cta) * rb * 64;
  L.bars = off;  // one weight barrier per sub-block
  off += kMaxSubBlocks * 8;
  L.sbsm = off;  // [sb_per_cta * subg][rb] (s, b - o s), o = weight_offset<DT>()
  off += static_cast<size_t>(sb_per_cta) * subg * rb * sizeof(float2);
  L.biasm = off;  // [rb] output bias
  off += static_cast<size_t>(rb) * sizeof(float);
  L.red = off;  // [kNW][rb][16] per-warp partials (columns swizzled by red_col)
  off += static_cast<size_t>(kNW) * rb * 16 * sizeof(float);
  L.fin = off;  // [ksplit][rb][16]: CTA partials pushed into the cluster leader
  // (at least 16 u64: the per-token maxima of the greedy epilogue)
  off += std::max(static_cast<size_t>(ksplit > 1 ? ksplit : 0) * rb * 16 * sizeof(float),
                  static_cast<size_t>(16 * sizeof(unsigned long long)));
  L.total = off;
  return L;
}

__device__ __forceinline__ void st_dsmem_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Kernel parameter blocks: one layer (every ordinary call), a group of
// same-shape layers, or one layer with an RNNT epilogue.  Separate layouts
// keep the common launch's parameters small (one map, one argument block).
enum GemvKind : int { kKindPlain = 0, kKindGroup = 1, kKindEpilogue = 2 };
template <int KIND>
struct GemvParams {
  CUtensorMap m[1];
  GemvArgs a[1];
  __device__ int count() const { return 1; }
};
template <>
struct GemvParams<kKindGroup> {
  CUtensorMap m[kGemvMaxGroup];
  GemvArgs a[kGemvMaxGroup];
  int n;
  __device__ int count() const { return n; }
};
template <>
struct GemvParams<kKindEpilogue> {
  CUtensorMap m[1];
  GemvArgs a[1];
  RnntEpilogue epi;
  __device__ int count() const { return 1; }
};

// Greedy epilogue, after this CTA folded token tile mt's maxima into
// epi.best: the last of the tile's `ctas` CTAs records the choices of its 16
// streams (one atomic round trip) and passes each emitted token on, as its id
// (last_token) or its embedding row (x).
__device__ void greedy_finish(const RnntEpilogue& epi, int M, int mt, unsigned ctas, int* scratch,
                              int tid) {
  if (tid == 0) {
    __threadfence();
    scratch[16] = atomicAdd(&epi.done[mt], 1u) == ctas - 1 ? 1 : 0;
    if (scratch[16]) __threadfence();
  }
  __syncthreads();
  if (scratch[16] == 0) return;
  if (tid < 16) {
    const int s = mt * 16 + tid;
    int out = -1;
    if (s < M) {
      const unsigned long long key = atomicExch(&epi.best[s], 0ull);  // read and clear
      if (epi.active[s]) {
        // every logit NaN: MLX returns index 0
        const int bi = key == 0ull ? 0 : static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key));
        if (bi == epi.blank) {
          epi.active[s] = 0;
        } else {
          const int n = epi.counts[s];
          if (n < epi.cap) {
            epi.tokens[static_cast<size_t>(s) * epi.cap + n] = bi;
            epi.token_frames[static_cast<size_t>(s) * epi.cap + n] = epi.frame;
          }
          epi.counts[s] = n + 1;
          out = bi;
        }
      }
    }
    scratch[tid] = out;
    if (epi.last_token != nullptr && out >= 0) epi.last_token[s] = out;
  }
  __syncthreads();
  const int per_row = epi.last_token != nullptr ? 0 : epi.H / 8;
  for (int i = tid; i < 16 * per_row; i += kThreads) {
    const int t = i / per_row, c8 = (i - t * per_row) * 8;
    if (scratch[t] < 0) continue;
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(epi.x) + static_cast<size_t>(mt * 16 + t) * epi.H + c8) =
        *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(epi.emb) +
                                        static_cast<size_t>(scratch[t]) * epi.H + c8);
  }
  if (tid == 0) epi.done[mt] = 0;
  __syncthreads();
}

template <int DT, int G, int RT, int KIND>
__global__ void __launch_bounds__(kThreads, 2) qgemv_kernel(const __grid_constant__ GemvParams<KIND> P) {
  constexpr int RB = 16 * RT;
  constexpr int SUBG = (G == 32) ? 2 : 1;  // groups per 64-wide sub-block
  extern __shared__ __align__(128) uint8_t smem[];

  const int S = gridDim.x;  // K-split factor == cluster size along x
  const int rank = blockIdx.x;
  // member of the group and band within it
  const int bands = (P.a[0].N + RB - 1) / RB;
  const int member = KIND == kKindGroup ? static_cast<int>(blockIdx.y) / bands : 0;
  const GemvArgs& a = P.a[member];
  const CUtensorMap* wmap = &P.m[member];
  const int n0 = (blockIdx.y - member * bands) * RB;
  const int nsb = (a.K + 63) >> 6;
  const int sb0 = rank * a.sb_per_cta;
  const int sbn = max(0, min(a.sb_per_cta, nsb - sb0));
  const int groups_per_row = a.K / G;

  const GemvSmem L = gemv_smem_layout(RT, a.sb_per_cta, SUBG, S);
  uint8_t* wt = smem + L.wt;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  float2* sbsm = reinterpret_cast<float2*>(smem + L.sbsm);
  float* biasm = reinterpret_cast<float*>(smem + L.biasm);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* fin = reinterpret_cast<float*>(smem + L.fin);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = lane & 3, r4 = lane >> 2;

  // ---- weight tile: independent of the previous kernel, issued first.
  if (tid == 0) {
    prefetch_tensormap(wmap);
    for (int j = 0; j < sbn; ++j) mbar_init(&bars[j], 1);
    fence_mbar_init();
    // weights are read once, unless token tiles are spread over grid.z
    const uint64_t pol = gridDim.z == 1 ? l2_policy_evict_first() : l2_policy_evict_normal();
    for (int j = 0; j < sbn; ++j) {
      mbar_arrive_expect_tx(&bars[j], RB * 64);
      tma_load_2d(wt + static_cast<size_t>(j) * RB * 64, wmap, (sb0 + j) * 64, n0, &bars[j], pol);
    }
  }

  // ---- group scales/biases (fp32 (s, b - o s)) and the output bias: all
  // loads issued back to back, then stored, so the CTA pays one latency.
  {
    const int per_row = sbn * SUBG;
    const int total = per_row * RB;
    float sv[kMaxSbPerThread], bv[kMaxSbPerThread];
#pragma unroll
    for (int i = 0; i < kMaxSbPerThread; ++i) {
      const int e = tid + i * kThreads;
      sv[i] = 0.f;
      bv[i] = 0.f;
      if (e < total) {
        const int row = e % RB, jh = e / RB;  // rows fastest: conflict-free float2 stores
        const int n = n0 + row;
        const int kfirst = (sb0 + jh / SUBG) * 64 + (jh % SUBG) * 32;
        if (n < a.N && kfirst < a.K) {
          const size_t gi = static_cast<size_t>(n) * groups_per_row + kfirst / G;
          sv[i] = ld_t<DT>(a.scales, gi);
          bv[i] = ld_t<DT>(a.biases, gi);
        }
      }
    }
    float bias_v = 0.f;
    if (a.bias != nullptr && tid < RB && n0 + tid < a.N) bias_v = ld_t<DT>(a.bias, n0 + tid);
#pragma unroll
    for (int i = 0; i < kMaxSbPerThread; ++i) {
      const int e = tid + i * kThreads;
      if (e < total) {
        const int row = e % RB, jh = e / RB;  // rows fastest: conflict-free float2 stores
        sbsm[jh * RB + row] = make_float2(sv[i], fmaf(-weight_offset<DT>(), sv[i], bv[i]));
      }
    }
    if (tid < RB) biasm[tid] = bias_v;
  }

  // Let the next kernel in the stream start its own weight prefetch.
  pdl_launch_dependents();
  __syncthreads();

  // ---- from here on the activations of the previous kernel are needed.
  pdl_wait();

  bool ok = true;
  const bool has_bias = a.bias != nullptr;
  const int mtiles = (a.M + 15) >> 4;
  // Token tiles blockIdx.z, blockIdx.z + gridDim.z, ... belong to this CTA.
  const int mt0 = blockIdx.z, mstep = gridDim.z;
  // All activation loads of this warp's sub-blocks in flight at once.
  const bool xw = x_rows_wide(a.x, a.ldx);
  uint4 xr[kSbPerWarp][2][2];
#pragma unroll
  for (int u = 0; u < kSbPerWarp; ++u) {
    const int j = warp + u * kNW;
    if (j < sbn) {
      const int kb = (sb0 + j) * 64;
      load_x_raw<G>(a.x, a.ldx, a.M, a.K, mt0 * 16 + r4, kb, c, xr[u][0][0], xr[u][0][1], xw);
      load_x_raw<G>(a.x, a.ldx, a.M, a.K, mt0 * 16 + 8 + r4, kb, c, xr[u][1][0], xr[u][1][1], xw);
    }
  }
  bool first_tile = true;
  for (int mt = mt0; mt < mtiles; mt += mstep) {

    float acc[RT][2][4];
#pragma unroll
    for (int i = 0; i < RT; ++i)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][nt][e] = 0.f;

#pragma unroll
    for (int u = 0; u < kSbPerWarp; ++u) {
      const int j = warp + u * kNW;
      if (j >= sbn) break;
      const XOperands<G> xo = x_operands<DT, G>(xr[u]);

      if (first_tile) ok = mbar_wait(&bars[j], 0, a.status) && ok;

      subblock_mma<DT, G, RT>(wt + static_cast<size_t>(j) * RB * 64,
                              sbsm + static_cast<size_t>(j) * SUBG * RB, xo, lane, acc);
    }

    first_tile = false;
    // Next token tile's activations: the loads overlap this tile's reduction.
    const int mt_next = mt + mstep;
    if (mt_next < mtiles) {
#pragma unroll
      for (int u = 0; u < kSbPerWarp; ++u) {
        const int j = warp + u * kNW;
        if (j < sbn) {
          const int kb = (sb0 + j) * 64;
          load_x_raw<G>(a.x, a.ldx, a.M, a.K, mt_next * 16 + r4, kb, c, xr[u][0][0], xr[u][0][1], xw);
          load_x_raw<G>(a.x, a.ldx, a.M, a.K, mt_next * 16 + 8 + r4, kb, c, xr[u][1][0],
                        xr[u][1][1], xw);
        }
      }
    }

    // ---- reduce: warps of this CTA through shared memory ...
#pragma unroll
    for (int i = 0; i < RT; ++i) {
      const int ra = 16 * i + r4, rb = ra + 8;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        *reinterpret_cast<float2*>(&red[(warp * RB + ra) * 16 + red_col(ra, 8 * nt + 2 * c)]) =
            make_float2(acc[i][nt][0], acc[i][nt][1]);
        *reinterpret_cast<float2*>(&red[(warp * RB + rb) * 16 + red_col(rb, 8 * nt + 2 * c)]) =
            make_float2(acc[i][nt][2], acc[i][nt][3]);
      }
    }
    __syncthreads();

    // element e = tok * RB + row: consecutive threads write consecutive n
    if (S == 1) {
      unsigned long long* best_s = reinterpret_cast<unsigned long long*>(fin);  // [16], greedy mode
      if (KIND == kKindEpilogue && a.mode == kGemvGreedy) {
        if (tid < 16) best_s[tid] = 0ull;
        __syncthreads();
      }
      for (int e = tid; e < RB * 16; e += kThreads) {
        const int row = e % RB, tok = e / RB;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kNW; ++w) v += red[(w * RB + row) * 16 + red_col(row, tok)];
        const int n = n0 + row, m = mt * 16 + tok;
        if (n < a.N && m < a.M) {
          const float o = epilogue_value<DT>(v, has_bias, biasm[row], a.act);
          const size_t off = static_cast<size_t>(m) * a.ldy + n;
          // the greedy head keeps only the per-stream maximum
          if (KIND != kKindEpilogue || a.mode != kGemvGreedy) st_t<DT>(a.y, off, o);
          if constexpr (KIND != kKindEpilogue) {
          } else if (a.mode == kGemvJointInput) {
            float d = o;
            if (P.epi.active[m]) st_t<DT>(P.epi.dec, off, o);
            else d = ld_t<DT>(P.epi.dec, off);
            const float en = ld_t<DT>(P.epi.enc, static_cast<size_t>(m) * P.epi.ld_enc + n);
            st_t<DT>(P.epi.fused, off, fmaxf(en + d, 0.0f));
          } else if (a.mode == kGemvGreedy && !isnan(o)) {
            // larger logit -> larger key; equal logits -> the smaller index
            const uint32_t u = __float_as_uint(o);
            const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
            atomicMax(&best_s[tok], (static_cast<unsigned long long>(ord) << 32) |
                                        (0xFFFFFFFFu - static_cast<uint32_t>(n)));
          }
        }
      }
      __syncthreads();
      if constexpr (KIND == kKindEpilogue) {
        if (a.mode == kGemvGreedy) {
          if (tid < 16 && mt * 16 + tid < a.M && best_s[tid] != 0ull)
            atomicMax(&P.epi.best[mt * 16 + tid], best_s[tid]);
          if (!P.epi.defer)
            greedy_finish(P.epi, a.M, mt, gridDim.x * gridDim.y, reinterpret_cast<int*>(red), tid);
        }
      }
    } else {
      // ... then every CTA of the cluster pushes its partial into the
      // leader's slot `rank`; one cluster barrier; the leader finishes.
      const uint32_t slot = mapa_shared(smem_u32(fin), 0) +
                            static_cast<uint32_t>(rank * RB * 16 * sizeof(float));
      for (int e = tid; e < RB * 16; e += kThreads) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kNW; ++w) v += red[(w * RB + e / 16) * 16 + red_col(e / 16, e % 16)];
        st_dsmem_f32(slot + static_cast<uint32_t>(e * sizeof(float)), v);
      }
      cluster_sync_all();
      if (rank == 0) {
        for (int e = tid; e < RB * 16; e += kThreads) {
          const int row = e % RB, tok = e / RB;
          float v = 0.f;
          for (int q = 0; q < S; ++q) v += fin[(q * RB + row) * 16 + tok];
          const int n = n0 + row, m = mt * 16 + tok;
          if (n < a.N && m < a.M)
            st_t<DT>(a.y, static_cast<size_t>(m) * a.ldy + n,
                     epilogue_value<DT>(v, has_bias, biasm[row], a.act));
        }
      }
      // the leader's slots are rewritten by the next token tile
      if (mt_next < mtiles) cluster_sync_all();
    }
  }

  if (!ok && tid == 0) {
    // A copy never completed: wait (bounded) once more for the copies in
    // flight before the shared memory is released.
    for (int j = 0; j < sbn; ++j) mbar_wait_bounded(&bars[j], 0, a.status);
  }
}

template <int DT, int G, int RT, int KIND>
cudaError_t launch_typed(const GemvPlan& plan, const GemvParams<KIND>& P, int count,
                         cudaStream_t stream, bool pdl) {
  constexpr int SUBG = (G == 32) ? 2 : 1;
  const GemvArgs& args = P.a[0];
  const GemvSmem L = gemv_smem_layout(RT, plan.sb_per_cta, SUBG, plan.ksplit);
  auto kern = qgemv_kernel<DT, G, RT, KIND>;
  static int configured_smem = 0;
  if (static_cast<int>(L.total) > configured_smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(L.total));
    if (e != cudaSuccess) return e;
    configured_smem = static_cast<int>(L.total);
  }
  cudaLaunchConfig_t cfg = {};
  // token tiles beyond the first spread over grid.z, within one wave
  const int bands = (args.N + 16 * RT - 1) / (16 * RT) * count;
  const int mtiles = (args.M + 15) / 16;
  const int zmax = std::max(1, (2 * plan.num_sms) / std::max(1, bands * plan.ksplit));
  cfg.gridDim = dim3(plan.ksplit, bands, std::min(mtiles, zmax));
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (plan.ksplit > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = plan.ksplit;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, P);
}

template <int DT, int G, int KIND>
cudaError_t launch_rt(const GemvPlan& plan, const GemvParams<KIND>& P, int count,
                      cudaStream_t stream, bool pdl) {
  switch (plan.rt) {
    case 1: return launch_typed<DT, G, 1, KIND>(plan, P, count, stream, pdl);
    case 2: return launch_typed<DT, G, 2, KIND>(plan, P, count, stream, pdl);
    case 4: return launch_typed<DT, G, 4, KIND>(plan, P, count, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

template <int KIND>
cudaError_t launch_kind(int dtype, int group, const GemvPlan& plan, const GemvParams<KIND>& P,
                        int count, cudaStream_t stream, bool pdl) {
  if (dtype != kF16 && dtype != kBF16) return cudaErrorInvalidValue;
  switch (group) {
    case 32:
      return dtype == kF16 ? launch_rt<kF16, 32, KIND>(plan, P, count, stream, pdl)
                           : launch_rt<kBF16, 32, KIND>(plan, P, count, stream, pdl);
    case 64:
      return dtype == kF16 ? launch_rt<kF16, 64, KIND>(plan, P, count, stream, pdl)
                           : launch_rt<kBF16, 64, KIND>(plan, P, count, stream, pdl);
    case 128:
      return dtype == kF16 ? launch_rt<kF16, 128, KIND>(plan, P, count, stream, pdl)
                           : launch_rt<kBF16, 128, KIND>(plan, P, count, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

GemvPlan plan_gemv(int N, int K, int num_sms) {
  const int nsb = (K + 63) / 64;
  // Measured on B200 (back-to-back launches, M = 14): the cluster reduction
  // costs more than it saves, so K is split only as far as the 16 sub-blocks
  // a CTA can hold require; rows per CTA grow only to stay within one wave of
  // two CTAs per SM.
  const int s = std::max(1, (nsb + kMaxSubBlocks - 1) / kMaxSubBlocks);
  const int spc = (nsb + s - 1) / s;
  GemvPlan best{4, s, spc, num_sms};
  for (int rt : {1, 2, 4}) {
    const int bands = (N + 16 * rt - 1) / (16 * rt);
    if (bands * s <= 2 * num_sms) {
      best = GemvPlan{rt, s, spc, num_sms};
      break;
    }
  }
  return best;
}

GemvPlan plan_gemv_rows(const GemvPlan& base, int N, int M) {
  const int mtiles = (M + 15) / 16;
  if (mtiles <= 1) return base;
  for (int rt : {1, 2, 4}) {
    if (rt < base.rt) continue;
    const int bands = (N + 16 * rt - 1) / (16 * rt);
    if (bands * base.ksplit * mtiles <= 2 * base.num_sms) {
      GemvPlan p = base;
      p.rt = rt;
      return p;
    }
  }
  GemvPlan p = base;
  p.rt = 4;
  return p;
}

cudaError_t launch_gemv_group(int dtype, int group, const GemvPlan& plan, const GemvMaps& maps,
                              const GemvGroup& g, cudaStream_t stream, bool pdl,
                              const RnntEpilogue* epi) {
  if (g.count < 1 || g.count > kGemvMaxGroup) return cudaErrorInvalidValue;
  for (int i = 0; i < g.count; ++i) {
    if (g.a[i].N != g.a[0].N || g.a[i].K != g.a[0].K || g.a[i].M != g.a[0].M ||
        g.a[i].sb_per_cta != g.a[0].sb_per_cta)
      return cudaErrorInvalidValue;
    // the RNNT epilogues need the whole K in one CTA, one member, their arguments
    if (g.a[i].mode != kGemvPlain && (epi == nullptr || plan.ksplit != 1 || g.count != 1))
      return cudaErrorInvalidValue;
  }
  if (epi != nullptr && g.a[0].mode != kGemvPlain) {
    GemvParams<kKindEpilogue> P;
    P.m[0] = maps.m[0];
    P.a[0] = g.a[0];
    P.epi = *epi;
    return launch_kind(dtype, group, plan, P, 1, stream, pdl);
  }
  if (g.count == 1) {
    GemvParams<kKindPlain> P;
    P.m[0] = maps.m[0];
    P.a[0] = g.a[0];
    return launch_kind(dtype, group, plan, P, 1, stream, pdl);
  }
  GemvParams<kKindGroup> P;
  for (int i = 0; i < g.count; ++i) {
    P.m[i] = maps.m[i];
    P.a[i] = g.a[i];
  }
  P.n = g.count;
  return launch_kind(dtype, group, plan, P, g.count, stream, pdl);
}

cudaError_t launch_gemv(int dtype, int group, const GemvPlan& plan, const CUtensorMap& wmap,
                        const GemvArgs& args, cudaStream_t stream, bool pdl) {
  GemvParams<kKindPlain> P;
  P.m[0] = wmap;
  P.a[0] = args;
  return launch_kind(dtype, group, plan, P, 1, stream, pdl);
}

}  // namespace cq
