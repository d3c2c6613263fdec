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
//    evict-first), together with the group scales/biases, BEFORE
//    griddepcontrol.wait: under programmatic dependent launch the weight
//    stream of this linear overlaps the tail of the previous kernel.
//  * The K-split CTAs of one band form a thread-block cluster and reduce their
//    fp32 partials through distributed shared memory: no global scratch, no
//    atomics, deterministic order.
//  * Tensor cores via mma.m16n8k16 (f16 x f16 -> f32): weight rows are the MMA
//    M dimension, tokens the N dimension.  A weight byte q becomes the f16
//    value 1024 + q with one PRMT (bits 0x64qq), exact; the 1024 offset is
//    folded into the group bias term:
//        y += s * sum(x * (1024 + q)) + (b - 1024 s) * sum(x)
//    so the dequantised weight is never rounded.  bf16 activations are moved
//    to f16 with a per-(token, 64-wide sub-block) power-of-two scale that is
//    undone in fp32, which is exact for every element within 2^-28 of the
//    block's largest magnitude.
//  * Each lane loads 16 contiguous weight bytes per row; the k-slot order of
//    the MMA fragments is permuted identically for A and B, so the MLX layout
//    is consumed as is (no repacking) and shared-memory reads are
//    conflict-free.
#include "common.cuh"
#include "qgemv.hpp"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>

namespace cq {

namespace {

constexpr int kNW = 4;            // warps per CTA
constexpr int kThreads = kNW * 32;
constexpr int kMaxSubBlocks = 16;  // sub-blocks (of 64 k) per CTA

struct GemvSmem {
  size_t wt, bars, sbsm, red, fin, total;
};

__host__ __device__ inline GemvSmem gemv_smem_layout(int rt, int sb_per_cta, int subg) {
  const int rb = 16 * rt;
  GemvSmem L{};
  size_t off = 0;
  L.wt = off;
  off += static_cast<size_t>(sb_per_cta) * rb * 64;
  off = (off + 127) & ~static_cast<size_t>(127);
  L.bars = off;
  off += kMaxSubBlocks * 8;
  L.sbsm = off;
  off += static_cast<size_t>(sb_per_cta) * subg * rb * sizeof(float2);
  L.red = off;
  off += static_cast<size_t>(kNW) * rb * 16 * sizeof(float);
  L.fin = off;
  off += static_cast<size_t>(rb) * 16 * sizeof(float);
  L.total = off;
  return L;
}

// Loads this lane's 16 activation values of one token for one 64-wide
// sub-block, converts them to f16 MMA B-fragments and returns the per-half
// sums of the converted values (reduced over the 4 lanes of the quad) and the
// inverse of the power-of-two scale that was applied.
//   G >= 64: values k = kb + 16c + [0, 16)
//   G == 32: values k = kb + 8c + [0, 8) and kb + 32 + 8c + [0, 8)
template <int DT, int G>
__device__ __forceinline__ void load_x_frag(const void* __restrict__ x, int ldx, int M, int K,
                                            int m, int kb, int c, uint32_t (&xb)[8],
                                            float (&xs)[2], float& inv) {
  uint4 r0 = make_uint4(0, 0, 0, 0), r1 = make_uint4(0, 0, 0, 0);
  if (m < M) {
    const uint16_t* xr = reinterpret_cast<const uint16_t*>(x) + static_cast<size_t>(m) * ldx;
    if constexpr (G >= 64) {
      const int k = kb + 16 * c;
      if (k < K) {
        r0 = ld_global_cg_v4(xr + k);
        r1 = ld_global_cg_v4(xr + k + 8);
      }
    } else {
      const int k0 = kb + 8 * c, k1 = kb + 32 + 8 * c;
      if (k0 < K) r0 = ld_global_cg_v4(xr + k0);
      if (k1 < K) r1 = ld_global_cg_v4(xr + k1);
    }
  }
  const uint32_t w[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
  float s0 = 0.f, s1 = 0.f;
  if constexpr (DT == kF16) {
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      xb[p] = w[p];
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[p]));
      if (p < 4) s0 += f.x + f.y;
      else s1 += f.x + f.y;
    }
    inv = 1.0f;
  } else {
    float v[16];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      v[2 * p] = __uint_as_float(w[p] << 16);
      v[2 * p + 1] = __uint_as_float(w[p] & 0xFFFF0000u);
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
    // scale = 2^(14 - floor(log2 amax)) puts the block maximum in [2^14, 2^15).
    const int e = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFF);
    int sh = e == 0 ? 0 : 141 - e;
    sh = max(-126, min(126, sh));
    const float scale = __uint_as_float(static_cast<uint32_t>(127 + sh) << 23);
    inv = __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const __half2 h = __floats2half2_rn(v[2 * p] * scale, v[2 * p + 1] * scale);
      xb[p] = *reinterpret_cast<const uint32_t*>(&h);
      const float2 f = __half22float2(h);
      if (p < 4) s0 += f.x + f.y;
      else s1 += f.x + f.y;
    }
  }
  s0 += __shfl_xor_sync(0xFFFFFFFFu, s0, 1);
  s0 += __shfl_xor_sync(0xFFFFFFFFu, s0, 2);
  s1 += __shfl_xor_sync(0xFFFFFFFFu, s1, 1);
  s1 += __shfl_xor_sync(0xFFFFFFFFu, s1, 2);
  if constexpr (G >= 64) {
    xs[0] = s0 + s1;
    xs[1] = 0.f;
  } else {
    xs[0] = s0;
    xs[1] = s1;
  }
}

template <int DT, int G, int RT>
__global__ void __launch_bounds__(kThreads)
    qgemv_kernel(const __grid_constant__ CUtensorMap wmap, const GemvArgs a) {
  constexpr int RB = 16 * RT;
  constexpr int SUBG = (G == 32) ? 2 : 1;  // groups per 64-wide sub-block
  extern __shared__ __align__(128) uint8_t smem[];

  const int S = gridDim.x;  // K-split factor == cluster size along x
  const int rank = blockIdx.x;
  const int n0 = blockIdx.y * RB;
  const int nsb = (a.K + 63) >> 6;
  const int sb0 = rank * a.sb_per_cta;
  const int sbn = max(0, min(a.sb_per_cta, nsb - sb0));
  const int groups_per_row = a.K / G;

  const GemvSmem L = gemv_smem_layout(RT, a.sb_per_cta, SUBG);
  uint8_t* wt = smem + L.wt;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  float2* sbsm = reinterpret_cast<float2*>(smem + L.sbsm);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* fin = reinterpret_cast<float*>(smem + L.fin);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = lane & 3, r4 = lane >> 2;

  // Let the next kernel in the stream start its own weight prefetch now.
  pdl_launch_dependents();

  // ---- weight tile: independent of the previous kernel, issued first.
  if (tid == 0) {
    prefetch_tensormap(&wmap);
    for (int j = 0; j < sbn; ++j) mbar_init(&bars[j], 1);
    fence_mbar_init();
    const uint64_t pol = l2_policy_evict_first();
    for (int j = 0; j < sbn; ++j) {
      mbar_arrive_expect_tx(&bars[j], RB * 64);
      tma_load_2d(wt + static_cast<size_t>(j) * RB * 64, &wmap, (sb0 + j) * 64, n0, &bars[j], pol);
    }
  }

  // ---- group scales/biases as fp32 (s, b - 1024 s), groups fastest.
  {
    const int per_row = sbn * SUBG;
    const int total = per_row * RB;
    for (int e = tid; e < total; e += kThreads) {
      const int row = e / per_row, jh = e - row * per_row;
      const int n = n0 + row;
      const int kfirst = (sb0 + jh / SUBG) * 64 + (jh % SUBG) * 32;
      float s = 0.f, b = 0.f;
      if (n < a.N && kfirst < a.K) {
        const size_t gi = static_cast<size_t>(n) * groups_per_row + kfirst / G;
        s = ld_t<DT>(a.scales, gi);
        b = ld_t<DT>(a.biases, gi);
      }
      sbsm[jh * RB + row] = make_float2(s, fmaf(-1024.0f, s, b));
    }
  }
  __syncthreads();

  // ---- from here on the activations of the previous kernel are needed.
  pdl_wait();

  bool ok = true;
  const int mtiles = (a.M + 15) >> 4;
  for (int mt = 0; mt < mtiles; ++mt) {
    float acc[RT][2][4];
#pragma unroll
    for (int i = 0; i < RT; ++i)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][nt][e] = 0.f;

    for (int j = warp; j < sbn; j += kNW) {
      const int kb = (sb0 + j) * 64;
      uint32_t xb[2][8];
      float xs[2][2], inv[2];
      load_x_frag<DT, G>(a.x, a.ldx, a.M, a.K, mt * 16 + r4, kb, c, xb[0], xs[0], inv[0]);
      load_x_frag<DT, G>(a.x, a.ldx, a.M, a.K, mt * 16 + 8 + r4, kb, c, xb[1], xs[1], inv[1]);
      // Token-side epilogue operands for the accumulator columns 2c, 2c+1.
      float xsA[2][SUBG], xsB[2][SUBG], ivA[2], ivB[2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
        for (int h = 0; h < SUBG; ++h) {
          xsA[nt][h] = __shfl_sync(0xFFFFFFFFu, xs[nt][h], 8 * c);
          xsB[nt][h] = __shfl_sync(0xFFFFFFFFu, xs[nt][h], 8 * c + 4);
        }
        ivA[nt] = __shfl_sync(0xFFFFFFFFu, inv[nt], 8 * c);
        ivB[nt] = __shfl_sync(0xFFFFFFFFu, inv[nt], 8 * c + 4);
      }

      if (mt == 0) ok = mbar_wait_bounded(&bars[j], 0, a.status) && ok;

      const uint8_t* wj = wt + static_cast<size_t>(j) * RB * 64;
      const float2* sbj = sbsm + static_cast<size_t>(j) * SUBG * RB;
#pragma unroll
      for (int i = 0; i < RT; ++i) {
        const int ra = 16 * i + r4, rb = ra + 8;
        uint32_t wa[4], wb[4];
        if constexpr (G >= 64) {
          const uint4 va = *reinterpret_cast<const uint4*>(wj + ra * 64 + 16 * c);
          const uint4 vb = *reinterpret_cast<const uint4*>(wj + rb * 64 + 16 * c);
          wa[0] = va.x; wa[1] = va.y; wa[2] = va.z; wa[3] = va.w;
          wb[0] = vb.x; wb[1] = vb.y; wb[2] = vb.z; wb[3] = vb.w;
        } else {
          const uint2 a0 = *reinterpret_cast<const uint2*>(wj + ra * 64 + 8 * c);
          const uint2 a1 = *reinterpret_cast<const uint2*>(wj + ra * 64 + 32 + 8 * c);
          const uint2 b0 = *reinterpret_cast<const uint2*>(wj + rb * 64 + 8 * c);
          const uint2 b1 = *reinterpret_cast<const uint2*>(wj + rb * 64 + 32 + 8 * c);
          wa[0] = a0.x; wa[1] = a0.y; wa[2] = a1.x; wa[3] = a1.y;
          wb[0] = b0.x; wb[1] = b0.y; wb[2] = b1.x; wb[3] = b1.y;
        }
        float d[2][SUBG][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int h = 0; h < SUBG; ++h)
#pragma unroll
            for (int e = 0; e < 4; ++e) d[nt][h][e] = 0.f;
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const int h = (SUBG == 2) ? (s >> 1) : 0;  // constant after unrolling
          // bytes 4s..4s+3 of this lane's 16: (b0,b1) -> k-slots 2c,2c+1;
          // (b2,b3) -> k-slots 2c+8, 2c+9.  0x64qq is the f16 value 1024 + q.
          const uint32_t a0 = __byte_perm(wa[s], 0x64646464u, 0x4140);
          const uint32_t a1 = __byte_perm(wb[s], 0x64646464u, 0x4140);
          const uint32_t a2 = __byte_perm(wa[s], 0x64646464u, 0x4342);
          const uint32_t a3 = __byte_perm(wb[s], 0x64646464u, 0x4342);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
            mma_16816_f16(d[nt][h], a0, a1, a2, a3, xb[nt][2 * s], xb[nt][2 * s + 1]);
        }
#pragma unroll
        for (int h = 0; h < SUBG; ++h) {
          const float2 sa = sbj[h * RB + ra];
          const float2 sb = sbj[h * RB + rb];
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const float t0 = fmaf(sa.x, d[nt][h][0], sa.y * xsA[nt][h]);
            const float t1 = fmaf(sa.x, d[nt][h][1], sa.y * xsB[nt][h]);
            const float t2 = fmaf(sb.x, d[nt][h][2], sb.y * xsA[nt][h]);
            const float t3 = fmaf(sb.x, d[nt][h][3], sb.y * xsB[nt][h]);
            if constexpr (DT == kF16) {
              acc[i][nt][0] += t0;
              acc[i][nt][1] += t1;
              acc[i][nt][2] += t2;
              acc[i][nt][3] += t3;
            } else {
              acc[i][nt][0] = fmaf(t0, ivA[nt], acc[i][nt][0]);
              acc[i][nt][1] = fmaf(t1, ivB[nt], acc[i][nt][1]);
              acc[i][nt][2] = fmaf(t2, ivA[nt], acc[i][nt][2]);
              acc[i][nt][3] = fmaf(t3, ivB[nt], acc[i][nt][3]);
            }
          }
        }
      }
    }

    // ---- reduce the K-split partials: warps of this CTA, then the cluster.
#pragma unroll
    for (int i = 0; i < RT; ++i) {
      const int ra = 16 * i + r4, rb = ra + 8;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        *reinterpret_cast<float2*>(&red[(warp * RB + ra) * 16 + 8 * nt + 2 * c]) =
            make_float2(acc[i][nt][0], acc[i][nt][1]);
        *reinterpret_cast<float2*>(&red[(warp * RB + rb) * 16 + 8 * nt + 2 * c]) =
            make_float2(acc[i][nt][2], acc[i][nt][3]);
      }
    }
    __syncthreads();

    if (S == 1) {
      for (int e = tid; e < RB * 16; e += kThreads) {
        const int row = e % RB, tok = e / RB;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kNW; ++w) v += red[(w * RB + row) * 16 + tok];
        const int n = n0 + row, m = mt * 16 + tok;
        if (n < a.N && m < a.M)
          st_t<DT>(a.y, static_cast<size_t>(m) * a.ldy + n, linear_epilogue<DT>(v, a.bias, n, a.act));
      }
      __syncthreads();
    } else {
      for (int e = tid; e < RB * 16; e += kThreads) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kNW; ++w) v += red[w * RB * 16 + e];
        fin[e] = v;
      }
      cluster_sync_all();
      const int r_lo = rank * RB / S, r_hi = (rank + 1) * RB / S, nr = r_hi - r_lo;
      const uint32_t fin_addr = smem_u32(fin);
      for (int e = tid; e < nr * 16; e += kThreads) {
        const int row = r_lo + e % nr, tok = e / nr;
        const uint32_t off = static_cast<uint32_t>((row * 16 + tok) * sizeof(float));
        float v = 0.f;
        for (int q = 0; q < S; ++q) v += ld_dsmem_f32(mapa_shared(fin_addr + off, q));
        const int n = n0 + row, m = mt * 16 + tok;
        if (n < a.N && m < a.M)
          st_t<DT>(a.y, static_cast<size_t>(m) * a.ldy + n, linear_epilogue<DT>(v, a.bias, n, a.act));
      }
      cluster_sync_all();
    }
  }

  if (!ok && tid == 0) {
    // A weight copy never completed: wait (bounded) once more for the copies
    // in flight before the shared memory is released.
    for (int j = 0; j < sbn; ++j) mbar_wait_bounded(&bars[j], 0, a.status);
  }
}

template <int DT, int G, int RT>
cudaError_t launch_typed(const GemvPlan& plan, const CUtensorMap& wmap, const GemvArgs& args,
                         cudaStream_t stream, bool pdl) {
  constexpr int SUBG = (G == 32) ? 2 : 1;
  const GemvSmem L = gemv_smem_layout(RT, plan.sb_per_cta, SUBG);
  auto kern = qgemv_kernel<DT, G, RT>;
  static int configured_smem = 0;
  if (static_cast<int>(L.total) > configured_smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(L.total));
    if (e != cudaSuccess) return e;
    configured_smem = static_cast<int>(L.total);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.ksplit, (args.N + 16 * RT - 1) / (16 * RT), 1);
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
  return cudaLaunchKernelEx(&cfg, kern, wmap, args);
}

template <int DT, int G>
cudaError_t launch_rt(const GemvPlan& plan, const CUtensorMap& wmap, const GemvArgs& args,
                      cudaStream_t stream, bool pdl) {
  switch (plan.rt) {
    case 1: return launch_typed<DT, G, 1>(plan, wmap, args, stream, pdl);
    case 2: return launch_typed<DT, G, 2>(plan, wmap, args, stream, pdl);
    case 4: return launch_typed<DT, G, 4>(plan, wmap, args, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

template <int DT>
cudaError_t launch_g(int group, const GemvPlan& plan, const CUtensorMap& wmap,
                     const GemvArgs& args, cudaStream_t stream, bool pdl) {
  switch (group) {
    case 32: return launch_rt<DT, 32>(plan, wmap, args, stream, pdl);
    case 64: return launch_rt<DT, 64>(plan, wmap, args, stream, pdl);
    case 128: return launch_rt<DT, 128>(plan, wmap, args, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

GemvPlan plan_gemv(int N, int K, int num_sms) {
  const int nsb = (K + 63) / 64;
  if (const char* env = std::getenv("CQ_GEMV_PLAN")) {
    int rt = 0, s = 0;
    if (std::sscanf(env, "%d,%d", &rt, &s) == 2 && (rt == 1 || rt == 2 || rt == 4) && s >= 1 &&
        s <= 8) {
      const int spc = (nsb + s - 1) / s;
      if (spc <= kMaxSubBlocks) return GemvPlan{rt, s, spc};
    }
  }
  GemvPlan best{4, 1, std::min(nsb, kMaxSubBlocks)};
  double best_score = -1e300;
  for (int rt : {4, 2, 1}) {
    const int rb = 16 * rt;
    const int bands = (N + rb - 1) / rb;
    for (int s = 1; s <= 8; ++s) {
      const int spc = (nsb + s - 1) / s;
      if (spc > kMaxSubBlocks) continue;
      if ((s - 1) * spc >= nsb) continue;  // every rank must own work
      const int ctas = bands * s;
      // SMs that receive work, discounted for warps left idle inside a CTA,
      // for cluster-reduction overhead and for very small tiles.
      const double busy = std::min(ctas, num_sms);
      const double warp_eff = std::min(spc, kNW) / static_cast<double>(kNW);
      const double waves = std::ceil(ctas / (2.0 * num_sms));
      const double score = busy * warp_eff / waves - 2.0 * (s - 1) + 0.5 * rt;
      if (score > best_score) {
        best_score = score;
        best = GemvPlan{rt, s, spc};
      }
    }
  }
  return best;
}

size_t gemv_smem_bytes(const GemvPlan& plan, int group) {
  return gemv_smem_layout(plan.rt, plan.sb_per_cta, group == 32 ? 2 : 1).total;
}

cudaError_t launch_gemv(int dtype, int group, const GemvPlan& plan, const CUtensorMap& wmap,
                        const GemvArgs& args, cudaStream_t stream, bool pdl) {
  if (dtype == kF16) return launch_g<kF16>(group, plan, wmap, args, stream, pdl);
  if (dtype == kBF16) return launch_g<kBF16>(group, plan, wmap, args, stream, pdl);
  return cudaErrorInvalidValue;
}

}  // namespace cq
