// One LSTM layer of one prediction step for every stream in ONE launch:
// gates = T(T(T(W_ih x) + T(W_hh h)) + bias), then the cell
// (LstmCell::forward, crates/nemotron-mlx/src/model/rnnt.rs:86-150) -- the
// work of two K1 launches and the cell kernel.
//
// The weight rows are interleaved at load time (row 4j + q holds gate q of
// hidden unit j), so one band of 16 * RT rows holds all four gates of 4 * RT
// hidden units.  FORM 0: the two products run as the two CTAs of a (2, 1, 1)
// cluster over the same band -- rank 0 multiplies the layer input by W_ih,
// rank 1 the previous hidden state by W_hh, each exactly as K1 does for one
// band (same sub-block order, same warp reduction: bit-identical partial
// sums); rank 1 pushes its partial tile into rank 0's shared memory, and rank
// 0 rounds each product to T, adds them and the gate bias in T and runs the
// cell.  FORM 1 (layer 0, whose input is always an embedding row): one CTA
// per band multiplies W_hh h and reads T(W_ih emb[token]) from a per-token
// table that FORM 0 made once with gi_out set; it can also finish the greedy
// choice the head deferred (token from the per-stream argmax key, band 0
// records it).  The new hidden state goes to a second buffer (other CTAs
// still read the old one); streams that are not stepping keep their state
// (h copied across, c untouched).
//
// Launch shape, per launch: token tiles spread over grid.z; the first of
// {64-row bands at one CTA per SM, 64-row bands at two per SM, 80-row bands
// at two per SM} whose grid fits one wave of resident CTAs, else 64-row
// bands at two per SM (a CTA walks several token tiles only past the grid
// limit, at one per SM).
#include "common.cuh"
#include "gemv_core.cuh"
#include "rnnt_ops.hpp"

namespace cq {

namespace {

// A band is 16 * RT interleaved gate rows = 4 * RT hidden units: RT 4 (64
// rows), or 5 (80 rows) where that keeps a launch within one wave.
constexpr int kNW = 8;
constexpr int kThreads = kNW * 32;
constexpr int kMaxSb = 16;  // K = hidden <= 1024
constexpr int kSbPerWarp = kMaxSb / kNW;

struct LstmSmem {
  size_t wt, bars, sbsm, red, fin, gb, total;
};

// rb rows per band; fin_bufs 2 where a CTA walks several token tiles.
__host__ __device__ inline LstmSmem lstm_smem_layout(int sbn, int subg, int rb, int fin_bufs) {
  LstmSmem L{};
  size_t off = 0;
  L.wt = off;  // [sbn][rb][64] u8, TMA destination
  off += static_cast<size_t>(sbn) * rb * 64;
  L.bars = off;
  off += kMaxSb * 8;
  L.sbsm = off;  // [sbn * subg][rb] (s, b - o s), o = weight_offset<DT>()
  off += static_cast<size_t>(sbn) * subg * rb * sizeof(float2);
  L.red = off;  // [8][rb][16] per-warp partials (columns swizzled by red_col)
  off += static_cast<size_t>(kNW) * rb * 16 * sizeof(float);
  L.fin = off;  // [fin_bufs tiles in flight][2 products][rb][16] of rank 0's band
  off += static_cast<size_t>(fin_bufs) * 2 * rb * 16 * sizeof(float);
  L.gb = off;  // [rb] the band's gate biases
  off += static_cast<size_t>(rb) * sizeof(float);
  L.total = off;
  return L;
}

__device__ __forceinline__ void st_dsmem_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

template <int DT>
__device__ __forceinline__ float sigmoid_t(float x) {
  return round_t<DT>(1.0f / (1.0f + expf(-x)));
}

// Loads issued where they stand (asm volatile keeps the compiler from
// sinking them to their use).
__device__ __forceinline__ int ld_volatile_s32(const int* p) {
  int v;
  asm volatile("ld.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_volatile_u16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.u16 %0, [%1];" : "=h"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint2 ld_volatile_v2u32(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

template <int DT>
__device__ __forceinline__ float widen_t(uint32_t bits16) {
  if constexpr (DT == kBF16) return __uint_as_float(bits16 << 16);
  else return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

template <int DT, int G, int RT, int MINB, int FORM>
__global__ void __launch_bounds__(kThreads, MINB)
    lstm_step_kernel(const __grid_constant__ LstmMaps maps, const LstmStepArgs a) {
  constexpr int SUBG = (G == 32) ? 2 : 1;
  constexpr int kRB = 16 * RT;
  constexpr int kUnits = kRB / 4;                                // hidden units per band
  constexpr int kCellIters = (kUnits * 16 + kThreads - 1) / kThreads;  // (unit, token) pairs
  constexpr int kFinBufs = MINB == 1 ? 2 : 1;
  extern __shared__ __align__(128) uint8_t smem[];
  // the product this CTA computes -- 0: W_ih x, 1: W_hh h (FORM 1: only that)
  const int rank = FORM == 1 ? 1 : static_cast<int>(blockIdx.x);
  const int n0 = blockIdx.y * kRB;
  const int H = a.H, K = a.H, N = 4 * a.H;
  const int sbn = (K + 63) >> 6;
  const int groups_per_row = K / G;
  const LstmSmem L = lstm_smem_layout(sbn, SUBG, kRB, kFinBufs);
  uint8_t* wt = smem + L.wt;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  float2* sbsm = reinterpret_cast<float2*>(smem + L.sbsm);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* fin = reinterpret_cast<float*>(smem + L.fin);
  float* gbias = reinterpret_cast<float*>(smem + L.gb);
  const CUtensorMap* wmap = RT == 4 ? &maps.m[rank] : &maps.m5[rank];
  const void* scales = rank == 0 ? a.scales_ih : a.scales_hh;
  const void* biases = rank == 0 ? a.biases_ih : a.biases_hh;
  const void* x = rank == 0 ? a.x : a.h_prev;
  const bool xw = x_rows_wide(x, H);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = lane & 3, r4 = lane >> 2;

  // ---- weight tile first: it does not depend on the previous kernel
  if (tid == 0) {
    prefetch_tensormap(wmap);
    for (int j = 0; j < sbn; ++j) mbar_init(&bars[j], 1);
    fence_mbar_init();
    const uint64_t pol = l2_policy_evict_normal();  // every token tile reads the band
    for (int j = 0; j < sbn; ++j) {
      mbar_arrive_expect_tx(&bars[j], kRB * 64);
      tma_load_2d(wt + static_cast<size_t>(j) * kRB * 64, wmap, j * 64, n0, &bars[j], pol);
    }
  }
  // ---- group scales / biases as (s, b - o s), o = weight_offset<DT>()
  for (int e = tid; e < sbn * SUBG * kRB; e += kThreads) {
    const int jh = e / kRB, row = e - jh * kRB;
    const int n = n0 + row;
    const int kfirst = (jh / SUBG) * 64 + (jh % SUBG) * 32;
    float sv = 0.f, bv = 0.f;
    if (n < N && kfirst < K) {
      const size_t gi = static_cast<size_t>(n) * groups_per_row + kfirst / G;
      sv = ld_t<DT>(scales, gi);
      bv = ld_t<DT>(biases, gi);
    }
    sbsm[e] = make_float2(sv, fmaf(-weight_offset<DT>(), sv, bv));
  }
  // ---- the band's gate biases (parameters of the model, like the scales)
  for (int e = tid; e < kRB; e += kThreads)
    gbias[e] = a.gate_bias != nullptr && n0 + e < N ? ld_t<DT>(a.gate_bias, n0 + e) : 0.0f;
  pdl_launch_dependents();
  __syncthreads();
  pdl_wait();

  bool ok = true;
  auto tile = [&](const int mt, const int round) {
    // FORM 1: this thread's table gates (pair p = unit p/16, stream
    // mt*16 + p%16), fetched before the product so the lookup (token id,
    // then row) overlaps the MMAs
    uint2 gi_bits[kCellIters];
    bool steps[kCellIters];  // deferred greedy choice: the stream steps
    // the cell's state reads, issued before the product so their latency
    // overlaps it: c (low half) and h_prev (high half) of each (unit, stream)
    // pair this thread updates -- only this thread writes them
    uint32_t ch_bits[kCellIters];
#pragma unroll
    for (int it = 0; it < kCellIters; ++it) {
      ch_bits[it] = 0u;
      const int p = tid + it * kThreads;
      const int s = mt * 16 + (p & 15), j = n0 / 4 + (p >> 4);
      if ((rank == 0 || FORM == 1) && a.gi_out == nullptr && p < kUnits * 16 && s < a.S && j < H) {
        const size_t hj = static_cast<size_t>(s) * H + j;
        ch_bits[it] = ld_volatile_u16(static_cast<const uint16_t*>(a.c) + hj) |
                      (ld_volatile_u16(static_cast<const uint16_t*>(a.h_prev) + hj) << 16);
      }
    }
#pragma unroll
    for (int it = 0; it < kCellIters; ++it) {
      gi_bits[it] = make_uint2(0u, 0u);
      steps[it] = false;
      const int p = tid + it * kThreads;
      if constexpr (FORM == 1) {
        const int s = mt * 16 + (p & 15);
        if (p < kUnits * 16 && s < a.S && n0 / 4 + (p >> 4) < H) {
          int tok;
          if (a.greedy_best != nullptr) {
            const unsigned long long key = ld_volatile_u64(a.greedy_best + s);
            tok = key == 0ull ? 0 : static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key));
            steps[it] = ld_volatile_s32(a.greedy_active + s) != 0 && tok != a.greedy_blank;
          } else {
            tok = ld_volatile_s32(a.gi_token + s);
          }
          gi_bits[it] = ld_volatile_v2u32(static_cast<const uint16_t*>(a.gi_table) +
                                          static_cast<size_t>(tok) * N + n0 + 4 * (p >> 4));
        }
      }
    }
    // band 0 records the deferred choice of its 16 streams (other CTAs that
    // read `active` after this write decide the same: a stream that emitted
    // blank reads 0 either way, one that emitted a token reads 1)
    if (FORM == 1 && a.greedy_best != nullptr && blockIdx.y == 0 && tid < 16) {
      const int s = mt * 16 + tid;
      if (s < a.S) {
        const unsigned long long key = ld_volatile_u64(a.greedy_best + s);
        const int tok = key == 0ull ? 0 : static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key));
        if (ld_volatile_s32(a.greedy_active + s) != 0) {
          if (tok == a.greedy_blank) {
            a.greedy_active[s] = 0;
          } else {
            const int n = a.counts[s];
            if (n < a.cap) {
              a.tokens[static_cast<size_t>(s) * a.cap + n] = tok;
              a.token_frames[static_cast<size_t>(s) * a.cap + n] = a.frame;
            }
            a.counts[s] = n + 1;
          }
        }
      }
    }
    if (FORM == 0 && a.clear_best != nullptr && blockIdx.y == 0 && rank == 0 && tid < 16 &&
        mt * 16 + tid < a.S)
      a.clear_best[mt * 16 + tid] = 0ull;
    // ---- activations of this token tile, all loads in flight at once
    uint4 xr[kSbPerWarp][2][2];
#pragma unroll
    for (int u = 0; u < kSbPerWarp; ++u) {
      const int j = warp + u * kNW;
      if (j < sbn) {
        load_x_raw<G>(x, H, a.S, K, mt * 16 + r4, j * 64, c, xr[u][0][0], xr[u][0][1], xw);
        load_x_raw<G>(x, H, a.S, K, mt * 16 + 8 + r4, j * 64, c, xr[u][1][0], xr[u][1][1], xw);
      }
    }
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
      ok = mbar_wait(&bars[j], 0, a.status) && ok;
      subblock_mma<DT, G, RT>(wt + static_cast<size_t>(j) * kRB * 64,
                               sbsm + static_cast<size_t>(j) * SUBG * kRB, xo, lane, acc);
    }
#pragma unroll
    for (int i = 0; i < RT; ++i) {
      const int ra = 16 * i + r4, rb = ra + 8;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        *reinterpret_cast<float2*>(&red[(warp * kRB + ra) * 16 + red_col(ra, 8 * nt + 2 * c)]) =
            make_float2(acc[i][nt][0], acc[i][nt][1]);
        *reinterpret_cast<float2*>(&red[(warp * kRB + rb) * 16 + red_col(rb, 8 * nt + 2 * c)]) =
            make_float2(acc[i][nt][2], acc[i][nt][3]);
      }
    }
    __syncthreads();
    // this CTA's product into rank 0's slot `rank` ([row][token], warp order)
    // fin alternates between two buffers: a CTA's push for the next tile is
    // preceded by this tile's cluster barrier, which rank 0 passes only
    // after it read the buffer before -- one barrier per tile suffices
    float* fbuf = fin + (kFinBufs == 2 ? (round & 1) : 0) * 2 * kRB * 16;
    if constexpr (FORM == 1) {
      for (int e = tid; e < kRB * 16; e += kThreads) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kNW; ++w) v += red[(w * kRB + e / 16) * 16 + red_col(e / 16, e % 16)];
        fbuf[kRB * 16 + e] = v;
      }
      __syncthreads();
    } else {
      const uint32_t slot = mapa_shared(smem_u32(fbuf), 0) +
                            static_cast<uint32_t>(rank * kRB * 16 * sizeof(float));
      for (int e = tid; e < kRB * 16; e += kThreads) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kNW; ++w) v += red[(w * kRB + e / 16) * 16 + red_col(e / 16, e % 16)];
        st_dsmem_f32(slot + static_cast<uint32_t>(e * sizeof(float)), v);
      }
      cluster_sync_all();
    }

    if (rank == 0 || FORM == 1) {
#pragma unroll
      for (int it = 0; it < kCellIters; ++it) {
        // one (hidden unit, token) pair per thread and pass
        const int p = tid + it * kThreads;
        const int u = p >> 4, t = p & 15;
        const int s = mt * 16 + t;
        const int j = n0 / 4 + u;
        if (p >= kUnits * 16 || s >= a.S || j >= H) continue;
        if (FORM == 0 && a.gi_out != nullptr) {
          // table row: the rounded ih product of the unit's 4 gates
#pragma unroll
          for (int q = 0; q < 4; ++q)
            st_t<DT>(a.gi_out, static_cast<size_t>(s) * N + n0 + 4 * u + q,
                     round_t<DT>(fbuf[(4 * u + q) * 16 + t]));
          continue;
        }
        const size_t hj = static_cast<size_t>(s) * H + j;
        const bool step = FORM == 1 && a.greedy_best != nullptr ? steps[it] : (a.all || a.active[s]);
        if (step) {
          float gi[4];
          if constexpr (FORM == 1) {
            // the four gates of unit j are adjacent in the interleaved row
            gi[0] = widen_t<DT>(gi_bits[it].x & 0xFFFFu);
            gi[1] = widen_t<DT>(gi_bits[it].x >> 16);
            gi[2] = widen_t<DT>(gi_bits[it].y & 0xFFFFu);
            gi[3] = widen_t<DT>(gi_bits[it].y >> 16);
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) gi[q] = round_t<DT>(fbuf[(4 * u + q) * 16 + t]);
          }
          float gate[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int row = 4 * u + q;
            const float gh = round_t<DT>(fbuf[kRB * 16 + row * 16 + t]);
            gate[q] = round_t<DT>(round_t<DT>(gi[q] + gh) + gbias[row]);
          }
          const float ig = sigmoid_t<DT>(gate[0]);
          const float fg = sigmoid_t<DT>(gate[1]);
          const float gg = round_t<DT>(tanhf(gate[2]));
          const float og = sigmoid_t<DT>(gate[3]);
          const float c_prev = widen_t<DT>(ch_bits[it] & 0xFFFFu);
          const float c_new = round_t<DT>(round_t<DT>(fg * c_prev) + round_t<DT>(ig * gg));
          const float h_new = round_t<DT>(og * round_t<DT>(tanhf(c_new)));
          st_t<DT>(a.c, hj, c_new);
          st_t<DT>(a.h_out, hj, h_new);
        } else {
          static_cast<uint16_t*>(a.h_out)[hj] = static_cast<uint16_t>(ch_bits[it] >> 16);  // state kept
        }
      }
    }
  };
  if constexpr (MINB == 1) {
    for (int mt = blockIdx.z, round = 0; mt < (a.S + 15) / 16; mt += gridDim.z, ++round)
      tile(mt, round);
  } else {
    tile(blockIdx.z, 0);  // launches at two CTAs per SM carry every token tile on grid.z
  }
  if (!ok && tid == 0)
    for (int j = 0; j < sbn; ++j) mbar_wait_bounded(&bars[j], 0, a.status);
}

// Launch units (clusters of `cluster` CTAs) of a configuration resident at
// once; the kernel's smem attribute must be set already.
int resident_units(const void* kern, cudaLaunchConfig_t cfg, int cluster) {
  int n = 0;
  if (cluster > 1) {
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = cluster;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
  } else {
    int per_sm = 0, dev = 0, sms = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, static_cast<int>(cfg.blockDim.x),
                                                      cfg.dynamicSmemBytes) == cudaSuccess &&
        cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
      n = per_sm * sms;
  }
  if (n < 1) {
    (void)cudaGetLastError();
    n = 1;
  }
  return n;
}

template <int DT, int G, int RT, int MINB, int FORM>
struct Variant {
  static constexpr int kCluster = FORM == 1 ? 1 : 2;
  static size_t smem(int H) {
    return lstm_smem_layout((H + 63) / 64, G == 32 ? 2 : 1, 16 * RT, MINB == 1 ? 2 : 1).total;
  }
  static cudaError_t prepare(size_t bytes) {
    static int configured = 0;
    if (static_cast<int>(bytes) <= configured) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(lstm_step_kernel<DT, G, RT, MINB, FORM>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e == cudaSuccess) configured = static_cast<int>(bytes);
    return e;
  }
  // launch units (clusters or CTAs) resident at once; 0 if it cannot launch
  // (cached for the last hidden size asked about: the shared memory follows it)
  static int resident(const cudaLaunchConfig_t& base, int H) {
    static int cache_h = -1, cache = 0;
    if (cache_h == H) return cache;
    cudaLaunchConfig_t cfg = base;
    cfg.dynamicSmemBytes = smem(H);
    cache_h = H;
    if (prepare(cfg.dynamicSmemBytes) != cudaSuccess) {
      (void)cudaGetLastError();
      cache = 0;
      return 0;
    }
    cache = resident_units(reinterpret_cast<const void*>(lstm_step_kernel<DT, G, RT, MINB, FORM>), cfg,
                           kCluster);
    return cache;
  }
  static cudaError_t launch(cudaLaunchConfig_t cfg, const LstmMaps& maps, const LstmStepArgs& a) {
    cfg.dynamicSmemBytes = smem(a.H);
    cfg.gridDim.y = (4 * a.H) / (16 * RT);
    cudaError_t e = prepare(cfg.dynamicSmemBytes);
    if (e != cudaSuccess) return e;
    return cudaLaunchKernelEx(&cfg, lstm_step_kernel<DT, G, RT, MINB, FORM>, maps, a);
  }
};

template <int DT, int G, int FORM>
cudaError_t launch_form(const LstmMaps& maps, const LstmStepArgs& a, cudaStream_t stream, bool pdl) {
  constexpr int kCluster = FORM == 1 ? 1 : 2;
  const int bands4 = (4 * a.H) / 64;
  const int bands5 = maps.has_m5 && (4 * a.H) % 80 == 0 ? (4 * a.H) / 80 : 0;
  const int mtiles = (a.S + 15) / 16;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kCluster, bands4, std::min(mtiles, 65535));
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (kCluster > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = kCluster;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  const int n_cluster_attrs = na;
  if (pdl) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  cudaLaunchConfig_t probe = cfg;  // occupancy queries see the cluster shape only
  probe.numAttrs = n_cluster_attrs;
  // One wave if possible: 64-row bands at one CTA per SM (most registers),
  // then two per SM, then 80-row bands at two per SM.  Past that, two per SM
  // in several waves (one CTA per SM walking tiles beyond the grid limit).
  using V41 = Variant<DT, G, 4, 1, FORM>;
  using V42 = Variant<DT, G, 4, 2, FORM>;
  using V52 = Variant<DT, G, 5, 2, FORM>;
  if (mtiles > 65535) return V41::launch(cfg, maps, a);
  if (bands4 * mtiles <= V41::resident(probe, a.H)) return V41::launch(cfg, maps, a);
  if (bands4 * mtiles <= V42::resident(probe, a.H)) return V42::launch(cfg, maps, a);
  if (bands5 > 0 && bands5 * mtiles <= V52::resident(probe, a.H)) return V52::launch(cfg, maps, a);
  return V42::launch(cfg, maps, a);
}

template <int DT, int G>
cudaError_t launch_g(const LstmMaps& maps, const LstmStepArgs& a, cudaStream_t stream, bool pdl) {
  if (a.gi_table != nullptr) {
    if (a.gi_token == nullptr || a.gi_out != nullptr) return cudaErrorInvalidValue;
    return launch_form<DT, G, 1>(maps, a, stream, pdl);
  }
  return launch_form<DT, G, 0>(maps, a, stream, pdl);
}

template <int DT>
cudaError_t launch_t(int group, const LstmMaps& maps, const LstmStepArgs& a, cudaStream_t stream,
                     bool pdl) {
  switch (group) {
    case 32: return launch_g<DT, 32>(maps, a, stream, pdl);
    case 64: return launch_g<DT, 64>(maps, a, stream, pdl);
    case 128: return launch_g<DT, 128>(maps, a, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

bool lstm_step_fits(int H, int group) {
  return H % 16 == 0 && H % 64 == 0 && H <= 64 * kMaxSb && (group == 32 || group == 64 || group == 128) &&
         H % group == 0;
}

cudaError_t launch_lstm_step(int dtype, int group, const LstmMaps& maps, const LstmStepArgs& a,
                             cudaStream_t stream, bool pdl) {
  if (!lstm_step_fits(a.H, group) || a.S < 1) return cudaErrorInvalidValue;
  if (dtype == kF16) return launch_t<kF16>(group, maps, a, stream, pdl);
  if (dtype == kBF16) return launch_t<kBF16>(group, maps, a, stream, pdl);
  return cudaErrorInvalidValue;
}

}  // namespace cq
