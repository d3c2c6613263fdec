// Persistent RNNT chunk decoder: the whole greedy loop of one chunk (every
// frame, up to max_symbols emissions per frame, every stream) in ONE
// cooperative launch, instead of ~10 dependent launches per emitted symbol.
//
// Work split.  The grid is at most one wave of co-resident CTAs.  Each CTA
// owns fixed slices of the three weight-bound products and keeps them for
// the whole chunk:
//   * joint head tiles (16 vocabulary rows each),
//   * LSTM hidden-unit groups (4 units = the 16 gate rows i, f, g, o of those
//     units, in both the input and the recurrent projection, so the cell
//     update is fused into the same CTA),
//   * decoder-projector tiles (16 rows each; their epilogue also forms the
//     joint input relu(enc + dec) of the next symbol).
// Phases are separated by a bounded grid barrier (global counter; a timeout
// records cq_device_status and aborts every CTA).  Per symbol: head -> barrier
// -> argmax (every CTA, from the head tiles' per-stream maxima) + LSTM layer 0
// -> barrier -> LSTM layer 1 .. -> barrier -> projector -> barrier.  When no
// stream is left active on a frame (all emitted blank) the remaining symbol
// iterations of that frame are skipped by every CTA alike.
//
// Products.  mma.sync m16n8k16 f16 x f16 -> f32 with weight rows as M and
// streams as N, exactly the K1 (qgemv.cu) formulation: a weight byte is the
// exact f16 1024 + q (one PRMT), the offset is folded into the group term
//   y += inv * (s * sum(x' (1024 + q)) + (b - 1024 s) * sum(x'))
// and bf16 activations x are staged in shared memory as f16 x' = x * 2^e with
// one power-of-two scale per (stream, 64-wide sub-block), inv = 2^-e.
// Rounding points are those of the launch-per-op path (rnnt_ops.cu) and of
// the reference (rnnt.rs): every linear rounds to T, then its output bias in
// T; the LSTM cell rounds after every op; the joint input relu(enc + dec) is
// f32, cast to T for the head.
#include <algorithm>

#include "common.cuh"
#include "rnnt_ops.hpp"

namespace cq {
namespace {

constexpr int kPT = 256;  // threads per CTA
constexpr int kPW = kPT / 32;

struct Bar {
  unsigned count;
  unsigned abort;
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier over a monotonic counter; bounded.  Returns false when
// the kernel must stop (a CTA timed out or aborted).
__device__ bool grid_sync(Bar* bar, unsigned& epoch, int* status) {
  __threadfence();
  __syncthreads();
  __shared__ int aborted;
  if (threadIdx.x == 0) {
    ++epoch;
    atomicAdd(&bar->count, 1u);
    const unsigned target = epoch * gridDim.x;
    int ab = 0;
    if (ld_acquire_u32(&bar->count) < target) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_u32(&bar->count) < target) {
        if (ld_acquire_u32(&bar->abort) != 0) {
          ab = 1;
          break;
        }
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(status, kStatusWaitTimeout);
          atomicExch(&bar->abort, 1u);
          ab = 1;
          break;
        }
        __nanosleep(32);
      }
    }
    __threadfence();
    aborted = ab;
  }
  __syncthreads();
  return aborted == 0;
}

template <int DT>
__device__ __forceinline__ float ldcg_t(const void* p, size_t i) {
  const uint16_t v = __ldcg(reinterpret_cast<const unsigned short*>(p) + i);
  if constexpr (DT == kBF16) return __uint_as_float(static_cast<uint32_t>(v) << 16);
  else return __half2float(__ushort_as_half(v));
}

// Shared-memory carve-up (bytes), sized for S8 stream rows and Kmax columns.
struct PLayout {
  int ldx;  // staged row stride in halves
  int slots;  // resident 16-row weight tiles
  size_t xs, xsum, xinv, w, sb, red, y, yg, act, tok, mbar, total;
};

// Resident weight tiles of one CTA: its head tiles, its LSTM unit groups'
// input and recurrent gate rows of every layer, its projector tiles.
__host__ __device__ inline int p_slots(int hmax, int gmax, int pmax, int layers) {
  return hmax + gmax * layers * 2 + pmax;
}

__host__ __device__ inline PLayout p_layout(int S8, int Kmax, int gmax, int slots) {
  PLayout L{};
  const int nsb = Kmax / 64;
  L.ldx = Kmax + 8;
  L.slots = slots;
  size_t o = 0;
  auto take = [&](size_t& dst, size_t bytes) {
    dst = o;
    o += (bytes + 15) / 16 * 16;
  };
  take(L.xs, static_cast<size_t>(S8) * L.ldx * 2);
  take(L.xsum, static_cast<size_t>(nsb) * S8 * 4);
  take(L.xinv, static_cast<size_t>(nsb) * S8 * 4);
  take(L.w, static_cast<size_t>(slots) * 16 * Kmax);
  take(L.sb, static_cast<size_t>(slots) * nsb * 16 * 8);
  take(L.red, static_cast<size_t>(kPW) * 16 * 8 * 4);
  take(L.y, static_cast<size_t>(16) * S8 * 4);
  take(L.yg, static_cast<size_t>(2) * gmax * 16 * S8 * 4);
  take(L.act, static_cast<size_t>(S8) * 4);
  take(L.tok, static_cast<size_t>(S8) * 4);
  take(L.mbar, 16);
  L.total = o;
  return L;
}

struct Ctx {
  const RnntChunkArgs* a;
  uint8_t* smem;
  PLayout L;
  int S8, nsb;
  uint32_t* phase;  // parity of the staging mbarrier (per CTA, in registers of the caller)
};

// Stages rows row(s) (K T values each) as scaled f16 for s < S (rows S..S8-1
// stay zero from the kernel's start), with per-(stream, sub-block) sums and
// inverse scales.  The raw rows arrive as one bulk copy each (the TMA engine,
// completion on an mbarrier: a few large requests instead of thousands of
// 16-byte ones); eight threads then convert each 64-wide sub-block in place.
template <int DT, class RowFn>
__device__ void stage(const Ctx& c, int S, int K, RowFn row) {
  __half* xs = reinterpret_cast<__half*>(c.smem + c.L.xs);
  float* xsum = reinterpret_cast<float*>(c.smem + c.L.xsum);
  float* xinv = reinterpret_cast<float*>(c.smem + c.L.xinv);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(c.smem + c.L.mbar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    if (lane == 0) {
      // earlier generic accesses (this CTA's reads of xs, other CTAs' writes
      // of the rows, acquired by the grid barrier) before the async-proxy copy
      asm volatile("fence.proxy.async.shared::cta;\n\tfence.proxy.async.global;" ::: "memory");
      mbar_arrive_expect_tx(mbar, static_cast<uint32_t>(S) * K * 2);
    }
    __syncwarp();
    // every CTA reads the same rows: start each CTA at a different row so the
    // requests for any one line are spread out in time
    const int rot = static_cast<int>((blockIdx.x * 37u) % static_cast<unsigned>(S));
    for (int i = lane; i < S; i += 32) {
      const int s = (i + rot) % S;
      bulk_copy_g2s(xs + static_cast<size_t>(s) * c.L.ldx, row(s), static_cast<uint32_t>(K) * 2, mbar);
    }
  }
  mbar_wait_bounded(mbar, *c.phase, c.a->status);
  *c.phase ^= 1u;
  const int nsb = K / 64;
  // 8 lanes per sub-block (one 16-byte chunk each), 4 sub-blocks per warp
  // step, and kIlp steps per thread interleaved so their shuffle chains overlap.
  constexpr int kIlp = 4;
  const int total = c.S8 * nsb * 8;
  for (int u0 = threadIdx.x; u0 < total; u0 += kPT * kIlp) {
    uint4 v[kIlp];
    float sum[kIlp], inv[kIlp], amax[kIlp];
#pragma unroll
    for (int r = 0; r < kIlp; ++r) {
      const int u = u0 + r * kPT;
      v[r] = make_uint4(0, 0, 0, 0);
      if (u < total) {
        const int blk = u / 8, part = u % 8;
        v[r] = *reinterpret_cast<const uint4*>(xs + static_cast<size_t>(blk / nsb) * c.L.ldx +
                                              (blk % nsb) * 64 + part * 8);
      }
      sum[r] = 0.0f;
      inv[r] = 1.0f;
      amax[r] = 0.0f;
    }
    if constexpr (DT == kBF16) {
#pragma unroll
      for (int r = 0; r < kIlp; ++r) {
        const uint32_t w[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          amax[r] = fmaxf(amax[r], fabsf(__uint_as_float(w[j] << 16)));
          amax[r] = fmaxf(amax[r], fabsf(__uint_as_float(w[j] & 0xFFFF0000u)));
        }
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int r = 0; r < kIlp; ++r) amax[r] = fmaxf(amax[r], __shfl_xor_sync(0xffffffffu, amax[r], o));
#pragma unroll
      for (int r = 0; r < kIlp; ++r) {
        // scale = 2^(14 - floor(log2 amax)): the sub-block maximum lands in [2^14, 2^15)
        const int e = static_cast<int>((__float_as_uint(amax[r]) >> 23) & 0xFF);
        int sh = e == 0 ? 0 : 141 - e;
        sh = max(-126, min(126, sh));
        const float scale = __uint_as_float(static_cast<uint32_t>(127 + sh) << 23);
        inv[r] = __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);
        const uint32_t w[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const __half2 h = __floats2half2_rn(__uint_as_float(w[j] << 16) * scale,
                                              __uint_as_float(w[j] & 0xFFFF0000u) * scale);
          o[j] = *reinterpret_cast<const uint32_t*>(&h);
          const float2 f = __half22float2(h);
          sum[r] += f.x + f.y;
        }
        v[r] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    } else {
#pragma unroll
      for (int r = 0; r < kIlp; ++r) {
        const uint32_t w[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
          sum[r] += f.x + f.y;
        }
      }
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1)
#pragma unroll
      for (int r = 0; r < kIlp; ++r) sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], o);
#pragma unroll
    for (int r = 0; r < kIlp; ++r) {
      const int u = u0 + r * kPT;
      if (u >= total) continue;
      const int blk = u / 8, part = u % 8;
      const int s = blk / nsb, kb = blk % nsb;
      if constexpr (DT == kBF16)
        *reinterpret_cast<uint4*>(xs + static_cast<size_t>(s) * c.L.ldx + kb * 64 + part * 8) = v[r];
      if (part == 0) {
        xsum[kb * c.S8 + s] = sum[r];
        xinv[kb * c.S8 + s] = inv[r];
      }
    }
  }
  __syncthreads();
}

// Loads the 16-row tile W[row(i)] (u8, K columns) and its (s, b - 1024 s)
// pairs per 64-wide sub-block into resident slot `slot`; rows with row(i) < 0
// are zero.  Loads only: the caller synchronises once after every slot.
template <int DT, class RowFn>
__device__ void load_tile(const Ctx& c, int slot, const uint8_t* __restrict__ q, const void* __restrict__ sc,
                          const void* __restrict__ bi, int K, int group, RowFn row) {
  const int nsb = K / 64, gpr = K / group, Kmax = c.nsb * 64;
  uint8_t* wsm = c.smem + c.L.w + static_cast<size_t>(slot) * 16 * Kmax;
  float2* sbsm = reinterpret_cast<float2*>(c.smem + c.L.sb) + static_cast<size_t>(slot) * c.nsb * 16;
  const int per_row = K / 16;
  for (int u = threadIdx.x; u < 16 * per_row; u += kPT) {
    const int i = u / per_row, c16 = u % per_row;
    const int r = row(i);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r >= 0) v = __ldg(reinterpret_cast<const uint4*>(q + static_cast<size_t>(r) * K + c16 * 16));
    *reinterpret_cast<uint4*>(wsm + i * K + c16 * 16) = v;
  }
  for (int u = threadIdx.x; u < 16 * nsb; u += kPT) {
    const int i = u % 16, kb = u / 16;
    const int r = row(i);
    float s = 0.0f, b = 0.0f;
    if (r >= 0) {
      const size_t gi = static_cast<size_t>(r) * gpr + (kb * 64) / group;
      s = ld_t<DT>(sc, gi);
      b = ld_t<DT>(bi, gi);
    }
    sbsm[kb * 16 + i] = make_float2(s, fmaf(-1024.0f, s, b));
  }
}

// y[i][s] (f32, 16 rows x S8 streams, into `yout`) = tile `slot` . x[s] over
// the staged x (K columns).
__device__ void mtile(const Ctx& c, int slot, int K, float* yout) {
  const int nsb = K / 64, Kmax = c.nsb * 64;
  const uint8_t* wsm = c.smem + c.L.w + static_cast<size_t>(slot) * 16 * Kmax;
  const float2* sbsm = reinterpret_cast<const float2*>(c.smem + c.L.sb) + static_cast<size_t>(slot) * c.nsb * 16;
  float* red = reinterpret_cast<float*>(c.smem + c.L.red);
  const __half* xs = reinterpret_cast<const __half*>(c.smem + c.L.xs);
  const float* xsum = reinterpret_cast<const float*>(c.smem + c.L.xsum);
  const float* xinv = reinterpret_cast<const float*>(c.smem + c.L.xinv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cq4 = lane & 3, r4 = lane >> 2;
  const int nt = c.S8 / 8;
  const int kpar = kPW / nt;  // warps per stream tile (S8 <= 64)
  const int tile = warp / kpar, ks = warp % kpar;
  if (tile < nt) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const int n0 = tile * 8;
    // Two sub-blocks per iteration, four k-step accumulators each: eight
    // independent MMAs in flight instead of one dependent chain.
    auto subblock = [&](int kb, float (&d)[4][4]) {
      const uint4 va = *reinterpret_cast<const uint4*>(wsm + r4 * K + kb * 64 + 16 * cq4);
      const uint4 vb = *reinterpret_cast<const uint4*>(wsm + (r4 + 8) * K + kb * 64 + 16 * cq4);
      const __half* xr = xs + static_cast<size_t>(n0 + r4) * c.L.ldx + kb * 64 + 16 * cq4;
      const uint4 x0 = *reinterpret_cast<const uint4*>(xr);
      const uint4 x1 = *reinterpret_cast<const uint4*>(xr + 8);
      const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
      const uint32_t xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
      for (int s4 = 0; s4 < 4; ++s4) {
        // bytes 4s4..4s4+3 of this lane's 16: (b0,b1) -> k-slots 2c,2c+1;
        // (b2,b3) -> k-slots 2c+8, 2c+9; 0x64qq is the f16 value 1024 + q.
        const uint32_t a0 = __byte_perm(wa[s4], 0x64646464u, 0x4140);
        const uint32_t a1 = __byte_perm(wb[s4], 0x64646464u, 0x4140);
        const uint32_t a2 = __byte_perm(wa[s4], 0x64646464u, 0x4342);
        const uint32_t a3 = __byte_perm(wb[s4], 0x64646464u, 0x4342);
#pragma unroll
        for (int e = 0; e < 4; ++e) d[s4][e] = 0.f;
        mma_16816_f16(d[s4], a0, a1, a2, a3, xw[2 * s4], xw[2 * s4 + 1]);
      }
    };
    auto fold = [&](int kb, const float (&d)[4][4]) {
      const float2 sa = sbsm[kb * 16 + r4], sb = sbsm[kb * 16 + r4 + 8];
      const int m0 = n0 + 2 * cq4;
      const float xs0 = xsum[kb * c.S8 + m0], xs1 = xsum[kb * c.S8 + m0 + 1];
      const float iv0 = xinv[kb * c.S8 + m0], iv1 = xinv[kb * c.S8 + m0 + 1];
      float t[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) t[e] = (d[0][e] + d[1][e]) + (d[2][e] + d[3][e]);
      acc[0] = fmaf(fmaf(sa.x, t[0], sa.y * xs0), iv0, acc[0]);
      acc[1] = fmaf(fmaf(sa.x, t[1], sa.y * xs1), iv1, acc[1]);
      acc[2] = fmaf(fmaf(sb.x, t[2], sb.y * xs0), iv0, acc[2]);
      acc[3] = fmaf(fmaf(sb.x, t[3], sb.y * xs1), iv1, acc[3]);
    };
    int kb = ks;
    for (; kb + kpar < nsb; kb += 2 * kpar) {
      float d0[4][4], d1[4][4];
      subblock(kb, d0);
      subblock(kb + kpar, d1);
      fold(kb, d0);
      fold(kb + kpar, d1);
    }
    if (kb < nsb) {
      float d0[4][4];
      subblock(kb, d0);
      fold(kb, d0);
    }
    float* rw = red + warp * 16 * 8;
    rw[r4 * 8 + 2 * cq4] = acc[0];
    rw[r4 * 8 + 2 * cq4 + 1] = acc[1];
    rw[(r4 + 8) * 8 + 2 * cq4] = acc[2];
    rw[(r4 + 8) * 8 + 2 * cq4 + 1] = acc[3];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 16 * c.S8; e += kPT) {
    const int i = e / c.S8, s = e % c.S8;
    const int t = s / 8, j = s % 8;
    float v = 0.0f;
    for (int k = 0; k < kpar; ++k) v += red[((t * kpar + k) * 16 + i) * 8 + j];
    yout[i * c.S8 + s] = v;
  }
  __syncthreads();
}

template <int DT>
__global__ void __launch_bounds__(kPT, 1) rnnt_chunk_kernel(const RnntChunkArgs args) {
  extern __shared__ __align__(16) uint8_t smem[];
  const RnntChunkArgs& a = args;
  const int S = a.S, H = a.H, J = a.J, V = a.V, Q = a.Q;
  const int S8 = (S + 7) / 8 * 8;
  const int Kmax = H > J ? H : J;
  const int G = gridDim.x, cta = blockIdx.x;
  const int HT = (V + 15) / 16, UG = H / 4, PT = (J + 15) / 16;
  const int gmax = (UG + G - 1) / G, hmax = (HT + G - 1) / G, pmax = (PT + G - 1) / G;
  uint32_t stage_phase = 0;
  Ctx c{&args, smem, p_layout(S8, Kmax, gmax, p_slots(hmax, gmax, pmax, a.layers)), S8, Kmax / 64,
        &stage_phase};
  // resident slot of this CTA's n-th head tile, LSTM (group, layer, matrix), projector tile
  auto head_slot = [&](int n) { return n; };
  auto lstm_slot = [&](int gi, int l, int m) { return hmax + (gi * a.layers + l) * 2 + m; };
  auto proj_slot = [&](int n) { return hmax + gmax * a.layers * 2 + n; };
  float* y = reinterpret_cast<float*>(smem + c.L.y);
  float* yg = reinterpret_cast<float*>(smem + c.L.yg);  // [2][gmax][16][S8]
  int* act = reinterpret_cast<int*>(smem + c.L.act);
  int* tok = reinterpret_cast<int*>(smem + c.L.tok);
  Bar* bar = reinterpret_cast<Bar*>(a.barrier);
  unsigned epoch = 0;
  int p = 0;  // ping-pong index of the current h buffers

  if (cta == 0)
    for (int s = threadIdx.x; s < S; s += kPT) a.counts[s] = 0;
  if (threadIdx.x == 0) {
    mbar_init(reinterpret_cast<uint64_t*>(smem + c.L.mbar), 1);
    fence_mbar_init();
  }
  // staged rows past the last stream stay zero
  for (int e = threadIdx.x; e < (S8 - S) * (c.L.ldx / 8); e += kPT)
    reinterpret_cast<uint4*>(smem + c.L.xs)[static_cast<size_t>(S) * (c.L.ldx / 8) + e] = make_uint4(0, 0, 0, 0);
  // This CTA's weight tiles stay in shared memory for the whole chunk.
  {
    int n = 0;
    for (int t = cta; t < HT; t += G, ++n)
      load_tile<DT>(c, head_slot(n), a.head_q, a.head_s, a.head_b, J, a.group,
                    [&](int i) { return t * 16 + i < V ? t * 16 + i : -1; });
    int gi = 0;
    for (int u = cta; u < UG; u += G, ++gi)
      for (int l = 0; l < a.layers; ++l) {
        auto gate_row = [&](int i) { return (i / 4) * H + 4 * u + (i % 4); };
        load_tile<DT>(c, lstm_slot(gi, l, 0), a.ih_q[l], a.ih_s[l], a.ih_b[l], H, a.group, gate_row);
        load_tile<DT>(c, lstm_slot(gi, l, 1), a.hh_q[l], a.hh_s[l], a.hh_b[l], H, a.group, gate_row);
      }
    n = 0;
    for (int t = cta; t < PT; t += G, ++n)
      load_tile<DT>(c, proj_slot(n), a.proj_q, a.proj_s, a.proj_b, H, a.group,
                    [&](int i) { return t * 16 + i < J ? t * 16 + i : -1; });
    __syncthreads();
  }

  // fused[s][j] = T(relu(enc[s, f][j] + dec[s][j])) for this CTA's projector rows
  auto joint_input = [&](int f) {
    for (int t = cta; t < PT; t += G)
      for (int e = threadIdx.x; e < 16 * S; e += kPT) {
        const int i = e % 16, s = e / 16, j = t * 16 + i;
        if (j >= J) continue;
        const float d = ldcg_t<DT>(a.dec, static_cast<size_t>(s) * J + j);
        const float en = ld_t<DT>(a.ep, (static_cast<size_t>(s) * Q + f) * J + j);
        st_t<DT>(a.fused, static_cast<size_t>(s) * J + j, fmaxf(en + d, 0.0f));
      }
  };

  bool run = true;
  for (int f = 0; f < Q && run; ++f) {
    joint_input(f);
    for (int s = threadIdx.x; s < S8; s += kPT) act[s] = s < S ? 1 : 0;
    run = grid_sync(bar, epoch, a.status);
    for (int k = 0; k < a.max_symbols && run; ++k) {
      // ---- joint head: per-stream maxima of this CTA's vocabulary tiles
      if (cta < HT) {
        stage<DT>(c, S, J, [&](int s) {
          return static_cast<const uint16_t*>(a.fused) + static_cast<size_t>(s) * J;
        });
        int n = 0;
        for (int t = cta; t < HT; t += G, ++n) {
          mtile(c, head_slot(n), J, y);
          for (int e = threadIdx.x; e < 4 * S8; e += kPT) {
            const int s = e / 4, q4 = e % 4;  // stream, quarter of the 16 rows
            float bv = -INFINITY;
            int bidx = 0x7fffffff;
            for (int i = 4 * q4; i < 4 * q4 + 4; ++i) {
              const int v = t * 16 + i;
              if (v >= V || s >= S) break;
              const float lv = linear_epilogue<DT>(y[i * S8 + s], a.head_bias, v, kActNone);
              if (lv > bv) {  // first maximum wins ties
                bv = lv;
                bidx = v;
              }
            }
#pragma unroll
            for (int o = 1; o < 4; o <<= 1) {
              const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
              const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
              if (ov > bv || (ov == bv && oi < bidx)) {
                bv = ov;
                bidx = oi;
              }
            }
            if (q4 != 0 || s >= S) continue;
            a.part[static_cast<size_t>(t) * S + s] = make_float2(bv, __int_as_float(bidx));
          }
          __syncthreads();
        }
      }
      if (!(run = grid_sync(bar, epoch, a.status))) break;

      // ---- greedy choice of every stream (each CTA, identically): 4 lanes per
      // stream, each with its share of the head tiles' partials loaded at once
      {
        constexpr int kLanes = 4, kPer = 32;  // up to 128 head tiles
        for (int s0 = threadIdx.x / kLanes; s0 < S8; s0 += kPT / kLanes) {
          const int s = s0, sub = threadIdx.x % kLanes;
          float2 pv[kPer];
#pragma unroll
          for (int i = 0; i < kPer; ++i) {
            const int t = sub + kLanes * i;
            pv[i] = (s < S && t < HT) ? __ldcg(&a.part[static_cast<size_t>(t) * S + s])
                                      : make_float2(-INFINITY, __int_as_float(0x7fffffff));
          }
          float bv = -INFINITY;
          int bidx = 0x7fffffff;
#pragma unroll
          for (int i = 0; i < kPer; ++i) {
            const int pi = __float_as_int(pv[i].y);
            if (pv[i].x > bv || (pv[i].x == bv && pi < bidx)) {
              bv = pv[i].x;
              bidx = pi;
            }
          }
#pragma unroll
          for (int o = 1; o < kLanes; o <<= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
            if (ov > bv || (ov == bv && oi < bidx)) {
              bv = ov;
              bidx = oi;
            }
          }
          if (bidx >= V) bidx = 0;  // every logit NaN: MLX returns index 0
          if (sub == 0 && s < S) {
            tok[s] = act[s] ? bidx : a.blank;
            if (act[s]) {
              if (bidx == a.blank) {
                act[s] = 0;
              } else if (cta == 0) {
                const int n = a.counts[s];
                if (n < a.cap) {
                  a.tokens[static_cast<size_t>(s) * a.cap + n] = bidx;
                  a.token_frames[static_cast<size_t>(s) * a.cap + n] = f;
                }
                a.counts[s] = n + 1;
              }
            }
          }
        }
        __syncthreads();
        int any = 0;
        for (int s = 0; s < S; ++s) any |= act[s];
        if (!any) break;  // every stream emitted blank: next frame (all CTAs agree)
      }

      // ---- prediction network: LSTM layers for the active streams
      for (int l = 0; l < a.layers && run; ++l) {
        const void* hin = a.h[l][p];
        void* hout = a.h[l][p ^ 1];
        if (cta < UG) {
          // input projection of this CTA's unit groups
          if (l == 0) {
            stage<DT>(c, S, H, [&](int s) {
              return static_cast<const uint16_t*>(a.emb) + static_cast<size_t>(tok[s]) * H;
            });
          } else {
            stage<DT>(c, S, H, [&](int s) {
              return static_cast<const uint16_t*>(a.h[l - 1][p ^ 1]) + static_cast<size_t>(s) * H;
            });
          }
          int gi = 0;
          for (int u = cta; u < UG; u += G, ++gi) mtile(c, lstm_slot(gi, l, 0), H, yg + gi * 16 * S8);
          // recurrent projection
          stage<DT>(c, S, H, [&](int s) {
            return static_cast<const uint16_t*>(hin) + static_cast<size_t>(s) * H;
          });
          gi = 0;
          for (int u = cta; u < UG; u += G, ++gi)
            mtile(c, lstm_slot(gi, l, 1), H, yg + (gmax + gi) * 16 * S8);
          // LstmCell::step_f32 for (unit, stream); inactive streams keep their state
          gi = 0;
          for (int u = cta; u < UG; u += G, ++gi) {
            const float* yih = yg + gi * 16 * S8;
            const float* yhh = yg + (gmax + gi) * 16 * S8;
            for (int e = threadIdx.x; e < 4 * S; e += kPT) {
              const int ui = e % 4, s = e / 4, j = 4 * u + ui;
              const size_t hj = static_cast<size_t>(s) * H + j;
              if (!act[s]) {
                st_t<DT>(hout, hj, ldcg_t<DT>(hin, hj));
                continue;
              }
              float gate[4];
#pragma unroll
              for (int qg = 0; qg < 4; ++qg) {
                const int i = qg * 4 + ui;
                const float ih = round_t<DT>(yih[i * S8 + s]);
                const float hh = round_t<DT>(yhh[i * S8 + s]);
                gate[qg] = round_t<DT>(round_t<DT>(ih + hh) +
                                       ld_t<DT>(a.lstm_bias[l], static_cast<size_t>(qg) * H + j));
              }
              const float ig = round_t<DT>(1.0f / (1.0f + expf(-gate[0])));
              const float fg = round_t<DT>(1.0f / (1.0f + expf(-gate[1])));
              const float gg = round_t<DT>(tanhf(gate[2]));
              const float og = round_t<DT>(1.0f / (1.0f + expf(-gate[3])));
              const float c_prev = ldcg_t<DT>(a.c[l], hj);
              const float c_new = round_t<DT>(round_t<DT>(fg * c_prev) + round_t<DT>(ig * gg));
              const float h_new = round_t<DT>(og * round_t<DT>(tanhf(c_new)));
              st_t<DT>(a.c[l], hj, c_new);
              st_t<DT>(hout, hj, h_new);
            }
          }
        }
        run = grid_sync(bar, epoch, a.status);
      }
      if (!run) break;

      // ---- decoder projector (+ the next symbol's joint input)
      if (cta < PT) {
        const void* hl = a.h[a.layers - 1][p ^ 1];
        stage<DT>(c, S, H, [&](int s) {
          return static_cast<const uint16_t*>(hl) + static_cast<size_t>(s) * H;
        });
        int n = 0;
        for (int t = cta; t < PT; t += G, ++n) {
          mtile(c, proj_slot(n), H, y);
          for (int e = threadIdx.x; e < 16 * S; e += kPT) {
            const int i = e % 16, s = e / 16, j = t * 16 + i;
            if (j >= J) continue;
            const size_t o = static_cast<size_t>(s) * J + j;
            float d = ldcg_t<DT>(a.dec, o);
            if (act[s]) {
              d = linear_epilogue<DT>(y[i * S8 + s], a.proj_bias, j, kActNone);
              st_t<DT>(a.dec, o, d);
            }
            const float en = ld_t<DT>(a.ep, (static_cast<size_t>(s) * Q + f) * J + j);
            st_t<DT>(a.fused, o, fmaxf(en + d, 0.0f));
          }
          __syncthreads();
        }
      }
      p ^= 1;
      run = grid_sync(bar, epoch, a.status);
    }
  }
  // leave the hidden state in buffer 0 for the next chunk: each CTA copies
  // its own units (no other CTA reads them any more in this launch)
  if (p == 1) {
    for (int l = 0; l < a.layers; ++l)
      for (int u = cta; u < UG; u += G)
        for (int e = threadIdx.x; e < 4 * S; e += kPT) {
          const size_t hj = static_cast<size_t>(e % S) * H + 4 * u + e / S;
          st_t<DT>(a.h[l][0], hj, ldcg_t<DT>(a.h[l][1], hj));
        }
  }
}

}  // namespace

size_t rnnt_chunk_smem_bytes(int S, int H, int J, int V, int layers, int grid) {
  const int S8 = (S + 7) / 8 * 8;
  const int Kmax = H > J ? H : J;
  const int gmax = (H / 4 + grid - 1) / grid;
  const int hmax = ((V + 15) / 16 + grid - 1) / grid;
  const int pmax = ((J + 15) / 16 + grid - 1) / grid;
  return p_layout(S8, Kmax, gmax, p_slots(hmax, gmax, pmax, layers)).total;
}

int rnnt_chunk_grid(int dtype, int S, int H, int J, int V, int layers, int num_sms) {
  if ((V + 15) / 16 > 128) return 0;  // the argmax keeps 32 partials in 4 lanes per stream
  const int want = std::max(std::max(H / 4, (V + 15) / 16), (J + 15) / 16);
  auto k = dtype == kBF16 ? rnnt_chunk_kernel<kBF16> : rnnt_chunk_kernel<kF16>;
  int g = std::min(want, num_sms);
  for (; g >= 1; --g) {
    const size_t smem = rnnt_chunk_smem_bytes(S, H, J, V, layers, g);
    if (smem > 227 * 1024) continue;  // fewer CTAs hold more tiles each: try more
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return 0;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kPT, smem) != cudaSuccess) return 0;
    if (per_sm * num_sms >= g) return g;
  }
  return 0;
}

cudaError_t launch_rnnt_chunk(int dtype, const RnntChunkArgs& a, int grid, cudaStream_t stream) {
  auto k = dtype == kBF16 ? rnnt_chunk_kernel<kBF16> : rnnt_chunk_kernel<kF16>;
  const size_t smem = rnnt_chunk_smem_bytes(a.S, a.H, a.J, a.V, a.layers, grid);
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: they wait on one another
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, a);
}

}  // namespace cq
