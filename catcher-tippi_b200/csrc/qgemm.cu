// K2: affine INT8 dequant-GEMM for many rows (concurrent streams stacked to
// M >= 128), on the 5th-generation tensor cores.
//
//   y[m, n] = sum_k x[m, k] * (s[n, k/g] * q[n, k] + b[n, k/g])      (T out)
//
// the operation behind QuantizedLinear::forward_array
// (crates/nemotron-mlx/src/model/layers.rs:298-310) at batched row counts.
//
// Per CTA: one output tile of 128 weight rows x TN tokens (224, or 128 where
// 224-token tiles would leave most SMs idle; the sizes below are for 224)
// over the full K (or its slice of a cluster's K split), 19 warps.  Everything moves in
// pairs of 64-wide k-tiles (128 k): one copy per pair for the activations
// and for the weights, one hand-off per pair from the dequantisers, and the
// MMA issuer waits and commits once per pair around eight MMAs (measured on
// B200: an issuer loop of four MMAs per wait/commit round leaves the tensor
// pipe idle ~35 % of the time, eight per round keeps it busy).
//   warp 0   weight producer: the packed weight pair [128 x 128] u8 (128B
//            swizzle) and its (scale, bias) blocks into a ring that the
//            dequant warps free, starting before griddepcontrol.wait (weights
//            do not depend on the previous kernel)
//   warp 1   tcgen05.mma issuer (one elected lane), kind::f16, M = 128 weight
//            rows (the A operand, read from tensor memory), N = 224 tokens
//            (the B operand, in shared memory), K = 16 per instruction; fp32
//            accumulator in tensor-memory columns 0..223; owns the
//            tensor-memory allocation
//   warp 2   activation producer, after the wait: the x pair [2][224 x 64]
//            f16 (128B swizzle, K-major) in one 3-D copy into a ring that
//            the MMA frees (a warp of its own: two producers spinning in one
//            warp starve each other)
//   warps 3-18 dequantisers: thread (w, lane) owns weight row
//            32 (w % 4) + lane -- the tensor-memory lanes its warp may write --
//            and 16 of each k-tile's 64 k; w = s * q + b in f16 (the byte
//            becomes the exact f16 1024 + q by one PRMT, 1024 is subtracted
//            exactly, then one fused multiply-add), stored with tcgen05.st
//            into one of three A pair buffers in tensor memory, so the
//            dequantisation runs up to two pairs ahead of the MMA and the
//            dequantised weights never pass through shared memory; after the
//            last pair the same warps run the epilogue (tcgen05.ld, row
//            scale, rounding to T, output bias, activation, stores).
// Both MMA operands are f16 (A and B of one MMA share the type): bf16
// activations are converted beforehand by qgemm_prepass (per-row power-of-two
// scale, undone in the epilogue), and the weights are dequantised to f16, whose
// 11-bit significand holds s*q + b more precisely than bf16 would.  Layers
// whose scales/biases leave the f16 normal range never reach this kernel.
// No multicast: every TMA load targets this CTA's own shared memory.
#include "common.cuh"
#include "qgemm.hpp"

#include <algorithm>
#include <cstdlib>

namespace cq {

namespace {

constexpr int kBM = kGemmBN;  // weight rows per CTA: the MMA's M (A operand, in tensor memory)
constexpr int kBK = 64;       // k per MMA group: one 128-byte swizzle atom of f16 (four K=16 MMAs)
constexpr int kQStages = 3;   // packed-weight ring of k-tile pairs (freed by the dequant warps)
constexpr int kABufs = 3;     // dequantised weight pairs in tensor memory
constexpr int kDequantWarps = 16;
constexpr int kThreads = (3 + kDequantWarps) * 32;
constexpr int kDequantWarp0 = 3;
// tensor memory: the fp32 accumulator D [128 lanes][kTN columns] at column 0,
// the dequantised weight pair buffers [128 lanes][64 columns] (128 f16 along
// K) from column 256
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemA0 = 256;
// Tokens per CTA (the MMA's N, the B operand in shared memory): kGemmTN for
// wide layers, kGemmTNSmall where kGemmTN-token tiles would leave most SMs
// idle; the activation ring of k-tile pairs (a stage is freed by the MMA)
// gets what the shared memory leaves.
template <int TN>
struct TileShape {
  static constexpr int kTN = TN;
  static constexpr int kXStages = TN > 128 ? 3 : 4;
  static_assert(TN <= 256 && TN % 32 == 0 && kBM == 128, "tile shape");
};
static_assert(kTmemA0 + 64 * kABufs <= kTmemCols, "tensor memory budget");

template <int SUBG, int TN>
struct GemmSmem {
  static constexpr int kTN = TileShape<TN>::kTN;
  static constexpr int kXStages = TileShape<TN>::kXStages;
  static constexpr int kX = kTN * kBK * 2;    // one k-tile of x, f16, 128B swizzle
  static constexpr int kXStage = 2 * kX;      // a k-tile pair: [2][kTN][64] f16
  static constexpr int kQ = kBM * 2 * kBK;    // packed u8 weights of a pair, [kBM][128], 128B swizzle
  static constexpr int kSB = kBM * SUBG * 4;  // f16 (scale, bias) per row and group, one k-tile
  static constexpr int kQStage = kQ + 2 * 1024;  // packed pair + its two (scale, bias) blocks
  static constexpr int kQOff = kXStages * kXStage;
  static constexpr int kRsOff = kQOff + kQStages * kQStage;  // [kTN] row scales (fp32)
  static constexpr int kBiasOff = kRsOff + kTN * 4;          // [kBM] output bias (fp32)
  static constexpr int kBarOff = kBiasOff + kBM * 4;
  // xfull/xempty[X], qfull/qempty[Q], afull/aempty[A], accum; tmem address word
  static constexpr int kBytes =
      kBarOff + (2 * kXStages + 2 * kQStages + 2 * kABufs + 1) * 8 + 16;
  static_assert(kSB <= 1024, "scale/bias slot");
  static_assert(kX % 1024 == 0 && kQStage % 1024 == 0, "swizzled tiles stay 1024-aligned");
  // the epilogue stages its output [kTN][kBM] T, or its K-split partial
  // [kTN][kBM + 4] fp32, in the idle rings
  static_assert(kTN * (kBM * 4 + 16) <= kRsOff, "epilogue staging fits the rings");
};

// --------------------------------------------------------------- tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D (+)= A * B with A in tensor memory ([128 lanes][K/2 columns] of f16
// pairs) and B in shared memory (descriptor)
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_mma_f16_ts_acc(uint32_t d_tmem, uint32_t a_tmem,
                                                  uint64_t b_desc, uint32_t idesc) {
  asm volatile("tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, 1;" ::"r"(d_tmem),
               "r"(a_tmem), "l"(b_desc), "r"(idesc)
               : "memory");
}
// 32 lanes x 8 columns of 32-bit: thread i of the warp writes lane (quarter*32+i)
__device__ __forceinline__ void tmem_st_32x32b_x8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// 32 lanes x 32 columns of 32-bit: thread i of the warp gets lane (quarter*32+i)
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: 8-row atoms of
// 128-byte rows, atoms 1024 bytes apart (SBO), LBO unused (1), version 1.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor: f32 accumulate, f16 A and B, both K-major, M = kBM,
// N = TN.
template <int TN>
__host__ __device__ constexpr uint32_t idesc_f16_f32() {
  return (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(TN >> 3) << 17) |
         (static_cast<uint32_t>(kBM >> 4) << 24);
}

template <int DT>
__device__ __forceinline__ uint16_t t_bits(float v) {
  if constexpr (DT == kBF16) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  else return __half_as_ushort(__float2half_rn(v));
}

// forward_array's epilogue for one accumulator value: the product rounded to
// T, plus the bias rounded to T, the activation rounded to T; returns T's
// bits (the last rounding is the conversion itself).  SiLU uses the fast
// exponential and division (a few fp32 ulps, far inside T's rounding step).
template <int DT, int ACT, bool BIAS>
__device__ __forceinline__ uint16_t finish_value(float acc, float rs, float bias) {
  float v = acc * rs;
  if constexpr (BIAS) v = round_t<DT>(v) + bias;
  if constexpr (ACT == kActSilu) {
    v = round_t<DT>(v);
    v = __fdividef(v, 1.0f + __expf(-v));
  } else if constexpr (ACT == kActRelu) {
    v = v > 0.f ? v : 0.f;  // relu commutes with the rounding
  }
  return t_bits<DT>(v);
}

template <int DT>
__device__ __forceinline__ uint16_t finish_value_any(float acc, float rs, float bias, bool has_bias,
                                                     int act) {
  if (act == kActSilu)
    return has_bias ? finish_value<DT, kActSilu, true>(acc, rs, bias)
                    : finish_value<DT, kActSilu, false>(acc, rs, bias);
  if (act == kActRelu)
    return has_bias ? finish_value<DT, kActRelu, true>(acc, rs, bias)
                    : finish_value<DT, kActRelu, false>(acc, rs, bias);
  return has_bias ? finish_value<DT, kActNone, true>(acc, rs, bias)
                  : finish_value<DT, kActNone, false>(acc, rs, bias);
}

// The single-CTA epilogue of one thread: its weight row (tensor-memory lane)
// over every fourth 32-token chunk from cg on, into the [token][row] staging
// tile (`out` already points at the row's column; `pitch` in elements).
template <int DT, int ACT, bool BIAS, int TN>
__device__ __forceinline__ void finish_rows(uint32_t tq, int cg, const float* rs_s, float bias,
                                            uint16_t* out, int pitch) {
#pragma unroll 1
  for (int c = cg; c < TN / 32; c += 4) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(tq + static_cast<uint32_t>(c * 32), r);
    tmem_wait_ld();
    const float4* rs4 = reinterpret_cast<const float4*>(rs_s + c * 32);
    uint16_t* o = out + c * 32 * pitch;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 s = rs4[j / 4];
      o[(j + 0) * pitch] = finish_value<DT, ACT, BIAS>(__uint_as_float(r[j + 0]), s.x, bias);
      o[(j + 1) * pitch] = finish_value<DT, ACT, BIAS>(__uint_as_float(r[j + 1]), s.y, bias);
      o[(j + 2) * pitch] = finish_value<DT, ACT, BIAS>(__uint_as_float(r[j + 2]), s.z, bias);
      o[(j + 3) * pitch] = finish_value<DT, ACT, BIAS>(__uint_as_float(r[j + 3]), s.w, bias);
    }
  }
}

template <int DT, int G, int TN>
__global__ void __launch_bounds__(kThreads, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap xmap_tile,
                 const __grid_constant__ CUtensorMap xmap_pair,
                 const __grid_constant__ CUtensorMap qmap, const GemmArgs a) {
  constexpr int SUBG = (G == 32) ? 2 : 1;
  using L = GemmSmem<SUBG, TN>;
  constexpr int kTN = L::kTN;
  constexpr int kXStages = L::kXStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* xfull = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* xempty = xfull + kXStages;
  uint64_t* qfull = xempty + kXStages;
  uint64_t* qempty = qfull + kQStages;
  uint64_t* afull = qempty + kQStages;
  uint64_t* aempty = afull + kABufs;
  uint64_t* accum = aempty + kABufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  float* rs_s = reinterpret_cast<float*>(smem + L::kRsOff);
  float* bias_s = reinterpret_cast<float*>(smem + L::kBiasOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kBM, m0 = blockIdx.y * kTN;
  const int KT = (a.K + kBK - 1) / kBK;
  // this CTA's k tiles: all of them, or its slice of a cluster's K split
  // (the host guarantees every slice is non-empty)
  const int nsplit = gridDim.z, split = blockIdx.z;
  const int per = (KT + nsplit - 1) / nsplit;
  const int kt0 = split * per;
  const int NKT = min(KT, kt0 + per) - kt0;
  const int NP = (NKT + 1) / 2;  // k-tile pairs (the last may hold one k-tile)

  if (threadIdx.x == 0) {
    prefetch_tensormap(&xmap_tile);
    prefetch_tensormap(&xmap_pair);
    prefetch_tensormap(&qmap);
    for (int s = 0; s < kXStages; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);  // tcgen05.commit
    }
    for (int s = 0; s < kQStages; ++s) {
      mbar_init(&qfull[s], 1);
      mbar_init(&qempty[s], kDequantWarps);  // one arrival per dequant warp
    }
    for (int b = 0; b < kABufs; ++b) {
      mbar_init(&afull[b], kDequantWarps);
      mbar_init(&aempty[b], 1);  // tcgen05.commit
    }
    mbar_init(accum, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;

  // Only the activations (and the row scales, and the output's readers) tie
  // this kernel to the previous one: the weights stream and are dequantised
  // ahead of griddepcontrol.wait, so a CTA launched early under programmatic
  // dependent launch has its first weight tiles ready when the activations
  // arrive.
  pdl_launch_dependents();

  bool ok = true;
  if (warp == 0) {
    // ------------------------------------------------------------ weights
    if (lane == 0) {
      // per k-tile pair: the packed weights [kBM][128] (zero past K) and the
      // pair's (scale, bias) blocks (contiguous in sb_tiles; the second only
      // inside K)
      const uint64_t pol = l2_policy_evict_normal();
      for (int j = 0; j < NP; ++j) {
        const int kt = kt0 + 2 * j;
        const int s = j % kQStages;
        const uint32_t ph = ((j / kQStages) & 1) ^ 1;
        if (!mbar_try_wait(&qempty[s], ph)) ok = mbar_wait_bounded(&qempty[s], ph, a.status) && ok;
        uint8_t* st = smem + L::kQOff + s * L::kQStage;
        const int nsb = kt + 1 < KT ? 2 : 1;
        mbar_arrive_expect_tx(&qfull[s], L::kQ + nsb * L::kSB);
        tma_load_2d(st, &qmap, kt * kBK, n0, &qfull[s], pol);
        bulk_copy_g2s(st + L::kQ,
                      reinterpret_cast<const uint8_t*>(a.sb_tiles) +
                          (static_cast<size_t>(blockIdx.x) * KT + kt) * L::kSB,
                      nsb * L::kSB, &qfull[s]);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ activations
    // (the previous kernel's output; a warp of its own: two producers spinning
    // in one warp starve each other)
    if (lane == 0) {
      pdl_wait();
      const uint64_t pol = l2_policy_evict_normal();
      for (int j = 0; j < NP; ++j) {
        const int kt = kt0 + 2 * j;
        const int s = j % kXStages;
        const uint32_t ph = ((j / kXStages) & 1) ^ 1;
        if (!mbar_try_wait(&xempty[s], ph)) ok = mbar_wait_bounded(&xempty[s], ph, a.status) && ok;
        uint8_t* st = smem + s * L::kXStage;
        mbar_arrive_expect_tx(&xfull[s], L::kXStage);
        if (kt + 1 < a.pair_tiles) {
          tma_load_3d(st, &xmap_pair, 0, m0, kt, &xfull[s], pol);
        } else {
          // the ragged end: one copy per k-tile, zero past K
          tma_load_2d(st, &xmap_tile, kt * kBK, m0, &xfull[s], pol);
          tma_load_2d(st + L::kX, &xmap_tile, (kt + 1) * kBK, m0, &xfull[s], pol);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // The tensor pipe keeps only a few MMAs queued: scalar work between two
      // MMAs idles it (measured: 128 cycles per 128x256x16 MMA back to back,
      // twice that with per-MMA descriptor arithmetic and out-of-line waits).
      // So the waits take an inline fast path and the operand addresses
      // advance by constants: the descriptor's start address field (bits
      // 0-13) holds address >> 4 and every buffer lies below 227 KB, so adding
      // never carries out of it; a tensor-memory column is the address's low
      // half.
      constexpr uint32_t idesc = idesc_f16_f32<kTN>();
      const uint64_t db0 = sw128_kmajor_desc(smem_u32(smem));
      const uint32_t ta0 = tmem_d + kTmemA0;
      for (int j = 0; j < NP; ++j) {
        const int s = j % kXStages, b = j % kABufs;
        const uint32_t px = (j / kXStages) & 1, pa = (j / kABufs) & 1;
        if (!mbar_try_wait(&xfull[s], px)) ok = mbar_wait_bounded(&xfull[s], px, a.status) && ok;
        if (!mbar_try_wait(&afull[b], pa)) ok = mbar_wait_bounded(&afull[b], pa, a.status) && ok;
        tc_fence_after();
        // K advances by 16 f16: 32 bytes (2 descriptor units) of the x tile,
        // 8 columns of the weight pair buffer
        const uint64_t db = db0 + static_cast<uint64_t>(s * (L::kXStage >> 4));
        const uint32_t ta = ta0 + static_cast<uint32_t>(b * 64);
        tc_mma_f16_ts(tmem_d, ta, db, idesc, j != 0);
        tc_mma_f16_ts_acc(tmem_d, ta + 8, db + 2, idesc);
        tc_mma_f16_ts_acc(tmem_d, ta + 16, db + 4, idesc);
        tc_mma_f16_ts_acc(tmem_d, ta + 24, db + 6, idesc);
        if (2 * j + 1 < NKT) {  // the pair's second k-tile
          const uint64_t db2 = db + static_cast<uint64_t>(L::kX >> 4);
          tc_mma_f16_ts_acc(tmem_d, ta + 32, db2, idesc);
          tc_mma_f16_ts_acc(tmem_d, ta + 40, db2 + 2, idesc);
          tc_mma_f16_ts_acc(tmem_d, ta + 48, db2 + 4, idesc);
          tc_mma_f16_ts_acc(tmem_d, ta + 56, db2 + 6, idesc);
        }
        tc_commit(&xempty[s]);  // the x pair consumed
        tc_commit(&aempty[b]);  // the dequantised pair consumed
      }
      tc_commit(accum);
    }
  } else {
    // ------------------------------------------------------------ dequant
    // Warp w writes tensor-memory lanes 32 (w % 4) .. + 31 (the lanes a warp
    // may access): weight row r = 32 (w % 4) + lane of the tile, and of its 64
    // k the 16 of column group cg = (w - 3) / 4, i.e. columns 8 cg .. 8 cg + 7.
    // w = s * q + b in f16: the byte becomes the exact f16 1024 + q by one
    // PRMT, 1024 is subtracted exactly, then one fused multiply-add (one
    // rounding).
    const int dw = warp - kDequantWarp0;
    const int quarter = warp & 3;
    const int cg = dw >> 2;
    const int row = quarter * 32 + lane;
    const int t = threadIdx.x - kDequantWarp0 * 32;
    for (int r = t; r < kBM; r += kDequantWarps * 32) {
      const int n = n0 + r;
      bias_s[r] = (a.bias != nullptr && n < a.N) ? ld_t<DT>(a.bias, n) : 0.0f;
    }
    const __half2 k1024 = __float2half2_rn(1024.0f);
    const int h = (G == 32) ? (cg >> 1) : 0;  // which 32-wide group of the k-tile
    const int sw = row & 7;  // 128B swizzle phase of the packed row
    const uint32_t ta_row = tmem_d + kTmemA0 + (static_cast<uint32_t>(quarter * 32) << 16) +
                            static_cast<uint32_t>(cg * 8);
    for (int j = 0; j < NP; ++j) {
      const int s = j % kQStages, b = j % kABufs;
      const uint32_t pq = (j / kQStages) & 1, pa = ((j / kABufs) & 1) ^ 1;
      if (!mbar_try_wait(&qfull[s], pq)) ok = mbar_wait_bounded(&qfull[s], pq, a.status) && ok;
      if (!mbar_try_wait(&aempty[b], pa)) ok = mbar_wait_bounded(&aempty[b], pa, a.status) && ok;
      tc_fence_after();
      const uint8_t* st = smem + L::kQOff + s * L::kQStage;
      const int nh = min(2, NKT - 2 * j);  // k-tiles in this pair
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        if (hh < nh) {
          const __half2 p = reinterpret_cast<const __half2*>(st + L::kQ + hh * L::kSB)[row * SUBG + h];
          const __half2 s2 = __low2half2(p), b2 = __high2half2(p);
          // logical 16-byte chunk 4 hh + cg of the 128B-swizzled packed row
          const uint4 qv =
              *reinterpret_cast<const uint4*>(st + row * 128 + ((((hh << 2) | cg) ^ sw) << 4));
          const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
          uint32_t out[8];
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint32_t lo = __byte_perm(qw[q4], 0x64646464u, 0x4140);  // 1024 + q0, 1024 + q1
            uint32_t hi = __byte_perm(qw[q4], 0x64646464u, 0x4342);  // 1024 + q2, 1024 + q3
            const __half2 wl = __hfma2(s2, __hsub2(*reinterpret_cast<__half2*>(&lo), k1024), b2);
            const __half2 wh = __hfma2(s2, __hsub2(*reinterpret_cast<__half2*>(&hi), k1024), b2);
            out[2 * q4] = *reinterpret_cast<const uint32_t*>(&wl);
            out[2 * q4 + 1] = *reinterpret_cast<const uint32_t*>(&wh);
          }
          tmem_st_32x32b_x8(ta_row + static_cast<uint32_t>(b * 64 + hh * 32), out);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&afull[b]);
        mbar_arrive(&qempty[s]);  // the pair's packed weights and scales consumed
      }
    }

    // ------------------------------------------------------------ epilogue
    // the row scales come from the previous kernel, and the output may be
    // one of its inputs
    pdl_wait();
    for (int r = t; r < kTN; r += kDequantWarps * 32) {
      const int m = m0 + r;
      rs_s[r] = (a.row_scale != nullptr && m < a.M) ? a.row_scale[m] : 1.0f;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kDequantWarps * 32) : "memory");
    ok = mbar_wait(accum, 0, a.status) && ok;
    tc_fence_after();
    // D [n = lane][m = column]: this warp's 32 lanes (weight rows) and every
    // fourth 32-token chunk from cg on
    const int nl = quarter * 32 + lane;
    const bool has_bias = a.bias != nullptr;
    const float bias_v = bias_s[nl];
    if (nsplit > 1) {
      // K split: park this CTA's fp32 partial [kTN][kBM + 4] in the idle
      // rings (a warp's 32 lanes write 32 consecutive floats of a row); the
      // cluster reduces it below
      float* part = reinterpret_cast<float*>(smem);
#pragma unroll 1
      for (int c = cg; c < kTN / 32; c += 4) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_d + (static_cast<uint32_t>(quarter * 32) << 16) + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) part[(c * 32 + j) * (kBM + 4) + nl] = __uint_as_float(r[j]);
      }
    } else {
      // finished T values go to a [kTN][kBM] tile (rows padded by 16 bytes)
      // in the idle rings, then leave in whole rows (16-byte stores)
      constexpr int kRowBytes = kBM * 2 + 16;
      uint16_t* ot = reinterpret_cast<uint16_t*>(smem) + nl;
      const uint32_t tq = tmem_d + (static_cast<uint32_t>(quarter * 32) << 16);
      // the activation and the bias are uniform: one specialised loop each
      if (a.act == kActSilu) {
        if (has_bias) finish_rows<DT, kActSilu, true, kTN>(tq, cg, rs_s, bias_v, ot, kRowBytes / 2);
        else finish_rows<DT, kActSilu, false, kTN>(tq, cg, rs_s, bias_v, ot, kRowBytes / 2);
      } else if (a.act == kActRelu) {
        if (has_bias) finish_rows<DT, kActRelu, true, kTN>(tq, cg, rs_s, bias_v, ot, kRowBytes / 2);
        else finish_rows<DT, kActRelu, false, kTN>(tq, cg, rs_s, bias_v, ot, kRowBytes / 2);
      } else {
        if (has_bias) finish_rows<DT, kActNone, true, kTN>(tq, cg, rs_s, bias_v, ot, kRowBytes / 2);
        else finish_rows<DT, kActNone, false, kTN>(tq, cg, rs_s, bias_v, ot, kRowBytes / 2);
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kDequantWarps * 32) : "memory");
      const bool vec_ok = (a.ldy % 8) == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0;
      constexpr int kPieces = kBM / 8;  // 16-byte pieces per row
      const uint8_t* otb = reinterpret_cast<const uint8_t*>(smem);
      for (int e = t; e < kTN * kPieces; e += kDequantWarps * 32) {
        const int rr = e / kPieces, pc = e % kPieces;
        const int mm = m0 + rr, n = n0 + pc * 8;
        if (mm >= a.M) continue;
        const uint4 v = *reinterpret_cast<const uint4*>(otb + rr * kRowBytes + pc * 16);
        if (vec_ok && n + 8 <= a.N) {
          *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(a.y) + static_cast<size_t>(mm) * a.ldy + n) = v;
        } else {
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
          for (int j = 0; j < 8; ++j) {
            const int nj = n + j;
            if (nj < a.N) {
              const uint16_t bits = static_cast<uint16_t>(j & 1 ? w[j / 2] >> 16 : w[j / 2] & 0xFFFFu);
              reinterpret_cast<uint16_t*>(a.y)[static_cast<size_t>(mm) * a.ldy + nj] = bits;
            }
          }
        }
      }
    }
  }

  if (nsplit > 1) {
    // every thread of every CTA in the cluster: the partial tiles are written
    cluster_sync_all();
    if (warp >= kDequantWarp0) {
      // this CTA reduces columns [rank * W, (rank + 1) * W) of the tile over
      // the cluster's partials in rank order, then applies the epilogue
      const int t = threadIdx.x - kDequantWarp0 * 32;
      const int W = kBM / nsplit, groups = W / 4;
      const int cbase = static_cast<int>(cluster_ctarank()) * W;
      const uint32_t part_s = smem_u32(smem);
      const bool vec4 = (a.ldy % 4) == 0 && (reinterpret_cast<uintptr_t>(a.y) & 7) == 0;
      for (int item = t; item < kTN * groups; item += kDequantWarps * 32) {
        const int row = item / groups, col = cbase + (item % groups) * 4;
        const uint32_t off = static_cast<uint32_t>(row * (kBM + 4) + col) * 4u;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int r = 0; r < nsplit; ++r) {
          const float4 v = ld_dsmem_v4(mapa_shared(part_s + off, static_cast<uint32_t>(r)));
          acc[0] += v.x;
          acc[1] += v.y;
          acc[2] += v.z;
          acc[3] += v.w;
        }
        const int m = m0 + row;
        if (m >= a.M) continue;
        const float rs = rs_s[row];
        uint16_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o[j] = finish_value_any<DT>(acc[j], rs, bias_s[col + j], a.bias != nullptr, a.act);
        const int n = n0 + col;
        uint16_t* yr = reinterpret_cast<uint16_t*>(a.y) + static_cast<size_t>(m) * a.ldy;
        if (vec4 && n + 4 <= a.N) {
          *reinterpret_cast<uint2*>(yr + n) =
              make_uint2(o[0] | (static_cast<uint32_t>(o[1]) << 16),
                         o[2] | (static_cast<uint32_t>(o[3]) << 16));
        } else {
          for (int j = 0; j < 4; ++j)
            if (n + j < a.N) yr[n + j] = o[j];
        }
      }
    }
    // the partials stay readable until every CTA of the cluster is done
    cluster_sync_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_d, kTmemCols);
  }
  (void)ok;
}

// bf16 -> f16 activations with a per-row power-of-two scale: the row maximum
// lands in [2^14, 2^15); row_scale[m] = 2^e undoes it in the epilogue.  One
// CTA per row; each thread keeps up to kPrepassChunks 16-byte chunks of the
// row in registers, so the row is read once with all loads in flight.
constexpr int kPrepassThreads = 128;
constexpr int kPrepassChunks = 8;  // rows up to 128 * 8 * 8 = 8192 wide

__global__ void __launch_bounds__(kPrepassThreads)
    qgemm_prepass_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int M, int K,
                         __half* __restrict__ xo, int ldo, float* __restrict__ row_scale) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  if (m >= M) return;
  const uint16_t* xr = reinterpret_cast<const uint16_t*>(x) + static_cast<size_t>(m) * ldx;
  uint4 u[kPrepassChunks];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kPrepassChunks; ++i) {
    const int k = (threadIdx.x + i * kPrepassThreads) * 8;
    if (k < K) {
      u[i] = *reinterpret_cast<const uint4*>(xr + k);
      const uint32_t w[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        amax = fmaxf(amax, fabsf(__uint_as_float(w[j] << 16)));
        amax = fmaxf(amax, fabsf(__uint_as_float(w[j] & 0xFFFF0000u)));
      }
    }
  }
  __shared__ float red[kPrepassThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = 0.f;
#pragma unroll
  for (int w = 0; w < kPrepassThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  const int e = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFF);
  int sh = e == 0 ? 0 : 141 - e;
  sh = max(-126, min(126, sh));
  const float scale = __uint_as_float(static_cast<uint32_t>(127 + sh) << 23);
  if (threadIdx.x == 0) row_scale[m] = __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);
  uint16_t* orow = reinterpret_cast<uint16_t*>(xo) + static_cast<size_t>(m) * ldo;
#pragma unroll
  for (int i = 0; i < kPrepassChunks; ++i) {
    const int k = (threadIdx.x + i * kPrepassThreads) * 8;
    if (k < K) {
      const uint32_t w[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint16_t lo = __half_as_ushort(__float2half_rn(__uint_as_float(w[j] << 16) * scale));
        const uint16_t hi = __half_as_ushort(__float2half_rn(__uint_as_float(w[j] & 0xFFFF0000u) * scale));
        o[j] = lo | (static_cast<uint32_t>(hi) << 16);
      }
      *reinterpret_cast<uint4*>(orow + k) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

template <int DT, int G, int TN>
cudaError_t launch_gemm_typed(const GemmActMaps& amaps, const CUtensorMap& qmap, const GemmArgs& a,
                              cudaStream_t stream, bool pdl) {
  using L = GemmSmem<(G == 32) ? 2 : 1, TN>;
  auto kern = qgemm_kernel<DT, G, TN>;
  static bool configured = false;
  const int smem = L::kBytes + 1024;  // + alignment slack
  static_assert(L::kBytes + 1024 <= 227 * 1024, "smem budget");
  if (amaps.tn != TN) return cudaErrorInvalidValue;  // the maps' boxes are TN rows
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const int splits = a.splits > 1 ? a.splits : 1;
  if (splits != 1 && splits != 2 && splits != 4) return cudaErrorInvalidValue;
  if (splits > 1) {
    // every split must own at least one k tile
    const int KT = (a.K + kBK - 1) / kBK, per = (KT + splits - 1) / splits;
    if ((splits - 1) * per >= KT) return cudaErrorInvalidValue;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + kBM - 1) / kBM, (a.M + TN - 1) / TN, splits);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (splits > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = splits;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, amaps.tile, amaps.pair, qmap, a);
}

template <int DT, int G>
cudaError_t launch_gemm_tn(const GemmActMaps& amaps, const CUtensorMap& qmap, const GemmArgs& a,
                           cudaStream_t stream, bool pdl) {
  if (a.tn == kGemmTN) return launch_gemm_typed<DT, G, kGemmTN>(amaps, qmap, a, stream, pdl);
  if (a.tn == kGemmTNSmall) return launch_gemm_typed<DT, G, kGemmTNSmall>(amaps, qmap, a, stream, pdl);
  return cudaErrorInvalidValue;
}

template <int DT>
cudaError_t launch_gemm_g(int group, const GemmActMaps& amaps, const CUtensorMap& qmap,
                          const GemmArgs& a, cudaStream_t stream, bool pdl) {
  switch (group) {
    case 32: return launch_gemm_tn<DT, 32>(amaps, qmap, a, stream, pdl);
    case 64: return launch_gemm_tn<DT, 64>(amaps, qmap, a, stream, pdl);
    case 128: return launch_gemm_tn<DT, 128>(amaps, qmap, a, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_gemm(int dtype, int group, const GemmActMaps& amaps, const CUtensorMap& qmap,
                        const GemmArgs& a, cudaStream_t stream, bool pdl) {
  if (dtype == kF16) return launch_gemm_g<kF16>(group, amaps, qmap, a, stream, pdl);
  if (dtype == kBF16) return launch_gemm_g<kBF16>(group, amaps, qmap, a, stream, pdl);
  return cudaErrorInvalidValue;
}

cudaError_t launch_gemm_prepass(const void* x, int ldx, int M, int K, void* xo, int ldo,
                                float* row_scale, cudaStream_t stream, bool pdl) {
  if (M == 0) return cudaSuccess;
  if (K % 8 != 0 || K > kPrepassThreads * kPrepassChunks * 8 || ldx % 8 != 0 || ldo % 8 != 0)
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M, 1, 1);
  cfg.blockDim = dim3(kPrepassThreads, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, qgemm_prepass_kernel, reinterpret_cast<const __nv_bfloat16*>(x),
                            ldx, M, K, reinterpret_cast<__half*>(xo), ldo, row_scale);
}

int gemm_tile_tokens(int M, int N, int K, int num_sms) {
  // The narrower tile when its tiles still fit one wave: at M = 896, N = 1024
  // and 2048 run on 56 / 112 CTAs instead of 32 / 64 (prepass + GEMM per
  // call in a graph: 12.0 -> 10.4 us and 12.8 -> 10.9 us) -- unless the wide
  // tile can split K four ways in one wave, which does better (1024 x 4096:
  // 18.0 us against 18.8 us for the narrow tile split two ways).
  const int nt = (N + kBM - 1) / kBM;
  if (nt * ((M + kGemmTNSmall - 1) / kGemmTNSmall) > num_sms) return kGemmTN;
  const int KT = (K + kBK - 1) / kBK;
  if (nt * ((M + kGemmTN - 1) / kGemmTN) * 4 <= num_sms && (KT + 3) / 4 >= 16) return kGemmTN;
  return kGemmTNSmall;
}

int gemm_splits(int M, int N, int K, int num_sms, int tn) {
  const int tiles = ((N + kBM - 1) / kBM) * ((M + tn - 1) / tn);
  const int KT = (K + kBK - 1) / kBK;
  // A CTA's k-tiles run at a fixed cadence set by its copy ring, whatever the
  // number of CTAs in flight, so splitting K over a cluster shortens the
  // mainloop as long as every slice still has an SM of its own (one wave);
  // the cluster reduction and the extra ring fill cost about as much as 16
  // k-tiles save.  Measured at M = 896 (prepass + GEMM per call, in a graph):
  // 1024 x 1024: 12.0 / 12.9 / 12.7 us unsplit / 2 / 4; 2048 x 1024: 12.8 /
  // 14.1 us unsplit / 2; 1024 x 4096: 27.6 / 21.3 / 18.0 us.
  constexpr int kMinTilesPerSlice = 16;
  for (int s : {4, 2}) {
    const int per = (KT + s - 1) / s;
    if (tiles * s <= num_sms && per >= kMinTilesPerSlice && (s - 1) * per < KT) return s;
  }
  return 1;
}

// (scale, bias) pairs as f16 in the GEMM's k-tile order:
// out[ntile][ktile][row][h], h over the 32-wide halves of a 64-wide k-tile
// when g = 32 (otherwise one pair per row and k-tile); zero past N and K.
template <int DT>
__global__ void build_sb_tiles_kernel(const void* __restrict__ scales,
                                      const void* __restrict__ biases, int N, int K, int G,
                                      int subg, __half2* __restrict__ out) {
  const int KT = (K + kBK - 1) / kBK;
  const int NT = (N + kGemmBN - 1) / kGemmBN;
  const size_t total = static_cast<size_t>(NT) * KT * kGemmBN * subg;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int h = static_cast<int>(i % subg);
    const int r = static_cast<int>((i / subg) % kGemmBN);
    const int kt = static_cast<int>((i / subg / kGemmBN) % KT);
    const int nt = static_cast<int>(i / subg / kGemmBN / KT);
    const int n = nt * kGemmBN + r, k = kt * kBK + h * 32;
    float sv = 0.f, bv = 0.f;
    if (n < N && k < K) {
      const size_t gi = static_cast<size_t>(n) * (K / G) + k / G;
      sv = ld_t<DT>(scales, gi);
      bv = ld_t<DT>(biases, gi);
    }
    out[i] = __halves2half2(__float2half_rn(sv), __float2half_rn(bv));
  }
}

size_t sb_tiles_bytes(int N, int K, int group) {
  const int KT = (K + kBK - 1) / kBK;
  const int NT = (N + kGemmBN - 1) / kGemmBN;
  return static_cast<size_t>(NT) * KT * kGemmBN * (group == 32 ? 2 : 1) * sizeof(__half2);
}

cudaError_t build_sb_tiles(int dtype, const void* scales, const void* biases, int N, int K,
                           int group, void* out, cudaStream_t stream) {
  const int subg = group == 32 ? 2 : 1;
  const size_t total = sb_tiles_bytes(N, K, group) / sizeof(__half2);
  const int block = 256;
  const int grid = static_cast<int>(std::min<size_t>((total + block - 1) / block, 65535));
  if (dtype == kF16)
    build_sb_tiles_kernel<kF16><<<grid, block, 0, stream>>>(scales, biases, N, K, group, subg,
                                                           reinterpret_cast<__half2*>(out));
  else if (dtype == kBF16)
    build_sb_tiles_kernel<kBF16><<<grid, block, 0, stream>>>(scales, biases, N, K, group, subg,
                                                            reinterpret_cast<__half2*>(out));
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace cq
