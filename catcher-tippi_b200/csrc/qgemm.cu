// K2: affine INT8 dequant-GEMM for many rows (concurrent streams stacked to
// M >= 128), on the 5th-generation tensor cores.
//
//   y[m, n] = sum_k x[m, k] * (s[n, k/g] * q[n, k] + b[n, k/g])      (T out)
//
// the operation behind QuantizedLinear::forward_array
// (crates/nemotron-mlx/src/model/layers.rs:298-310) at batched row counts.
//
// Per CTA: one 128 x BN output tile over the full K, 18 warps:
//   warp 0   TMA producer: x tile [128 x 64] f16 (128B swizzle) and the packed
//            weight tile [BN x 64] u8 (64B swizzle) into a 4-stage ring
//   warp 1   tcgen05.mma issuer (one elected lane), kind::f16, M=128, N=BN,
//            K=16 per instruction, fp32 accumulator in tensor memory; owns the
//            tensor-memory allocation
//   warps 2-17 dequantisers: half a weight row per thread (sixteen warps, so
//            that the PRMT -> subtract -> FMA chains of four warps per
//            scheduler hide each other's latency), w = s * q + b in f16
//            (the byte becomes the exact f16 1024 + q by one PRMT, 1024 is
//            subtracted exactly, then one fused multiply-add), written into
//            the 128B-swizzled K-major layout the MMA reads; after the last
//            k-tile the same warps run the epilogue (tcgen05.ld, row scale,
//            rounding to T, output bias, activation, stores).
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

constexpr int kBM = 128;  // MMA M (tokens)
constexpr int kBK = 64;   // k per stage: one 128-byte swizzle atom of f16
constexpr int kStages = 4;  // TMA ring depth
constexpr int kBBufs = 2;   // dequantised weight tiles (double buffer)
constexpr int kDequantWarps = 16;
constexpr int kThreads = (2 + kDequantWarps) * 32;
constexpr int kDequantWarp0 = 2;

template <int BN, int SUBG>
struct GemmSmem {
  static constexpr int kA = kBM * kBK * 2;   // x tile, f16, 128B swizzle (16 KB)
  static constexpr int kQ = BN * kBK;        // packed u8 weights, 64B swizzle
  static constexpr int kSB = BN * SUBG * 4;  // f16 (scale, bias) per row and group
  static constexpr int kStage = kA + kQ + 2048;  // TMA stage, 1024-aligned
  static constexpr int kB = BN * kBK * 2;    // dequantised f16 weights, 128B swizzle
  static constexpr int kBOff = kStages * kStage;
  static constexpr int kBiasOff = kBOff + kBBufs * kB;  // [BN] output bias (fp32)
  static constexpr int kBarOff = kBiasOff + BN * 4;
  // full[S], empty[S], bfull[2], bempty[2], accum; tmem address word
  static constexpr int kBytes = kBarOff + (2 * kStages + 2 * kBBufs + 1) * 8 + 16;
  static_assert(kSB <= 2048, "scale/bias slot");
  static_assert(kStage % 1024 == 0 && kB % 1024 == 0, "swizzled tiles stay 1024-aligned");
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
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
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

// Instruction descriptor: f32 accumulate, f16 A and B, both K-major, M=128, N=BN.
template <int BN>
__host__ __device__ constexpr uint32_t idesc_f16_f32() {
  return (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(BN >> 3) << 17) |
         (static_cast<uint32_t>(kBM >> 4) << 24);
}

template <int DT, int G, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap qmap,
                 const GemmArgs a) {
  constexpr int SUBG = (G == 32) ? 2 : 1;
  // each dequant thread takes kChunks of the four 16-byte chunks of one row
  constexpr int kChunks = 4 * BN / (kDequantWarps * 32);
  static_assert(kChunks >= 1 && 4 % kChunks == 0 && (kDequantWarps * 32) % BN == 0,
                "chunks per dequant thread");
  using L = GemmSmem<BN, SUBG>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + kStages;
  uint64_t* bfull = empty + kStages;
  uint64_t* bempty = bfull + kBBufs;
  uint64_t* accum = bempty + kBBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  float* bias_s = reinterpret_cast<float*>(smem + L::kBiasOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * kBM;
  const int KT = (a.K + kBK - 1) / kBK;
  // this CTA's k tiles: all of them, or its slice of a cluster's K split
  // (the host guarantees every slice is non-empty)
  const int nsplit = gridDim.z, split = blockIdx.z;
  const int per = (KT + nsplit - 1) / nsplit;
  const int kt0 = split * per;
  const int NKT = min(KT, kt0 + per) - kt0;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&amap);
    prefetch_tensormap(&qmap);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDequantWarps + 1);  // dequant warps (q, scales) + MMA commit (x)
    }
    for (int b = 0; b < kBBufs; ++b) {
      mbar_init(&bfull[b], kDequantWarps);  // one arrival per dequant warp
      mbar_init(&bempty[b], 1);  // tcgen05.commit
    }
    mbar_init(accum, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;

  pdl_launch_dependents();
  pdl_wait();

  bool ok = true;
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_normal();
      for (int i = 0; i < NKT; ++i) {
        const int kt = kt0 + i;
        const int s = i % kStages;
        const uint32_t ph = (i / kStages) & 1;
        ok = mbar_wait_bounded(&empty[s], ph ^ 1, a.status) && ok;
        uint8_t* st = smem + s * L::kStage;
        mbar_arrive_expect_tx(&full[s], L::kA + L::kQ + L::kSB);
        tma_load_2d(st, &amap, kt * kBK, m0, &full[s], pol);
        tma_load_2d(st + L::kA, &qmap, kt * kBK, n0, &full[s], pol);
        // the k-tile's (scale, bias) pairs of the BN rows: one contiguous block
        bulk_copy_g2s(st + L::kA + L::kQ,
                      reinterpret_cast<const uint8_t*>(a.sb_tiles) +
                          (static_cast<size_t>(blockIdx.x) * KT + kt) * L::kSB,
                      L::kSB, &full[s]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32<BN>();
      for (int i = 0; i < NKT; ++i) {
        const int s = i % kStages, b = i % kBBufs;
        ok = mbar_wait_bounded(&full[s], (i / kStages) & 1, a.status) && ok;
        ok = mbar_wait_bounded(&bfull[b], (i / kBBufs) & 1, a.status) && ok;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * L::kStage);
        const uint32_t b_addr = smem_u32(smem + L::kBOff + b * L::kB);
#pragma unroll
        for (int ks = 0; ks < kBK / 16; ++ks) {
          // advancing K by 16 f16 = 32 bytes inside the swizzle atom
          tc_mma_f16(tmem_d, sw128_kmajor_desc(a_addr + 32 * ks), sw128_kmajor_desc(b_addr + 32 * ks),
                     idesc, (i | ks) != 0);
        }
        tc_commit(&empty[s]);   // x tile consumed
        tc_commit(&bempty[b]);  // dequantised tile consumed
      }
      tc_commit(accum);
    }
  } else {
    // ------------------------------------------------------------ dequant
    constexpr int kDT = kDequantWarps * 32;
    const int t = threadIdx.x - kDequantWarp0 * 32;
    const int row = t % BN, cfirst = (t / BN) * kChunks;  // chunks cfirst .. cfirst + kChunks - 1
    for (int r = t; r < BN; r += kDT) {
      const int n = n0 + r;
      bias_s[r] = (a.bias != nullptr && n < a.N) ? ld_t<DT>(a.bias, n) : 0.0f;
    }
    const __half2 k1024 = __float2half2_rn(1024.0f);
    for (int i = 0; i < NKT; ++i) {
      const int s = i % kStages, b = i % kBBufs;
      ok = mbar_wait_bounded(&full[s], (i / kStages) & 1, a.status) && ok;
      ok = mbar_wait_bounded(&bempty[b], ((i / kBBufs) & 1) ^ 1, a.status) && ok;
      const uint8_t* st = smem + s * L::kStage;
      const __half2* sbp = reinterpret_cast<const __half2*>(st + L::kA + L::kQ);
      uint8_t* bt = smem + L::kBOff + b * L::kB;
      // this row's (scale, bias) for the k-tile's group(s), f16
      __half2 s2[2], b2[2];
#pragma unroll
      for (int h = 0; h < SUBG; ++h) {
        const __half2 p = sbp[row * SUBG + h];
        s2[h] = __low2half2(p);
        b2[h] = __high2half2(p);
      }
      if constexpr (SUBG == 1) {
        s2[1] = s2[0];
        b2[1] = b2[0];
      }
      const uint8_t* qrow = st + L::kA + row * 64;  // 64B-swizzled u8 row
      uint8_t* brow = bt + row * 128;               // 128B-swizzled f16 row
      const int sw64 = (row >> 1) & 3, sw128 = row & 7;
#pragma unroll
      for (int cc = 0; cc < kChunks; ++cc) {
        const int c = cfirst + cc;
        // logical 16-byte chunk c of the packed row = k0 + 16c .. k0 + 16c + 15
        const uint4 qv = *reinterpret_cast<const uint4*>(qrow + ((c ^ sw64) << 4));
        const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
        const int h = (G == 32) ? (c >> 1) : 0;
        uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t lo = __byte_perm(qw[i], 0x64646464u, 0x4140);  // 1024 + q0, 1024 + q1
          uint32_t hi = __byte_perm(qw[i], 0x64646464u, 0x4342);  // 1024 + q2, 1024 + q3
          const __half2 ql = __hsub2(*reinterpret_cast<__half2*>(&lo), k1024);
          const __half2 qh = __hsub2(*reinterpret_cast<__half2*>(&hi), k1024);
          const __half2 wl = __hfma2(s2[h], ql, b2[h]);
          const __half2 wh = __hfma2(s2[h], qh, b2[h]);
          out[2 * i] = *reinterpret_cast<const uint32_t*>(&wl);
          out[2 * i + 1] = *reinterpret_cast<const uint32_t*>(&wh);
        }
        // 16 f16 = two 16-byte chunks (2c, 2c+1) of the 128-byte row
        *reinterpret_cast<uint4*>(brow + (((2 * c) ^ sw128) << 4)) =
            make_uint4(out[0], out[1], out[2], out[3]);
        *reinterpret_cast<uint4*>(brow + (((2 * c + 1) ^ sw128) << 4)) =
            make_uint4(out[4], out[5], out[6], out[7]);
      }
      fence_proxy_async_shared();  // generic-proxy writes -> tensor-core reads
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bfull[b]);
        mbar_arrive(&empty[s]);  // packed weights and scales of stage s consumed
      }
    }

    // ------------------------------------------------------------ epilogue
    // the dequant warps wrote bias_s; make it visible to each other
    asm volatile("bar.sync 1, %0;" ::"n"(kDequantWarps * 32) : "memory");
    ok = mbar_wait_bounded(accum, 0, a.status) && ok;
    tc_fence_after();
    const int quarter = warp & 3;  // TMEM lanes this warp may read
    // warps sharing a lane quarter split the columns
    constexpr int kColSplit = kDequantWarps / 4;
    const int csub = (warp - kDequantWarp0) / 4;
    const int m = m0 + quarter * 32 + lane;
    const float rs = (a.row_scale != nullptr && m < a.M) ? a.row_scale[m] : 1.0f;
    const bool has_bias = a.bias != nullptr;
    const bool vec_ok = (a.ldy % 8) == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0;
    if (nsplit > 1) {
      // K split: park this CTA's partial tile [128][BN] in the (now idle)
      // stage buffers, rows padded by 4 floats so a warp's 16-byte writes of
      // 32 rows spread over all banks; the cluster reduces it below.
      float* part = reinterpret_cast<float*>(smem);
      const int row = quarter * 32 + lane;
#pragma unroll 1
      for (int c0 = csub * 32; c0 < BN; c0 += 32 * kColSplit) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_d + (static_cast<uint32_t>(quarter * 32) << 16) + c0, r);
        tmem_wait_ld();
        float4* dst = reinterpret_cast<float4*>(part + row * (BN + 4) + c0);
#pragma unroll
        for (int v = 0; v < 8; ++v)
          dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                               __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
      }
    } else {
      // Finished T values go to a [128][BN] tile in the (idle) stage buffers,
      // rows padded by 16 bytes so a warp's 16-byte writes of 8 rows hit all
      // banks; the tile then leaves in whole rows (each warp writes 32
      // consecutive 16-byte pieces of one row: fully coalesced).
      constexpr int kRowBytes = BN * 2 + 16;
      uint8_t* ot = smem;
      const int row = quarter * 32 + lane;
#pragma unroll 1
      for (int c0 = csub * 32; c0 < BN; c0 += 32 * kColSplit) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_d + (static_cast<uint32_t>(quarter * 32) << 16) + c0, r);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float o2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int jj = 2 * j + e;
            float v = round_t<DT>(__uint_as_float(r[jj]) * rs);
            if (has_bias) v = round_t<DT>(v + bias_s[c0 + jj]);
            if (a.act == kActSilu) v = round_t<DT>(v / (1.0f + expf(-v)));
            else if (a.act == kActRelu) v = v > 0.f ? v : 0.f;
            o2[e] = v;
          }
          if constexpr (DT == kBF16) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(o2[0], o2[1]);
            pk[j] = *reinterpret_cast<const uint32_t*>(&h);
          } else {
            const __half2 h = __floats2half2_rn(o2[0], o2[1]);
            pk[j] = *reinterpret_cast<const uint32_t*>(&h);
          }
        }
        uint4* dst = reinterpret_cast<uint4*>(ot + row * kRowBytes + c0 * 2);
#pragma unroll
        for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kDequantWarps * 32) : "memory");
      constexpr int kPieces = BN / 8;  // 16-byte pieces per row
      const int t = threadIdx.x - kDequantWarp0 * 32;
      for (int e = t; e < kBM * kPieces; e += kDequantWarps * 32) {
        const int rr = e / kPieces, pc = e % kPieces;
        const int mm = m0 + rr, n = n0 + pc * 8;
        if (mm >= a.M) continue;
        const uint4 v = *reinterpret_cast<const uint4*>(ot + rr * kRowBytes + pc * 16);
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
      const int W = BN / nsplit, groups = W / 4;
      const int cbase = static_cast<int>(cluster_ctarank()) * W;
      const uint32_t part_s = smem_u32(smem);
      const bool vec4 = (a.ldy % 4) == 0 && (reinterpret_cast<uintptr_t>(a.y) & 7) == 0;
      for (int item = t; item < kBM * groups; item += kDequantWarps * 32) {
        const int row = item / groups, col = cbase + (item % groups) * 4;
        const uint32_t off = static_cast<uint32_t>(row * (BN + 4) + col) * 4u;
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
        const float rs = a.row_scale != nullptr ? a.row_scale[m] : 1.0f;
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float v = round_t<DT>(acc[j] * rs);
          if (a.bias != nullptr) v = round_t<DT>(v + bias_s[col + j]);
          if (a.act == kActSilu) v = round_t<DT>(v / (1.0f + expf(-v)));
          else if (a.act == kActRelu) v = v > 0.f ? v : 0.f;
          o[j] = v;
        }
        const int n = n0 + col;
        if (vec4 && n + 4 <= a.N) {
          uint32_t pk[2];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            if constexpr (DT == kBF16) {
              const __nv_bfloat162 h = __floats2bfloat162_rn(o[2 * j], o[2 * j + 1]);
              pk[j] = *reinterpret_cast<const uint32_t*>(&h);
            } else {
              const __half2 h = __floats2half2_rn(o[2 * j], o[2 * j + 1]);
              pk[j] = *reinterpret_cast<const uint32_t*>(&h);
            }
          }
          *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(a.y) + static_cast<size_t>(m) * a.ldy +
                                    n) = make_uint2(pk[0], pk[1]);
        } else {
          for (int j = 0; j < 4; ++j)
            if (n + j < a.N) st_t<DT>(a.y, static_cast<size_t>(m) * a.ldy + n + j, o[j]);
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
    tmem_dealloc(tmem_d, BN);
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

template <int DT, int G, int BN>
cudaError_t launch_gemm_typed(const CUtensorMap& amap, const CUtensorMap& qmap, const GemmArgs& a,
                              cudaStream_t stream, bool pdl) {
  using L = GemmSmem<BN, (G == 32) ? 2 : 1>;
  auto kern = qgemm_kernel<DT, G, BN>;
  static bool configured = false;
  const int smem = L::kBytes + 1024;  // + alignment slack
  static_assert(GemmSmem<BN, (G == 32) ? 2 : 1>::kBytes + 1024 <= 227 * 1024, "smem budget");
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
  cfg.gridDim = dim3((a.N + BN - 1) / BN, (a.M + kBM - 1) / kBM, splits);
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
  return cudaLaunchKernelEx(&cfg, kern, amap, qmap, a);
}

template <int DT>
cudaError_t launch_gemm_g(int group, const CUtensorMap& amap, const CUtensorMap& qmap,
                          const GemmArgs& a, cudaStream_t stream, bool pdl) {
  switch (group) {
    case 32: return launch_gemm_typed<DT, 32, kGemmBN>(amap, qmap, a, stream, pdl);
    case 64: return launch_gemm_typed<DT, 64, kGemmBN>(amap, qmap, a, stream, pdl);
    case 128: return launch_gemm_typed<DT, 128, kGemmBN>(amap, qmap, a, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_gemm(int dtype, int group, const CUtensorMap& amap, const CUtensorMap& qmap,
                        const GemmArgs& a, cudaStream_t stream, bool pdl) {
  if (dtype == kF16) return launch_gemm_g<kF16>(group, amap, qmap, a, stream, pdl);
  if (dtype == kBF16) return launch_gemm_g<kBF16>(group, amap, qmap, a, stream, pdl);
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

int gemm_splits(int M, int N, int K, int num_sms) {
  const int tiles = ((N + kGemmBN - 1) / kGemmBN) * ((M + kBM - 1) / kBM);
  const int KT = (K + kBK - 1) / kBK;
  // A CTA's k-tiles run at a fixed cadence set by its copy ring, whatever the
  // number of CTAs in flight, so splitting K over a cluster shortens the call
  // as long as every slice still has an SM of its own (one wave).
  for (int s : {4, 2}) {
    const int per = (KT + s - 1) / s;
    if (tiles * s <= num_sms && KT >= 2 * s && (s - 1) * per < KT) return s;
  }
  return 1;
}

size_t gemm_smem_bytes() { return GemmSmem<kGemmBN, 2>::kBytes + 1024; }

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
