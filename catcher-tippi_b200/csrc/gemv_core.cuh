// Arithmetic of the small-M dequant-GEMV (K1, qgemv.cu): activation loads and
// their conversion to f16 MMA operands, the per-64-k-sub-block tensor-core
// step over a weight tile in shared memory, and the output rounding.
//
// Operation: y[m, n] = sum_k x[m, k] * (s[n, k/g] * q[n, k] + b[n, k/g]) in
// the MLX affine INT8 layout (QuantizedLinear::forward_array,
// crates/nemotron-mlx/src/model/layers.rs:298-310).  Weight rows are the MMA M
// dimension, tokens the N dimension (two n8 tiles = 16 tokens).  A weight byte
// q becomes the f16 value 1024 + q with one PRMT (bits 0x64qq), exact; the
// offset is folded into the group bias term
//     y += s * sum(x * (1024 + q)) + (b - 1024 s) * sum(x)
// so the dequantised weight is never rounded.  bf16 activations move to f16
// with a per-(token, 64-wide sub-block) power-of-two scale undone in fp32.
// Each lane reads 16 contiguous weight bytes per row; the k-slot order of the
// MMA fragments is permuted identically for A and B, so the MLX layout is
// consumed as is.
#pragma once

#include "common.cuh"

namespace cq {

// Column of (weight row, token) in the cross-warp reduction buffers
// ([warp][row][16] floats): the token index is XORed with an even mask built
// from row bits 1..3 (bit 1 -> 8, bit 2 -> 2, bit 3 -> 4).  The float2
// partial stores of a half-warp (rows r4 = 0..3 x lanes c) then fall on
// disjoint banks, and the sums read rows-fastest (32 lanes = 16 rows x 2
// tokens at 16 rows per CTA) hit 32 distinct banks; with 32 or more rows the
// reads are 2-way.  An even mask keeps each float2 pair adjacent.
__device__ __forceinline__ int red_col(int row, int tok) {
  return tok ^ (((row & 2) << 2) | ((row & 12) >> 1));
}

// Raw activation loads of one token for one 64-wide sub-block (this lane's 16
// values; zeros past M and past K):
//   G >= 64: k = kb + 16c + [0, 16)
//   G == 32: k = kb + 8c + [0, 8) and kb + 32 + 8c + [0, 8)
template <int G>
__device__ __forceinline__ void load_x_raw(const void* __restrict__ x, int ldx, int M, int K, int m,
                                           int kb, int c, uint4& r0, uint4& r1) {
  r0 = make_uint4(0, 0, 0, 0);
  r1 = make_uint4(0, 0, 0, 0);
  if (m >= M) return;
  const uint16_t* xr = reinterpret_cast<const uint16_t*>(x) + static_cast<size_t>(m) * ldx;
  if constexpr (G >= 64) {
    r0 = ld_global_cg_v4(xr + kb + 16 * c);
    r1 = ld_global_cg_v4(xr + kb + 16 * c + 8);
  } else {
    r0 = ld_global_cg_v4(xr + kb + 8 * c);
    if (kb + 32 < K) r1 = ld_global_cg_v4(xr + kb + 32 + 8 * c);
  }
}

// Converts this lane's 16 raw activation values into f16 MMA B-fragments and
// returns the inverse of the power-of-two scale that was applied (bf16: one
// scale per token and 64-wide sub-block, shared by the quad's 4 lanes).
template <int DT>
__device__ __forceinline__ void x_frag(const uint4& r0, const uint4& r1, uint32_t (&xb)[8],
                                       float& inv) {
  const uint32_t w[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
  if constexpr (DT == kF16) {
#pragma unroll
    for (int p = 0; p < 8; ++p) xb[p] = w[p];
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
    }
  }
}

template <int DT>
__device__ __forceinline__ float epilogue_value(float acc, bool has_bias, float bias, int act) {
  float o = round_t<DT>(acc);
  if (has_bias) o = round_t<DT>(o + bias);
  if (act == kActSilu) {
    o = round_t<DT>(o / (1.0f + expf(-o)));
  } else if (act == kActRelu) {
    o = o > 0.0f ? o : 0.0f;
  }
  return o;
}

// Token-side operands of one 64-wide sub-block for this lane: B fragments of
// both 8-token halves, and the activation sums / inverse scales the epilogue
// of the accumulator columns 2c, 2c+1 needs.
template <int G>
struct XOperands {
  static constexpr int SUBG = (G == 32) ? 2 : 1;
  uint32_t xb[2][8];
  float xsA[2][SUBG], xsB[2][SUBG], ivA[2], ivB[2];
};

// xr: this lane's raw loads (load_x_raw) for tokens r4 and r4 + 8.
// The per-(token, group) sums of the converted activations, which the group
// term of the epilogue needs, come from the tensor pipe: an MMA with an
// all-ones A fragment sums each token's sixteen k-slots of a k-step, and
// lands them in the accumulator layout the epilogue reads (columns 2c and
// 2c + 1 = tokens 2c and 2c + 1), so no unpacking, adds or shuffles are
// needed for them.
template <int DT, int G>
__device__ __forceinline__ XOperands<G> x_operands(const uint4 (&xr)[2][2], int lane) {
  constexpr int SUBG = XOperands<G>::SUBG;
  const int c = lane & 3;
  XOperands<G> o;
  float inv[2];
  x_frag<DT>(xr[0][0], xr[0][1], o.xb[0], inv[0]);
  x_frag<DT>(xr[1][0], xr[1][1], o.xb[1], inv[1]);
  constexpr uint32_t kOnes = 0x3C003C00u;  // f16 1.0 twice
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    float sm[SUBG][4];
#pragma unroll
    for (int h = 0; h < SUBG; ++h)
#pragma unroll
      for (int e = 0; e < 4; ++e) sm[h][e] = 0.f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const int h = (SUBG == 2) ? (s >> 1) : 0;  // k-steps 0, 1 / 2, 3: the two 32-wide groups
      mma_16816_f16(sm[h], kOnes, kOnes, kOnes, kOnes, o.xb[nt][2 * s], o.xb[nt][2 * s + 1]);
    }
#pragma unroll
    for (int h = 0; h < SUBG; ++h) {
      o.xsA[nt][h] = sm[h][0];
      o.xsB[nt][h] = sm[h][1];
    }
    o.ivA[nt] = __shfl_sync(0xFFFFFFFFu, inv[nt], 8 * c);
    o.ivB[nt] = __shfl_sync(0xFFFFFFFFu, inv[nt], 8 * c + 4);
  }
  return o;
}

// One 64-wide sub-block of a band of RB = 16 * RT weight rows: wj is the
// [RB][64] u8 tile in shared memory, sbj the [SUBG][RB] (s, b - 1024 s) pairs;
// accumulates into acc[row tile][token half][fragment].
template <int DT, int G, int RT>
__device__ __forceinline__ void subblock_mma(const uint8_t* wj, const float2* sbj,
                                             const XOperands<G>& xo, int lane,
                                             float (&acc)[RT][2][4]) {
  constexpr int SUBG = XOperands<G>::SUBG;
  constexpr int RB = 16 * RT;
  const int c = lane & 3, r4 = lane >> 2;
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
        mma_16816_f16(d[nt][h], a0, a1, a2, a3, xo.xb[nt][2 * s], xo.xb[nt][2 * s + 1]);
    }
#pragma unroll
    for (int h = 0; h < SUBG; ++h) {
      const float2 sa = sbj[h * RB + ra];
      const float2 sb = sbj[h * RB + rb];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const float t0 = fmaf(sa.x, d[nt][h][0], sa.y * xo.xsA[nt][h]);
        const float t1 = fmaf(sa.x, d[nt][h][1], sa.y * xo.xsB[nt][h]);
        const float t2 = fmaf(sb.x, d[nt][h][2], sb.y * xo.xsA[nt][h]);
        const float t3 = fmaf(sb.x, d[nt][h][3], sb.y * xo.xsB[nt][h]);
        if constexpr (DT == kF16) {
          acc[i][nt][0] += t0;
          acc[i][nt][1] += t1;
          acc[i][nt][2] += t2;
          acc[i][nt][3] += t3;
        } else {
          acc[i][nt][0] = fmaf(t0, xo.ivA[nt], acc[i][nt][0]);
          acc[i][nt][1] = fmaf(t1, xo.ivB[nt], acc[i][nt][1]);
          acc[i][nt][2] = fmaf(t2, xo.ivA[nt], acc[i][nt][2]);
          acc[i][nt][3] = fmaf(t3, xo.ivB[nt], acc[i][nt][3]);
        }
      }
    }
  }
}

}  // namespace cq
