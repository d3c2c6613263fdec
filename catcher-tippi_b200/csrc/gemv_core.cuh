// Arithmetic of the small-M dequant-GEMV (K1, qgemv.cu): activation loads,
// the per-64-k-sub-block tensor-core step over a weight tile in shared
// memory, and the output rounding.
//
// Operation: y[m, n] = sum_k x[m, k] * (s[n, k/g] * q[n, k] + b[n, k/g]) in
// the MLX affine INT8 layout (QuantizedLinear::forward_array,
// crates/nemotron-mlx/src/model/layers.rs:298-310).  Weight rows are the MMA M
// dimension, tokens the N dimension (two n8 tiles = 16 tokens).  The
// activations are the B operand in their own type, as loaded; the weight
// bytes become exact values of that type offset by a constant o, and the
// offset is folded into the group bias term
//     y += s * sum(x * (o + q)) + (b - o s) * sum(x)
// so the dequantised weight is never rounded:
//   f16:  q -> 1024 + q with one PRMT (bits 0x64qq), o = 1024;
//   bf16: q = l + 128 h (l < 128) -> two A fragments, 128 + l (bits 0x43,l)
//         and 128 h (0x4300 or 0), accumulated by two MMAs, o = 128.
// Each lane reads 16 contiguous weight bytes per row; the k-slot order of the
// MMA fragments is permuted identically for A and B, so the MLX layout is
// consumed as is.
#pragma once

#include "common.cuh"

namespace cq {

// The constant o that the A-fragment values of a weight byte q carry (o + q).
template <int DT>
__host__ __device__ constexpr float weight_offset() {
  return DT == kBF16 ? 128.0f : 1024.0f;
}

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
// wide (x and every row 32-byte aligned, x_rows_wide): the G >= 64 lane's 32
// bytes come in one 256-bit load.  Two 16-byte loads would each touch all four
// 32-byte sectors of the quad's 128 bytes by halves, so the sectors would
// cross from L2 twice.
template <int G>
__device__ __forceinline__ void load_x_raw(const void* __restrict__ x, int ldx, int M, int K, int m,
                                           int kb, int c, uint4& r0, uint4& r1, bool wide) {
  r0 = make_uint4(0, 0, 0, 0);
  r1 = make_uint4(0, 0, 0, 0);
  if (m >= M) return;
  const uint16_t* xr = reinterpret_cast<const uint16_t*>(x) + static_cast<size_t>(m) * ldx;
  if constexpr (G >= 64) {
    if (wide) {
      ld_global_cg_v8(xr + kb + 16 * c, r0, r1);
    } else {
      r0 = ld_global_cg_v4(xr + kb + 16 * c);
      r1 = ld_global_cg_v4(xr + kb + 16 * c + 8);
    }
  } else {
    r0 = ld_global_cg_v4(xr + kb + 8 * c);
    if (kb + 32 < K) r1 = ld_global_cg_v4(xr + kb + 32 + 8 * c);
  }
}

// Whether load_x_raw may use 256-bit loads on x[., ldx] (16-bit elements).
__device__ __forceinline__ bool x_rows_wide(const void* x, int ldx) {
  return ((reinterpret_cast<uintptr_t>(x) | (static_cast<uintptr_t>(ldx) * 2)) & 31) == 0;
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
// both 8-token halves, and the activation sums the group term of the
// accumulator columns 2c, 2c+1 needs.
template <int G>
struct XOperands {
  static constexpr int SUBG = (G == 32) ? 2 : 1;
  uint32_t xb[2][8];
  float xsA[2][SUBG], xsB[2][SUBG];
};

// xr: this lane's raw loads (load_x_raw) for tokens r4 and r4 + 8; the 16-bit
// pairs are the B fragments as they are.  The per-(token, group) activation
// sums come from the tensor pipe: an MMA with an all-ones A fragment sums
// each token's sixteen k-slots of a k-step, and lands them in the accumulator
// layout the epilogue reads (columns 2c and 2c + 1 = tokens 2c and 2c + 1),
// so no unpacking, adds or shuffles are needed for them.
template <int DT, int G>
__device__ __forceinline__ XOperands<G> x_operands(const uint4 (&xr)[2][2]) {
  constexpr int SUBG = XOperands<G>::SUBG;
  XOperands<G> o;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const uint4& r0 = xr[nt][0];
    const uint4& r1 = xr[nt][1];
    o.xb[nt][0] = r0.x; o.xb[nt][1] = r0.y; o.xb[nt][2] = r0.z; o.xb[nt][3] = r0.w;
    o.xb[nt][4] = r1.x; o.xb[nt][5] = r1.y; o.xb[nt][6] = r1.z; o.xb[nt][7] = r1.w;
  }
  // 1.0 twice in the activations' type
  constexpr uint32_t kOnes = DT == kBF16 ? 0x3F803F80u : 0x3C003C00u;
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
      mma_16816<DT>(sm[h], kOnes, kOnes, kOnes, kOnes, o.xb[nt][2 * s], o.xb[nt][2 * s + 1]);
    }
#pragma unroll
    for (int h = 0; h < SUBG; ++h) {
      o.xsA[nt][h] = sm[h][0];
      o.xsB[nt][h] = sm[h][1];
    }
  }
  return o;
}

// One 64-wide sub-block of a band of RB = 16 * RT weight rows: wj is the
// [RB][64] u8 tile in shared memory, sbj the [SUBG][RB] (s, b - o s) pairs
// (o = weight_offset<DT>()); accumulates into acc[row tile][token half][fragment].
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
      // (b2,b3) -> k-slots 2c+8, 2c+9.
      if constexpr (DT == kBF16) {
        // 0x43qq with bit 7 of qq cleared is the bf16 value 128 + (q & 127);
        // (0x0080 per set bit 7) * 0x86 = 0x4300 is the bf16 value 128.
        const uint32_t p0 = __byte_perm(wa[s], 0x43434343u, 0x4140);
        const uint32_t p1 = __byte_perm(wb[s], 0x43434343u, 0x4140);
        const uint32_t p2 = __byte_perm(wa[s], 0x43434343u, 0x4342);
        const uint32_t p3 = __byte_perm(wb[s], 0x43434343u, 0x4342);
        const uint32_t l0 = p0 & 0xFF7FFF7Fu, h0 = (p0 & 0x00800080u) * 0x86u;
        const uint32_t l1 = p1 & 0xFF7FFF7Fu, h1 = (p1 & 0x00800080u) * 0x86u;
        const uint32_t l2 = p2 & 0xFF7FFF7Fu, h2 = (p2 & 0x00800080u) * 0x86u;
        const uint32_t l3 = p3 & 0xFF7FFF7Fu, h3 = (p3 & 0x00800080u) * 0x86u;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          mma_16816_bf16(d[nt][h], l0, l1, l2, l3, xo.xb[nt][2 * s], xo.xb[nt][2 * s + 1]);
          mma_16816_bf16(d[nt][h], h0, h1, h2, h3, xo.xb[nt][2 * s], xo.xb[nt][2 * s + 1]);
        }
      } else {
        // 0x64qq is the f16 value 1024 + q.
        const uint32_t a0 = __byte_perm(wa[s], 0x64646464u, 0x4140);
        const uint32_t a1 = __byte_perm(wb[s], 0x64646464u, 0x4140);
        const uint32_t a2 = __byte_perm(wa[s], 0x64646464u, 0x4342);
        const uint32_t a3 = __byte_perm(wb[s], 0x64646464u, 0x4342);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
          mma_16816_f16(d[nt][h], a0, a1, a2, a3, xo.xb[nt][2 * s], xo.xb[nt][2 * s + 1]);
      }
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
        acc[i][nt][0] += t0;
        acc[i][nt][1] += t1;
        acc[i][nt][2] += t2;
        acc[i][nt][3] += t3;
      }
    }
  }
}

}  // namespace cq
