/*
 * CPU oracle for the affine group-wise INT8 quantized linear (TEST INFRASTRUCTURE).
 *
 * This file is the checker, not the product: only the test suite, the smoke
 * entry and the benchmark's CPU-baseline leg load it.  The CUDA library never
 * links it and never falls back to it.
 *
 * What it restates (reference paths are relative to the Catcher workspace):
 *   - crates/nemotron-mlx/src/model/layers.rs:298-310  QuantizedLinear::forward_array:
 *       x is cast to the layer dtype T, y = quantized_matmul(x, q, s, b,
 *       transpose=true, group, bits=8) in T, then y = y + output_bias in T.
 *   - crates/nemotron-mlx/src/model/layers.rs:283-296  forward_f32: host f32 in,
 *       f32 out (the T result widened).
 *   - crates/nemotron-mlx/src/weights/artifact.rs:222-240,294-300  packed arrays
 *       `__qweight` (u32 [N, K/4]), `__scales` / `__biases` (T [N, K/g]).
 *   - mlx-rs 0.25.3 / mlx-sys 0.2.0 (MLX C++), `quantize` / `dequantize` /
 *     `quantized_matmul` with bits=8 (absent from the reference tree; restated
 *     from MLX's published affine_quantize, the fp32 form of its CPU stream):
 *       per row and per group of g consecutive elements along K, with the
 *       group's min and max taken in fp32:
 *         the edge is the extreme of larger magnitude (min when |min| > |max|,
 *         else max), step = max((max - min) / 255, 1e-7) carrying the edge's
 *         sign, q0 = round(edge / step); when q0 != 0 the scale is edge / q0
 *         and the bias is the edge (so the edge is represented exactly and the
 *         scale is negative when the edge is the max), otherwise the scale
 *         stays step and the bias is 0;
 *         q = clamp(round((w - bias) / scale), 0, 255) from the fp32 scale and
 *         bias, which are then rounded to T for storage;
 *         w_hat = scale * q + bias from the stored T values;
 *       round = round half to even; codes packed 4 per uint32 from the least
 *       significant byte up, so on a little-endian host the u32 [N, K/4] array
 *       is byte-identical to a uint8 [N, K] row-major array.
 *
 * Accumulation is fp32 (oracle_qmatmul) or fp64 (oracle_qmatmul_f64, unrounded)
 * over the dequantised fp32 weight; the output is rounded to T once (the
 * quantized_matmul result) and, when an output bias is present, rounded to T
 * again after the bias add, matching the two rounding points of forward_array.
 *
 * Parity pinning: the reference's own known-answer tests for this path
 * (crates/nemotron-mlx/tests/quantized_matmul.rs:24-47, model_layers.rs:35-78,
 * weight_roundtrip.rs:50-115) are tolerance tests against unquantised f32; the
 * oracle is pinned to those at the reference's tolerances.  MLX itself cannot
 * run here, so bit-level agreement with MLX's Metal rounding is unpinned.
 *
 * dtype codes: 0 = f16, 1 = bf16, 2 = f32 (scales/biases/activations as float).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_F16 0
#define ORACLE_BF16 1
#define ORACLE_F32 2

static inline uint32_t f32_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}
static inline float bits_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* IEEE binary16 -> binary32 (exact). */
float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    if (exp == 0) {
        if (man == 0) return bits_f32(sign);
        /* subnormal: man * 2^-24 */
        float v = (float)man * 5.9604644775390625e-08f;
        return sign ? -v : v;
    }
    if (exp == 31) return bits_f32(sign | 0x7F800000u | (man << 13));
    return bits_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

/* binary32 -> binary16, round to nearest even, with subnormals and overflow. */
uint16_t oracle_f32_to_f16(float f) {
    uint32_t x = f32_bits(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u);
    if (ax >= 0x477FF000u) return sign | 0x7C00u; /* >= 65520 rounds to inf */
    if (ax < 0x38800000u) {                         /* below 2^-14: subnormal */
        int e = (int)(ax >> 23);
        if (e < 102) return sign;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        int shift = 126 - e;
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 112u;
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

float oracle_bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

uint16_t oracle_f32_to_bf16(float f) {
    uint32_t x = f32_bits(f);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)(((x >> 16) & 0x8000u) | 0x7FC0u);
    x += 0x7FFFu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

static inline float load_t(const void* p, size_t i, int dtype) {
    if (dtype == ORACLE_F32) return ((const float*)p)[i];
    uint16_t v = ((const uint16_t*)p)[i];
    return dtype == ORACLE_BF16 ? oracle_bf16_to_f32(v) : oracle_f16_to_f32(v);
}

static inline void store_t(void* p, size_t i, float v, int dtype) {
    if (dtype == ORACLE_F32) {
        ((float*)p)[i] = v;
    } else {
        ((uint16_t*)p)[i] = dtype == ORACLE_BF16 ? oracle_f32_to_bf16(v) : oracle_f32_to_f16(v);
    }
}

/* Round to T and widen back (identity for f32). */
static inline float round_t(float v, int dtype) {
    if (dtype == ORACLE_F32) return v;
    if (dtype == ORACLE_BF16) return oracle_bf16_to_f32(oracle_f32_to_bf16(v));
    return oracle_f16_to_f32(oracle_f32_to_f16(v));
}

void oracle_round_array(const float* in, size_t n, int dtype, void* out) {
    for (size_t i = 0; i < n; ++i) store_t(out, i, in[i], dtype);
}

void oracle_widen_array(const void* in, size_t n, int dtype, float* out) {
    for (size_t i = 0; i < n; ++i) out[i] = load_t(in, i, dtype);
}

int oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/*
 * Affine 8-bit quantisation of a row-major [N, K] matrix, groups of g along K,
 * in MLX's edge/sign form (file header).  `round_input` != 0 first rounds w to
 * T, as the reference's call sites do (layers.rs:266-269 and artifact.rs:295-297
 * cast the weight to f16 before `quantize`).
 * q: N*K bytes (the u32 [N, K/4] packing); scales/biases: T [N, K/g].
 */
void oracle_quantize_group(const float* v, int g, uint8_t* q, float* scale_out, float* bias_out) {
    float lo = INFINITY, hi = -INFINITY;
    for (int k = 0; k < g; ++k) {
        lo = v[k] < lo ? v[k] : lo;
        hi = v[k] > hi ? v[k] : hi;
    }
    const int low_edge = fabsf(lo) > fabsf(hi);
    float step = (hi - lo) / 255.0f;
    step = step > 1e-7f ? step : 1e-7f;
    float scale = low_edge ? step : -step;
    const float edge = low_edge ? lo : hi;
    const float q0 = rintf(edge / scale);
    float bias = 0.0f;
    if (q0 != 0.0f) {
        scale = edge / q0;
        bias = edge;
    }
    for (int k = 0; k < g; ++k) {
        float c = rintf((v[k] - bias) / scale);
        c = c < 0.0f ? 0.0f : (c > 255.0f ? 255.0f : c);
        q[k] = (uint8_t)c;
    }
    *scale_out = scale;
    *bias_out = bias;
}

void oracle_quantize(const float* w, int N, int K, int g, int dtype, int round_input,
                     uint8_t* q, void* scales, void* biases) {
    const int groups = K / g;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        float v[128];
        for (int j = 0; j < groups; ++j) {
            const float* src = w + (size_t)n * K + (size_t)j * g;
            for (int k = 0; k < g; ++k) v[k] = round_input ? round_t(src[k], dtype) : src[k];
            float scale, bias;
            oracle_quantize_group(v, g, q + (size_t)n * K + (size_t)j * g, &scale, &bias);
            store_t(scales, (size_t)n * groups + j, scale, dtype);
            store_t(biases, (size_t)n * groups + j, bias, dtype);
        }
    }
}

/* w_hat = scale * q + bias in fp32 from the stored T scale/bias. */
void oracle_dequantize(const uint8_t* q, const void* scales, const void* biases, int N, int K,
                       int g, int dtype, float* w) {
    const int groups = K / g;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        for (int k = 0; k < K; ++k) {
            size_t gi = (size_t)n * groups + k / g;
            w[(size_t)n * K + k] =
                load_t(scales, gi, dtype) * (float)q[(size_t)n * K + k] + load_t(biases, gi, dtype);
        }
    }
}

/* Epilogue activation applied to the widened T result (0 none, 1 SiLU, 2 ReLU). */
static inline float apply_act(float v, int act) {
    if (act == 1) return v / (1.0f + expf(-v));
    if (act == 2) return v > 0.0f ? v : 0.0f;
    return v;
}

/*
 * y[M, N] = round_T(round_T(x . dequant(W)^T) + bias), fp32 accumulation.
 * x: T [M, K]; bias: T [N] or NULL; act applied after the bias add and
 * rounded to T (the fused epilogue of the encoder call sites).
 * The per-row dequantised weight is built once and reused for all M rows.
 */
void oracle_qmatmul(const void* x, int M, int K, const uint8_t* q, const void* scales,
                    const void* biases, const void* bias, int N, int g, int dtype, int act,
                    void* y) {
    const int groups = K / g;
    float* xf = (float*)malloc(sizeof(float) * (size_t)M * K);
    for (size_t i = 0; i < (size_t)M * K; ++i) xf[i] = load_t(x, i, dtype);
#pragma omp parallel
    {
        float* wrow = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
        for (int n = 0; n < N; ++n) {
            const uint8_t* qr = q + (size_t)n * K;
            for (int j = 0; j < groups; ++j) {
                float s = load_t(scales, (size_t)n * groups + j, dtype);
                float b = load_t(biases, (size_t)n * groups + j, dtype);
                for (int k = 0; k < g; ++k) wrow[j * g + k] = s * (float)qr[j * g + k] + b;
            }
            float bn = bias ? load_t(bias, (size_t)n, dtype) : 0.0f;
            for (int m = 0; m < M; ++m) {
                const float* xr = xf + (size_t)m * K;
                /* eight fixed partial sums: deterministic and vectorisable */
                float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                int k = 0;
                for (; k + 8 <= K; k += 8)
                    for (int l = 0; l < 8; ++l) acc[l] += xr[k + l] * wrow[k + l];
                for (; k < K; ++k) acc[k & 7] += xr[k] * wrow[k];
                float sum = ((acc[0] + acc[1]) + (acc[2] + acc[3])) +
                            ((acc[4] + acc[5]) + (acc[6] + acc[7]));
                float v = round_t(sum, dtype);
                if (bias) v = round_t(v + bn, dtype);
                if (act) v = round_t(apply_act(v, act), dtype);
                store_t(y, (size_t)m * N + n, v, dtype);
            }
        }
        free(wrow);
    }
    free(xf);
}

/* Same contraction in fp64, unrounded result (plus bias), for accuracy checks. */
void oracle_qmatmul_f64(const void* x, int M, int K, const uint8_t* q, const void* scales,
                        const void* biases, const void* bias, int N, int g, int dtype,
                        double* y) {
    const int groups = K / g;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        for (int m = 0; m < M; ++m) {
            double acc = 0.0;
            for (int k = 0; k < K; ++k) {
                size_t gi = (size_t)n * groups + k / g;
                double w = (double)load_t(scales, gi, dtype) * (double)q[(size_t)n * K + k] +
                           (double)load_t(biases, gi, dtype);
                acc += (double)load_t(x, (size_t)m * K + k, dtype) * w;
            }
            if (bias) acc += (double)load_t(bias, (size_t)n, dtype);
            y[(size_t)m * N + n] = acc;
        }
    }
}

/* Unquantised fp32 reference matmul (the reference tests' fp32_reference). */
void oracle_f32_linear(const float* x, int M, int K, const float* w, int N, const float* bias,
                       float* y) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
        for (int n = 0; n < N; ++n) {
            float sum = bias ? bias[n] : 0.0f;
            for (int k = 0; k < K; ++k) sum += x[(size_t)m * K + k] * w[(size_t)n * K + k];
            y[(size_t)m * N + n] = sum;
        }
    }
}
