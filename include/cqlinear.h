/*
 * cqlinear.h - C ABI of the B200 affine INT8 quantized linear.
 *
 * This boundary stands in for the quantized-linear call sites of Catcher's
 * nemotron-mlx crate.  Each entry names the reference interface it replaces
 * (paths relative to the Catcher workspace).
 *
 * Conventions
 *   - Plain pointers and sizes only; no CUDA or framework types.  `stream` is
 *     a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Every call returns a cq_status; no C++ exception crosses the ABI.  On
 *     failure cq_last_error() returns a thread-local message (mirrors
 *     catcher_last_error, crates/catcher-ffi/src/lib.rs:30-32).
 *   - A handle may be used from one thread at a time (the caller serialises
 *     calls per handle, as the reference's MLX-backed layers require);
 *     distinct handles are independent and may run on distinct streams.
 *   - Weights use the MLX affine layout: qweight u32 [N, K/4] holding four
 *     8-bit codes per word from the least significant byte up, scales and
 *     biases of dtype T [N, K/g]; w_hat = scale * q + bias.
 *   - Supported group sizes: 32, 64, 128 (crates/nemotron-mlx/src/weights/
 *     manifest.rs:206-220).  K must be a multiple of the group size.
 */
#ifndef CQLINEAR_H
#define CQLINEAR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes; numeric values follow catcher.h (crates/catcher-ffi/include/catcher.h:30-37). */
typedef int32_t cq_status;
enum {
    CQ_OK = 0,
    CQ_INVALID_ARGUMENT = -1, /* null pointer, shape, group size, alignment */
    CQ_RUNTIME_ERROR = -3     /* CUDA error or device watchdog timeout */
};

/* Element type T of activations, outputs, scales, biases and output bias. */
typedef int32_t cq_dtype;
enum {
    CQ_F16 = 0,  /* the reference's artifact dtype (artifact.rs:294-300) */
    CQ_BF16 = 1,
    CQ_F32 = 2   /* backend::quantized_matmul keeps f32 scales (backend/mod.rs:78-93) */
};

/* Optional fused epilogue activation, applied to the T result and re-rounded to T. */
typedef int32_t cq_act;
enum { CQ_ACT_NONE = 0, CQ_ACT_SILU = 1, CQ_ACT_RELU = 2 };

typedef struct cq_linear cq_linear;

/* Thread-local message for the last failed call on this thread ("" if none).
 * Replaces catcher_last_error (crates/catcher-ffi/src/lib.rs:30-32, :779-786). */
const char *cq_last_error(void);

/* Library version string. */
const char *cq_version(void);

/* Nonzero when a CUDA device of compute capability 10.x is usable.
 * Replaces backend::is_metal_available (crates/nemotron-mlx/src/backend/mod.rs:28-38). */
int32_t cq_is_device_available(void);

/*
 * Binds packed affine INT8 arrays to a new layer on `device`; the arrays may
 * be in host or device memory (unified addressing) and the handle owns a
 * device copy.  bias_or_null: T [output_dims] or NULL (no
 * output bias, equivalent to the zero bias the reference substitutes).
 * Replaces QuantizedLinear::from_artifact (crates/nemotron-mlx/src/model/layers.rs:221-256).
 */
cq_status cq_linear_create(const uint32_t *qweight, const void *scales, const void *biases,
                           const void *bias_or_null, int32_t output_dims, int32_t input_dims,
                           int32_t group_size, cq_dtype dtype, int32_t device, cq_linear **out);

/*
 * Quantises a row-major f32 [output_dims, input_dims] weight on the device
 * (the weight is first rounded to T) and binds it with an f32 output bias of
 * bias_len == output_dims values (rounded to T).
 * Replaces QuantizedLinear::from_f32 (crates/nemotron-mlx/src/model/layers.rs:259-280),
 * including its "linear weight/bias mismatch" and "incompatible with group size" errors.
 */
cq_status cq_linear_create_from_f32(const float *weight, size_t weight_len, int32_t output_dims,
                                    int32_t input_dims, const float *bias, size_t bias_len,
                                    int32_t group_size, cq_dtype dtype, int32_t device,
                                    cq_linear **out);

/*
 * New layer whose output rows are the concatenation of `count` layers with
 * equal input_dims, group size, dtype and device (e.g. q, k, v projections
 * sharing one input, crates/nemotron-mlx/src/model/encoder.rs:194-206, run as
 * one launch).  Missing output biases are filled with zeros.
 * No single reference counterpart: composes QuantizedLinear instances.
 */
cq_status cq_linear_concat(cq_linear *const *parts, int32_t count, cq_linear **out);

/*
 * y[rows, N] = x[rows, K] . dequant(W)^T (+ bias), device pointers in T,
 * asynchronous on `stream`.  x rows must be 16-byte aligned.
 * Replaces QuantizedLinear::forward_array (crates/nemotron-mlx/src/model/layers.rs:298-310)
 * and PointwiseConv1d::forward_f32's row-flattened matmul (layers.rs:342-351).
 */
cq_status cq_linear_forward(cq_linear *layer, const void *x, int32_t rows, void *y, void *stream);

/*
 * As cq_linear_forward with explicit leading dimensions (elements; ldx a
 * multiple of 8 for 16-bit T) and a fused activation: the encoder call sites'
 * SiLU after FFN linear1 (crates/nemotron-mlx/src/model/encoder.rs:323-336) and
 * ReLU after the prompt projector's first linear (prompt.rs:105-140).
 */
cq_status cq_linear_forward_ex(cq_linear *layer, const void *x, int32_t ldx, int32_t rows, void *y,
                               int32_t ldy, cq_act act, void *stream);

/*
 * Host f32 in, host f32 out, synchronous: x is rounded to T, run through
 * forward_array, and the T result widened to f32.  Fails with
 * "invalid model shape: linear input has {len} values, expected {rows}x{K}".
 * Replaces QuantizedLinear::forward_f32 (crates/nemotron-mlx/src/model/layers.rs:283-296).
 */
cq_status cq_linear_forward_f32(cq_linear *layer, const float *input, size_t input_len,
                                int32_t rows, float *output, size_t output_len);

/*
 * The tensor-core GEMM's activation format, for producers that can emit it
 * directly (this library's encoder LayerNorm does): x bf16 [rows, ldx] ->
 * x16 f16 [rows, input_dims] (row stride input_dims, 16-byte aligned) and
 * row_scale fp32 [rows]; each row is scaled by the power of two that puts its
 * largest magnitude in [2^14, 2^15), and row_scale holds the inverse, which
 * the GEMM's epilogue applies.  Only for calls that run the tensor-core GEMM:
 * bf16 layers at rows >= 256 whose scales fit f16 (else CQ_INVALID_ARGUMENT).
 * Asynchronous on `stream`.  No reference counterpart: an implementation
 * format of this library's batched path.
 */
cq_status cq_linear_prescale_activations(cq_linear *layer, const void *x, int32_t ldx,
                                         int32_t rows, void *x16, float *row_scale, void *stream);

/*
 * cq_linear_forward_ex on activations already in the tensor-core format
 * (cq_linear_prescale_activations): bit-identical results, without the
 * conversion launch.  Same restrictions; asynchronous on `stream`.
 */
cq_status cq_linear_forward_prescaled(cq_linear *layer, const void *x16, const float *row_scale,
                                      int32_t rows, void *y, int32_t ldy, cq_act act,
                                      void *stream);

/*
 * Sizes the layer's workspace for calls of up to max_rows rows.  Calls with
 * rows >= 256 run on the tensor-core GEMM; for bf16 layers that path stages
 * the activations as f16 in a per-layer workspace that is otherwise
 * allocated on the first such call.  Reserve before capturing calls into a
 * CUDA graph.  No reference counterpart (MLX allocates inside its graph).
 */
cq_status cq_linear_reserve(cq_linear *layer, int32_t max_rows);

/*
 * cq_linear_forward_ex without any device allocation, for callers that
 * cannot allocate device memory once a stream is running: a transcriber fed
 * from a real-time audio path, or a host held to a GPU memory budget fixed at
 * start-up, cannot afford a cudaMalloc mid-stream (it can block for
 * milliseconds, synchronises with queued work, and can fail under memory
 * pressure).  The only scratch the layer needs -- the f16 copy of bf16
 * activations that calls with rows >= 256 stage before the tensor-core GEMM --
 * comes from an 8 MiB array that is part of the library's device image, held
 * by every GPU that loads the library until the process exits.  Limit:
 * rows * input_dims * 2 (rounded up to 256) + rows * 4 bytes <= 8 MiB, e.g.
 * 896 rows at input_dims 4096; larger calls fail with CQ_INVALID_ARGUMENT and
 * a message naming the limit.  The first such call on a device looks the
 * array's device address up (once per device), so make it before any stream
 * capture; a first call on a capturing stream fails with CQ_INVALID_ARGUMENT
 * and says so.  The looked-up address, like every handle of this library,
 * does not survive a cudaDeviceReset.  All calls share the array and it keeps
 * the last call's contents (every call overwrites what it reads); calls that
 * overlap on the GPU race, so serialise them (one stream, or events).
 * No counterpart in the reference: MLX allocates inside its own graph.
 */
cq_status cq_linear_forward_noalloc(cq_linear *layer, const void *x, int32_t ldx, int32_t rows,
                                    void *y, int32_t ldy, cq_act act, void *stream);

/* Dimensions and type of a layer (layers.rs:312-318). */
int32_t cq_linear_input_dims(const cq_linear *layer);
int32_t cq_linear_output_dims(const cq_linear *layer);
int32_t cq_linear_group_size(const cq_linear *layer);
cq_dtype cq_linear_dtype(const cq_linear *layer);

/* Device pointers of the layer's packed arrays (any out-pointer may be NULL). */
cq_status cq_linear_device_arrays(const cq_linear *layer, const void **qweight,
                                  const void **scales, const void **biases, const void **bias);

/* Copies the layer's packed arrays into caller memory (host or device; any
 * pointer may be NULL): qweight u32 [N, K/4], scales/biases T [N, K/g], bias
 * T [N] (zeros when the layer has none).  Synchronous.  The inverse of
 * cq_linear_create, e.g. to write an artifact (weights/artifact.rs:222-240). */
cq_status cq_linear_copy_arrays(const cq_linear *layer, uint32_t *qweight, void *scales,
                                void *biases, void *bias);

/* Frees the layer and its device arrays.  NULL, and handles borrowed from an
 * encoder (cq_encoder_linear), are a no-op. */
void cq_linear_destroy(cq_linear *layer);

/*
 * Quantises the f32 weight to affine INT8 (f32 scales/biases) on the device
 * and returns input . dequant(weight)^T as f32, synchronously.
 * Replaces backend::quantized_matmul (crates/nemotron-mlx/src/backend/mod.rs:41-94),
 * with its error texts "input has {} values, expected {}x{}", "weight has {}
 * values, expected {}x{}", "group size must be positive", "input dimension {}
 * is not divisible by group size {}" (tests/quantized_matmul.rs:49-75).
 */
cq_status cq_quantized_matmul(const float *input, size_t input_len, size_t rows,
                              size_t input_dims, const float *weight, size_t weight_len,
                              size_t output_dims, size_t group_size, float *output,
                              size_t output_len);

/*
 * Device-pointer affine quantisation, groups along the last axis: w f32
 * [rows, cols] -> qweight u32 [rows, cols/4], scales/biases T [rows, cols/g].
 * round_input != 0 rounds w to T first.  Asynchronous on `stream`.
 * Replaces mlx_rs::ops::quantize(w, g, 8) (layers.rs:269, artifact.rs:296-297).
 */
cq_status cq_quantize(const float *w, int32_t rows, int32_t cols, int32_t group_size,
                      cq_dtype dtype, int32_t round_input, uint32_t *qweight, void *scales,
                      void *biases, void *stream);

/*
 * Device-pointer dequantisation to f32 [rows, cols], asynchronous.
 * Replaces mlx_rs::ops::dequantize as used by Artifact::dequantize_to_f32
 * (crates/nemotron-mlx/src/weights/artifact.rs:183-200).
 */
cq_status cq_dequantize(const uint32_t *qweight, const void *scales, const void *biases,
                        int32_t rows, int32_t cols, int32_t group_size, cq_dtype dtype, float *w,
                        void *stream);

/*
 * Reads and clears the device watchdog word of `device` (0 = clean; nonzero
 * = a kernel gave up on a bounded wait).  Synchronises the device first.
 * No reference counterpart (MLX reports device errors through eval()).
 */
cq_status cq_device_status(int32_t device, int32_t *status);

/*
 * Checks the device watchdog of `device`: one kernel waits, through the same
 * bounded wait the TMA pipelines use, on a barrier that nothing arrives on;
 * after the wait's limit (2 s) it sets the timeout bit of the watchdog word
 * and returns.  CQ_OK when that happened; the word stays set, so calls that
 * check it (cq_linear_forward_f32) report CQ_RUNTIME_ERROR until
 * cq_device_status reads and clears it.  Faults, traps and hangs nothing.
 * No reference counterpart.
 */
cq_status cq_device_watchdog_check(int32_t device);

#ifdef __cplusplus
}
#endif

#endif /* CQLINEAR_H */
