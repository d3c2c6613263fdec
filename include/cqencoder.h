/*
 * cqencoder.h - C ABI of the B200 streaming FastConformer encoder.
 *
 * The encoder composes the affine INT8 quantized linears of cqlinear.h with
 * the supporting ops of one cache-aware streaming chunk: Conv2D subsampling,
 * 24 FastConformer blocks (LayerNorms, relative-position attention with a
 * sliding K/V window, the convolution module with its depthwise cache) and the
 * language-prompt projector.  It stands in for StreamingEncoder
 * (crates/nemotron-mlx/src/model/encoder.rs:567-655) and its layers; tensors
 * are named as in the reference artifact (crates/nemotron-mlx/src/weights/
 * manifest.rs:105-335), so an artifact loader binds them one name at a time
 * (from_artifact).  Conventions (status codes, cq_last_error, one thread per
 * handle, void* streams) are those of cqlinear.h.
 *
 * Several streams are encoded in lock step by one state: every chunk call
 * advances all of them by the same number of mel frames.  Rows of the
 * per-chunk tensors are stream-major: row = stream * frames + frame.
 */
#ifndef CQENCODER_H
#define CQENCODER_H

#include "cqlinear.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cq_encoder cq_encoder;
typedef struct cq_encoder_state cq_encoder_state;

/* Architecture constants (EncoderConfig, encoder.rs:922-955, plus the
 * subsampling and prompt-projector widths StreamingEncoder binds). */
typedef struct {
    int32_t hidden;          /* 1024 */
    int32_t ff;              /* 4096 */
    int32_t layers;          /* 24 */
    int32_t heads;           /* 8 */
    int32_t conv_kernel;     /* 9: depthwise kernel, cache of kernel-1 frames */
    int32_t sliding_window;  /* 57: attention keeps sliding_window-1 cached frames */
    int32_t mel_bins;        /* 128 */
    int32_t sub_channels;    /* 256 */
    int32_t num_prompts;     /* 128: one-hot width of the prompt projector */
    int32_t prompt_hidden;   /* 2048 */
    int32_t group_size;      /* 64 (the reference artifact uses 128) */
} cq_encoder_config;

/* Fills `cfg` with the published checkpoint's values (EncoderConfig::nemotron_3_5). */
void cq_encoder_default_config(cq_encoder_config *cfg);

/* An encoder with every tensor unset.  dtype T (CQ_F16 or CQ_BF16) is the
 * type of activations, quantisation parameters and unquantised tensors. */
cq_status cq_encoder_create(const cq_encoder_config *cfg, cq_dtype dtype, int32_t device,
                            cq_encoder **out);

/*
 * Binds one quantized linear by its artifact name, e.g.
 * "encoder.layers.3.self_attn.q_proj.weight"; arrays as cq_linear_create
 * (host or device memory), bias_or_null T [output_dims].  The dimensions must
 * be those the configuration implies for that name.
 * Replaces QuantizedLinear::from_artifact at the encoder's call sites
 * (encoder.rs:67-105, :300-318, :350-371, :736-757, prompt.rs:46-66).
 */
cq_status cq_encoder_set_linear(cq_encoder *enc, const char *name, const uint32_t *qweight,
                                const void *scales, const void *biases, const void *bias_or_null,
                                int32_t output_dims, int32_t input_dims, int32_t group_size);

/*
 * Binds one unquantised tensor (host f32, rounded to T on the device) by its
 * artifact name: LayerNorm weights/biases, bias_u / bias_v, the depthwise
 * kernels ("...conv.depthwise_conv.weight" [hidden, 1, kernel]) and the
 * subsampling Conv2D weights/biases ([channels, 1, 3, 3]).  `len` must equal
 * the element count of the name's shape.
 * Replaces Artifact::f16_to_f32 at LayerNorm::from_artifact (layers.rs:483-489),
 * DepthwiseConv1d::from_artifact (layers.rs:365-391), Fp16Conv2d::from_artifact
 * (layers.rs:47-74) and RelativePositionAttention::from_artifact (encoder.rs:74-82).
 */
cq_status cq_encoder_set_tensor(cq_encoder *enc, const char *name, const float *values,
                                size_t len);

/* Copies an unquantised tensor back to host f32 (T values widened). */
cq_status cq_encoder_get_tensor(const cq_encoder *enc, const char *name, float *values,
                                size_t len);

/* Borrowed handle of a bound quantized linear (valid while `enc` lives); use
 * cq_linear_device_arrays to read its packed arrays.  NULL if unset/unknown. */
const cq_linear *cq_encoder_linear(const cq_encoder *enc, const char *name);

/* Seeded synthetic weights for every tensor, generated and quantised on the
 * device: linears N(0, 0.02) (+ N(0, 0.02) output biases where the artifact
 * has them), LayerNorm weights 1 + N(0, 0.1), depthwise and Conv2D kernels
 * N(0, 1/3), every other unquantised tensor N(0, 0.02). */
cq_status cq_encoder_init_random(cq_encoder *enc, uint64_t seed);

/* Number of tensor names and the i-th name (linears first), for loaders. */
int32_t cq_encoder_tensor_count(const cq_encoder *enc);
const char *cq_encoder_tensor_name(const cq_encoder *enc, int32_t index);

void cq_encoder_destroy(cq_encoder *enc);

/*
 * Streaming state of `streams` utterances (StreamingEncoderCache,
 * encoder.rs:560-564, :623-639): subsampling caches, per layer the attention
 * window (sliding_window-1 frames) and the depthwise cache, all zero, plus
 * the per-chunk workspaces for chunks of up to max_mel_frames log-mel frames.
 * Every tensor of `enc` must be bound.  The prompt of every stream starts as
 * 101 ("auto", prompt.rs PROMPT_DICTIONARY).
 */
cq_status cq_encoder_state_create(cq_encoder *enc, int32_t streams, int32_t max_mel_frames,
                                  cq_encoder_state **out);

/* Per-stream prompt ids (LanguagePrompt::id, prompt.rs:18-34), each below num_prompts. */
cq_status cq_encoder_state_set_prompts(cq_encoder_state *st, const int32_t *prompt_ids,
                                       int32_t count);

/* Encoder frames the next chunk of `mel_frames` frames produces (the first
 * chunk of a state differs: its subsampling sees one extra zero frame). */
int32_t cq_encoder_state_output_frames(const cq_encoder_state *st, int32_t mel_frames);

/*
 * Encodes one chunk of every stream: mel f32 device [streams, mel_frames,
 * mel_bins] -> out T device [streams * frames, hidden], frames =
 * cq_encoder_state_output_frames(st, mel_frames).  Asynchronous on `stream`.
 * Calls after the first replay a CUDA graph of the whole chunk, captured on
 * first use for each (mel_frames, mel, out) triple.
 * Replaces StreamingEncoder::encode_chunk (encoder.rs:641-655).
 */
cq_status cq_encoder_encode_chunk(cq_encoder_state *st, const float *mel, int32_t mel_frames,
                                  void *out, void *stream);

/* Chunks encoded so far. */
int32_t cq_encoder_state_chunks(const cq_encoder_state *st);

/* Kernels one chunk launches (nodes of the captured chunk graph; 0 before the
 * first graph is captured). */
int32_t cq_encoder_state_kernels_per_chunk(const cq_encoder_state *st);

/* Zeroes every cache (a new utterance on every stream). Synchronous. */
cq_status cq_encoder_state_reset(cq_encoder_state *st);

/* Programmatic dependent launch between the state's kernels: 1 (the default
 * unless the environment sets CQ_PDL=0) or 0.  With another stream's work
 * overlapping the encoder on the same GPU (an RNNT decoder pipelined beside
 * it), 0 can be faster: kernels launched early hold SM room while they wait.
 * Synchronous; drops the captured chunk graphs. */
cq_status cq_encoder_state_set_pdl(cq_encoder_state *st, int32_t enable);

void cq_encoder_state_destroy(cq_encoder_state *st);

#ifdef __cplusplus
}
#endif

#endif /* CQENCODER_H */
