/*
 * cqrnnt.h - C ABI of the B200 batched RNNT greedy decoder.
 *
 * Stands in for StreamingRnntDecoder (crates/nemotron-mlx/src/model/rnnt.rs:
 * 336-388): the encoder projector, the LSTM prediction network with its
 * embedding (PredictionNetwork, :228-290), the ReLU joint and vocabulary head
 * (JointNetwork, :293-334) and the greedy loop of at most max_symbols tokens
 * per frame.  Tensors are named as in the reference artifact
 * (crates/nemotron-mlx/src/weights/manifest.rs:149-194).  Conventions are
 * those of cqlinear.h.
 *
 * A state decodes several streams in lock step over the frames of a chunk;
 * each stream follows its own greedy path (it stops emitting on a frame at its
 * own blank) and keeps its own LSTM state across chunks.
 */
#ifndef CQRNNT_H
#define CQRNNT_H

#include "cqlinear.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cq_rnnt cq_rnnt;
typedef struct cq_rnnt_state cq_rnnt_state;

typedef struct {
    int32_t enc_hidden;    /* 1024: encoder output width */
    int32_t pred_hidden;   /* 640: embedding and LSTM width */
    int32_t joint_hidden;  /* 640: projector outputs, joint input */
    int32_t vocab;         /* 13088 in the checkpoint; 1025 in the batched benchmark */
    int32_t blank;         /* vocab - 1 (13087 in the checkpoint, rnnt.rs:263) */
    int32_t lstm_layers;   /* 2 */
    int32_t max_symbols;   /* 10 per frame (rnnt.rs:357) */
    int32_t group_size;    /* 64 */
} cq_rnnt_config;

/* vocab 1025 (blank 1024), the rest as the checkpoint. */
void cq_rnnt_default_config(cq_rnnt_config *cfg);

cq_status cq_rnnt_create(const cq_rnnt_config *cfg, cq_dtype dtype, int32_t device, cq_rnnt **out);

/*
 * Binds one quantized tensor by artifact name: "encoder_projector.weight",
 * "decoder.decoder_projector.weight", "joint.head.weight" (with output biases),
 * "decoder.lstm.weight_ih_l{l}", "decoder.lstm.weight_hh_l{l}" and
 * "decoder.embedding.weight" (dequantised to T once, QuantizedEmbedding,
 * rnnt.rs:186-201).  Arrays as cq_linear_create.
 * Replaces QuantizedLinear::from_artifact at rnnt.rs:86-111, :252-266, :296-303, :341-349.
 */
cq_status cq_rnnt_set_linear(cq_rnnt *dec, const char *name, const uint32_t *qweight,
                             const void *scales, const void *biases, const void *bias_or_null,
                             int32_t output_dims, int32_t input_dims, int32_t group_size);

/* Binds "decoder.lstm.bias_ih_l{l}" / "decoder.lstm.bias_hh_l{l}" (host f32,
 * [4 * pred_hidden]); the cell adds them in T (LstmCell::from_artifact). */
cq_status cq_rnnt_set_tensor(cq_rnnt *dec, const char *name, const float *values, size_t len);
cq_status cq_rnnt_get_tensor(const cq_rnnt *dec, const char *name, float *values, size_t len);

/* Borrowed handle of a bound quantized tensor (the embedding included). */
const cq_linear *cq_rnnt_linear(const cq_rnnt *dec, const char *name);

/* Seeded synthetic weights: linears N(0, 0.02) with N(0, 0.02) output biases,
 * embedding N(0, 1), LSTM biases N(0, 0.02). */
cq_status cq_rnnt_init_random(cq_rnnt *dec, uint64_t seed);

/* One launch per LSTM layer step (enable != 0, the default where the shapes
 * fit) or separate ih, hh and cell launches; both give the same bits.  For
 * states created afterwards.  No reference counterpart. */
cq_status cq_rnnt_set_fused_lstm(cq_rnnt *dec, int32_t enable);

int32_t cq_rnnt_tensor_count(const cq_rnnt *dec);
const char *cq_rnnt_tensor_name(const cq_rnnt *dec, int32_t index);
void cq_rnnt_destroy(cq_rnnt *dec);

/*
 * Prediction state of `streams` utterances (PredictionState, rnnt.rs:210-226),
 * already advanced by the initial blank step, for chunks of up to max_frames
 * encoder frames.  Every tensor of `dec` must be bound.
 */
cq_status cq_rnnt_state_create(cq_rnnt *dec, int32_t streams, int32_t max_frames,
                               cq_rnnt_state **out);

/* Token slots per stream of one chunk: max_frames * max_symbols. */
int32_t cq_rnnt_state_capacity(const cq_rnnt_state *st);

/*
 * Greedy decode of one chunk of every stream: encoded T device [streams *
 * frames, enc_hidden] (row = stream * frames + frame, row stride ld) ->
 * device int32 tokens[streams][capacity], token_frames[streams][capacity]
 * (frame within the chunk) and counts[streams].  Asynchronous; replays a CUDA
 * graph captured on first use for each argument set.
 * Replaces StreamingRnntDecoder::decode_frames (rnnt.rs:364-388).
 */
cq_status cq_rnnt_decode_chunk(cq_rnnt_state *st, const void *encoded, int32_t ld, int32_t frames,
                               int32_t *tokens, int32_t *token_frames, int32_t *counts,
                               void *stream);

/*
 * Selects how chunks run.  enable = 0 (the default): a CUDA graph of one
 * launch per op, every frame running max_symbols iterations with per-stream
 * masks.  enable != 0: one persistent cooperative launch per chunk (every CTA
 * keeps its weight tiles in shared memory; bounded grid barriers between the
 * head, LSTM and projector phases) that skips a frame's remaining iterations
 * once every stream has emitted blank -- the faster choice when frames mostly
 * end early (trained models), the slower one when every frame emits the
 * maximum.  Fails with CQ_INVALID_ARGUMENT if the shapes do not fit it (more
 * than 64 streams, hidden sizes not multiples of 64, group sizes below 64).
 */
cq_status cq_rnnt_state_set_persistent(cq_rnnt_state *st, int32_t enable);

/* Programmatic dependent launch between the state's kernels: 1 (the default
 * unless the environment sets CQ_PDL=0) or 0 (see cq_encoder_state_set_pdl).
 * Synchronous; drops the captured chunk graphs. */
cq_status cq_rnnt_state_set_pdl(cq_rnnt_state *st, int32_t enable);

/* Kernels one chunk launches (nodes of the captured graph; 0 before capture). */
int32_t cq_rnnt_state_kernels_per_chunk(const cq_rnnt_state *st);

/* New utterances on every stream: zero LSTM state, initial blank step. Synchronous. */
cq_status cq_rnnt_state_reset(cq_rnnt_state *st);

void cq_rnnt_state_destroy(cq_rnnt_state *st);

#ifdef __cplusplus
}
#endif

#endif /* CQRNNT_H */
