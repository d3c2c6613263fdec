/*
 * cqartifact.h - C ABI of the MLX release-artifact reader.
 *
 * An artifact is a directory holding manifest.json (format_version, model_id
 * and, per tensor, its shape and storage: "F16" or {"Int8Affine":
 * {"group_size": g}}) and weights.safetensors (an Int8Affine tensor W is stored
 * as the arrays "W.__qweight" U32 [N, K/4], "W.__scales" and "W.__biases" F16
 * [N, K/g]; an F16 tensor under its own name).  Stands in for Artifact
 * (crates/nemotron-mlx/src/weights/artifact.rs:156-252) and the from_artifact
 * constructors that bind it (QuantizedLinear::from_artifact, layers.rs:222-256;
 * StreamingEncoder::from_artifact, encoder.rs:586-640;
 * StreamingRnntDecoder::from_artifact, rnnt.rs:336-362).  Conventions are
 * those of cqlinear.h; errors carry the reference's texts ("missing artifact
 * tensor X", "missing artifact array X", "tensor X has incompatible storage
 * F16").
 */
#ifndef CQARTIFACT_H
#define CQARTIFACT_H

#include "cqencoder.h"
#include "cqlinear.h"
#include "cqrnnt.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cq_artifact cq_artifact;

typedef enum {
    CQ_STORAGE_INT8_AFFINE = 0,
    CQ_STORAGE_F16 = 1,
    CQ_STORAGE_F32 = 2,
    CQ_STORAGE_I32 = 3
} cq_storage;

/* Artifact::load (artifact.rs:157-163): parses the manifest and maps the
 * weights file read-only.  The mapping lives until cq_artifact_close. */
cq_status cq_artifact_open(const char *dir, cq_artifact **out);
void cq_artifact_close(cq_artifact *art);

const char *cq_artifact_model_id(const cq_artifact *art);
int32_t cq_artifact_format_version(const cq_artifact *art);
/* Manifest tensors in name order. */
int32_t cq_artifact_tensor_count(const cq_artifact *art);
const char *cq_artifact_tensor_name(const cq_artifact *art, int32_t index);

/* Artifact::tensor_info (artifact.rs:166-168): rank, shape (up to max_rank
 * dimensions written), storage and group size (0 unless Int8Affine).
 * CQ_INVALID_ARGUMENT with "missing artifact tensor X" if absent. */
cq_status cq_artifact_tensor_info(const cq_artifact *art, const char *name, int32_t *rank,
                                  int64_t *shape, int32_t max_rank, int32_t *storage,
                                  int32_t *group_size);

/* Artifact::f16_to_f32 (artifact.rs:200-211) into host values[len]; len must
 * equal the tensor's element count. */
cq_status cq_artifact_f16_to_f32(const cq_artifact *art, const char *name, float *values,
                                 size_t len);

/* QuantizedLinear::from_artifact (layers.rs:222-256): an owned layer on
 * `device` in `dtype` (F16 scales, quantization biases and output bias are
 * rounded to bf16 when dtype is CQ_BF16).  bias_name NULL: zero output bias. */
cq_status cq_linear_from_artifact(const cq_artifact *art, const char *weight_name,
                                  const char *bias_name_or_null, cq_dtype dtype, int32_t device,
                                  cq_linear **out);

/* Binds every tensor the encoder's configuration names (StreamingEncoder::
 * from_artifact_with_config, encoder.rs:590-640); linears with output biases
 * read "<prefix>.bias" beside "<prefix>.weight". */
cq_status cq_encoder_bind_artifact(cq_encoder *enc, const cq_artifact *art);

/* Binds every tensor of the RNNT decoder (StreamingRnntDecoder::from_artifact,
 * rnnt.rs:336-362): projectors, head, embedding, LSTM weights and biases. */
cq_status cq_rnnt_bind_artifact(cq_rnnt *dec, const cq_artifact *art);

#ifdef __cplusplus
}
#endif

#endif /* CQARTIFACT_H */
