/*
 * catcher.h - the transcription C ABI of Catcher, over the B200 pipeline.
 *
 * Same entry points, status codes, session states and error behaviour as the
 * reference's ABI (crates/catcher-ffi/include/catcher.h:12-113,
 * crates/catcher-ffi/src/lib.rs:251-586), so a host written against it
 * (the Swift app, the stdio host) links against this library unchanged for
 * ASR.  Behind it: the GPU log-mel frontend, the cache-aware FastConformer
 * encoder and the RNNT greedy decoder (one stream per handle), the window
 * scheduler of StreamingTranscriber (crates/nemotron-mlx/src/model/stream.rs)
 * and the Metaspace tokenizer decode (crates/nemotron-mlx/src/tokenizer.rs).
 *
 * Differences from the reference, by design of this library's scope:
 *  - no speaker diarization: a non-NULL diar_model_path makes catcher_create
 *    fail with a message saying so; catcher_segments always returns "[]" and
 *    catcher_warning always NULL (the reference's ASR-only behaviour);
 *  - the transcript is the tokenizer's decode without the OpenCC simplified
 *    to traditional Chinese conversion (text post-processing is not part of
 *    this library);
 *  - the keyword-spotting entries (catcher_kws_*, sherpa-onnx) are not
 *    provided.
 * Threading: one thread at a time per handle; distinct handles are
 * independent.  Errors of a handle are kept on the handle
 * (catcher_last_error(handle)); errors without a handle (NULL handle, failed
 * catcher_create) are thread-local (catcher_last_error(NULL)).
 */
#ifndef CATCHER_H
#define CATCHER_H

#include <stddef.h>
#include <stdint.h>

#include "cqencoder.h"
#include "cqrnnt.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct catcher_handle catcher_handle_t;
typedef int32_t catcher_status_t;

/* catcher.h:30-37 of the reference.  push/finish return CATCHER_OK when the
 * call decoded new tokens, CATCHER_NO_UPDATE otherwise. */
enum {
    CATCHER_OK = 0,
    CATCHER_NO_UPDATE = 1,
    CATCHER_COMMAND_DETECTED = 2,
    CATCHER_INVALID_ARGUMENT = -1,
    CATCHER_INVALID_STATE = -2,
    CATCHER_RUNTIME_ERROR = -3,
};

/*
 * Loads the release artifact directory asr_model_path (manifest.json,
 * weights.safetensors, tokenizer.json) onto GPU 0 and returns an idle handle,
 * or NULL with catcher_last_error(NULL) set.  language is a prompt code
 * ("en-US", "zh-TW", "auto", ...; "unsupported language prompt: X"),
 * lookahead one of 0, 3, 6, 13 encoder frames ("unsupported lookahead N;
 * supported values are [3, 0, 6, 13]").  The architecture is Nemotron 3.5's
 * (24 blocks, d 1024, 8 heads; prediction network 640) with the group size and
 * the vocabulary of the artifact; the tokenizer's pad id is 0 and its blank
 * id the vocabulary's last.  Every host-side check (paths, language,
 * lookahead, tokenizer) runs before any device work.
 * Replaces catcher_create (crates/catcher-ffi/src/lib.rs:251-303).
 */
catcher_handle_t *catcher_create(const char *asr_model_path, const char *diar_model_path,
                                 const char *language, uint32_t lookahead);

/*
 * catcher_create for other geometries: the encoder and RNNT configurations
 * are given (f16 or bf16 compute, any device).  No counterpart in the
 * reference, whose transcriber fixes the architecture.
 */
catcher_handle_t *catcher_create_config(const char *asr_model_path, const char *language,
                                        uint32_t lookahead, const cq_encoder_config *encoder,
                                        const cq_rnnt_config *rnnt, cq_dtype dtype,
                                        int32_t device);

/* Clears caches and text for a new utterance (lib.rs:310-343). */
catcher_status_t catcher_start(catcher_handle_t *handle);

/* Pushes count mono f32 16 kHz samples (samples may be NULL when count is 0);
 * CATCHER_INVALID_STATE unless a session was started and not finished
 * (lib.rs:362-399). */
catcher_status_t catcher_push_audio(catcher_handle_t *handle, const float *samples, size_t count);

/* Decodes the zero-padded last window and closes the session (lib.rs:414-416). */
catcher_status_t catcher_finish(catcher_handle_t *handle);

/* catcher_finish, then drops the tokens whose frame starts at or after
 * cutoff_ms (80 ms per encoder frame; lib.rs:423-425, :606-611). */
catcher_status_t catcher_finish_before(catcher_handle_t *handle, uint64_t cutoff_ms);

/* The current UTF-8 transcript, borrowed until the next mutating call or
 * catcher_destroy; NULL for a NULL handle (lib.rs:432-444). */
const char *catcher_text(const catcher_handle_t *handle);

/* Transcript of the tokens whose frame starts before cutoff_ms, without
 * changing the session; borrowed until the next mutating call, the next
 * catcher_text_before or catcher_destroy (lib.rs:454-484). */
const char *catcher_text_before(catcher_handle_t *handle, uint64_t cutoff_ms);

/* "[]" (no diarization model; lib.rs:497-511). */
const char *catcher_segments(const catcher_handle_t *handle);

/* NULL (no diarization model; lib.rs:528-545). */
const char *catcher_warning(const catcher_handle_t *handle);

/* The handle's last error, or this thread's for a NULL handle (lib.rs:552-566). */
const char *catcher_last_error(const catcher_handle_t *handle);

/* Releases the handle; NULL is accepted (lib.rs:573-584). */
void catcher_destroy(catcher_handle_t *handle);

#ifdef __cplusplus
}
#endif

#endif /* CATCHER_H */
