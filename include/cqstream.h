/*
 * cqstream.h - C ABI of the streaming window scheduler and the tokenizer
 * decode that catcher.h is built on, for hosts that drive the encoder and the
 * RNNT decoder themselves (cqencoder.h, cqrnnt.h, cqlogmel.h).  Host code
 * only: nothing here touches a GPU.
 */
#ifndef CQSTREAM_H
#define CQSTREAM_H

#include <stddef.h>
#include <stdint.h>

#include "cqlinear.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cq_chunk_scheduler cq_chunk_scheduler;
typedef struct cq_tokenizer cq_tokenizer;

/*
 * AudioChunkScheduler over StreamingChunkPlan::new(nemotron_3_5, lookahead)
 * (crates/nemotron-mlx/src/model/stream.rs:17-128, encoder.rs:941-994): a
 * centered first window of (8 * lookahead) * 160 + 200 samples
 * (1 + 8 * lookahead mel frames), then uncentered windows of
 * 8 * (lookahead + 1) * 160 + 400 samples, each starting 256 samples before
 * its first frame.  lookahead must be 0, 3, 6 or 13.
 */
cq_status cq_chunk_scheduler_create(int32_t lookahead, cq_chunk_scheduler **out);

/* Appends count samples; *windows = how many windows they completed (read
 * them with cq_chunk_scheduler_window before the next push/finish).  Pushing
 * after finish fails: "streaming audio session is already finished". */
cq_status cq_chunk_scheduler_push(cq_chunk_scheduler *s, const float *samples, size_t count,
                                  int32_t *windows);

/* The zero-padded last window, if any (*windows = 0 or 1); the scheduler is
 * closed until cq_chunk_scheduler_reset. */
cq_status cq_chunk_scheduler_finish(cq_chunk_scheduler *s, int32_t *windows);

/* Window `index` of the last push/finish: its sample count (always), and,
 * when samples is not NULL, up to capacity samples, whether it is centered
 * and its mel frame count. */
cq_status cq_chunk_scheduler_window(const cq_chunk_scheduler *s, int32_t index, float *samples,
                                    size_t capacity, size_t *count, int32_t *center,
                                    int32_t *mel_frames);

/* Clears buffered audio and begins a new utterance. */
cq_status cq_chunk_scheduler_reset(cq_chunk_scheduler *s);
void cq_chunk_scheduler_destroy(cq_chunk_scheduler *s);

/*
 * Tokenizer::from_json (crates/nemotron-mlx/src/tokenizer.rs:36-67): a
 * tokenizer.json with a BPE model and a Metaspace decoder ("unsupported
 * tokenizer model or decoder: A + B" otherwise).
 */
cq_status cq_tokenizer_from_json(const char *path, uint32_t pad_token_id, uint32_t blank_token_id,
                                 cq_tokenizer **out);

/* Tokenizer::decode (tokenizer.rs:69-87): pad and blank are skipped, special
 * tokens too when strip_special; "token id N is absent from tokenizer.json"
 * for unknown ids.  *text is borrowed until the next decode or destroy. */
cq_status cq_tokenizer_decode(cq_tokenizer *t, const uint32_t *ids, size_t count,
                              int32_t strip_special, const char **text);
void cq_tokenizer_destroy(cq_tokenizer *t);

#ifdef __cplusplus
}
#endif

#endif /* CQSTREAM_H */
