/*
 * cqchain.h - C ABI of the persistent linear-chain executor.
 *
 * A chain is a fixed sequence of quantized-linear calls on small token counts
 * (1..255 rows; the batch-1 streaming chunk has 14), planned once and then run
 * as ONE cooperative kernel launch per cq_linear_chain_run.  A run computes
 * exactly what calling cq_linear_forward_ex for every step in order on the
 * same stream computes (QuantizedLinear::forward_array,
 * crates/nemotron-mlx/src/model/layers.rs:298-310, once per linear as the
 * encoder blocks do, crates/nemotron-mlx/src/model/encoder.rs), within the
 * quantized-linear parity bar (the K reduction is split differently); it
 * replaces that sequence of launches, not an entry point of the reference.
 *
 * Dependencies come from the buffers: a step waits for earlier steps that
 * write memory it reads, read memory it writes or write memory it writes.  A
 * step whose input is (a column range of) the output of exactly one earlier
 * step, row for row, reads that output through a tagged copy -- each 8-byte
 * word carries two values and the launch's tag, so values are consumed as
 * they land, without a completion round trip.
 * Buffers are device memory that stays valid for the chain's lifetime; runs
 * of one chain must be ordered (one stream, or events).  Conventions are those
 * of cqlinear.h.
 */
#ifndef CQCHAIN_H
#define CQCHAIN_H

#include "cqlinear.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cq_linear_chain cq_linear_chain;

typedef struct {
    const cq_linear *layer;
    const void *x;   /* T device [rows, ldx], 16-byte aligned rows */
    int32_t ldx;
    int32_t rows;    /* 1..255 */
    void *y;         /* T device [rows, ldy] */
    int32_t ldy;
    int32_t act;     /* CQ_ACT_* applied to the rounded output */
} cq_chain_step;

/* Every layer on one device with one dtype (f16 or bf16) and group size. */
cq_status cq_linear_chain_create(const cq_chain_step *steps, int32_t count, cq_linear_chain **out);

/* Asynchronous on `stream` (NULL: the legacy default stream); capturable in a
 * CUDA graph. */
cq_status cq_linear_chain_run(cq_linear_chain *chain, void *stream);

/* Work decomposition of step `index`: weight rows per work item, 64-wide K
 * sub-blocks per item, K slices, the step's first work item and item count,
 * the earlier step whose tagged output it reads (-1 = none; such a step is
 * read value by value as it is produced, with no completion wait), and the
 * earlier steps whose completion it waits for (-1 = none; up to three).  For
 * tests and profiling. */
cq_status cq_linear_chain_step_info(const cq_linear_chain *chain, int32_t index, int32_t *rows_per_item,
                                    int32_t *subblocks_per_item, int32_t *kslices,
                                    int32_t *first_item, int32_t *items, int32_t *reads_tagged,
                                    int32_t *waits_for);

/* Profiling: with enable != 0 every later run records, per work item, six
 * %globaltimer stamps in ns (weight copies issued; consumers started; inputs
 * ready; weights ready; slot released; item done); work item t runs on CTA
 * t % grid.  cq_linear_chain_read_profile copies the last run's stamps,
 * [items][6], to host memory (len = items * 6). */
cq_status cq_linear_chain_profile(cq_linear_chain *chain, int32_t enable);
cq_status cq_linear_chain_read_profile(const cq_linear_chain *chain, uint64_t *stamps, size_t len);

/* Work items over all steps, and CTAs of a run (one per SM). */
int32_t cq_linear_chain_items(const cq_linear_chain *chain);
int32_t cq_linear_chain_grid(const cq_linear_chain *chain);

void cq_linear_chain_destroy(cq_linear_chain *chain);

#ifdef __cplusplus
}
#endif

#endif /* CQCHAIN_H */
